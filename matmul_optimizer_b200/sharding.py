"""N-sharding of one GEMM across the GPUs of a node (no reference counterpart: the reference is
single-GPU).

C is split into column slabs: slab r covers columns [r*w, min((r+1)*w, n)) with
w = roundup16(ceil(n / g)).  Rank r holds the full A and a contiguous copy of its B slab on its
own GPU and computes its C slab with the ordinary 1-GPU call, so the data path has no
collective and no peer access, and (the kernel's K order being the same for every shape) each
slab is bit-identical to the same columns of a 1-GPU run.  An optional all-gather of the slabs
(NCCL through torch.distributed) plus a column re-layout rebuilds C on every rank.

The partition comes from the library (mo_shard_partition), so the Python side and the C
runner agree by construction.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import numpy as np


@dataclass(frozen=True)
class Slab:
    rank: int
    begin: int
    width: int


def partition(n: int, g: int) -> List[Slab]:
    from . import shard_partition

    begins, widths = shard_partition(n, g)
    return [Slab(r, b, w) for r, (b, w) in enumerate(zip(begins, widths))]


def slab_columns(b: np.ndarray, slab: Slab) -> np.ndarray:
    """Contiguous copy of B[:, slab] (the bytes a rank copies to its GPU)."""
    return np.ascontiguousarray(b[:, slab.begin:slab.begin + slab.width])


def padded_block(c_slab: np.ndarray, block_width: int) -> np.ndarray:
    """Rank's all-gather send buffer: its [m, width] slab flattened into m*block_width
    elements (the tail of a narrower last slab is zero padding)."""
    m = c_slab.shape[0]
    out = np.zeros(m * block_width, dtype=c_slab.dtype)
    out[: c_slab.size] = c_slab.reshape(-1)
    return out


def assemble(gathered: np.ndarray, slabs: Sequence[Slab], m: int) -> np.ndarray:
    """Host-side column re-layout of an all-gather result (the same mapping the device kernel
    mo_unshard_columns applies): block r of `gathered` holds slab r row-major."""
    n = sum(s.width for s in slabs)
    block = gathered.reshape(len(slabs), -1)
    out = np.empty((m, n), dtype=gathered.dtype)
    for s in slabs:
        if s.width:
            out[:, s.begin:s.begin + s.width] = block[s.rank, : m * s.width].reshape(m, s.width)
    return out


def row_shard(m: int, g: int, rank: int) -> tuple:
    """Rows [begin, end) of A that rank `rank` holds in host memory when A is sharded by rows
    for the end-to-end path; every rank's shard is padded to ceil(m / g) rows for the
    all-gather."""
    h = -(-m // g)
    begin = min(rank * h, m)
    return begin, min(begin + h, m), h


def gemm_sharded_from_host(a_rows_host, a_shard_dev, a_full_dev, b_slab_host, c_slab_host,
                           m: int, k: int, slab_width: int, stream=None, group=None) -> int:
    """One rank's step of the N-sharded GEMM from host buffers.

    Each rank holds only its row shard of A (`a_rows_host`, padded to the shard height) and its
    column slab of B in page-locked host memory.  The shard goes up over PCIe; the full A is
    assembled on every GPU by an all-gather over NVLink (NCCL; `a_full_dev` holds g shards,
    its first m rows are A); then B's slab goes up, the slab GEMMs run and C's slab comes down,
    overlapped by the library (mo_gemm_b_from_host).  Each rank moves 1/g of A plus its slab of
    B over PCIe, instead of all of A.  Returns the library's status code."""
    import torch
    import torch.distributed as dist

    from . import gemm_b_from_host

    a_shard_dev.copy_(a_rows_host, non_blocking=True)
    # NCCL has no int16; the bits travel as bfloat16 unchanged.
    dist.all_gather_into_tensor(a_full_dev.view(torch.bfloat16), a_shard_dev.view(torch.bfloat16),
                                group=group)
    return gemm_b_from_host(a_full_dev.data_ptr(), b_slab_host.data_ptr(), c_slab_host.data_ptr(),
                            m, slab_width, k, 0, stream)
