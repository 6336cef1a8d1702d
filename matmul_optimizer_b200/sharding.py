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
