"""The N>1 host path on CPU: two gloo ranks partition C by columns through the library's
partition, compute their slabs (numpy stands in for the GPU GEMM here), all-gather padded
slabs, re-layout, and get the full product; the max-over-ranks timing reduce is checked too."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from matmul_optimizer_b200 import sharding


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        a = rng.integers(-4, 5, size=(m, k)).astype(np.float32)
        b = rng.integers(-4, 5, size=(k, n)).astype(np.float32)
        slabs = sharding.partition(n, world)
        mine = slabs[rank]
        c_slab = a @ sharding.slab_columns(b, mine)
        block = sharding.padded_block(c_slab, slabs[0].width)
        gathered = torch.empty(world * block.size, dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, torch.from_numpy(block))
        full = sharding.assemble(gathered.numpy(), slabs, m)
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, bool(np.array_equal(full, a @ b)), float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n", [(2, 7776), (2, 100), (3, 64)])
def test_two_rank_shard_gather_roundtrip(world, n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 37, n, 24, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in results] == [True] * world
    assert [r[2] for r in results] == [float(world)] * world


def test_assemble_matches_partition_edges():
    slabs = sharding.partition(7776, 8)
    m = 5
    full = np.arange(m * 7776, dtype=np.int32).reshape(m, 7776)
    blocks = np.concatenate([sharding.padded_block(sharding.slab_columns(full, s), slabs[0].width) for s in slabs])
    assert np.array_equal(sharding.assemble(blocks, slabs, m), full)


def test_row_shards_cover_a():
    """The end-to-end path's row shards of A (padded to equal height for the all-gather) cover
    every row once, and the gathered buffer's first m rows are A."""
    from matmul_optimizer_b200 import sharding

    for m, g in [(6464, 8), (6464, 3), (1, 4), (10, 4)]:
        a = np.arange(m * 3, dtype=np.int16).reshape(m, 3)
        shards = []
        for r in range(g):
            r0, r1, h = sharding.row_shard(m, g, r)
            block = np.zeros((h, 3), dtype=np.int16)
            block[: r1 - r0] = a[r0:r1]
            shards.append(block)
        gathered = np.concatenate(shards)
        assert np.array_equal(gathered[:m], a)
