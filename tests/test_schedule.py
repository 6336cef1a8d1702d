"""Host checks of the kernel's work schedules (no GPU).

mo_gemm_schedule lists the work units of a plan with the kernel's own schedule functions
compiled for the host (csrc/gemm_kernel.cuh: tile_coords, unit_at, sk_range, sk_owner,
sk_tile_pieces).  These tests check, over the BASELINE shapes and their slabs and a sweep of
ragged shapes, with the cost model's choice and with stream-K forced, that every K chunk of
every tile is computed exactly once, and that the stream-K pieces of a split tile form one head,
any middles and one tail in the order the epilogue's fix-up relies on.  The reference's kernel
has no schedule of this kind
(src/kernels/bf16_gemm_v1.cu launches one CTA per output tile); the GPU parity tests then check
the bits these schedules produce.
"""

from __future__ import annotations

import numpy as np
import pytest

import matmul_optimizer_b200 as mo

SHAPES = [
    (6464, 7776, 7232), (6464, 976, 7232), (6464, 1952, 7232), (6464, 3888, 7232), (6464, 944, 7232),
    (8192, 8192, 8192), (4096, 28672, 8192), (4096, 3584, 8192), (4096, 7168, 8192),
    (1, 7776, 7232), (16, 7776, 7232), (129, 7776, 7232), (1000, 7776, 7232), (3333, 7776, 7232),
    (1000, 1000, 1000), (300, 1000, 4096), (129, 1000, 20000), (257, 392, 520), (513, 640, 72),
    (127, 264, 8), (2048, 2056, 4096), (5000, 3000, 7232), (256, 2000, 16384),
]


def check_schedule(m: int, n: int, k: int, num_sms: int = 148) -> dict:
    units = mo.schedule(m, n, k, num_sms)
    plan = mo.select_plan(m, n, k, num_sms)
    fields = {name: units[:, i] for i, name in enumerate(mo.SCHEDULE_FIELDS)}
    bm, bn = plan["block_m"], plan["block_n"]
    mblocks, nblocks = -(-m // bm), -(-n // bn)
    nkb = -(-k // 64)
    q = plan["num_chunks"] if plan["split"] == 0 else plan["num_chunks"]
    assert units.shape[0] > 0
    assert fields["m_block"].min() >= 0 and fields["m_block"].max() < mblocks
    assert fields["n_block"].min() >= 0 and fields["n_block"].max() < nblocks
    assert fields["chunk_begin"].min() >= 0 and (fields["chunk_end"] > fields["chunk_begin"]).all()
    # Every K chunk of every tile exactly once.
    cover = np.zeros((mblocks, nblocks, q), dtype=np.int32)
    for u in units:
        cover[u[2], u[3], u[4]:u[5]] += 1
    assert (cover == 1).all(), (m, n, k, np.argwhere(cover != 1)[:5])
    # Clusters' positions run 0, 1, 2, ... in order.
    for c in np.unique(fields["cluster"]):
        pos = fields["position"][fields["cluster"] == c]
        assert (pos == np.arange(len(pos))).all()
    # Stream-K pieces: one head (from chunk 0) and one tail (to the last chunk) per split tile,
    # pieces of one tile on distinct clusters, heads and middles before a cluster's whole tiles,
    # tails after them.
    pieces = units[fields["sk_tile"] >= 0]
    if len(pieces):
        assert plan["stream_k"] == 1
        sk_tiles = np.unique(pieces[:, 6])
        clusters = plan["grid"] // plan["cta_group"]
        leftover = plan["num_tiles"] % clusters
        # Workspace slots and arrival words exist for the leftover tiles only (a leftover tile
        # that one cluster runs whole is not split).
        assert sk_tiles.min() >= 0 and sk_tiles.max() < leftover
        assert leftover * plan["cta_group"] <= 1024  # arrival words of one region
        for st in sk_tiles:
            tp = pieces[pieces[:, 6] == st]
            tp = tp[np.argsort(tp[:, 4])]
            assert len(tp) >= 2
            assert len({(r[2], r[3]) for r in tp}) == 1
            assert tp[0, 4] == 0 and tp[-1, 5] == q
            assert (tp[1:, 4] == tp[:-1, 5]).all()
            assert len(np.unique(tp[:, 0])) == len(tp)
        for c in np.unique(fields["cluster"]):
            cu = units[fields["cluster"] == c]
            kinds = []
            for u in cu:
                if u[6] < 0:
                    kinds.append(1)
                elif u[5] == q and u[4] > 0:
                    kinds.append(2)
                else:
                    kinds.append(0)
            assert kinds == sorted(kinds), (c, kinds)
    return {"units": units, "plan": plan}


@pytest.mark.parametrize("shape", SHAPES)
def test_schedule_covers_every_chunk_once(shape):
    check_schedule(*shape)


@pytest.mark.parametrize("shape", SHAPES)
def test_forced_stream_k_schedule_covers_every_chunk_once(shape, monkeypatch):
    monkeypatch.setenv("MO_GEMM_STREAMK", "1")
    check_schedule(*shape)


@pytest.mark.parametrize("variant", ["pair256", "1x256", "1x128", "1x64", "pair128"])
@pytest.mark.parametrize("shape", [(6464, 976, 7232), (1000, 1000, 1000), (300, 1000, 4096), (4096, 3584, 8192)])
def test_every_variant_schedule_with_stream_k(shape, variant, monkeypatch):
    monkeypatch.setenv("MO_GEMM_VARIANT", variant)
    monkeypatch.setenv("MO_GEMM_STREAMK", "1")
    check_schedule(*shape)


def test_ragged_sweep_schedules(monkeypatch):
    rng = np.random.default_rng(11)
    for mode in ("", "1"):
        monkeypatch.setenv("MO_GEMM_STREAMK", mode)
        for _ in range(40):
            m = int(rng.integers(1, 9000))
            n = int(rng.integers(1, 1200)) * 8
            k = int(rng.integers(1, 1400)) * 8
            check_schedule(m, n, k)


def test_slab8_stream_k_plan():
    """The 8-GPU slab 6464x976: 104 pair tiles on 74 clusters.  One whole tile per cluster, then
    the 30 leftover tiles' 120 K chunks two to a cluster over 60 clusters: every split tile is a
    head (chunks 0-1) and a tail (chunks 2-3) on two clusters, and no cluster runs more than two
    stream-K chunks."""
    units = check_schedule(6464, 976, 7232)["units"]
    pieces = units[units[:, 6] >= 0]
    assert len(np.unique(pieces[:, 6])) == 30 and len(pieces) == 60
    assert ((pieces[:, 5] - pieces[:, 4]) == 2).all()
    whole = units[units[:, 6] < 0]
    assert len(whole) == 74 and len(np.unique(whole[:, 0])) == 74


def test_schedule_and_plan_reject_bad_arguments(monkeypatch):
    """mo_gemm_schedule validates like the launch: a null count, a negative capacity, a
    non-positive dimension or SM count, and an invalid override each return an error code."""
    import ctypes

    lib = mo.load_library()
    count = ctypes.c_int(0)
    assert lib.mo_gemm_schedule(64, 64, 64, 148, None, 0, None) == mo.MO_ERR_NULL_POINTER
    assert lib.mo_gemm_schedule(64, 64, 64, 148, None, 4, ctypes.byref(count)) == mo.MO_ERR_NULL_POINTER
    assert lib.mo_gemm_schedule(64, 64, 64, 148, None, -1, ctypes.byref(count)) == mo.MO_ERR_BAD_ARGUMENT
    assert lib.mo_gemm_schedule(0, 64, 64, 148, None, 0, ctypes.byref(count)) == mo.MO_ERR_BAD_DIMS
    assert lib.mo_gemm_schedule(64, 64, 64, 0, None, 0, ctypes.byref(count)) == mo.MO_ERR_BAD_ARGUMENT
    # A capacity below the total writes only that many units and still reports the total.
    total = len(mo.schedule(6464, 976, 7232))
    buf = (ctypes.c_int * (7 * 3))()
    assert lib.mo_gemm_schedule(6464, 976, 7232, 148, buf, 3, ctypes.byref(count)) == mo.MO_OK
    assert count.value == total and total > 3
    monkeypatch.setenv("MO_GEMM_STREAMK", "7")
    assert lib.mo_gemm_schedule(64, 64, 64, 148, None, 0, ctypes.byref(count)) == mo.MO_ERR_BAD_ARGUMENT
    with pytest.raises(mo.MoGemmError):
        mo.select_plan(64, 64, 64, 148)
