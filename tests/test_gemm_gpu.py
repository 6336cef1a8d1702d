"""Parity of the sm_100a GEMM (through the C ABI) against the CPU oracle.

Tolerances, per element (written here so the bar is visible in the test):
  * the reference runner's rule  |out - ref_fp32| <= 0.15 + 0.01 |ref_fp32|
    (src/runner/main.cpp:324-365, configs/fixed_bf16_gemm_v1.json:32-38);
  * the north-star bound          |out - exact| <= 2^-7 |exact| + 1e-2 sqrt(K) max|A| max|B| / K
    against the float64 product of the same BF16 inputs;
  * BF16 bit agreement with the reference's RNE(C_ref_fp32) on at least 97 % of elements
    (the two FP32 sums differ only in summation order, so mismatches are rounding-boundary
    cases only).
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import matmul_optimizer_b200 as mo
from oracle import bf16_oracle as orc
from tests.gpu_utils import gemm_dev, run_gemm, to_device, to_host

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
BF16_AGREEMENT = 0.97


def check_against_oracle(out, a_bits, b_bits, ref32=None, ref16=None, exact=None):
    if ref32 is None:
        ref32 = orc.reference_gemm_fp32(a_bits, b_bits)
    if ref16 is None:
        ref16 = orc.float32_to_bf16_bits(ref32)
    res = orc.evaluate_correctness(out, ref32, ref16)
    assert res["passed"], res
    if exact is None:
        exact = orc.reference_gemm_fp64(a_bits, b_bits)
    ns = orc.check_north_star(out, exact, a_bits, b_bits)
    assert ns["passed"], ns
    agree = float(np.mean(out.reshape(-1) == ref16.reshape(-1)))
    assert agree >= BF16_AGREEMENT, agree
    return res, ns, agree


def test_small_golden_cases(cuda_device):
    data = np.load(GOLDEN / "small_cases.npz")
    index = json.loads((GOLDEN / "small_cases_index.json").read_text())
    for entry in index:
        key = entry["key"]
        a, b = data[f"{key}_a"], data[f"{key}_b"]
        out = run_gemm(a, b)
        check_against_oracle(out, a, b, data[f"{key}_c32"], data[f"{key}_c16"])


@pytest.mark.parametrize("shape", [(1, 8, 8), (3, 16, 24), (127, 264, 8), (128, 256, 64),
                                   (255, 392, 520), (300, 8, 4096), (64, 4104, 64),
                                   (513, 640, 72), (1000, 1000, 1000)])
def test_edge_shapes(cuda_device, shape):
    m, n, k = shape
    case = orc.make_uniform_case(m, n, k, seed=11 + m + n + k)
    out = run_gemm(case.a_bits, case.b_bits)
    check_against_oracle(out, case.a_bits, case.b_bits)


def test_hero_shape_seed_3407(cuda_device):
    pins = json.loads((GOLDEN / "hero_pins.json").read_text())
    m, n, k = pins["shape"]
    case = orc.make_uniform_case(m, n, k, 3407)
    seed = pins["seeds"]["3407"]
    # The inputs on this machine are the reference's inputs, byte for byte.
    assert orc.sha256_bytes(case.a_bits) == seed["sha256_A_bf16"]
    assert orc.sha256_bytes(case.b_bits) == seed["sha256_B_bf16"]
    out = run_gemm(case.a_bits, case.b_bits)
    ref32 = orc.reference_gemm_fp32(case.a_bits, case.b_bits)
    res = orc.evaluate_correctness(out, ref32, orc.float32_to_bf16_bits(ref32))
    assert res["passed"], res
    rows, cols = np.array(pins["sample_rows"]), np.array(pins["sample_cols"])
    exact = np.array(seed["c_exact_f64_samples"])
    ns = orc.check_north_star(out[rows, cols], exact, case.a_bits, case.b_bits)
    assert ns["passed"], ns
    # The reference's own C_ref_fp32 at the pinned positions agrees with ours within its rule.
    ref_samples = np.array(seed["c_ref_fp32_samples"], dtype=np.float32)
    got = orc.bf16_bits_to_float32(out[rows, cols]).astype(np.float64)
    assert np.all(np.abs(got - ref_samples) <= 0.15 + 0.01 * np.abs(ref_samples))


@pytest.mark.parametrize("m", [1, 16, 129, 1000, 3333])
def test_ragged_sweep(cuda_device, m):
    case = orc.make_uniform_case(m, 7776, 7232, 3407)
    out = run_gemm(case.a_bits, case.b_bits)
    ref32 = orc.reference_gemm_fp32(case.a_bits, case.b_bits)
    res = orc.evaluate_correctness(out, ref32, orc.float32_to_bf16_bits(ref32))
    assert res["passed"], res
    agree = float(np.mean(out == orc.float32_to_bf16_bits(ref32)))
    assert agree >= BF16_AGREEMENT, agree
    ns = orc.check_north_star(out, orc.reference_gemm_fp64(case.a_bits, case.b_bits), case.a_bits, case.b_bits)
    assert ns["passed"], ns


def test_hero_north_star_row_band(cuda_device):
    """Every element of a 512-row band of the hero output meets the north-star bound against
    the float64 product (the near-zero outputs are where a single FP32 TMEM accumulator over
    K = 7232 fails it)."""
    case = orc.make_uniform_case(6464, 7776, 7232, 1729)
    out = run_gemm(case.a_bits, case.b_bits)
    rows = slice(6464 - 512, 6464)  # includes the ragged last row band
    exact = orc.reference_gemm_fp64(case.a_bits[rows], case.b_bits)
    ns = orc.check_north_star(out[rows], exact, case.a_bits, case.b_bits)
    assert ns["passed"], ns


@pytest.mark.parametrize("shape", [(256, 512, 16384), (128, 264, 32768), (64, 1024, 65536)])
def test_north_star_long_k(cuda_device, shape):
    """The two-level accumulation keeps the north-star bound at K well beyond the hero's."""
    m, n, k = shape
    case = orc.make_uniform_case(m, n, k, seed=k)
    out = run_gemm(case.a_bits, case.b_bits)
    ns = orc.check_north_star(out, orc.reference_gemm_fp64(case.a_bits, case.b_bits), case.a_bits, case.b_bits)
    assert ns["passed"], ns


@pytest.mark.parametrize("which", ["square_8192", "llm_4096x28672x8192"])
def test_north_star_k8192_row_band(cuda_device, which):
    if which == "square_8192":
        case = orc.make_uniform_case(8192, 8192, 8192, 3407)
    else:
        case = orc.make_normal_case(4096, 28672, 8192, 3407, 9713, 1.0, 0.02)
    out = run_gemm(case.a_bits, case.b_bits)
    rows = slice(0, 128)
    ns = orc.check_north_star(out[rows], orc.reference_gemm_fp64(case.a_bits[rows], case.b_bits),
                              case.a_bits, case.b_bits)
    assert ns["passed"], ns


def test_nshard_bit_identical(cuda_device):
    case = orc.make_uniform_case(6464, 7776, 7232, 9713)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    full = to_host(gemm_dev(a, b))
    for g in (2, 4, 8):
        begins, widths = mo.shard_partition(7776, g)
        for begin, width in zip(begins, widths):
            slab_b = b[:, begin:begin + width].contiguous()
            slab = to_host(gemm_dev(a, slab_b))
            assert np.array_equal(slab, full[:, begin:begin + width]), (g, begin, width)


@pytest.mark.parametrize("g", [2, 8])
def test_gemm_nshard_entry_point_on_one_device(cuda_device, g):
    """mo_gemm_nshard, the C ABI's multi-device entry, with every slab on device 0 (each on its
    own stream): each slab is bit-identical to the same columns of the 1-GPU call, and the
    caller's current device is restored."""
    m, n, k = 6464, 7776, 7232
    case = orc.make_uniform_case(m, n, k, seed=9713)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    full = to_host(gemm_dev(a, b))
    begins, widths = mo.shard_partition(n, g)
    b_slabs = [b[:, b0:b0 + w].contiguous() for b0, w in zip(begins, widths)]
    c_slabs = [torch.full((m, w), 0x7FC0, dtype=torch.int16, device="cuda:0") for w in widths]
    streams = [torch.cuda.Stream() for _ in range(g)]
    torch.cuda.synchronize()
    mo.gemm_nshard([0] * g, [a.data_ptr()] * g, [t.data_ptr() for t in b_slabs],
                   [t.data_ptr() for t in c_slabs], m, k, widths, streams)
    torch.cuda.synchronize()
    assert torch.cuda.current_device() == 0
    for b0, w, c in zip(begins, widths, c_slabs):
        assert np.array_equal(to_host(c), full[:, b0:b0 + w]), (g, b0, w)
    assert mo.read_watchdog(clear=True) == 0


def test_deterministic(cuda_device):
    case = orc.make_uniform_case(2048, 2048, 4096, 5)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    first = to_host(gemm_dev(a, b))
    for _ in range(3):
        assert np.array_equal(first, to_host(gemm_dev(a, b)))


def test_no_writes_outside_c(cuda_device):
    m, n, k = 259, 264, 200
    case = orc.make_uniform_case(m, n, k, 3)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    guard = 4096
    buf = torch.full((guard * 2 + m * n,), 0x5A5A, dtype=torch.int16, device="cuda:0")
    c = buf[guard:guard + m * n]
    rc = mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream())
    assert rc == mo.MO_OK
    torch.cuda.synchronize()
    host = buf.cpu().numpy()
    assert np.all(host[:guard] == 0x5A5A) and np.all(host[guard + m * n:] == 0x5A5A)
    check_against_oracle(host[guard:guard + m * n].view(np.uint16).reshape(m, n), case.a_bits, case.b_bits)


@pytest.mark.parametrize("shape,offsets", [((5, 7, 9), (0, 0, 0)), ((3, 1001, 1003), (0, 0, 0)),
                                           ((130, 264, 60), (2, 0, 0)), ((64, 64, 64), (2, 6, 10)),
                                           ((257, 390, 7230), (0, 2, 4)), ((1000, 999, 1001), (0, 0, 0))])
def test_unaligned_layouts_through_padded_copies(cuda_device, shape, offsets):
    """k or n not a multiple of 8, or a pointer off a 16-byte boundary: the call copies A and B
    into padded buffers, runs the tensor-core GEMM there and copies C back.  The result meets the
    reference rule and the north-star bound, and nothing outside C is written."""
    m, n, k = shape
    case = orc.make_uniform_case(m, n, k, seed=3 * m + 5 * n + k)
    oa, ob, oc = (o // 2 for o in offsets)  # element offsets from 16-byte aligned bases
    guard = 64
    a_buf = torch.from_numpy(np.concatenate([np.zeros(oa, np.uint16), case.a_bits.reshape(-1)]).view(np.int16)).cuda()
    b_buf = torch.from_numpy(np.concatenate([np.zeros(ob, np.uint16), case.b_bits.reshape(-1)]).view(np.int16)).cuda()
    c_buf = torch.full((guard + oc + m * n + guard,), 0x5A5A, dtype=torch.int16, device="cuda:0")
    c_ptr = c_buf.data_ptr() + 2 * (guard + oc)
    rc = mo.launch(a_buf.data_ptr() + 2 * oa, b_buf.data_ptr() + 2 * ob, c_ptr, m, n, k,
                   torch.cuda.current_stream())
    assert rc == mo.MO_OK, mo.error_string(rc)
    torch.cuda.synchronize()
    host = c_buf.cpu().numpy()
    assert np.all(host[:guard + oc] == 0x5A5A) and np.all(host[guard + oc + m * n:] == 0x5A5A)
    out = host[guard + oc:guard + oc + m * n].view(np.uint16).reshape(m, n)
    check_against_oracle(out, case.a_bits, case.b_bits)
    assert mo.read_watchdog(clear=True) == 0


def test_error_codes_and_watchdog(cuda_device):
    a = torch.zeros((64, 64), dtype=torch.int16, device="cuda:0")
    c = torch.zeros((64, 64), dtype=torch.int16, device="cuda:0")
    s = torch.cuda.current_stream()
    assert mo.launch(0, a.data_ptr(), c.data_ptr(), 64, 64, 64, s) == mo.MO_ERR_NULL_POINTER
    assert mo.launch(a.data_ptr(), a.data_ptr(), c.data_ptr(), 0, 64, 64, s) == mo.MO_ERR_BAD_DIMS
    assert mo.launch(a.data_ptr() + 1, a.data_ptr(), c.data_ptr(), 8, 8, 8, s) == mo.MO_ERR_UNSUPPORTED
    assert mo.launch_bf16_gemm_v1(a.data_ptr(), a.data_ptr(), c.data_ptr(), 64, 64, 64, s)
    assert mo.read_watchdog(clear=True) == 0
    # A wait nobody completes: the bounded wait expires, the flag records it, the context lives.
    mo.selftest_wait_timeout(20000)
    assert mo.read_watchdog(clear=True) == 6
    assert mo.read_watchdog(clear=False) == 0
    case = orc.make_uniform_case(130, 264, 200, 1)
    check_against_oracle(run_gemm(case.a_bits, case.b_bits), case.a_bits, case.b_bits)


def test_unshard_columns(cuda_device):
    m, n, g = 37, 7776, 8
    begins, widths = mo.shard_partition(n, g)
    w = widths[0]
    rng = np.random.default_rng(0)
    full = rng.integers(-30000, 30000, size=(m, n), dtype=np.int16)
    gathered = np.zeros((g, m * w), dtype=np.int16)
    for i, (b0, wi) in enumerate(zip(begins, widths)):
        gathered[i, :m * wi] = full[:, b0:b0 + wi].reshape(-1)
    gd = torch.from_numpy(gathered).cuda()
    out = torch.empty((m, n), dtype=torch.int16, device="cuda:0")
    mo.unshard_columns(gd.data_ptr(), out.data_ptr(), m, widths, m * w, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), full)


def test_square_8192(cuda_device):
    case = orc.make_uniform_case(8192, 8192, 8192, 3407)
    out = run_gemm(case.a_bits, case.b_bits)
    ref32 = orc.reference_gemm_fp32(case.a_bits, case.b_bits)
    res = orc.evaluate_correctness(out, ref32, orc.float32_to_bf16_bits(ref32))
    assert res["passed"], res


@pytest.mark.parametrize("shape", [(98304, 4096, 128), (1, 1 << 20, 64), (65536, 64, 1024)])
def test_many_tiles_sampled(cuda_device, shape):
    """Large tile counts for the persistent schedule: 6144 pair tiles (83 waves), a 1-row GEMM
    16384 column blocks wide, and a tall, thin C.  A sample of rows is checked against the
    float64 product; the rest of C must not keep the canary the buffer was filled with."""
    m, n, k = shape
    rng = np.random.default_rng(m + n + k)
    a_bits = orc.float32_to_bf16_bits(rng.uniform(-1, 1, (m, k)).astype(np.float32))
    b_bits = orc.float32_to_bf16_bits(rng.uniform(-1, 1, (k, n)).astype(np.float32))
    a, b = to_device(a_bits), to_device(b_bits)
    c = torch.full((m, n), 0x7FC1, dtype=torch.int16, device="cuda:0")  # a NaN canary
    rc = mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream())
    assert rc == mo.MO_OK, mo.error_string(rc)
    torch.cuda.synchronize()
    assert not bool((c == 0x7FC1).any())
    rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, 256)]))
    out = to_host(c[torch.from_numpy(rows).cuda()])
    exact = orc.reference_gemm_fp64(a_bits[rows], b_bits)
    ns = orc.check_north_star(out, exact, a_bits, b_bits)
    assert ns["passed"], ns
    assert mo.read_watchdog(clear=True) == 0


@pytest.mark.parametrize("shape", [(139264, 16384, 64), (270336, 64, 8192), (64, 270336, 8192)])
def test_operands_past_32_bit_element_offsets(cuda_device, shape):
    """One operand holds more than 2^31 elements (C, then A, then B; about 4.5 GB each), so a
    32-bit element offset anywhere in the kernel, the tensor maps or the host planning would
    wrap.  The inputs are drawn on the device; sampled rows and columns of C are checked
    against the float64 product, and no element of C may keep the canary."""
    m, n, k = shape
    assert max(m * n, m * k, k * n) > 2**31
    gen = torch.Generator(device="cuda:0").manual_seed(m + n + k)
    a = torch.empty((m, k), dtype=torch.bfloat16, device="cuda:0").uniform_(-1, 1, generator=gen)
    b = torch.empty((k, n), dtype=torch.bfloat16, device="cuda:0").uniform_(-1, 1, generator=gen)
    a, b = a.view(torch.int16), b.view(torch.int16)
    c = torch.full((m, n), 0x7FC1, dtype=torch.int16, device="cuda:0")  # a NaN canary
    rc = mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream())
    assert rc == mo.MO_OK, mo.error_string(rc)
    torch.cuda.synchronize()
    assert not bool((c == 0x7FC1).any())
    rng = np.random.default_rng(k)
    rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, 128)]))
    cols = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, 512)]))
    r_idx, c_idx = torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()
    a_s, b_s = to_host(a[r_idx]), to_host(b[:, c_idx])
    out = to_host(c[r_idx][:, c_idx])
    ns = orc.check_north_star(out, orc.reference_gemm_fp64(a_s, b_s), a_s, b_s)
    assert ns["passed"], ns
    assert mo.read_watchdog(clear=True) == 0


def test_non_finite_inputs_propagate(cuda_device):
    """An Inf in A and a NaN in B reach C where IEEE arithmetic puts them: the Inf's row of C is
    +-Inf (NaN where it meets the NaN), the NaN's column is NaN, and every other element is
    finite and inside the bound.  The NaN/Inf pattern equals the oracle's FP32 product."""
    m, n, k = 192, 264, 200
    case = orc.make_uniform_case(m, n, k, seed=77)
    a_bits, b_bits = case.a_bits.copy(), case.b_bits.copy()
    a_bits[3, 17] = 0x7F80   # +Inf
    b_bits[150, 5] = 0x7FC0  # NaN
    out = run_gemm(a_bits, b_bits)
    ref32 = orc.reference_gemm_fp32(a_bits, b_bits)
    got = orc.bf16_bits_to_float32(out)
    assert np.array_equal(np.isnan(got), np.isnan(ref32))
    assert np.array_equal(np.isposinf(got), np.isposinf(ref32))
    assert np.array_equal(np.isneginf(got), np.isneginf(ref32))
    assert np.isnan(got[:, 5]).all() and not np.isfinite(got[3]).any()
    finite = np.isfinite(ref32)
    rows = np.array([r for r in range(m) if r != 3])
    cols = np.array([c for c in range(n) if c != 5])
    clean = out[np.ix_(rows, cols)]
    exact = orc.reference_gemm_fp64(case.a_bits[rows], case.b_bits[:, cols])
    assert finite[np.ix_(rows, cols)].all()
    assert orc.check_north_star(clean, exact, case.a_bits, case.b_bits)["passed"]


def test_llm_projection(cuda_device):
    case = orc.make_normal_case(4096, 28672, 8192, 3407, 9713, 1.0, 0.02)
    out = run_gemm(case.a_bits, case.b_bits)
    ref32 = orc.reference_gemm_fp32(case.a_bits, case.b_bits)
    res = orc.evaluate_correctness(out, ref32, orc.float32_to_bf16_bits(ref32))
    assert res["passed"], res
    agree = float(np.mean(out == orc.float32_to_bf16_bits(ref32)))
    assert agree >= BF16_AGREEMENT, agree


VARIANTS = ["pair256", "1x256", "1x128", "1x64", "pair128"]


@pytest.mark.parametrize("shape", [(1, 7776, 7232), (16, 7776, 7232), (129, 7776, 7232),
                                   (300, 1000, 4096), (256, 392, 30000),
                                   (192, 520, 4000), (257, 392, 3000)])  # 96-row 1-CTA tiles
def test_variants_and_split_bit_identical(cuda_device, monkeypatch, shape):
    """Every kernel variant, split across CTAs or not, gives the same bits: the K chunks depend
    on K alone and their FP32 sums run in the same order.  The result also meets the oracle."""
    m, n, k = shape
    case = orc.make_uniform_case(m, n, k, seed=m + n + k)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    outs = {}
    for variant in VARIANTS:
        for split in ("0", "1"):
            monkeypatch.setenv("MO_GEMM_VARIANT", variant)
            monkeypatch.setenv("MO_GEMM_SPLIT", split)
            outs[(variant, split)] = to_host(gemm_dev(a, b))
    monkeypatch.delenv("MO_GEMM_VARIANT")
    monkeypatch.delenv("MO_GEMM_SPLIT")
    ref = to_host(gemm_dev(a, b))  # the cost model's own choice
    for key, out in outs.items():
        assert np.array_equal(out, ref), key
    assert mo.read_watchdog(clear=True) == 0
    exact = orc.reference_gemm_fp64(case.a_bits, case.b_bits)
    assert orc.check_north_star(ref, exact, case.a_bits, case.b_bits)["passed"]


@pytest.mark.parametrize("shape", [(6464, 976, 7232), (1000, 7776, 7232), (300, 1000, 4096),
                                   (256, 392, 30000), (1, 7776, 7232), (129, 1000, 20000)])
def test_stream_k_bit_identical(cuda_device, monkeypatch, shape):
    """The stream-K schedule (the last partial wave's K chunks spread over every cluster, the
    split tiles finished from their pieces' FP32 results) gives the same bits as whole tiles, for
    every kernel variant: the head piece's running sum plus the later chunks in order is the
    same sequence of FP32 adds.  (6464, 976) is the hero's column slab on 8 GPUs."""
    m, n, k = shape
    case = orc.make_uniform_case(m, n, k, seed=3 * m + n + k)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    monkeypatch.setenv("MO_GEMM_SPLIT", "0")
    outs = {}
    for variant in VARIANTS:
        for sk in ("0", "1"):
            monkeypatch.setenv("MO_GEMM_VARIANT", variant)
            monkeypatch.setenv("MO_GEMM_STREAMK", sk)
            outs[(variant, sk)] = to_host(gemm_dev(a, b))
    for name in ("MO_GEMM_VARIANT", "MO_GEMM_STREAMK", "MO_GEMM_SPLIT"):
        monkeypatch.delenv(name)
    ref = to_host(gemm_dev(a, b))  # the cost model's own choice
    for key, out in outs.items():
        assert np.array_equal(out, ref), key
    assert mo.read_watchdog(clear=True) == 0
    exact = orc.reference_gemm_fp64(case.a_bits, case.b_bits)
    assert orc.check_north_star(ref, exact, case.a_bits, case.b_bits)["passed"]


@pytest.mark.parametrize("shape", [(6464, 976, 7232), (300, 1000, 4096), (129, 1000, 20000),
                                   (1000, 7776, 7232), (4096, 3584, 8192), (6464, 3888, 7232),
                                   (129, 7776, 7232)])
def test_stream_k_repeated_launches_bit_identical(cuda_device, monkeypatch, shape):
    """A split tile is finished by its tail piece from the head's published running sum (and any
    middle piece's chunks): the same FP32 adds in the same order as whole tiles, launch after
    launch.  (4096, 3584, 8192) is the LLM projection's 8-GPU slab, whose split tiles have a head,
    middles and a tail on five clusters; (6464, 3888, 7232) splits 46 tiles three ways;
    (129, 7776, 7232) is the skinny case the cost model spreads over every cluster with no
    whole wave (31 pair tiles, 124 chunks on 74 clusters)."""
    m, n, k = shape
    case = orc.make_uniform_case(m, n, k, seed=7 * m + n + k)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    monkeypatch.setenv("MO_GEMM_SPLIT", "0")
    monkeypatch.setenv("MO_GEMM_STREAMK", "0")
    ref = to_host(gemm_dev(a, b))
    monkeypatch.setenv("MO_GEMM_STREAMK", "1")
    for rep in range(5):
        assert np.array_equal(to_host(gemm_dev(a, b)), ref), rep
    assert mo.read_watchdog(clear=True) == 0


@pytest.mark.parametrize("shape,env", [((6464, 976, 7232), {}),
                                       ((300, 1000, 4096), {"MO_GEMM_STREAMK": "1"}),
                                       ((300, 1000, 4096), {"MO_GEMM_SPLIT": "1"}),
                                       ((1000, 1000, 1000), {}),
                                       ((130, 262, 60), {})])  # padded copies (k, n % 8 != 0)
def test_cuda_graph_capture_and_replay(cuda_device, monkeypatch, shape, env):
    """A launch captured into a CUDA graph replays to the eager bits, replay after replay.  A
    stream-K launch (the 8-GPU slab; a forced one) counts its pieces in arrival words of its own,
    zeroed in the graph before the kernel, since the device's per-launch epochs cannot be
    replayed; the K-split and stream-K workspaces become graph memory nodes."""
    m, n, k = shape
    for key, value in env.items():
        monkeypatch.setenv(key, value)
    case = orc.make_uniform_case(m, n, k, seed=5 * m + n + k)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    eager = to_host(gemm_dev(a, b))
    side = torch.cuda.Stream()
    c = torch.zeros((m, n), dtype=torch.int16, device="cuda:0")
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up on the capture stream
        assert mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, side) == mo.MO_OK
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        rc = mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, side)
    assert rc == mo.MO_OK, mo.error_string(rc)
    for _ in range(3):
        c.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert np.array_equal(to_host(c), eager)
    del graph
    assert mo.read_watchdog(clear=True) == 0


def test_workspace_pool_is_kept_then_released(cuda_device, monkeypatch):
    """A call that needs a workspace leaves it in the library's pool for the next call, and
    mo_release_workspace gives it back."""
    m, n, k = 6464, 976, 7232  # stream-K: 30 split tiles
    monkeypatch.setenv("MO_GEMM_STREAMK", "1")
    a = torch.zeros((m, k), dtype=torch.int16, device="cuda:0")
    b = torch.zeros((k, n), dtype=torch.int16, device="cuda:0")
    c = torch.zeros((m, n), dtype=torch.int16, device="cuda:0")
    assert mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream()) == mo.MO_OK
    torch.cuda.synchronize()
    assert mo.release_workspace() >= 30 * 2 * 5 * 128 * 256 * 4
    assert mo.release_workspace() == 0
    assert mo.read_watchdog(clear=True) == 0


def test_stream_k_workspace_grows_moves_and_survives_release(cuda_device, monkeypatch):
    """The stream-K workspace stays with a stream's arrival-word region between launches: a
    larger split later on the same stream grows it, more streams than regions take regions over
    (after a wait for the previous owner), and mo_release_workspace frees every kept workspace,
    after which launches allocate afresh.  Every launch gives the whole-tile bits."""
    monkeypatch.setenv("MO_GEMM_SPLIT", "0")
    shapes = [(300, 1000, 4096), (6464, 976, 7232)]  # the second needs the larger workspace
    cases = {}
    for m, n, k in shapes:
        case = orc.make_uniform_case(m, n, k, seed=m + 3 * n + k)
        a, b = to_device(case.a_bits), to_device(case.b_bits)
        monkeypatch.setenv("MO_GEMM_STREAMK", "0")
        cases[(m, n, k)] = (a, b, to_host(gemm_dev(a, b)))
    monkeypatch.setenv("MO_GEMM_STREAMK", "1")
    streams = [torch.cuda.Stream() for _ in range(18)]  # more streams than the 16 regions

    def run_all(order):
        outs = []
        for i, shape in enumerate(order):
            a, b, _ = cases[shape]
            m, n, k = shape
            out = torch.empty((m, n), dtype=torch.int16, device="cuda:0")
            s = streams[i % len(streams)]
            s.wait_stream(torch.cuda.current_stream())
            assert mo.launch(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, s) == mo.MO_OK
            outs.append((shape, out))
        torch.cuda.synchronize()
        for shape, out in outs:
            assert np.array_equal(to_host(out), cases[shape][2]), shape

    torch.cuda.synchronize()
    run_all([shapes[0]] * 18 + [shapes[1]] * 18 + [shapes[0], shapes[1]] * 9)
    assert mo.release_workspace() > 0
    run_all([shapes[1], shapes[0]] * 3)
    assert mo.release_workspace() > 0
    assert mo.release_workspace() == 0
    assert mo.read_watchdog(clear=True) == 0


def test_reference_tile_override_values_give_the_default_bits(cuda_device, monkeypatch):
    """Every MATMUL_FIXED_MAIN_TILE_N value of the reference's sweep
    (scripts/sweep_fixed_main_tiles.py:20) is a valid plan on the hero shape, and each gives
    the bits of the analytic choice: the K chunks depend on K alone."""
    case = orc.make_uniform_case(6464, 7776, 7232, 1729)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    monkeypatch.delenv("MATMUL_FIXED_MAIN_TILE_N", raising=False)
    want = to_host(gemm_dev(a, b))
    small = torch.empty((1, 8), dtype=torch.int16, device="cuda:0")
    for width in (32, 64, 96, 128, 160, 192, 256, 320, 384, 480):
        monkeypatch.setenv("MATMUL_FIXED_MAIN_TILE_N", str(width))
        assert mo.launch_bf16_gemm_v1(a.data_ptr(), b.data_ptr(), small.data_ptr(), 1, 8, 8,
                                      torch.cuda.current_stream())  # not the hero: ignored
        got = to_host(gemm_dev(a, b))
        assert np.array_equal(got, want), width
    monkeypatch.setenv("MATMUL_FIXED_MAIN_TILE_N", "97")
    c = torch.empty((6464, 7776), dtype=torch.int16, device="cuda:0")
    assert not mo.launch_bf16_gemm_v1(a.data_ptr(), b.data_ptr(), c.data_ptr(), 6464, 7776, 7232,
                                      torch.cuda.current_stream())
    assert mo.read_watchdog(clear=True) == 0


def test_bad_overrides_are_rejected(cuda_device, monkeypatch):
    a = torch.zeros((64, 64), dtype=torch.int16, device="cuda:0")
    monkeypatch.setenv("MO_GEMM_VARIANT", "huge")
    assert mo.launch(a.data_ptr(), a.data_ptr(), a.data_ptr(), 64, 64, 64, torch.cuda.current_stream()) == mo.MO_ERR_BAD_ARGUMENT
    monkeypatch.setenv("MO_GEMM_VARIANT", "1x64")
    monkeypatch.setenv("MO_GEMM_SPLIT", "2")
    assert mo.launch(a.data_ptr(), a.data_ptr(), a.data_ptr(), 64, 64, 64, torch.cuda.current_stream()) == mo.MO_ERR_BAD_ARGUMENT
    monkeypatch.setenv("MO_GEMM_SPLIT", "0")
    monkeypatch.setenv("MO_GEMM_STREAMK", "yes")
    assert mo.launch(a.data_ptr(), a.data_ptr(), a.data_ptr(), 64, 64, 64, torch.cuda.current_stream()) == mo.MO_ERR_BAD_ARGUMENT


@pytest.mark.parametrize("shape,slabs", [((6464, 7776, 7232), 0), ((6464, 7776, 7232), 1),
                                         ((1000, 7776, 7232), 3), ((1, 7776, 7232), 0),
                                         ((257, 392, 520), 2)])
def test_gemm_from_host_matches_device_path(cuda_device, shape, slabs):
    """mo_gemm_from_host (A up, then B in column slabs overlapped with the slab GEMMs and the C
    downloads) gives the device path's bits: the slab GEMMs sum exactly what the whole GEMM
    sums."""
    m, n, k = shape
    case = orc.make_uniform_case(m, n, k, seed=m + 3 * n + k)
    a_h = torch.from_numpy(case.a_bits.view(np.int16)).pin_memory()
    b_h = torch.from_numpy(case.b_bits.view(np.int16)).pin_memory()
    c_h = torch.full((m, n), 0x7FC0, dtype=torch.int16).pin_memory()  # NaN fill
    want = to_host(gemm_dev(to_device(case.a_bits), to_device(case.b_bits)))
    stream = torch.cuda.current_stream()
    for _ in range(2):  # the second call reuses the pool's buffers
        rc = mo.gemm_from_host(a_h.data_ptr(), b_h.data_ptr(), c_h.data_ptr(), m, n, k, slabs, stream)
        assert rc == mo.MO_OK, mo.error_string(rc)
        stream.synchronize()
        assert np.array_equal(c_h.numpy().view(np.uint16), want)
    assert mo.read_watchdog(clear=True) == 0


def test_gemm_from_host_rejects_bad_arguments(cuda_device):
    buf = torch.zeros(64 * 64, dtype=torch.int16).pin_memory()
    p = buf.data_ptr()
    assert mo.gemm_from_host(0, p, p, 64, 64, 64) == mo.MO_ERR_NULL_POINTER
    assert mo.gemm_from_host(p, p, p, 0, 64, 64) == mo.MO_ERR_BAD_DIMS
    assert mo.gemm_from_host(p, p, p, 64, 64, 60) == mo.MO_ERR_UNSUPPORTED
    assert mo.gemm_from_host(p, p, p, 64, 64, 64, -1) == mo.MO_ERR_BAD_ARGUMENT


def test_stream_k_on_two_streams(cuda_device, monkeypatch):
    """Stream-K launches on two streams get separate counter regions (a region is handed to
    another stream only after a wait), so interleaved launches still give the same bits."""
    monkeypatch.setenv("MO_GEMM_STREAMK", "1")
    monkeypatch.setenv("MO_GEMM_VARIANT", "pair256")
    m, n, k = 6464, 976, 7232
    case = orc.make_uniform_case(m, n, k, seed=97)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    want = to_host(gemm_dev(a, b))
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.empty((m, n), dtype=torch.int16, device="cuda:0") for _ in range(6)]
    torch.cuda.synchronize()
    for i, out in enumerate(outs):
        rc = mo.launch(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, streams[i % 2])
        assert rc == mo.MO_OK
    torch.cuda.synchronize()
    for out in outs:
        assert np.array_equal(to_host(out), want)
    assert mo.read_watchdog(clear=True) == 0


def test_gemm_b_from_host_with_resident_a(cuda_device):
    """mo_gemm_b_from_host (A already on the device, B and C on the host) gives the device
    path's bits; the sharded end-to-end step uses it after gathering A."""
    m, n, k = 1000, 2000, 7232
    case = orc.make_uniform_case(m, n, k, seed=31)
    a = to_device(case.a_bits)
    b_h = torch.from_numpy(case.b_bits.view(np.int16)).pin_memory()
    c_h = torch.full((m, n), 0x7FC0, dtype=torch.int16).pin_memory()
    want = to_host(gemm_dev(a, to_device(case.b_bits)))
    stream = torch.cuda.current_stream()
    rc = mo.gemm_b_from_host(a.data_ptr(), b_h.data_ptr(), c_h.data_ptr(), m, n, k, 0, stream)
    assert rc == mo.MO_OK, mo.error_string(rc)
    stream.synchronize()
    assert np.array_equal(c_h.numpy().view(np.uint16), want)
    assert mo.read_watchdog(clear=True) == 0


def test_back_to_back_dependent_gemms(cuda_device):
    """Two GEMMs launched back to back on one stream, the second reading the first's output as
    its A: with programmatic dependent launch the second may start before the first ends, and
    its grid-dependency wait must still order every read of C after the first GEMM's writes."""
    m, k, n, p = 2048, 2048, 2048, 1024
    case = orc.make_uniform_case(m, n, k, seed=5)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    e = to_device(orc.make_uniform_case(8, p, n, seed=6).b_bits)  # [n, p] BF16 bits
    stream = torch.cuda.current_stream()
    c = torch.empty((m, n), dtype=torch.int16, device="cuda:0")
    d = torch.empty((m, p), dtype=torch.int16, device="cuda:0")
    # Reference: the two GEMMs with a synchronisation between them.
    assert mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, stream) == mo.MO_OK
    torch.cuda.synchronize()
    assert mo.launch(c.data_ptr(), e.data_ptr(), d.data_ptr(), m, p, n, stream) == mo.MO_OK
    torch.cuda.synchronize()
    want = to_host(d)
    for _ in range(5):
        c.fill_(0x7FC0)  # NaN: a read of C before the first GEMM's writes would show
        d.zero_()
        assert mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, stream) == mo.MO_OK
        assert mo.launch(c.data_ptr(), e.data_ptr(), d.data_ptr(), m, p, n, stream) == mo.MO_OK
        torch.cuda.synchronize()
        assert np.array_equal(to_host(d), want)
    assert mo.read_watchdog(clear=True) == 0
