"""The oracle (CPU restatement of the reference's generator and check) is pinned against
fixtures produced by running the reference's own code (tests/golden/make_golden.py)."""

import ctypes
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import bf16_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"
ORACLE_DIR = Path(__file__).resolve().parent.parent / "oracle"


@pytest.fixture(scope="module")
def coracle():
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "all"], check=True)
    lib = ctypes.CDLL(str(ORACLE_DIR / "_build" / "liboracle_gemm.so"))
    p = ctypes.c_void_p
    lib.oracle_bf16_to_f32.argtypes = [p, p, ctypes.c_int64]
    lib.oracle_f32_to_bf16.argtypes = [p, p, ctypes.c_int64]
    lib.oracle_gemm_f64.argtypes = [p, p, p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.oracle_gemm_f32_rows.argtypes = [p, p, p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.oracle_check.argtypes = [p, p, ctypes.c_int64, ctypes.c_double, ctypes.c_double, p]
    lib.oracle_check.restype = ctypes.c_int
    return lib


def ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def test_codec_matches_reference_kat(coracle):
    kat = json.loads((GOLDEN / "codec_kat.json").read_text())
    f32_bits = np.array(kat["f32_bits"], dtype=np.uint32)
    want = np.array(kat["bf16_bits"], dtype=np.uint16)
    with np.errstate(over="ignore", invalid="ignore"):
        got = orc.float32_to_bf16_bits(f32_bits.view(np.float32))
    assert np.array_equal(got, want)
    widened = orc.bf16_bits_to_float32(want).view(np.uint32)
    assert np.array_equal(widened, np.array(kat["widened_f32_bits"], dtype=np.uint32))
    out = np.empty_like(want)
    coracle.oracle_f32_to_bf16(ptr(f32_bits), ptr(out), want.size)
    assert np.array_equal(out, want)


def test_small_cases_inputs_and_reference(coracle):
    data = np.load(GOLDEN / "small_cases.npz")
    index = json.loads((GOLDEN / "small_cases_index.json").read_text())
    assert len(index) >= 10
    for e in index:
        key, m, n, k, seed = e["key"], e["m"], e["n"], e["k"], e["seed"]
        case = orc.make_uniform_case(m, n, k, seed)
        # The seeded draw and RNE codec reproduce the reference's files bit for bit.
        assert np.array_equal(case.a_bits, data[f"{key}_a"]), key
        assert np.array_equal(case.b_bits, data[f"{key}_b"]), key
        assert orc.sha256_bytes(case.a_bits) == e["checksums"]["A_bf16"]
        assert orc.sha256_bytes(case.b_bits) == e["checksums"]["B_bf16"]
        # FP32 product: equal up to BLAS summation order.
        c32 = orc.reference_gemm_fp32(case.a_bits, case.b_bits)
        ref32 = data[f"{key}_c32"]
        assert np.allclose(c32, ref32, rtol=1e-5, atol=1e-5 * np.sqrt(k)), key
        assert np.mean(orc.float32_to_bf16_bits(c32) == data[f"{key}_c16"]) > 0.99
        # C float64 restatement agrees with numpy float64.
        c64 = np.empty((m, n), dtype=np.float64)
        coracle.oracle_gemm_f64(ptr(case.a_bits), ptr(case.b_bits), ptr(c64), m, n, k)
        assert np.allclose(c64, orc.reference_gemm_fp64(case.a_bits, case.b_bits), rtol=1e-12, atol=1e-12)


def test_check_rule_matches_reference_runner(coracle):
    data = np.load(GOLDEN / "small_cases.npz")
    key = "130x264x200_s3407"
    ref32, ref16 = data[f"{key}_c32"], data[f"{key}_c16"]
    res = orc.evaluate_correctness(ref16, ref32, ref16)
    assert res["passed"] and res["bf16_exact_match"] and res["atol"] == 0.15 and res["rtol"] == 0.01
    bad = ref16.copy()
    bad[3, 7] = orc.float32_to_bf16_bits(np.array([ref32[3, 7] + 4.0], dtype=np.float32))[0]
    res2 = orc.evaluate_correctness(bad, ref32, ref16)
    assert not res2["passed"] and not res2["bf16_exact_match"]
    stats = np.zeros(3)
    assert coracle.oracle_check(ptr(bad), ptr(ref32), bad.size, 0.15, 0.01, ptr(stats)) == 0
    assert stats[0] == pytest.approx(res2["max_abs_err"])
    assert stats[2] == pytest.approx(res2["mean_abs_err"])
    # A NaN output fails both the numpy and the C rule.
    nan = ref16.copy()
    nan[0, 0] = 0x7FC0
    assert not orc.evaluate_correctness(nan, ref32, ref16)["passed"]
    assert coracle.oracle_check(ptr(nan), ptr(ref32), nan.size, 0.15, 0.01, ptr(stats)) == 0


def test_north_star_bound_formula():
    ref = np.array([0.0, 1.0, -128.0])
    b = orc.north_star_bound(ref, 7232, 1.0, 1.0)
    assert b[0] == pytest.approx(1e-2 / np.sqrt(7232))
    assert b[2] == pytest.approx(128 * 2 ** -7 + 1e-2 / np.sqrt(7232))


@pytest.mark.parametrize("seed", [3407, 9713, 1729])
def test_hero_inputs_pinned(seed):
    pins = json.loads((GOLDEN / "hero_pins.json").read_text())
    m, n, k = pins["shape"]
    case = orc.make_uniform_case(m, n, k, seed)
    p = pins["seeds"][str(seed)]
    assert orc.sha256_bytes(case.a_bits) == p["sha256_A_bf16"]
    assert orc.sha256_bytes(case.b_bits) == p["sha256_B_bf16"]
    rows, cols = np.array(pins["sample_rows"]), np.array(pins["sample_cols"])
    a = orc.bf16_bits_to_float32(case.a_bits[rows]).astype(np.float64)
    b = orc.bf16_bits_to_float32(case.b_bits[:, cols]).astype(np.float64)
    exact = np.einsum("ik,ki->i", a, b)
    assert np.allclose(exact, p["c_exact_f64_samples"], rtol=1e-12, atol=1e-9)
    # The reference's FP32 C_ref samples sit within FP32 accumulation error of the exact value.
    assert np.allclose(p["c_ref_fp32_samples"], exact, rtol=1e-4, atol=1e-3)


def test_evaluate_on_planted_error_in_oracle():
    """A mistake planted in the oracle's output (not in any GPU path) is caught by both rules."""
    case = orc.make_uniform_case(64, 64, 256, 5)
    ref32 = orc.reference_gemm_fp32(case.a_bits, case.b_bits)
    ref16 = orc.float32_to_bf16_bits(ref32)
    planted = ref16.copy()
    planted[10, 20] = orc.float32_to_bf16_bits(np.array([ref32[10, 20] + 1.0], dtype=np.float32))[0]
    assert not orc.evaluate_correctness(planted, ref32, ref16)["passed"]
    assert not orc.check_north_star(planted, orc.reference_gemm_fp64(case.a_bits, case.b_bits),
                                    case.a_bits, case.b_bits)["passed"]


def test_full_matrix_check_agrees_with_whole_matrix_rules():
    """The row-blocked full-matrix check reports what the whole-matrix functions report, and a
    mistake planted in the oracle's output is found at the planted position."""
    case = orc.make_uniform_case(300, 264, 1000, 17)
    ref32 = orc.reference_gemm_fp32(case.a_bits, case.b_bits)
    good = orc.float32_to_bf16_bits(ref32)
    planted = good.copy()
    planted[257, 33] = orc.float32_to_bf16_bits(np.array([ref32[257, 33] + 0.5], dtype=np.float32))[0]
    res = orc.full_matrix_check({"good": good, "planted": planted}, case.a_bits, case.b_bits, block_rows=64)
    exact = orc.reference_gemm_fp64(case.a_bits, case.b_bits)
    ns = orc.check_north_star(good, exact, case.a_bits, case.b_bits)
    g = res["good"]
    assert g["elements"] == 300 * 264
    assert g["reference_rule"]["passed"] and g["north_star"]["passed"]
    assert g["north_star"]["worst_ratio"] == pytest.approx(ns["worst_ratio"])
    assert g["north_star"]["frac_abs_term_bound"] == pytest.approx(ns["frac_abs_term_bound"])
    assert g["bf16_agreement"] > 0.99
    p = res["planted"]
    assert not p["reference_rule"]["passed"]  # 0.5 > 0.15 + 0.01 |ref| for |ref| < 35
    assert not p["north_star"]["passed"]
    assert p["north_star"]["worst_at"] == [257, 33]
