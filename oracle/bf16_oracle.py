"""CPU oracle for the fixed BF16 GEMM path: TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may
import this module, and only as the checker or the timed CPU baseline; the product
(matmul_optimizer_b200) never calls into oracle/.

It restates, in numpy, the reference's dataset generator and result check:

* ``float32_to_bf16_bits`` / ``bf16_bits_to_float32``: the round-to-nearest-even codec of
  scripts/generate_fixed_bf16_dataset.py:32-48 (``(u + 0x7FFF + lsb) >> 16``; NaN is not
  special-cased there, so it is not special-cased here either);
* ``generate_uniform_f32``: ``rng.random(float32) * (hi - lo) + lo`` (generator :66-69), with
  A drawn before B from one ``default_rng(seed)`` (generator :104-108);
* ``reference_gemm_fp32``: ``A_q @ B_q`` in float32 (generator :118-122) followed by RNE to
  BF16 (generator :128);
* ``evaluate_correctness``: the runner's check, pass iff every element satisfies
  ``|out - ref| <= atol + rtol * |ref|`` plus max_abs / max_rel / mean_abs and the BF16 exact
  match flag (src/runner/main.cpp:324-365), atol 0.15 / rtol 0.01 by default
  (configs/fixed_bf16_gemm_v1.json:32-38);
* ``north_star_bound``: the stated tolerance of the build,
  ``|err| <= 2^-7 * |ref| + 1e-2 * sqrt(K) * max|A| * max|B| / K`` per element.

Parity pin: the restatement is checked against fixtures produced by importing the
reference generator itself (tests/golden/make_golden.py, committed with its outputs).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np

HERO_M, HERO_N, HERO_K = 6464, 7776, 7232
HERO_SEEDS = (3407, 9713, 1729)
DEFAULT_ATOL = 0.15
DEFAULT_RTOL = 0.01


def float32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """RNE float32 -> BF16 bit patterns (generator :32-40)."""
    if x.dtype != np.float32:
        raise TypeError(f"expected float32, got {x.dtype}")
    u = x.view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    return ((u + (np.uint32(0x7FFF) + lsb)) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_float32(bits: np.ndarray) -> np.ndarray:
    """Widen BF16 bit patterns to float32 (generator :43-48)."""
    if bits.dtype != np.uint16:
        raise TypeError(f"expected uint16, got {bits.dtype}")
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def generate_uniform_f32(rng: np.random.Generator, shape, low: float, high: float) -> np.ndarray:
    """Uniform [low, high) float32 draw exactly as generator :66-69."""
    arr = rng.random(shape, dtype=np.float32)
    arr = arr * np.float32(high - low) + np.float32(low)
    return np.ascontiguousarray(arr, dtype=np.float32)


def generate_normal_f32(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    """Normal(0, std) float32 draw for the LLM-projection config (no reference counterpart:
    the reference only has the uniform distribution)."""
    arr = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    return np.ascontiguousarray(arr, dtype=np.float32)


@dataclass
class Case:
    a_bits: np.ndarray  # uint16 [m, k]
    b_bits: np.ndarray  # uint16 [k, n]

    @property
    def shape(self):
        m, k = self.a_bits.shape
        return m, self.b_bits.shape[1], k


def make_uniform_case(m: int, n: int, k: int, seed: int, low: float = -1.0, high: float = 1.0) -> Case:
    """A then B from one default_rng(seed), quantised to BF16 (generator :104-112)."""
    rng = np.random.default_rng(seed)
    a = generate_uniform_f32(rng, (m, k), low, high)
    b = generate_uniform_f32(rng, (k, n), low, high)
    return Case(float32_to_bf16_bits(a), float32_to_bf16_bits(b))


def make_normal_case(m: int, n: int, k: int, seed_a: int, seed_b: int, std_a: float, std_b: float) -> Case:
    """Activations ~ N(0, std_a) from seed_a, weights ~ N(0, std_b) from seed_b, both BF16."""
    a = generate_normal_f32(np.random.default_rng(seed_a), (m, k), std_a)
    b = generate_normal_f32(np.random.default_rng(seed_b), (k, n), std_b)
    return Case(float32_to_bf16_bits(a), float32_to_bf16_bits(b))


def reference_gemm_fp32(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """FP32 CPU GEMM on the BF16-quantised inputs (generator :118-122)."""
    a = np.ascontiguousarray(bf16_bits_to_float32(a_bits))
    b = np.ascontiguousarray(bf16_bits_to_float32(b_bits))
    return np.ascontiguousarray(a @ b, dtype=np.float32)


def reference_gemm_fp64(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Float64 GEMM on the same inputs: a near-exact value for error accounting."""
    a = bf16_bits_to_float32(a_bits).astype(np.float64)
    b = bf16_bits_to_float32(b_bits).astype(np.float64)
    return a @ b


def evaluate_correctness(out_bits: np.ndarray, ref_fp32: np.ndarray, ref_bf16_bits: np.ndarray,
                         atol: float = DEFAULT_ATOL, rtol: float = DEFAULT_RTOL) -> dict:
    """The runner's correctness check (src/runner/main.cpp:324-365)."""
    out = bf16_bits_to_float32(out_bits.reshape(-1)).astype(np.float64)
    ref = ref_fp32.reshape(-1).astype(np.float64)
    abs_err = np.abs(out - ref)
    rel_err = abs_err / np.maximum(np.abs(ref), 1.0e-12)
    tol = atol + rtol * np.abs(ref)
    return {
        "passed": bool(np.all(abs_err <= tol)),
        "max_abs_err": float(abs_err.max()) if abs_err.size else 0.0,
        "max_rel_err": float(rel_err.max()) if rel_err.size else 0.0,
        "mean_abs_err": float(abs_err.mean()) if abs_err.size else 0.0,
        "bf16_exact_match": bool(np.array_equal(out_bits.reshape(-1), ref_bf16_bits.reshape(-1))),
        "atol": atol,
        "rtol": rtol,
    }


def north_star_bound(ref: np.ndarray, k: int, max_a: float, max_b: float) -> np.ndarray:
    """Per-element tolerance 2^-7 |ref| + 1e-2 sqrt(K) max|A| max|B| / K."""
    return np.abs(ref) * 2.0 ** -7 + 1.0e-2 * np.sqrt(k) * max_a * max_b / k


def check_north_star(out_bits: np.ndarray, ref: np.ndarray, a_bits: np.ndarray, b_bits: np.ndarray) -> dict:
    """Applies north_star_bound to a BF16 result; reports the worst margin."""
    k = a_bits.shape[1]
    max_a = float(np.abs(bf16_bits_to_float32(a_bits)).max()) if a_bits.size else 0.0
    max_b = float(np.abs(bf16_bits_to_float32(b_bits)).max()) if b_bits.size else 0.0
    out = bf16_bits_to_float32(out_bits).astype(np.float64)
    ref64 = ref.astype(np.float64)
    err = np.abs(out - ref64)
    bound = north_star_bound(ref64, k, max_a, max_b)
    ratio = err / bound
    worst = int(np.argmax(ratio)) if ratio.size else 0
    abs_term = 1.0e-2 * np.sqrt(k) * max_a * max_b / k
    return {
        "passed": bool(np.all(err <= bound)),
        "worst_ratio": float(ratio.reshape(-1)[worst]) if ratio.size else 0.0,
        "max_abs_err": float(err.max()) if err.size else 0.0,
        "frac_abs_term_bound": float(np.mean(abs_term > np.abs(ref64) * 2.0 ** -7)) if ref64.size else 0.0,
    }


def full_matrix_check(outs: dict, a_bits: np.ndarray, b_bits: np.ndarray,
                      atol: float = DEFAULT_ATOL, rtol: float = DEFAULT_RTOL,
                      block_rows: int = 512) -> dict:
    """Checks every element of one or more BF16 results of the same product, row block by row
    block, so that full-size outputs (hero, square 8192, the LLM projection) are checked whole
    without holding several full-size float64 temporaries.

    ``outs`` maps a name to a uint16 [m, n] result.  Per result it reports:

    * ``reference_rule``: the runner's check (src/runner/main.cpp:324-365) against the FP32
      product of this module (generator :118-122), with max_abs / max_rel / mean_abs;
    * ``north_star``: ``north_star_bound`` against the float64 product, with the worst ratio
      err / bound, where it sits, and the fraction of elements whose bound is dominated by the
      absolute term;
    * ``bf16_agreement``: the fraction of elements equal to RNE(FP32 product) (generator :128).
    """
    m, k = a_bits.shape
    n = b_bits.shape[1]
    max_a = float(np.abs(bf16_bits_to_float32(a_bits)).max()) if a_bits.size else 0.0
    max_b = float(np.abs(bf16_bits_to_float32(b_bits)).max()) if b_bits.size else 0.0
    abs_term = 1.0e-2 * np.sqrt(k) * max_a * max_b / k
    b32 = np.ascontiguousarray(bf16_bits_to_float32(b_bits))
    b64 = b32.astype(np.float64)
    acc = {name: {"ref_pass": True, "ref_max_abs": 0.0, "ref_max_rel": 0.0, "ref_sum_abs": 0.0,
                  "ns_pass": True, "ns_worst": -1.0, "ns_where": (0, 0), "ns_max_abs": 0.0,
                  "abs_bound": 0, "agree": 0} for name in outs}
    for r0 in range(0, m, block_rows):
        r1 = min(m, r0 + block_rows)
        a32 = np.ascontiguousarray(bf16_bits_to_float32(a_bits[r0:r1]))
        ref32 = (a32 @ b32).astype(np.float64)
        ref16 = float32_to_bf16_bits(ref32.astype(np.float32))
        exact = a32.astype(np.float64) @ b64
        bound = np.abs(exact) * 2.0 ** -7 + abs_term
        tol = atol + rtol * np.abs(ref32)
        n_abs = int(np.count_nonzero(abs_term > np.abs(exact) * 2.0 ** -7))
        for name, out_bits in outs.items():
            s = acc[name]
            blk = out_bits[r0:r1]
            out = bf16_bits_to_float32(blk).astype(np.float64)
            err_ref = np.abs(out - ref32)
            s["ref_pass"] &= bool(np.all(err_ref <= tol))
            s["ref_max_abs"] = max(s["ref_max_abs"], float(err_ref.max()))
            s["ref_max_rel"] = max(s["ref_max_rel"], float((err_ref / np.maximum(np.abs(ref32), 1.0e-12)).max()))
            s["ref_sum_abs"] += float(err_ref.sum())
            err = np.abs(out - exact)
            ratio = err / bound
            i = int(np.argmax(ratio))
            s["ns_pass"] &= bool(np.all(err <= bound))
            if ratio.reshape(-1)[i] > s["ns_worst"]:
                s["ns_worst"] = float(ratio.reshape(-1)[i])
                s["ns_where"] = (r0 + i // n, i % n)
            s["ns_max_abs"] = max(s["ns_max_abs"], float(err.max()))
            s["abs_bound"] += n_abs
            s["agree"] += int(np.count_nonzero(blk == ref16))
    total = m * n
    result = {}
    for name, s in acc.items():
        result[name] = {
            "elements": total,
            "reference_rule": {"passed": s["ref_pass"], "max_abs_err": s["ref_max_abs"],
                               "max_rel_err": s["ref_max_rel"], "mean_abs_err": s["ref_sum_abs"] / total,
                               "atol": atol, "rtol": rtol},
            "north_star": {"passed": s["ns_pass"], "worst_ratio": s["ns_worst"],
                           "worst_at": [int(s["ns_where"][0]), int(s["ns_where"][1])],
                           "max_abs_err": s["ns_max_abs"], "abs_term": abs_term,
                           "frac_abs_term_bound": s["abs_bound"] / total},
            "bf16_agreement": s["agree"] / total,
        }
    return result


def sha256_bytes(arr: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()
