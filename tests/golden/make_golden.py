#!/usr/bin/env python3
"""Generates the committed golden fixtures by running the REFERENCE's own dataset generator.

Run on a machine that has the reference checkout (named by --reference, default
MO_REFERENCE_ROOT); the GPU box never runs this script, it only reads its outputs:

* small_cases.npz  - for each small shape/seed, the files the reference's ``write_case``
                     (scripts/generate_fixed_bf16_dataset.py:91-183) writes: A/B BF16 bits,
                     C_ref_fp32 and C_ref_bf16, read back from disk.
* hero_pins.json   - for the hero shape 6464x7776x7232 and the three configured seeds
                     (configs/fixed_bf16_gemm_v1.json:39-52): sha256 of A.bf16.bin and
                     B.bf16.bin, sha256 of C_ref_bf16.bin, and C_ref_fp32 at 1024 fixed
                     positions plus the float64 value of the same dot products.
* codec_kat.json   - float32 bit patterns and the BF16 bits the reference codec
                     (generator :32-48) gives for them: ties, subnormals, infinities, NaN.

Usage: python tests/golden/make_golden.py --reference <reference checkout> [--skip-hero]
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import platform
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# Small shapes: (m, n, k).  n and k are multiples of 8 (the GPU path's TMA stride rule) and
# cover single rows, ragged M/N tails, K below one 64-wide block, and K tails.
SMALL_SHAPES = [
    (1, 16, 16),
    (7, 24, 40),
    (16, 64, 64),
    (128, 256, 64),
    (129, 136, 72),
    (130, 264, 200),
    (257, 520, 136),
    (24, 200, 1000),
]
SMALL_SEEDS = [3407, 9713]
LARGE_SMALL_SEEDS = [1729]  # one seed for the shapes above 64 Ki elements of B


def load_reference_generator(ref_root: Path):
    path = ref_root / "scripts" / "generate_fixed_bf16_dataset.py"
    spec = importlib.util.spec_from_file_location("ref_generate_fixed_bf16_dataset", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses look the module up by name
    spec.loader.exec_module(mod)
    return mod


def run_reference_case(gen, m: int, n: int, k: int, seed: int, workdir: Path) -> dict:
    config = {
        "gemm": {"m": m, "n": n, "k": k, "layout_a": "row_major", "layout_b": "row_major",
                 "layout_c": "row_major", "input_dtype": "bf16", "accumulator_dtype": "fp32",
                 "output_dtype": "bf16"},
        "distribution": {"name": "uniform", "low": -1.0, "high": 1.0},
    }
    case = gen.CaseConfig(case_id=f"case_{m}x{n}x{k}_seed_{seed}", seed=seed)
    summary = gen.write_case(workdir, config, case, force=True)
    case_dir = workdir / "cases" / case.case_id
    return {
        "dir": case_dir,
        "checksums": summary["checksums"],
        "a": np.fromfile(case_dir / "A.bf16.bin", dtype=np.uint16).reshape(m, k),
        "b": np.fromfile(case_dir / "B.bf16.bin", dtype=np.uint16).reshape(k, n),
        "c32": np.fromfile(case_dir / "C_ref_fp32.bin", dtype=np.float32).reshape(m, n),
        "c16": np.fromfile(case_dir / "C_ref_bf16.bin", dtype=np.uint16).reshape(m, n),
    }


def make_small(gen, out: Path) -> None:
    arrays = {}
    index = []
    with tempfile.TemporaryDirectory() as td:
        for (m, n, k) in SMALL_SHAPES:
            seeds = SMALL_SEEDS if k * n <= 65536 else LARGE_SMALL_SEEDS
            for seed in seeds:
                r = run_reference_case(gen, m, n, k, seed, Path(td))
                key = f"{m}x{n}x{k}_s{seed}"
                arrays[f"{key}_a"] = r["a"]
                arrays[f"{key}_b"] = r["b"]
                arrays[f"{key}_c32"] = r["c32"]
                arrays[f"{key}_c16"] = r["c16"]
                index.append({"key": key, "m": m, "n": n, "k": k, "seed": seed,
                              "checksums": r["checksums"]})
    np.savez_compressed(out / "small_cases.npz", **arrays)
    (out / "small_cases_index.json").write_text(json.dumps(index, indent=1) + "\n")


def make_hero(gen, out: Path) -> None:
    m, n, k = 6464, 7776, 7232
    rng = np.random.default_rng(20240601)
    rows = rng.integers(0, m, size=1024)
    cols = rng.integers(0, n, size=1024)
    pins = {"shape": [m, n, k], "numpy": np.__version__, "machine": platform.machine(),
            "sample_rows": rows.tolist(), "sample_cols": cols.tolist(), "seeds": {}}
    with tempfile.TemporaryDirectory() as td:
        for seed in (3407, 9713, 1729):
            r = run_reference_case(gen, m, n, k, seed, Path(td))
            a = gen.bf16_bits_to_float32(r["a"]).astype(np.float64)
            b = gen.bf16_bits_to_float32(r["b"]).astype(np.float64)
            exact = np.einsum("ik,ki->i", a[rows, :], b[:, cols])
            pins["seeds"][str(seed)] = {
                "sha256_A_bf16": r["checksums"]["A_bf16"],
                "sha256_B_bf16": r["checksums"]["B_bf16"],
                "sha256_C_ref_bf16": r["checksums"]["C_ref_bf16"],
                "sha256_C_ref_fp32": r["checksums"]["C_ref_fp32"],
                "c_ref_fp32_samples": r["c32"][rows, cols].astype(float).tolist(),
                "c_exact_f64_samples": exact.tolist(),
                "c_ref_bf16_samples": r["c16"][rows, cols].astype(int).tolist(),
            }
            for f in r["dir"].iterdir():
                f.unlink()
    (out / "hero_pins.json").write_text(json.dumps(pins) + "\n")


def make_codec(gen, out: Path) -> None:
    specials = [0x00000000, 0x80000000, 0x3F800000, 0xBF800000, 0x7F7FFFFF, 0xFF7FFFFF,
                0x7F800000, 0xFF800000, 0x00000001, 0x007FFFFF, 0x00800000,
                0x3F808000, 0x3F818000, 0x3F807FFF, 0x3F808001, 0x3F80FFFF,
                0x7F7F8000, 0x7FC00000, 0x7F800001, 0xFFFFFFFF, 0x33800000, 0x40490FDB]
    rng = np.random.default_rng(7)
    rand = rng.integers(0, 2 ** 32, size=2000, dtype=np.uint64).astype(np.uint32)
    bits = np.concatenate([np.array(specials, dtype=np.uint32), rand])
    with np.errstate(over="ignore", invalid="ignore"):
        out_bits = gen.float32_to_bf16_bits(bits.view(np.float32))
    widened = gen.bf16_bits_to_float32(out_bits).view(np.uint32)
    (out / "codec_kat.json").write_text(json.dumps({
        "f32_bits": bits.astype(int).tolist(),
        "bf16_bits": out_bits.astype(int).tolist(),
        "widened_f32_bits": widened.astype(int).tolist(),
    }) + "\n")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=os.environ.get("MO_REFERENCE_ROOT"),
                    required=not os.environ.get("MO_REFERENCE_ROOT"),
                    help="the reference checkout (default: MO_REFERENCE_ROOT)")
    ap.add_argument("--skip-hero", action="store_true")
    args = ap.parse_args()
    gen = load_reference_generator(args.reference)
    make_codec(gen, HERE)
    make_small(gen, HERE)
    if not args.skip_hero:
        make_hero(gen, HERE)


if __name__ == "__main__":
    main()
