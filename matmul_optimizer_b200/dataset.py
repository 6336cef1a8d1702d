"""Dataset cases in the reference's on-disk format, the input contract of the runner.

Layout per case (reference configs/fixed_bf16_gemm_v1.json:53-65, writer
scripts/generate_fixed_bf16_dataset.py:91-183)::

    <root>/<dataset_id>/manifest.json
    <root>/<dataset_id>/cases/<case_id>/{A.bf16.bin,B.bf16.bin,C_ref_fp32.bin,C_ref_bf16.bin,
                                         meta.json,checksums.json}

A and B are drawn exactly as the reference draws them (one ``default_rng(seed)``, A before B,
``random(float32) * (high - low) + low``, round-to-nearest-even to BF16), so a case written
here is byte-identical to the reference's for the same config and seed.  The BASELINE
configs the reference does not have (square 8192, the LLM projection with normal
distributions, the ragged sweep) are added as extra config files in the package's ``configs/``.

C_ref is the FP32 product of the quantised inputs, as in the reference (numpy/BLAS float32,
generator :122), then RNE to BF16.  Writing C_ref can be skipped (``with_reference=False``)
for perf-only cases.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import shutil
from pathlib import Path
from typing import Dict, Iterable, Optional

import numpy as np

CONFIG_DIR = Path(__file__).resolve().parent / "configs"


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> BF16 bits, the codec of generator :32-40."""
    if x.dtype != np.float32:
        raise TypeError(f"expected float32, got {x.dtype}")
    u = x.view(np.uint32)
    return ((u + (np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widening BF16 bits -> float32 (generator :43-48)."""
    if bits.dtype != np.uint16:
        raise TypeError(f"expected uint16, got {bits.dtype}")
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def draw_inputs(m: int, n: int, k: int, seed: int, distribution: Dict) -> tuple:
    """BF16 bit matrices A[m,k], B[k,n] for one case."""
    name = distribution.get("name", "uniform")
    if name == "uniform":
        rng = np.random.default_rng(seed)
        lo, hi = float(distribution["low"]), float(distribution["high"])
        a = rng.random((m, k), dtype=np.float32) * np.float32(hi - lo) + np.float32(lo)
        b = rng.random((k, n), dtype=np.float32) * np.float32(hi - lo) + np.float32(lo)
    elif name == "normal":
        seed_b = int(distribution.get("seed_b", seed + 1))
        a = np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32) * np.float32(distribution["std_a"])
        b = np.random.default_rng(seed_b).standard_normal((k, n), dtype=np.float32) * np.float32(distribution["std_b"])
    else:
        raise ValueError(f"unknown distribution {name!r}")
    return (np.ascontiguousarray(f32_to_bf16_bits(np.ascontiguousarray(a, dtype=np.float32))),
            np.ascontiguousarray(f32_to_bf16_bits(np.ascontiguousarray(b, dtype=np.float32))))


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def write_case(dataset_dir: Path, gemm: Dict, distribution: Dict, case_id: str, seed: int,
               force: bool = False, with_reference: bool = True) -> Dict:
    m, n, k = int(gemm["m"]), int(gemm["n"]), int(gemm["k"])
    case_dir = dataset_dir / "cases" / case_id
    if case_dir.exists():
        if not force:
            raise FileExistsError(f"{case_dir} already exists; use force=True to overwrite")
        shutil.rmtree(case_dir)
    case_dir.mkdir(parents=True)
    a_bits, b_bits = draw_inputs(m, n, k, seed, distribution)
    files = {"A_bf16": case_dir / "A.bf16.bin", "B_bf16": case_dir / "B.bf16.bin"}
    a_bits.tofile(files["A_bf16"])
    b_bits.tofile(files["B_bf16"])
    if with_reference:
        c32 = np.ascontiguousarray(bf16_bits_to_f32(a_bits) @ bf16_bits_to_f32(b_bits), dtype=np.float32)
        files["C_ref_fp32"] = case_dir / "C_ref_fp32.bin"
        files["C_ref_bf16"] = case_dir / "C_ref_bf16.bin"
        c32.tofile(files["C_ref_fp32"])
        f32_to_bf16_bits(c32).tofile(files["C_ref_bf16"])
    checksums = {name: _sha256(p) for name, p in files.items()}
    (case_dir / "checksums.json").write_text(json.dumps(checksums, indent=2) + "\n")
    meta = {
        "case_id": case_id, "seed": seed, "m": m, "n": n, "k": k,
        "layout_a": gemm.get("layout_a", "row_major"), "layout_b": gemm.get("layout_b", "row_major"),
        "layout_c": gemm.get("layout_c", "row_major"), "distribution": distribution,
        "input_dtype": "bf16", "accumulator_dtype": "fp32", "output_dtype": "bf16",
        "files": {name: p.name for name, p in files.items()} | {"checksums": "checksums.json"},
        "sizes_bytes": {name: p.stat().st_size for name, p in files.items()},
    }
    (case_dir / "meta.json").write_text(json.dumps(meta, indent=2) + "\n")
    return {"case_id": case_id, "seed": seed, "checksums": checksums,
            "total_bytes": sum(meta["sizes_bytes"].values())}


def load_config(path: Path) -> Dict:
    return json.loads(Path(path).read_text())


def generate(config: Dict, output_root: Path, cases: Optional[Iterable[str]] = None,
             force: bool = False, with_reference: bool = True) -> Dict:
    """Writes the manifest and the selected cases of a dataset config."""
    dataset_dir = Path(output_root) / config["dataset_id"]
    dataset_dir.mkdir(parents=True, exist_ok=True)
    selected = set(cases) if cases else None
    chosen = [c for c in config["cases"] if selected is None or c["case_id"] in selected]
    if not chosen:
        raise ValueError("no cases selected")
    manifest = {key: config[key] for key in ("dataset_id", "description", "gemm", "distribution",
                                             "benchmark_policy", "correctness_policy") if key in config}
    manifest["generated_cases"] = [c["case_id"] for c in chosen]
    (dataset_dir / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    out = [write_case(dataset_dir, config["gemm"], config["distribution"], c["case_id"], int(c["seed"]),
                      force=force, with_reference=with_reference) for c in chosen]
    return {"dataset_id": config["dataset_id"], "dataset_dir": str(dataset_dir), "generated_cases": out}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Write GEMM dataset cases in the reference's format")
    ap.add_argument("--config", type=Path, default=CONFIG_DIR / "fixed_bf16_gemm_v1.json")
    ap.add_argument("--output-root", type=Path, default=Path("artifacts/datasets"))
    ap.add_argument("--cases", nargs="*", default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--no-reference", action="store_true", help="skip C_ref (perf-only cases)")
    args = ap.parse_args(argv)
    summary = generate(load_config(args.config), args.output_root, args.cases, args.force,
                       not args.no_reference)
    print(json.dumps({"dataset_dir": summary["dataset_dir"],
                      "cases": [c["case_id"] for c in summary["generated_cases"]]}))


if __name__ == "__main__":
    main()
