"""The product's dataset writer produces the reference's on-disk case format, byte for byte
on the inputs (checksums of the reference's own write_case, tests/golden)."""

import json
from pathlib import Path

import numpy as np

from matmul_optimizer_b200 import dataset

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_cases_match_reference_checksums(tmp_path):
    index = json.loads((GOLDEN / "small_cases_index.json").read_text())
    data = np.load(GOLDEN / "small_cases.npz")
    for e in index[:6]:
        out = dataset.write_case(tmp_path, {"m": e["m"], "n": e["n"], "k": e["k"]},
                                 {"name": "uniform", "low": -1.0, "high": 1.0},
                                 f"c_{e['key']}", e["seed"])
        assert out["checksums"]["A_bf16"] == e["checksums"]["A_bf16"]
        assert out["checksums"]["B_bf16"] == e["checksums"]["B_bf16"]
        case_dir = tmp_path / "cases" / f"c_{e['key']}"
        meta = json.loads((case_dir / "meta.json").read_text())
        assert (meta["m"], meta["n"], meta["k"]) == (e["m"], e["n"], e["k"])
        assert set(meta["files"]) >= {"A_bf16", "B_bf16", "C_ref_fp32", "C_ref_bf16", "checksums"}
        c16 = np.fromfile(case_dir / "C_ref_bf16.bin", dtype=np.uint16).reshape(e["m"], e["n"])
        assert np.mean(c16 == data[f"{e['key']}_c16"]) > 0.99


def test_generate_manifest_and_configs(tmp_path):
    for cfg_path in sorted(dataset.CONFIG_DIR.glob("*.json")):
        cfg = dataset.load_config(cfg_path)
        assert {"dataset_id", "gemm", "distribution", "cases"} <= set(cfg)
    cfg = dataset.load_config(dataset.CONFIG_DIR / "fixed_bf16_gemm_v1.json")
    assert (cfg["gemm"]["m"], cfg["gemm"]["n"], cfg["gemm"]["k"]) == (6464, 7776, 7232)
    assert [c["seed"] for c in cfg["cases"]] == [3407, 9713, 1729]
    small = dict(cfg, gemm=dict(cfg["gemm"], m=32, n=64, k=48))
    summary = dataset.generate(small, tmp_path, cases=["case_01_seed_9713"])
    manifest = json.loads((Path(summary["dataset_dir"]) / "manifest.json").read_text())
    assert manifest["correctness_policy"]["initial_atol"] == 0.15
    assert manifest["generated_cases"] == ["case_01_seed_9713"]


def test_normal_distribution_config():
    a, b = dataset.draw_inputs(64, 128, 256, 3407, {"name": "normal", "std_a": 1.0, "std_b": 0.02, "seed_b": 9713})
    af = dataset.bf16_bits_to_f32(a)
    bf = dataset.bf16_bits_to_f32(b)
    assert 0.9 < af.std() < 1.1 and 0.018 < bf.std() < 0.022
