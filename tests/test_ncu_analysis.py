"""Blackwell retarget of the reference's ncu analysis (scripts/ncu_analysis.py), tested on
exports of real gb100 captures of this repository's kernel (tests/fixtures/ncu_gb100), as the
reference tests its parser on sm_86 exports (tests/test_ncu_rich_handoff.py:146-220)."""

import json
from pathlib import Path

import pytest

from matmul_optimizer_b200 import ncu_analysis as na

FIX = Path(__file__).resolve().parent / "fixtures" / "ncu_gb100"
CONFIGS = Path(na.__file__).resolve().parent / "configs"
HERO_FLOPS = 2.0 * 6464 * 7776 * 7232
HERO_BYTES = 2.0 * (6464 * 7232 + 7232 * 7776 + 6464 * 7776)


def test_wide_raw_page_headline():
    rec = na.read_csv(FIX / "raw_gemm_hero.csv")
    assert len(rec) == 1
    s = na.summarize_launch(rec[0], HERO_FLOPS, HERO_BYTES)
    assert "gemm_bf16_sm100_kernel<2, 128, 6>" in s["kernel"]
    assert s["duration_us"] == pytest.approx(474.208)
    assert s["sm_clock_hz"] == pytest.approx(1.4987e9, rel=1e-3)
    assert s["tensor_pipe_pct"] == pytest.approx(89.83, abs=0.01)
    assert s["dram_bytes"] == pytest.approx(735.14496e6 + 99.744256e6)
    assert s["dram_traffic_ratio"] == pytest.approx(2.724, abs=1e-3)
    assert s["achieved_tflops"] == pytest.approx(1533.1, abs=0.5)
    # Section-qualified names (FBSP.TriageCompute.dram__throughput...) are found by suffix.
    assert na._suffix_lookup(rec[0], "dram__throughput.avg.pct_of_peak_sustained_elapsed") is not None
    assert s["cluster_dim_x"] == 2 and s["grid_size"] == 148 and s["dynamic_smem_bytes"] == pytest.approx(230552)
    assert next(iter(s["stalls"])) == "long_scoreboard"


def test_long_log_two_kernels():
    recs = na.read_csv(FIX / "metrics_gemm_vs_cublas.csv")
    kernels = {r["Kernel Name"][1] for r in recs}
    assert any(k.startswith("nvjet") for k in kernels) and any("gemm_bf16" in k for k in kernels)
    ours = na.summarize_launch([r for r in recs if "gemm_bf16" in r["Kernel Name"][1]][0])
    cublas = na.summarize_launch([r for r in recs if "nvjet" in r["Kernel Name"][1]][0])
    assert ours["tensor_pipe_pct"] == pytest.approx(76.28, abs=0.01)
    assert cublas["tensor_pipe_pct"] == pytest.approx(92.19, abs=0.01)
    assert cublas["grid_size"] == 884 and ours["grid_size"] == 148


def test_launch_shares():
    shares = na.launch_shares(na.read_csv(FIX / "launches_bench_hero.csv"))
    assert sum(r["share"] for r in shares) == pytest.approx(1.0)
    top = shares[0]
    assert "gemm_bf16_sm100_kernel" in top["kernel"] and top["launches"] == 11
    assert top["share"] == pytest.approx(0.591, abs=0.001)


def test_classification_rules():
    base = {"tensor_pipe_pct": 90.0, "l2_throughput_pct": 40.0, "dram_throughput_pct": 20.0, "duration_us": 400.0,
            "dram_traffic_ratio": 1.2, "stalls": {}}
    assert [c["class"] for c in na.classify(base)] == ["tensor_bound_near_peak"]
    low = dict(base, tensor_pipe_pct=50.0)
    assert na.classify(low)[0] == {"class": "tensor_core_underutilization", "severity": "high",
                                   "evidence": "tcgen05 pipe active 50.0% of peak"}
    classes = {c["class"] for c in na.classify(dict(base, l2_throughput_pct=85.0, dram_throughput_pct=80.0,
                                                    duration_us=10.0, dram_traffic_ratio=3.0,
                                                    stalls={"barrier": 9.0, "wait": 1.0}))}
    assert classes >= {"l2_bandwidth_bound", "dram_bandwidth_bound", "launch_or_tail_bound",
                       "dram_traffic_excess", "synchronization_barrier"}
    assert "tensor_bound_near_peak" not in classes


def test_delta_and_cli(tmp_path):
    a = na.analyze(FIX / "raw_gemm_hero.csv", kernel_regex="gemm_bf16", previous=FIX / "raw_gemm_hero_prev.csv",
                   launches=FIX / "launches_bench_hero.csv", flops=HERO_FLOPS, algorithmic_bytes=HERO_BYTES)
    d = a["delta_vs_previous"]
    assert d["tensor_pipe_pct"]["delta"] == pytest.approx(89.834 - 76.758, abs=1e-3)
    assert d["duration_us"]["delta"] < 0
    with pytest.raises(ValueError):
        na.analyze(FIX / "raw_gemm_hero.csv", kernel_regex="no_such_kernel")
    out_json, out_md = tmp_path / "a.json", tmp_path / "a.md"
    na.main(["--raw", str(FIX / "raw_gemm_hero.csv"), "--previous", str(FIX / "raw_gemm_hero_prev.csv"),
             "--flops", str(HERO_FLOPS), "--bytes", str(HERO_BYTES), "--out-json", str(out_json), "--out-md", str(out_md)])
    j = json.loads(out_json.read_text())
    assert j["schema_version"] == na.SCHEMA_VERSION and j["bottlenecks"]
    md = out_md.read_text()
    assert "tcgen05 pipe active (%) | 89.8" in md and "Change vs previous capture" in md


def test_metric_list_names_exist_on_gb100():
    """Every counter of the gb100 metric list is present in a real gb100 capture."""
    names = [ln.strip() for ln in (CONFIGS / "ncu_metrics_core_gb100.txt").read_text().splitlines() if ln.strip()]
    rec = na.read_csv(FIX / "raw_gemm_hero.csv")[0]
    missing = [n for n in names if na._suffix_lookup(rec, n) is None]
    assert not missing, missing
    assert set(na.HEADLINE_METRICS.values()) >= set(names) - {"launch__occupancy_limit_registers"}
