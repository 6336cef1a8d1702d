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


# ---- the drop-in interface of the reference's scripts/ncu_analysis.py (schema_version 2) ----
# Shaped after the reference's tests (tests/test_ncu_rich_handoff.py:146-365), on gb100 exports.
import os
import subprocess
import sys

HEADLINE = ["sm__pipe_tc_cycles_active.avg.pct_of_peak_sustained_elapsed",
            "sm__throughput.avg.pct_of_peak_sustained_elapsed",
            "lts__throughput.avg.pct_of_peak_sustained_elapsed",
            "dram__bytes_read.sum", "dram__bytes_write.sum", "launch__registers_per_thread"]
SUMMARY_KEYS = {"schema_version", "status", "source_run_id", "source_run_dir", "analysis_path", "kernel_name",
                "block_size", "grid_size", "registers_per_thread", "shared_mem_per_block_allocated", "launch",
                "headline_metrics", "stall_breakdown", "bottleneck_classes", "top_findings", "top_source_hotspots",
                "delta_vs_previous_run", "handoff", "raw_csv_path", "raw_rep_path", "raw_details_csv_path",
                "import_raw_csv_path", "details_page_csv_path", "source_csv_path", "artifacts"}


def _stage(tmp_path, name, headline, raw=None, details=None, source=None):
    run = tmp_path / "runs" / name
    run.mkdir(parents=True)
    (run / "ncu_metrics.csv").write_text((FIX / headline).read_text())
    if raw:
        (run / "ncu_import_raw.csv").write_text((FIX / raw).read_text())
        (run / "ncu_details.csv").write_text((FIX / raw).read_text())
    if details is not None:
        (run / "ncu_details_page.csv").write_text(details)
    if source is not None:
        (run / "ncu_source.csv").write_text(source)
    (run / "ncu_profile.ncu-rep").write_text("fixture report\n")
    return run


def _analyze(run, previous=None, source_reason=None):
    details = run / "ncu_details_page.csv"
    source = run / "ncu_source.csv"
    raw = run / "ncu_import_raw.csv"
    a = na.analyze_run(run_dir=run, source_run_id=run.name, headline_csv_path=run / "ncu_metrics.csv",
                       import_raw_path=raw if raw.exists() else None,
                       details_page_path=details if details.exists() else None,
                       source_csv_path=source if source.exists() else None, rep_path=run / "ncu_profile.ncu-rep",
                       wanted_headline_metrics=HEADLINE, previous_analysis_path=previous,
                       source_unavailable_reason=source_reason, legacy_import_raw_alias=run / "ncu_details.csv",
                       return_codes={"rep": 0, "headline_csv": 0, "import_raw": 0, "details_page": None,
                                     "source_page": 1})
    return a, na.write_analysis_outputs(run_dir=run, analysis=a)


def test_dropin_parsers_on_gb100_exports():
    wide = na.parse_wide_csv_records(FIX / "raw_gemm_hero.csv")
    assert len(wide) == 1 and na.parse_wide_csv_records(FIX / "metrics_gemm_vs_cublas.csv") == []
    launch = na.build_launch(wide[0], None)
    assert "gemm_bf16_sm100_kernel<2, 128, 6>" in launch["kernel_name"]
    assert launch["block_size"] == "(384, 1, 1)" and launch["grid_size"] == "(148, 1, 1)"
    assert launch["registers_per_thread"] == 168.0 and launch["cluster_size"] == 2.0
    longs = na.long_csv_records(FIX / "metrics_gemm_vs_cublas.csv")
    assert len(longs) == 4
    primary = na.select_primary_record(longs)  # the longest launch
    assert primary["Kernel Name"].startswith("void mo::")
    kv = na.parse_name_value_metrics(FIX / "metrics_gemm_vs_cublas.csv")
    assert kv["launch__grid_size"] == 884.0  # the last launch listed (cuBLAS) wins, as in the reference
    units = na.units_of(FIX / "raw_gemm_hero.csv")
    assert units["gpu__time_duration.sum"] == "us" and units["dram__bytes_read.sum"] == "Mbyte"


def test_dropin_analysis_schema_units_and_classes(tmp_path):
    run = _stage(tmp_path, "r_hero", "raw_gemm_hero.csv")
    a, (json_path, md_path) = _analyze(run)
    assert a["schema_version"] == 2 and a["status"] == "available"
    for key in ("launch", "headline_metrics", "stall_breakdown", "memory_hierarchy", "occupancy_latency",
                "tensor_core_utilization", "rules", "section_highlights", "source_hotspots", "artifacts",
                "bottleneck_classes", "delta_vs_previous_run", "handoff"):
        assert key in a, key
    # Display units (usecond, Mbyte) are turned into ns and bytes for the derived fields.
    assert a["launch"]["duration_ns"] == pytest.approx(474208.0)
    assert a["memory_hierarchy"]["dram_bytes"] == pytest.approx(834.889216e6)
    assert a["tensor_core_utilization"]["tensor_pipe_active_pct"] == pytest.approx(89.83, abs=0.01)
    assert a["headline_metrics"]["sm__pipe_tc_cycles_active.avg.pct_of_peak_sustained_elapsed"] == pytest.approx(89.83, abs=0.01)
    # A tensor-bound launch at 90 % tcgen05 activity is not flagged as under-using the tensor core,
    # and one CTA per SM (the design) is not an occupancy finding.
    ids = [c["class_id"] for c in a["bottleneck_classes"]]
    assert "tensor_core_underutilization" not in ids and "occupancy_latency_hiding_issue" not in ids
    top = a["stall_breakdown"][0]
    assert top["stall_group"] == "long_scoreboard" and top["by_design"] is True
    assert a["source_hotspots"] and a["handoff"]["node_c"]["target_hotspots"]
    guard = {g["metric_name"]: g["guardrail"] for g in a["handoff"]["node_c"]["guardrail_metrics"]}
    assert guard["sm__pipe_tc_cycles_active.avg.pct_of_peak_sustained_elapsed"] == "non_decreasing"
    assert json_path.name == "ncu_analysis.json" and md_path.read_text().startswith("# NCU analysis")
    assert set(na.build_rich_summary_from_analysis(a)) >= SUMMARY_KEYS


def test_dropin_flags_an_underused_tensor_pipe_and_computes_deltas(tmp_path):
    prev = _stage(tmp_path, "r_prev", "raw_gemm_hero_prev.csv")
    _, (prev_json, _) = _analyze(prev)
    cur = _stage(tmp_path, "r_cur", "metrics_gemm_vs_cublas.csv")
    a, _ = _analyze(cur, previous=prev_json)
    assert a["launch"]["kernel_name"].startswith("void mo::")
    tc = a["tensor_core_utilization"]["tensor_pipe_active_pct"]
    assert tc < 85.0
    top = a["bottleneck_classes"][0]
    assert top["class_id"] == "tensor_core_underutilization" and top["rank"] == 1
    assert top["severity_score"] == pytest.approx(85.0 - tc, abs=1e-3)
    delta = a["delta_vs_previous_run"]
    assert delta["baseline_run_id"] == "r_prev"
    d = delta["headline_metrics"]["sm__pipe_tc_cycles_active.avg.pct_of_peak_sustained_elapsed"]
    assert d["trend"] == "regressed" and d["delta"] < 0
    findings = [f["finding_id"] for f in a["handoff"]["node_b"]["top_findings"]]
    assert "finding::tensor_core_underutilization" in findings
    assert any(f.startswith("finding::delta::") for f in findings)


def test_dropin_details_page_rules_and_hotspots(tmp_path):
    """Of a details page, the speed-of-light throughputs and ncu's rules become hotspots and rules;
    rows that describe the kernel's design (occupancy, L1 hit rate) do not, and other kernels' rows
    are ignored."""
    kernel = na.parse_wide_csv_records(FIX / "raw_gemm_hero.csv")[0]["Kernel Name"]
    details = ('"ID","Kernel Name","Section Name","Metric Name","Metric Unit","Metric Value","Rule Name",'
               '"Rule Type","Rule Description","Estimated Speedup Type","Estimated Speedup"\n'
               f'"0","{kernel}","GPU Speed Of Light Throughput","DRAM Throughput","%","21.0","","","","",""\n'
               f'"0","{kernel}","Occupancy","Achieved Occupancy","%","18.7","","","","",""\n'
               f'"0","{kernel}","Memory Workload Analysis","L1/TEX Hit Rate","%","0.0","","","","",""\n'
               f'"0","{kernel}","Memory Workload Analysis","","","","L2OperandReReads","WRN",'
               '"DRAM traffic is 2.7x the algorithmic bytes: memory operand re-reads across raster groups","global","4.5"\n'
               '"1","other_kernel","GPU Speed Of Light Throughput","DRAM Throughput","%","90.0","","","","",""\n')
    run = _stage(tmp_path, "r_details", "raw_gemm_hero.csv", details=details)
    a, _ = _analyze(run)
    assert [r["rule_name"] for r in a["rules"]] == ["L2OperandReReads"]
    rule = a["rules"][0]
    assert rule["severity"] == "warning" and rule["estimated_speedup_pct"] == 4.5
    metrics = {h["metric_name"]: h for h in a["source_hotspots"]}
    assert "DRAM Throughput" in metrics and metrics["DRAM Throughput"]["metric_value"] == 21.0
    assert "Achieved Occupancy" not in metrics and "L1/TEX Hit Rate" not in metrics
    assert any(h["scope_name"] == "tcgen05_pipe" for h in a["source_hotspots"])
    # A low-DRAM launch is not called memory bound because a rule's text mentions memory.
    assert "global_memory_bound" not in [c["class_id"] for c in a["bottleneck_classes"]]
    assert rule["rule_id"] in [rid for h in a["section_highlights"] for rid in h["rule_ids"]]


def test_dropin_skips_a_disassembly_source_page(tmp_path):
    """A source page exported as disassembly (Address, Source) is never parsed: hotspots come from
    the headline counters and the artifact says why."""
    run = _stage(tmp_path, "r_sass", "raw_gemm_hero.csv", source='"Address","Source"\n"0x0","(elided)"\n')
    a, _ = _analyze(run)
    src = a["artifacts"]["source_page"]
    assert src["status"] == "available" and src["structured_hotspots_available"] is False
    assert "disassembly" in src["unavailable_reason"]
    assert all(h["scope_type"] == "section" for h in a["source_hotspots"])


def test_dropin_reference_cli_writes_outputs(tmp_path):
    run = _stage(tmp_path, "r_cli", "raw_gemm_hero.csv")
    cmd = [sys.executable, str(Path(na.__file__)), "--run-dir", str(run), "--source-run-id", "r_cli",
           "--headline-csv", str(run / "ncu_metrics.csv"), "--headline-metric", HEADLINE[0]]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr
    out = json.loads((run / "ncu_analysis.json").read_text())
    assert out["source_run_id"] == "r_cli" and HEADLINE[0] in out["headline_metrics"]


def test_dropin_serves_the_reference_eval_kernel(tmp_path, reference_root):
    """The reference's own scripts/eval_kernel.py, with this module in place of its ncu_analysis,
    parses a gb100 export and builds its ncu summary from our analysis."""
    import importlib.util

    scripts = reference_root / "scripts"
    sys.modules["ncu_analysis"] = na
    try:
        spec = importlib.util.spec_from_file_location("ref_eval_kernel", scripts / "eval_kernel.py")
        ek = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(ek)
    finally:
        del sys.modules["ncu_analysis"]
    assert ek.ncu_analysis is na
    run = _stage(tmp_path, "r_ek", "raw_gemm_hero.csv")
    metrics = ek.parse_ncu_csv(run / "ncu_metrics.csv")
    assert "gemm_bf16_sm100_kernel" in metrics["Kernel Name"]
    a, (json_path, _) = _analyze(run)
    summary = ek.build_ncu_summary(full_metrics=metrics, headline_metrics={}, csv_path=run / "ncu_metrics.csv",
                                   rep_path=run / "ncu_profile.ncu-rep", import_raw_path=None, details_page_path=None,
                                   source_csv_path=None, legacy_import_raw_alias=None, analysis=a,
                                   analysis_json_path=json_path)
    assert summary["analysis_path"] == "ncu_analysis.json" and summary["schema_version"] == 2
    text = ek.render_markdown_ncu_summary(summary)
    assert "gemm_bf16_sm100_kernel" in text


def test_dropin_on_a_full_gb100_capture(tmp_path):
    """A --set full capture of the 2-GPU column slab (6464x3888x7232) exported as eval_kernel.py
    exports it: the raw page (trimmed to the counters read here) and the details page with ncu's
    gb100 rules (Rule Type WRN/OPT/INF, Rule Description, Estimated Speedup)."""
    details = (FIX / "details_gemm_slab2.csv").read_text()
    run = _stage(tmp_path, "r_slab2", "raw_gemm_slab2.csv", raw="raw_gemm_slab2.csv", details=details)
    a, _ = _analyze(run)
    assert a["launch"]["duration_ns"] == pytest.approx(263200.0)
    assert a["memory_hierarchy"]["dram_bytes"] == pytest.approx(436.786944e6 + 49.98656e6)
    assert a["tensor_core_utilization"]["tensor_pipe_active_pct"] == pytest.approx(83.77, abs=0.01)
    rules = {r["rule_name"]: r for r in a["rules"]}
    assert "HighPipeUtilization" in rules and rules["HighPipeUtilization"]["severity"] == "optimization"
    assert "TC is the highest-utilized pipeline" in rules["HighPipeUtilization"]["message"]
    assert rules["SOLBottleneck"]["severity"] == "info"
    assert all(r["severity"] in ("error", "warning", "optimization", "info") for r in a["rules"])
    assert a["rules"][0]["importance_score"] >= a["rules"][-1]["importance_score"]
    # Hotspots come from the details page's section metrics; every one names its section.
    assert a["source_hotspots"] and all(h["section_name"] for h in a["source_hotspots"])
    ids = [c["class_id"] for c in a["bottleneck_classes"]]
    assert ids[0] == "tensor_core_underutilization"  # 83.8 % < 85 %
    assert a["handoff"]["node_b"]["code_regions_to_investigate"]
    summary = na.build_rich_summary_from_analysis(a)
    assert set(summary) >= SUMMARY_KEYS and summary["details_page_csv_path"].endswith("ncu_details_page.csv")
