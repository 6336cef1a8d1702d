"""Nsight Compute analysis for the B200 GEMM: the reference's scripts/ncu_analysis.py retargeted
to Blackwell (gb100) counters.

The reference parses sm_86 exports (tensor pipe, SM/DRAM/L2 throughput, four stall reasons;
configs/ncu_metrics_core.txt, analysis `analyze_run` :1450, bottleneck classes :719-996).  This
module reads the two CSV layouts `ncu` writes:

* "wide": `ncu -i rep.ncu-rep --page raw --csv` has one header row of metric names, one units
  row, then one row per captured launch.  Section-qualified names such as
  `FBSP.TriageCompute.dram__throughput...` are matched by their metric suffix.
* "long": `ncu --metrics ... --csv --log-file f.csv` has one row per (launch, metric) with
  columns `ID, Kernel Name, ..., Metric Name, Metric Unit, Metric Value`.

It reports, per launch:

* the tcgen05 tensor-pipe activity (`sm__pipe_tc_cycles_active`);
* TMA activity and bytes;
* the tensor core's shared-memory reads;
* L2 throughput and hit rate;
* DRAM bytes against the algorithmic bytes of the GEMM;
* warp stall ratios;
* the launch shape.

It then classifies the bottleneck with Blackwell thresholds and can diff two runs.  It also
turns a launch list into per-kernel time shares.  The agent-loop hand-offs of the reference
(node_b/node_c, state files) are outside this path and are not reproduced.

CLI:
    python -m matmul_optimizer_b200.ncu_analysis --raw prof.csv [--previous prev.csv]
        [--launches launches.csv] [--flops F] [--bytes B] [--kernel REGEX]
        [--out-json a.json] [--out-md a.md]
"""

from __future__ import annotations

import argparse
import csv
import json
import re
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence

SCHEMA_VERSION = 1

# gb100 counters this analysis reads (also the list in configs/ncu_metrics_core_gb100.txt).
HEADLINE_METRICS = {
    "duration_us": "gpu__time_duration.sum",
    "sm_clock_hz": "sm__cycles_elapsed.avg.per_second",
    "tensor_pipe_pct": "sm__pipe_tc_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "tensor_subpipe_pct": "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "tma_pipe_pct": "sm__pipe_tma_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "tma_inst_pct": "sm__inst_executed_pipe_tma.avg.pct_of_peak_sustained_active",
    "tma_load_bytes": "l1tex__m_xbar2l1tex_read_bytes_mem_global_op_tma_ld.sum",
    "tc_smem_read_pct": "l1tex__data_pipe_tc_wavefronts_mem_shared.sum.pct_of_peak_sustained_elapsed",
    "l2_throughput_pct": "lts__throughput.avg.pct_of_peak_sustained_elapsed",
    "l2_hit_rate_pct": "lts__t_sector_hit_rate.pct",
    "dram_read_bytes": "dram__bytes_read.sum",
    "dram_write_bytes": "dram__bytes_write.sum",
    "dram_throughput_pct": "dram__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm_throughput_pct": "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "warps_active_pct": "sm__warps_active.avg.pct_of_peak_sustained_active",
    "registers_per_thread": "launch__registers_per_thread",
    "grid_size": "launch__grid_size",
    "block_size": "launch__block_size",
    "cluster_dim_x": "launch__cluster_dim_x",
    "dynamic_smem_bytes": "launch__shared_mem_per_block_dynamic",
}

STALL_PREFIX = "smsp__average_warps_issue_stalled_"
STALL_SUFFIX = "_per_issue_active.ratio"

# Unit multipliers to a base unit (seconds for time, bytes for sizes, hertz for clocks).
UNIT_SCALE = {
    "ns": 1e-9, "us": 1e-6, "usecond": 1e-6, "ms": 1e-3, "msecond": 1e-3, "s": 1.0,
    "byte": 1.0, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9,
    "byte/block": 1.0, "kbyte/block": 1e3,
    "hz": 1.0, "khz": 1e3, "mhz": 1e6, "ghz": 1e9,
}

# Blackwell thresholds (percent of peak unless noted).
TENSOR_GOOD_PCT = 85.0
TENSOR_LOW_PCT = 60.0
L2_BOUND_PCT = 80.0
DRAM_BOUND_PCT = 75.0
TRAFFIC_EXCESS_RATIO = 2.0
SHORT_KERNEL_US = 20.0
STALL_DOMINANT_SHARE = 0.35


def _num(text: Any) -> Optional[float]:
    if text is None:
        return None
    if isinstance(text, (int, float)):
        return float(text)
    t = str(text).strip().replace(",", "")
    if t in ("", "n/a", "N/A", "-"):
        return None
    try:
        return float(t)
    except ValueError:
        return None


def _scaled(value: Optional[float], unit: str, base: str) -> Optional[float]:
    """Convert `value` in `unit` to the base unit family of `base` ('s', 'byte' or 'hz')."""
    if value is None:
        return None
    u = (unit or "").strip().lower()
    if u in UNIT_SCALE:
        return value * UNIT_SCALE[u]
    return value  # unitless or already base


def _suffix_lookup(record: Dict[str, tuple], name: str) -> Optional[tuple]:
    if name in record:
        return record[name]
    for key, val in record.items():
        if key.endswith("." + name) or key.split(".", 2)[-1] == name:
            return val
    return None


def read_wide_csv(path: Path) -> List[Dict[str, tuple]]:
    """Rows of an `ncu --page raw --csv` export: one dict per launch, metric -> (unit, value)."""
    rows = list(csv.reader(Path(path).read_text().splitlines()))
    rows = [r for r in rows if r and not r[0].startswith("==")]
    if len(rows) < 3:
        return []
    header, units = rows[0], rows[1]
    out = []
    for r in rows[2:]:
        out.append({h: (u, v) for h, u, v in zip(header, units, r)})
    return out


def read_long_csv(path: Path) -> List[Dict[str, tuple]]:
    """Rows of an `ncu --csv --log-file` export, grouped into one dict per launch ID."""
    lines = [ln for ln in Path(path).read_text().splitlines() if ln and not ln.startswith("==")]
    reader = csv.DictReader(lines)
    launches: Dict[str, Dict[str, tuple]] = {}
    for row in reader:
        lid = row.get("ID")
        if lid is None:
            continue
        rec = launches.setdefault(lid, {"ID": ("", lid), "Kernel Name": ("", row.get("Kernel Name", "")),
                                        "Block Size": ("", row.get("Block Size", "")),
                                        "Grid Size": ("", row.get("Grid Size", ""))})
        rec[row["Metric Name"]] = (row.get("Metric Unit", ""), row.get("Metric Value", ""))
    return [launches[k] for k in sorted(launches, key=lambda x: int(x) if x.isdigit() else x)]


def read_csv(path: Path) -> List[Dict[str, tuple]]:
    head = Path(path).read_text().splitlines()[:3]
    is_long = any("Metric Name" in h and "Metric Value" in h for h in head)
    return read_long_csv(path) if is_long else read_wide_csv(path)


def summarize_launch(record: Dict[str, tuple], flops: Optional[float] = None,
                     algorithmic_bytes: Optional[float] = None) -> Dict[str, Any]:
    """Headline numbers of one launch, in base units (seconds, bytes, hertz, percent)."""
    s: Dict[str, Any] = {"kernel": record.get("Kernel Name", ("", ""))[1], "id": record.get("ID", ("", ""))[1]}
    for key, metric in HEADLINE_METRICS.items():
        hit = _suffix_lookup(record, metric)
        if hit is None:
            s[key] = None
            continue
        unit, raw = hit
        val = _num(raw)
        if key == "duration_us":
            sec = _scaled(val, unit, "s")
            s[key] = None if sec is None else sec * 1e6
        elif key.endswith("_bytes"):
            s[key] = _scaled(val, unit, "byte")
        elif key == "sm_clock_hz":
            s[key] = _scaled(val, unit, "hz")
        else:
            s[key] = val
    stalls = {}
    for name, (unit, raw) in record.items():
        base = name.split(".", 2)[-1] if name.count(".") > 2 else name
        if base.startswith(STALL_PREFIX) and base.endswith(STALL_SUFFIX):
            v = _num(raw)
            if v is not None:
                stalls[base[len(STALL_PREFIX):-len(STALL_SUFFIX)]] = v
    s["stalls"] = dict(sorted(stalls.items(), key=lambda kv: -kv[1]))
    rd, wr = s.get("dram_read_bytes"), s.get("dram_write_bytes")
    s["dram_bytes"] = None if rd is None or wr is None else rd + wr
    dur = s.get("duration_us")
    if flops and dur:
        s["achieved_tflops"] = flops / (dur * 1e-6) / 1e12
    if algorithmic_bytes and s["dram_bytes"]:
        s["dram_traffic_ratio"] = s["dram_bytes"] / algorithmic_bytes
    return s


def classify(summary: Dict[str, Any]) -> List[Dict[str, Any]]:
    """Bottleneck classes for a GEMM launch, most important first, each with its evidence."""
    out: List[Dict[str, Any]] = []

    def add(cls: str, severity: str, evidence: str):
        out.append({"class": cls, "severity": severity, "evidence": evidence})

    tc = summary.get("tensor_pipe_pct")
    l2 = summary.get("l2_throughput_pct")
    dram = summary.get("dram_throughput_pct")
    dur = summary.get("duration_us")
    ratio = summary.get("dram_traffic_ratio")
    stalls = summary.get("stalls") or {}
    if dur is not None and dur < SHORT_KERNEL_US:
        add("launch_or_tail_bound", "high", f"kernel lasts {dur:.1f} us (< {SHORT_KERNEL_US:.0f} us)")
    if tc is not None:
        if tc < TENSOR_LOW_PCT:
            add("tensor_core_underutilization", "high", f"tcgen05 pipe active {tc:.1f}% of peak")
        elif tc < TENSOR_GOOD_PCT:
            add("tensor_core_underutilization", "medium", f"tcgen05 pipe active {tc:.1f}% of peak")
    if l2 is not None and l2 >= L2_BOUND_PCT:
        add("l2_bandwidth_bound", "high", f"L2 throughput {l2:.1f}% of peak")
    if dram is not None and dram >= DRAM_BOUND_PCT:
        add("dram_bandwidth_bound", "high", f"DRAM throughput {dram:.1f}% of peak")
    if ratio is not None and ratio > TRAFFIC_EXCESS_RATIO:
        add("dram_traffic_excess", "medium",
            f"DRAM traffic {ratio:.2f}x the algorithmic bytes (operand re-reads across raster groups)")
    if stalls:
        total = sum(stalls.values())
        top, val = next(iter(stalls.items()))
        if total > 0 and val / total >= STALL_DOMINANT_SHARE:
            cls = {"long_scoreboard": "memory_or_tmem_latency", "barrier": "synchronization_barrier",
                   "membar": "memory_fence", "wait": "fixed_latency_wait",
                   "mio_throttle": "shared_memory_pressure", "short_scoreboard": "shared_memory_pressure",
                   "sleeping": "warp_sleep"}.get(top, f"stall_{top}")
            add(cls, "low", f"{top} stalls are {100 * val / total:.0f}% of sampled issue stalls "
                            "(warp-specialised kernels park most warps on barriers by design)")
    if tc is not None and tc >= TENSOR_GOOD_PCT and not any(c["severity"] == "high" for c in out):
        add("tensor_bound_near_peak", "info", f"tcgen05 pipe active {tc:.1f}%: the kernel is tensor-bound")
    return out


def diff(prev: Dict[str, Any], cur: Dict[str, Any]) -> Dict[str, Any]:
    """Current minus previous for the numeric headline fields both runs have."""
    out = {}
    for key in list(HEADLINE_METRICS) + ["dram_bytes", "achieved_tflops", "dram_traffic_ratio"]:
        a, b = prev.get(key), cur.get(key)
        if isinstance(a, (int, float)) and isinstance(b, (int, float)):
            out[key] = {"previous": a, "current": b, "delta": b - a}
    return out


def launch_shares(records: Sequence[Dict[str, tuple]]) -> List[Dict[str, Any]]:
    """Per-kernel launch count, total device time and share of a launch list."""
    agg: Dict[str, List[float]] = {}
    for rec in records:
        hit = _suffix_lookup(rec, "gpu__time_duration.sum")
        if hit is None:
            continue
        sec = _scaled(_num(hit[1]), hit[0], "s")
        if sec is None:
            continue
        name = rec.get("Kernel Name", ("", "?"))[1]
        agg.setdefault(name, []).append(sec)
    total = sum(sum(v) for v in agg.values()) or 1.0
    rows = [{"kernel": k, "launches": len(v), "total_us": sum(v) * 1e6, "us_per_launch": sum(v) / len(v) * 1e6,
             "share": sum(v) / total} for k, v in agg.items()]
    return sorted(rows, key=lambda r: -r["total_us"])


def analyze(raw: Path, kernel_regex: Optional[str] = None, previous: Optional[Path] = None,
            launches: Optional[Path] = None, flops: Optional[float] = None,
            algorithmic_bytes: Optional[float] = None) -> Dict[str, Any]:
    """Full analysis of one capture (optionally against a previous capture and a launch list)."""
    pattern = re.compile(kernel_regex) if kernel_regex else None

    def pick(records):
        chosen = [r for r in records if pattern is None or pattern.search(r.get("Kernel Name", ("", ""))[1])]
        if not chosen:
            raise ValueError(f"no launch matches {kernel_regex!r}")
        return chosen[-1]

    cur = summarize_launch(pick(read_csv(raw)), flops, algorithmic_bytes)
    result: Dict[str, Any] = {"schema_version": SCHEMA_VERSION, "source": str(raw), "launch": cur,
                              "bottlenecks": classify(cur)}
    if previous is not None:
        prev = summarize_launch(pick(read_csv(previous)), flops, algorithmic_bytes)
        result["previous"] = {"source": str(previous), "launch": prev}
        result["delta_vs_previous"] = diff(prev, cur)
    if launches is not None:
        result["launch_shares"] = launch_shares(read_csv(launches))
    return result


def _fmt(v: Any, digits: int = 1) -> str:
    if v is None:
        return "n/a"
    if isinstance(v, float):
        return f"{v:,.{digits}f}"
    return str(v)


def render_markdown(a: Dict[str, Any]) -> str:
    s = a["launch"]
    lines = [f"# ncu analysis: `{s['kernel'][:100]}`", "",
             f"Source: `{a['source']}` (launch ID {s['id']})", "",
             "| metric | value |", "|---|---|"]
    rows = [("duration (us)", s.get("duration_us")), ("SM clock (GHz)", (s.get("sm_clock_hz") or 0) / 1e9 or None),
            ("tcgen05 pipe active (%)", s.get("tensor_pipe_pct")), ("TMA pipe active (%)", s.get("tma_pipe_pct")),
            ("tensor-core smem reads (% of peak)", s.get("tc_smem_read_pct")),
            ("L2 throughput (%)", s.get("l2_throughput_pct")), ("L2 hit rate (%)", s.get("l2_hit_rate_pct")),
            ("DRAM throughput (%)", s.get("dram_throughput_pct")),
            ("TMA load bytes (MB)", (s.get("tma_load_bytes") or 0) / 1e6 or None),
            ("DRAM read (MB)", (s.get("dram_read_bytes") or 0) / 1e6 or None),
            ("DRAM write (MB)", (s.get("dram_write_bytes") or 0) / 1e6 or None),
            ("DRAM traffic / algorithmic bytes", s.get("dram_traffic_ratio")),
            ("achieved TFLOP/s", s.get("achieved_tflops")), ("warps active (%)", s.get("warps_active_pct")),
            ("registers / thread", s.get("registers_per_thread")), ("grid", s.get("grid_size")),
            ("cluster x", s.get("cluster_dim_x"))]
    for name, val in rows:
        lines.append(f"| {name} | {_fmt(val, 3 if isinstance(val, float) and abs(val) < 10 else 1)} |")
    lines += ["", "## Bottlenecks", ""]
    for b in a["bottlenecks"]:
        lines.append(f"- **{b['class']}** ({b['severity']}): {b['evidence']}")
    if s.get("stalls"):
        lines += ["", "## Issue-stall ratios (warps stalled per issue)", ""]
        lines += [f"- {k}: {v:.3f}" for k, v in list(s["stalls"].items())[:6]]
    if "delta_vs_previous" in a:
        lines += ["", "## Change vs previous capture", "", "| metric | previous | current | delta |", "|---|---|---|---|"]
        for k, d in a["delta_vs_previous"].items():
            lines.append(f"| {k} | {_fmt(d['previous'], 3)} | {_fmt(d['current'], 3)} | {_fmt(d['delta'], 3)} |")
    if "launch_shares" in a:
        lines += ["", "## Launch list", "", "| kernel | launches | total us | us/launch | share |", "|---|---:|---:|---:|---:|"]
        for r in a["launch_shares"]:
            lines.append(f"| `{r['kernel'][:80]}` | {r['launches']} | {r['total_us']:.1f} | "
                         f"{r['us_per_launch']:.1f} | {100 * r['share']:.1f}% |")
    return "\n".join(lines) + "\n"


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Blackwell ncu analysis of a GEMM capture")
    ap.add_argument("--raw", type=Path, required=True, help="ncu raw-page CSV (wide) or --csv log (long)")
    ap.add_argument("--kernel", default=None, help="regex selecting the launch (default: last)")
    ap.add_argument("--previous", type=Path, default=None)
    ap.add_argument("--launches", type=Path, default=None, help="launch-list CSV for time shares")
    ap.add_argument("--flops", type=float, default=None, help="algorithmic FLOPs per launch")
    ap.add_argument("--bytes", type=float, default=None, help="algorithmic bytes per launch")
    ap.add_argument("--out-json", type=Path, default=None)
    ap.add_argument("--out-md", type=Path, default=None)
    args = ap.parse_args(argv)
    result = analyze(args.raw, args.kernel, args.previous, args.launches, args.flops, args.bytes)
    if args.out_json:
        args.out_json.write_text(json.dumps(result, indent=2) + "\n")
    md = render_markdown(result)
    if args.out_md:
        args.out_md.write_text(md)
    if not args.out_json and not args.out_md:
        print(md)


if __name__ == "__main__":
    main()
