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
turns a launch list into per-kernel time shares.

Drop-in interface (second half of this file).  The reference's orchestrator
scripts/eval_kernel.py does ``import ncu_analysis`` and calls ``analyze_run``,
``write_analysis_outputs``, ``build_rich_summary_from_analysis``, ``parse_wide_csv_records``,
``select_primary_record`` and ``parse_name_value_metrics`` (eval_kernel.py:57, :161,
:267-270, :505-527).  Those functions exist here with the reference's signatures and the
reference's analysis schema (schema_version 2: launch, headline metrics, stall breakdown,
memory hierarchy, occupancy, tensor-core utilisation, rules, section highlights, hotspots,
bottleneck classes, delta vs the previous run, node_b / node_c hand-off), so that this file,
placed as scripts/ncu_analysis.py, serves the reference's ``--ncu`` flow.  What differs is the
reading of the counters: the tensor pipe is the tcgen05 pipe (sm__pipe_tc_cycles_active), the
stalls are gb100's per-issue ratios, and the thresholds are those of a persistent,
warp-specialised sm_100a GEMM (one CTA per SM, so register and shared-memory occupancy limits
are the design, not a finding).  The module uses the standard library only, so it runs as a
top-level module as well as inside the package.  A source page that ncu exported as
disassembly (columns Address, Source) is detected and skipped, never parsed.

CLI:
    python -m matmul_optimizer_b200.ncu_analysis --raw prof.csv [--previous prev.csv]
        [--launches launches.csv] [--flops F] [--bytes B] [--kernel REGEX]
        [--out-json a.json] [--out-md a.md]
    python ncu_analysis.py --run-dir DIR --source-run-id ID [--headline-csv F]
        [--import-raw-csv F] [--details-page-csv F] [--source-csv F] [--rep-path F]
        [--previous-analysis F] [--headline-metric M ...]     (the reference's CLI)
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import math
import re
import sys
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional, Sequence, Tuple

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


# ========================================================================================
# Drop-in interface of the reference's scripts/ncu_analysis.py (schema_version 2)
# ========================================================================================
# The names, signatures and output keys below are the reference's (analyze_run :1450,
# write_analysis_outputs :1734, build_rich_summary_from_analysis :1683, parsers :212-350),
# because scripts/eval_kernel.py and the agent loop read them; the reading of the counters is
# Blackwell's.

HANDOFF_SCHEMA_VERSION = 2
TOP_FINDINGS = 6
TOP_HOTSPOTS = 8

# Counters behind each derived field, gb100 first, then the sm_86 names the reference's
# metrics file asks for (an export may carry either).
# Elapsed before active: a persistent kernel's prologue and tail count against it.
_TENSOR_PIPE = ("sm__pipe_tc_cycles_active.avg.pct_of_peak_sustained_elapsed",
                "sm__pipe_tc_cycles_active.avg.pct_of_peak_sustained_active",
                "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
                "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active")
_TMA_PIPE = ("sm__pipe_tma_cycles_active.avg.pct_of_peak_sustained_elapsed",
             "sm__pipe_tma_cycles_active.avg.pct_of_peak_sustained_active")
_SM_THROUGHPUT = ("sm__throughput.avg.pct_of_peak_sustained_elapsed",)
_WARPS_ACTIVE = ("sm__warps_active.avg.pct_of_peak_sustained_active",)
_DRAM_PCT = ("dram__throughput.avg.pct_of_peak_sustained_elapsed", "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed")
_LTS_PCT = ("lts__throughput.avg.pct_of_peak_sustained_elapsed",)
_L2_HIT = ("lts__t_sector_hit_rate.pct",)
_COMPUTE_MEM = ("gpu__compute_memory_throughput.avg.pct_of_peak_sustained_elapsed",)
_TC_SMEM = ("l1tex__data_pipe_tc_wavefronts_mem_shared.sum.pct_of_peak_sustained_elapsed",)
_BANK_READS = ("l1tex__data_bank_reads.avg.pct_of_peak_sustained_elapsed",)
_BANK_WRITES = ("l1tex__data_bank_writes.avg.pct_of_peak_sustained_elapsed",)
_DURATION = ("gpu__time_duration.sum", "gpu__time_duration.avg", "gpu__time_duration")

# Issue-stall counters: gb100's per-issue ratios and the sm_86 per-warp percentages.
_STALL_PATTERNS = (
    (re.compile(r"^smsp__average_warps_issue_stalled_(\w+?)_per_issue_active\.ratio$"), "ratio"),
    (re.compile(r"^smsp__warp_issue_stalled_(\w+?)_per_warp_active\.pct$"), "pct"),
)
# Stall reasons that a warp-specialised TMA/tcgen05 kernel shows by design: its producer, MMA
# and epilogue warps sleep on mbarriers (long_scoreboard covers the mbarrier try_wait loop).
_BY_DESIGN_STALLS = {"long_scoreboard", "barrier", "sleeping", "wait", "membar"}

# Speed-of-light rows of a details page (percent of peak): the busiest is the bound.
_SOL_METRICS = {"Compute (SM) Throughput", "Memory Throughput", "DRAM Throughput", "L1/TEX Cache Throughput",
                "L2 Cache Throughput"}

# Blackwell thresholds for the classes (percent of peak).
_TENSOR_TARGET = 85.0     # a healthy sm_100a GEMM mainloop keeps tcgen05 this busy
_DRAM_HIGH = 70.0
_LTS_HIGH = 75.0
_TC_SMEM_HIGH = 85.0
_SHORT_US = 20.0


def _to_float(value: Any) -> Optional[float]:
    """A finite float from a CSV cell ('1,234.5', '87.2%', 'n/a' ...), else None."""
    if value is None:
        return None
    if isinstance(value, (int, float)):
        v = float(value)
        return v if math.isfinite(v) else None
    text = str(value).strip().replace(",", "")
    if text.endswith("%"):
        text = text[:-1]
    if not text or text.lower() in ("n/a", "none", "nan", "-"):
        return None
    try:
        v = float(text)
    except ValueError:
        return None
    return v if math.isfinite(v) else None


def _value(cell: Any) -> Any:
    v = _to_float(cell)
    if v is not None:
        return v
    text = "" if cell is None else str(cell).strip()
    return text or None


def _slug(text: Any) -> str:
    out = re.sub(r"[^0-9a-z]+", "_", str(text or "").lower()).strip("_")
    return out or "unknown"


def _csv_rows(path: Optional[Path]) -> List[List[str]]:
    """Rows of an ncu CSV export, without ncu's '==PROF==' / '==WARNING==' lines."""
    if path is None or not Path(path).exists():
        return []
    lines = [ln for ln in Path(path).read_text(encoding="utf-8", errors="replace").splitlines()
             if ln.strip() and not ln.lstrip().startswith("==")]
    return [[c.strip() for c in row] for row in csv.reader(io.StringIO("\n".join(lines)))]


def _looks_like_units(row: Sequence[str]) -> bool:
    """The row under an ncu raw-page header that holds units ('%', 'byte', 'nsecond', ...)."""
    if not row or any(_to_float(c) is not None for c in row):  # units rows hold no numbers
        return False
    unitish = sum(1 for c in row if c == "" or c in ("%",) or (c.replace("/", "").isalpha() and len(c) <= 16))
    return unitish >= max(3, int(0.6 * len(row)))


def _lookup(record: Optional[Dict[str, Any]], names: Iterable[str]) -> Any:
    """First present, non-empty value among `names` (exact, else a section-qualified
    'SECTION.metric' column ending in the name)."""
    if not record:
        return None
    for name in names:
        if record.get(name) not in (None, ""):
            return _value(record[name])
    for name in names:
        for key, val in record.items():
            if key.endswith("." + name) and val not in (None, ""):
                return _value(val)
    return None


def _rel(path: Optional[Path], base: Optional[Path]) -> Optional[str]:
    if path is None:
        return None
    path = Path(path)
    if base is not None:
        try:
            return path.relative_to(base).as_posix()
        except ValueError:
            pass
    return path.as_posix()


def _cell(row: Dict[str, Any], names: Iterable[str]) -> Optional[str]:
    """Case-insensitive column lookup returning non-empty text."""
    lower = {str(k).strip().lower(): k for k in row}
    for name in names:
        key = lower.get(name.lower())
        if key is not None and str(row.get(key) or "").strip():
            return str(row[key]).strip()
    return None


def parse_wide_csv_records(path: Optional[Path]) -> List[Dict[str, str]]:
    """One dict per launch from a wide raw-page export (`ncu --csv --page raw`, or
    `ncu --import rep --csv --page raw`): header row with 'ID' and 'Kernel Name', an optional
    units row, then one row per launch."""
    rows = _csv_rows(path)
    head = next((i for i, r in enumerate(rows) if "ID" in r and "Kernel Name" in r), None)
    if head is None or "Metric Name" in rows[head]:  # a long export: see long_csv_records
        return []
    header = rows[head]
    body = rows[head + 1:]
    if body and _looks_like_units(body[0]):
        body = body[1:]
    name_col = header.index("Kernel Name")
    return [dict(zip(header, r)) for r in body
            if len(r) == len(header) and r[name_col].strip()]


_BASE_SCALE = {
    "nsecond": ("ns", 1.0), "usecond": ("ns", 1e3), "msecond": ("ns", 1e6), "second": ("ns", 1e9),
    "ns": ("ns", 1.0), "us": ("ns", 1e3), "ms": ("ns", 1e6), "s": ("ns", 1e9),
    "byte": ("byte", 1.0), "kbyte": ("byte", 1e3), "mbyte": ("byte", 1e6), "gbyte": ("byte", 1e9),
    "tbyte": ("byte", 1e12), "kibyte": ("byte", 1024.0), "mibyte": ("byte", 1024.0 ** 2),
    "byte/block": ("byte", 1.0), "kbyte/block": ("byte", 1e3),
}


def units_of(path: Optional[Path]) -> Dict[str, str]:
    """metric -> unit of an ncu export: the units row under a wide header, or the 'Metric Unit'
    column of a long export.  Section-qualified columns are also listed by metric name."""
    rows = _csv_rows(path)
    out: Dict[str, str] = {}
    head = next((i for i, r in enumerate(rows) if "ID" in r and "Kernel Name" in r), None)
    if head is not None and "Metric Name" not in rows[head] and head + 1 < len(rows) \
            and _looks_like_units(rows[head + 1]):
        for name, unit in zip(rows[head], rows[head + 1]):
            out[name] = unit
            if "." in name and "__" in name:
                out.setdefault(name[name.rfind(".", 0, name.find("__")) + 1:], unit)
        return out
    head = next((i for i, r in enumerate(rows) if "Metric Name" in r and "Metric Unit" in r), None)
    if head is not None:
        ni, ui = rows[head].index("Metric Name"), rows[head].index("Metric Unit")
        for r in rows[head + 1:]:
            if len(r) > max(ni, ui) and r[ni]:
                out[r[ni]] = r[ui]
    return out


def _in_base(value: Any, unit: Optional[str], base: str) -> Optional[float]:
    """`value` in `unit` converted to ns or bytes (`base`); a missing unit means base already."""
    v = _to_float(value)
    if v is None:
        return None
    scale = _BASE_SCALE.get((unit or "").strip().lower())
    return v * scale[1] if scale is not None and scale[0] == base else v


def parse_name_value_metrics(path: Optional[Path]) -> Dict[str, Any]:
    """metric -> value from a long export (columns 'Metric Name' and 'Metric Value'); the last
    launch wins when several are listed."""
    rows = _csv_rows(path)
    head = next((i for i, r in enumerate(rows) if "Metric Name" in r and "Metric Value" in r), None)
    if head is None:
        return {}
    ni, vi = rows[head].index("Metric Name"), rows[head].index("Metric Value")
    out: Dict[str, Any] = {}
    for r in rows[head + 1:]:
        if len(r) > max(ni, vi) and r[ni]:
            out[r[ni]] = _value(r[vi])
    return out


def long_csv_records(path: Optional[Path]) -> List[Dict[str, str]]:
    """One dict per launch from a long export (`ncu --metrics ... --csv`): the launch columns
    (ID, Kernel Name, Block Size, Grid Size ...) plus metric -> value."""
    rows = _csv_rows(path)
    head = next((i for i, r in enumerate(rows) if "ID" in r and "Metric Name" in r and "Metric Value" in r), None)
    if head is None:
        return []
    header = rows[head]
    ni, vi = header.index("Metric Name"), header.index("Metric Value")
    fixed = [i for i, h in enumerate(header) if h not in ("Metric Name", "Metric Unit", "Metric Value")]
    launches: Dict[str, Dict[str, str]] = {}
    for r in rows[head + 1:]:
        if len(r) != len(header):
            continue
        rec = launches.setdefault(r[header.index("ID")], {header[i]: r[i] for i in fixed})
        rec[r[ni]] = r[vi]
    return [rec for rec in launches.values() if rec.get("Kernel Name")]


def parse_generic_rows(path: Optional[Path]) -> List[Dict[str, str]]:
    """Rows of a details-page (or source-page) export as dicts, units rows dropped."""
    rows = _csv_rows(path)
    if len(rows) < 2:
        return []
    header = rows[0]
    out = []
    for r in rows[1:]:
        d = {h: (r[i] if i < len(r) else "") for i, h in enumerate(header)}
        if any(d.values()) and not _looks_like_units(list(d.values())):
            out.append(d)
    return out


def source_page_is_disassembly(path: Optional[Path]) -> bool:
    """True when a source-page export holds disassembly (columns Address, Source) instead of
    metric rows correlated with CUDA source lines; such a file is not read further."""
    rows = _csv_rows(path)
    return any(r[:2] == ["Address", "Source"] for r in rows[:3])


def select_primary_record(records: Sequence[Dict[str, str]]) -> Optional[Dict[str, str]]:
    """The dominant launch: the longest (gpu__time_duration, else elapsed cycles), ties broken
    by SM throughput."""
    if not records:
        return None

    def key(rec):
        dur = _lookup(rec, _DURATION + ("sm__cycles_elapsed.sum", "sm__cycles_elapsed.max"))
        thr = _lookup(rec, _SM_THROUGHPUT)
        return (dur if isinstance(dur, float) else 0.0, thr if isinstance(thr, float) else 0.0)

    return max(records, key=key)


def build_launch(headline_record: Optional[Dict[str, Any]], raw_record: Optional[Dict[str, Any]]) -> Dict[str, Any]:
    """Launch shape of the dominant kernel (headline export over the full raw page)."""
    merged: Dict[str, Any] = dict(raw_record or {})
    merged.update(headline_record or {})
    return {
        "kernel_name": _cell(merged, ("Kernel Name", "kernel_name")),
        "block_size": _cell(merged, ("Block Size", "launch__block_size", "block_size")),
        "grid_size": _cell(merged, ("Grid Size", "launch__grid_size", "grid_size")),
        "registers_per_thread": _lookup(merged, ("launch__registers_per_thread",)),
        "shared_mem_per_block_allocated": _lookup(merged, ("launch__shared_mem_per_block_allocated",
                                                           "launch__shared_mem_per_block")),
        "cluster_size": _lookup(merged, ("launch__cluster_dim_x",)),
        "dynamic_shared_mem_per_block": _lookup(merged, ("launch__shared_mem_per_block_dynamic",)),
        "duration_ns": _lookup(merged, _DURATION),
    }


def filter_headline_metrics(record: Optional[Dict[str, Any]], wanted: Sequence[str]) -> Dict[str, Any]:
    return {name: _lookup(record, (name,)) for name in wanted if _lookup(record, (name,)) is not None}


def build_stall_breakdown(record: Optional[Dict[str, Any]]) -> List[Dict[str, Any]]:
    """Issue stalls by reason, largest first.  gb100 reports warps stalled per issued
    instruction; the share of the total is the importance."""
    found: Dict[str, Tuple[str, float]] = {}
    for key, val in (record or {}).items():
        base = key[key.find("smsp__"):] if "smsp__" in key else key  # drop a 'SECTION.' qualifier
        for pattern, _kind in _STALL_PATTERNS:
            m = pattern.match(base)
            v = _to_float(val)
            if m and v is not None and m.group(1) not in found:
                found[m.group(1)] = (base, v)
    total = sum(v for _, v in found.values()) or 1.0
    out = []
    for reason, (metric, v) in found.items():
        share = 100.0 * v / total
        design = reason in _BY_DESIGN_STALLS
        out.append({
            "finding_id": f"stall::{reason}",
            "stall_group": reason,
            "metric_name": metric,
            "metric_value": v,
            "share_pct": round(share, 2),
            "by_design": design,
            "importance_score": round(share * (0.25 if design else 1.0), 4),
            "explanation": (f"{reason.replace('_', ' ')} accounts for {share:.1f}% of issue stalls"
                            + (" (warps of a warp-specialised kernel wait on mbarriers by design)" if design else "")
                            + "."),
        })
    out.sort(key=lambda d: d["importance_score"], reverse=True)
    return out


def build_memory_hierarchy(record: Optional[Dict[str, Any]]) -> Dict[str, Any]:
    rd = _lookup(record, ("dram__bytes_read.sum",))
    wr = _lookup(record, ("dram__bytes_write.sum",))
    return {
        "compute_memory_throughput_pct": _lookup(record, _COMPUTE_MEM),
        "dram_throughput_pct": _lookup(record, _DRAM_PCT),
        "lts_throughput_pct": _lookup(record, _LTS_PCT),
        "l2_hit_rate_pct": _lookup(record, _L2_HIT),
        "l1tex_bank_reads_pct": _lookup(record, _BANK_READS),
        "l1tex_bank_writes_pct": _lookup(record, _BANK_WRITES),
        "tensor_core_smem_reads_pct": _lookup(record, _TC_SMEM),
        "tma_load_bytes": _lookup(record, ("l1tex__m_xbar2l1tex_read_bytes_mem_global_op_tma_ld.sum",
                                           "l1tex__m_xbar2l1tex_read_bytes.sum")),
        "dram_bytes": (rd + wr) if isinstance(rd, float) and isinstance(wr, float) else None,
    }


def build_occupancy_latency(record: Optional[Dict[str, Any]]) -> Dict[str, Any]:
    return {
        "active_warps_pct": _lookup(record, _WARPS_ACTIVE),
        "occupancy_limit_registers": _lookup(record, ("launch__occupancy_limit_registers",)),
        "occupancy_limit_shared_mem": _lookup(record, ("launch__occupancy_limit_shared_mem",)),
        "occupancy_limit_blocks": _lookup(record, ("launch__occupancy_limit_blocks",)),
        "registers_per_thread": _lookup(record, ("launch__registers_per_thread",)),
        "shared_mem_per_block_allocated": _lookup(record, ("launch__shared_mem_per_block_allocated",)),
    }


def build_tensor_core_utilization(record: Optional[Dict[str, Any]]) -> Dict[str, Any]:
    return {
        "tensor_pipe_active_pct": _lookup(record, _TENSOR_PIPE),
        "tensor_pipe_counter": next((n for n in _TENSOR_PIPE if _lookup(record, (n,)) is not None), None),
        "tma_pipe_active_pct": _lookup(record, _TMA_PIPE),
        "sm_throughput_pct": _lookup(record, _SM_THROUGHPUT),
        "active_warps_pct": _lookup(record, _WARPS_ACTIVE),
    }


def row_matches_kernel(row: Dict[str, str], kernel_name: Optional[str]) -> bool:
    other = _cell(row, ("Kernel Name", "kernel_name"))
    return not kernel_name or not other or other == kernel_name


def build_rules(rows: Sequence[Dict[str, str]], kernel_name: Optional[str]) -> List[Dict[str, Any]]:
    """ncu's rule results from the details page (rows with a rule name), most severe first."""
    weight = {"error": 25.0, "warning": 15.0, "optimization": 10.0, "info": 5.0}
    # gb100 details pages carry the rule's kind in 'Rule Type' (WRN, OPT, INF) and its text in
    # 'Rule Description'; other exports name them Severity and Rule Message.
    kinds = {"wrn": "warning", "err": "error", "opt": "optimization", "inf": "info"}
    out = []
    for i, row in enumerate(rows):
        name = _cell(row, ("Rule Name", "Rule", "rule_name"))
        if not name or not row_matches_kernel(row, kernel_name):
            continue
        severity = (_cell(row, ("Severity", "Rule Severity", "severity", "Rule Type")) or "info").lower()
        severity = kinds.get(severity, severity)
        metric = _cell(row, ("Metric Name", "Metric", "metric_name"))
        raw = _cell(row, ("Metric Value", "Value", "metric_value"))
        est = _to_float(_cell(row, ("Estimated Speedup", "Speedup", "estimated_speedup")))
        out.append({
            "rule_id": f"rule::{_slug(name)}::{i}",
            "rule_name": name,
            "severity": severity,
            "section_name": _cell(row, ("Section Name", "Section", "section_name")),
            "metric_name": metric,
            "metric_value": _value(raw),
            "message": _cell(row, ("Rule Message", "Rule Description", "Message", "Description", "Advice")) or name,
            "estimated_speedup_pct": est,
            "location": _cell(row, ("Source Location", "Location")),
            "importance_score": weight.get(severity, 0.0) + (est or 0.0),
        })
    out.sort(key=lambda d: d["importance_score"], reverse=True)
    return out


def build_hotspot_from_row(row: Dict[str, str], *, index: int) -> Optional[Dict[str, Any]]:
    """A hotspot from one details-page or source-page row that names a metric.  Source rows
    carry a CUDA file and line (-lineinfo builds); details rows carry a section."""
    metric = _cell(row, ("Metric Name", "Metric", "metric_name"))
    if not metric:
        return None
    value = _to_float(_cell(row, ("Metric Value", "Value", "metric_value")))
    unit = _cell(row, ("Metric Unit", "Unit", "metric_unit"))
    file_ = _cell(row, ("Source File", "File", "Filename", "File Name", "source_file"))
    line = _cell(row, ("Line", "Line Number", "line"))
    func = _cell(row, ("Function Name", "Function", "Device Function", "function_name"))
    section = _cell(row, ("Section Name", "Section", "section_name"))
    rule = _cell(row, ("Rule Name", "Rule"))
    if file_:
        scope_type, scope_name, location = "cuda_source", func or file_, f"{file_}:{line}" if line else file_
    elif func:
        scope_type, scope_name, location = "device_function", func, func
    else:
        scope_type, scope_name, location = "section", section or "unknown_section", section
        # Of a details page's section rows only ncu's rules and the speed-of-light throughputs
        # point at a bottleneck; occupancy, L1 hit rate or divergence figures describe a
        # warp-specialised TMA kernel's design, not a problem.
        if not rule and metric not in _SOL_METRICS:
            return None
    explicit = _to_float(_cell(row, ("Importance Score", "Importance", "Contribution", "Estimated Speedup")))
    if explicit is not None:
        score = explicit
    elif metric in _SOL_METRICS:
        score = value or 0.0  # the busiest unit is the bound
    elif value is None:
        score = 0.0
    elif (unit or "") == "%":
        # Percent of peak: a low tensor or throughput figure is the problem; a high stall is.
        lowered = metric.lower()
        score = value if "stall" in lowered else max(0.0, 100.0 - value) if any(
            t in lowered for t in ("throughput", "active", "utiliz", "hit rate", "occupancy")) else value
    else:
        score = min(abs(value), 15.0)
    if section:
        score += 5.0
    return {
        "hotspot_id": f"hotspot::{scope_type}::{_slug(scope_name)}::{_slug(location or metric)}::{_slug(metric)}",
        "scope_type": scope_type,
        "scope_name": scope_name,
        "location": location,
        "metric_name": metric,
        "metric_value": value if value is not None else _value(_cell(row, ("Metric Value", "Value"))),
        "metric_unit": unit,
        "importance_score": float(score),
        "explanation": _cell(row, ("Description", "Rule Description", "Rule Message", "Message"))
                       or f"{scope_name}: {metric} = {value if value is not None else 'n/a'}{unit or ''}.",
        "section_name": section,
        "source_row_index": index,
    }


def dedupe_hotspots(hotspots: Sequence[Dict[str, Any]]) -> List[Dict[str, Any]]:
    best: Dict[str, Dict[str, Any]] = {}
    for h in hotspots:
        if h["hotspot_id"] not in best or h["importance_score"] > best[h["hotspot_id"]]["importance_score"]:
            best[h["hotspot_id"]] = h
    return sorted(best.values(), key=lambda h: h["importance_score"], reverse=True)


def _synthetic_hotspots(launch: Dict[str, Any], tensor: Dict[str, Any], memory: Dict[str, Any],
                        stalls: Sequence[Dict[str, Any]]) -> List[Dict[str, Any]]:
    """Hotspots from the headline counters when no page names one: the tcgen05 pipe, the
    operand feed (L2), DRAM and the largest stalls."""
    kernel = launch.get("kernel_name") or "kernel"
    out = []

    def add(scope, section, metric, value, score, text):
        out.append({"hotspot_id": f"hotspot::section::{scope}", "scope_type": "section", "scope_name": scope,
                    "location": kernel, "metric_name": metric, "metric_value": value, "metric_unit": "%",
                    "importance_score": float(score), "explanation": text, "section_name": section})

    tp = tensor.get("tensor_pipe_active_pct")
    if isinstance(tp, float):
        add("tcgen05_pipe", "Compute", tensor.get("tensor_pipe_counter"), tp, max(0.0, 100.0 - tp),
            f"The tcgen05 tensor pipe is active {tp:.1f}% of the time.")
    lts = memory.get("lts_throughput_pct")
    if isinstance(lts, float):
        add("l2_operand_feed", "Memory", _LTS_PCT[0], lts, lts * 0.5,
            f"L2 throughput is {lts:.1f}% of peak (TMA operand loads into shared memory).")
    dram = memory.get("dram_throughput_pct")
    if isinstance(dram, float):
        add("dram_throughput", "Memory", _DRAM_PCT[0], dram, dram * 0.5, f"DRAM throughput is {dram:.1f}% of peak.")
    for st in stalls[:2]:
        add(f"stall_{st['stall_group']}", "Scheduler", st["metric_name"], st["metric_value"],
            st["importance_score"], st["explanation"])
    return dedupe_hotspots(out)


def build_section_highlights(hotspots: Sequence[Dict[str, Any]], rules: Sequence[Dict[str, Any]],
                             stall_breakdown: Sequence[Dict[str, Any]]) -> List[Dict[str, Any]]:
    """The strongest hotspot or rule of each ncu section."""
    by_section: Dict[str, Dict[str, Any]] = {}

    def offer(section, metric, value, score, summary, rule_id=None, hotspot_id=None):
        cur = by_section.setdefault(section, {"section_id": f"section::{_slug(section)}", "section_name": section,
                                              "metric_name": metric, "metric_value": value, "importance_score": -1.0,
                                              "summary": summary, "rule_ids": [], "hotspot_ids": []})
        if rule_id:
            cur["rule_ids"].append(rule_id)
        if hotspot_id:
            cur["hotspot_ids"].append(hotspot_id)
        if score > cur["importance_score"]:
            cur.update(metric_name=metric, metric_value=value, importance_score=score, summary=summary)

    for h in hotspots:
        offer(h.get("section_name") or h.get("scope_name") or "unknown_section", h["metric_name"], h["metric_value"],
              h["importance_score"], h["explanation"], hotspot_id=h["hotspot_id"])
    for r in rules:
        offer(r.get("section_name") or "rule_only", r["metric_name"], r["metric_value"], r["importance_score"],
              r["message"], rule_id=r["rule_id"])
    if stall_breakdown and "Scheduler" not in by_section:
        st = stall_breakdown[0]
        offer("Scheduler", st["metric_name"], st["metric_value"], st["importance_score"], st["explanation"])
    return sorted(by_section.values(), key=lambda d: d["importance_score"], reverse=True)


def _evidence(kind: str, ref_id: str, metric: Any, value: Any, summary: str) -> Dict[str, Any]:
    return {"kind": kind, "ref_id": ref_id, "metric_name": metric, "metric_value": value, "summary": summary}


def classify_bottlenecks(launch: Dict[str, Any], stall_breakdown: Sequence[Dict[str, Any]],
                         memory_hierarchy: Dict[str, Any], occupancy_latency: Dict[str, Any],
                         tensor_core_utilization: Dict[str, Any], rules: Sequence[Dict[str, Any]],
                         section_highlights: Sequence[Dict[str, Any]],
                         hotspots: Sequence[Dict[str, Any]]) -> List[Dict[str, Any]]:
    """The reference's bottleneck classes (class ids kept for its consumers), scored with
    Blackwell thresholds for a persistent, warp-specialised tcgen05 GEMM, plus one class of
    its own: l2_operand_feed_bound (TMA operand loads limited by the L2 -> SM feed)."""
    classes: List[Dict[str, Any]] = []

    def add(class_id, score, summary, evidence):
        if score > 0 and evidence:
            classes.append({"class_id": class_id, "severity_score": round(float(score), 4), "summary": summary,
                            "evidence": evidence})

    tp = tensor_core_utilization.get("tensor_pipe_active_pct")
    tp = tp if isinstance(tp, float) else None
    dram = memory_hierarchy.get("dram_throughput_pct")
    lts = memory_hierarchy.get("lts_throughput_pct")
    tc_smem = memory_hierarchy.get("tensor_core_smem_reads_pct")
    warps = occupancy_latency.get("active_warps_pct")
    dur_ns = launch.get("duration_ns")
    stalls = {s["stall_group"]: s for s in stall_breakdown}
    tensor_gap = max(0.0, _TENSOR_TARGET - tp) if tp is not None else 0.0
    counter = tensor_core_utilization.get("tensor_pipe_counter") or _TENSOR_PIPE[0]

    if tp is not None and tensor_gap > 0:
        add("tensor_core_underutilization", tensor_gap,
            f"The tcgen05 pipe is active {tp:.1f}% of the time, below the {_TENSOR_TARGET:.0f}% a "
            "persistent sm_100a GEMM mainloop sustains.",
            [_evidence("headline_metric", f"metric::{counter}", counter, tp,
                       f"tcgen05 pipe active {tp:.1f}%.")]
            + ([_evidence("source_hotspot", hotspots[0]["hotspot_id"], hotspots[0]["metric_name"],
                          hotspots[0]["metric_value"], hotspots[0]["explanation"])] if hotspots else []))
    if isinstance(lts, float) and lts > _LTS_HIGH:
        add("l2_operand_feed_bound", (lts - _LTS_HIGH) + 0.5 * tensor_gap,
            f"L2 throughput {lts:.1f}% of peak: the TMA operand loads are near the L2 -> SM feed limit.",
            [_evidence("headline_metric", f"metric::{_LTS_PCT[0]}", _LTS_PCT[0], lts, f"L2 throughput {lts:.1f}%.")])
    mem_score, mem_ev = 0.0, []
    if isinstance(dram, float) and dram > _DRAM_HIGH:
        mem_score += dram - _DRAM_HIGH
        mem_ev.append(_evidence("headline_metric", f"metric::{_DRAM_PCT[0]}", _DRAM_PCT[0], dram,
                                f"DRAM throughput {dram:.1f}% of peak."))
    # A rule about memory only counts when DRAM or L2 is busy enough to matter.
    memory_busy = (isinstance(dram, float) and dram > 50.0) or (isinstance(lts, float) and lts > _LTS_HIGH)
    if memory_busy and any("memory" in (r.get("message") or "").lower() for r in rules[:5]) and rules:
        mem_score += 5.0
        mem_ev.append(_evidence("rule", rules[0]["rule_id"], rules[0].get("metric_name") or rules[0]["rule_name"],
                                rules[0].get("metric_value"), rules[0]["message"]))
    add("global_memory_bound", mem_score, "DRAM throughput is high: the launch is bound by HBM traffic.", mem_ev)
    if isinstance(tc_smem, float) and tc_smem > _TC_SMEM_HIGH:
        add("shared_memory_bottleneck", tc_smem - _TC_SMEM_HIGH,
            f"The tensor core reads shared memory at {tc_smem:.1f}% of peak.",
            [_evidence("headline_metric", f"metric::{_TC_SMEM[0]}", _TC_SMEM[0], tc_smem,
                       f"tensor-core shared-memory reads {tc_smem:.1f}%.")])
    # One CTA per SM is the design of a persistent warp-specialised kernel, so occupancy limits
    # are not findings; few active warps only matter when the tensor pipe is idle too.
    if isinstance(warps, float) and warps < 10.0 and tensor_gap > 20.0:
        add("occupancy_latency_hiding_issue", (10.0 - warps) + 0.25 * tensor_gap,
            f"Only {warps:.1f}% of warp slots are active while the tensor pipe idles.",
            [_evidence("headline_metric", f"metric::{_WARPS_ACTIVE[0]}", _WARPS_ACTIVE[0], warps,
                       f"active warps {warps:.1f}%.")])
    bar = stalls.get("barrier")
    if bar is not None and tensor_gap > 0:
        add("synchronization_barrier_issue", bar["share_pct"] * tensor_gap / 100.0,
            "Barrier stalls coincide with an under-used tensor pipe: hand-offs between the warp roles "
            "may be on the critical path.",
            [_evidence("stall_breakdown", bar["finding_id"], bar["metric_name"], bar["metric_value"], bar["explanation"])])
    if isinstance(dur_ns, float) and dur_ns < _SHORT_US * 1e3:
        add("tail_overhead_or_generic_path_issue", (_SHORT_US * 1e3 - dur_ns) / 1e3,
            f"The launch lasts {dur_ns / 1e3:.1f} us: prologue, first loads and the store tail weigh on it.",
            [_evidence("launch", "launch::duration", _DURATION[0], dur_ns, f"{dur_ns / 1e3:.1f} us per launch.")])
    classes.sort(key=lambda c: c["severity_score"], reverse=True)
    for rank, c in enumerate(classes, start=1):
        c["rank"] = rank
    return classes


def _direction(metric: str) -> str:
    lowered = (metric or "").lower()
    if any(t in lowered for t in ("stall", "conflict", "bank", "replay", "bytes", "duration", "throttle", "scoreboard")):
        return "lower_better"
    if any(t in lowered for t in ("active", "throughput", "hit_rate", "occupancy", "utiliz", "ipc")):
        return "higher_better"
    return "lower_better"


def _trend(metric: str, prev: Optional[float], cur: Optional[float]) -> Tuple[Optional[float], str]:
    if prev is None or cur is None:
        return None, "unknown"
    d = cur - prev
    if abs(d) < 1e-9:
        return d, "flat"
    better = d > 0 if _direction(metric) == "higher_better" else d < 0
    return d, "improved" if better else "regressed"


def compute_delta_vs_previous_run(previous: Optional[Dict[str, Any]], current: Dict[str, Any]) -> Dict[str, Any]:
    """Headline, stall and hotspot changes against a previous analysis (reference :1269)."""
    empty = {"baseline_run_id": None, "headline_metrics": {}, "stall_breakdown": [],
             "source_hotspots": {"improved": [], "regressed": [], "new": [], "disappeared": []}}
    if not previous:
        return empty
    head = {}
    ph, ch = previous.get("headline_metrics") or {}, current.get("headline_metrics") or {}
    for name in sorted(set(ph) | set(ch)):
        d, t = _trend(name, _to_float(ph.get(name)), _to_float(ch.get(name)))
        head[name] = {"previous": ph.get(name), "current": ch.get(name), "delta": d, "trend": t}
    prev_stalls = {s["stall_group"]: s for s in previous.get("stall_breakdown") or []}
    stalls = []
    for s in current.get("stall_breakdown") or []:
        pv = _to_float((prev_stalls.get(s["stall_group"]) or {}).get("metric_value"))
        d, t = _trend(s["metric_name"], pv, _to_float(s["metric_value"]))
        stalls.append({"stall_group": s["stall_group"], "metric_name": s["metric_name"], "previous": pv,
                       "current": s["metric_value"], "delta": d, "trend": t})
    stalls.sort(key=lambda x: abs(x["delta"] or 0.0), reverse=True)
    prev_h = {h["hotspot_id"]: h for h in previous.get("source_hotspots") or []}
    cur_h = {h["hotspot_id"]: h for h in current.get("source_hotspots") or []}
    buckets: Dict[str, List[Dict[str, Any]]] = {"improved": [], "regressed": [], "new": [], "disappeared": []}
    for hid, h in cur_h.items():
        if hid not in prev_h:
            buckets["new"].append(dict(h, trend="new"))
            continue
        p = prev_h[hid]
        d, t = _trend(h["metric_name"], _to_float(p.get("metric_value")), _to_float(h.get("metric_value")))
        entry = {k: h.get(k) for k in ("hotspot_id", "scope_type", "scope_name", "location", "metric_name", "explanation")}
        entry.update(previous=_to_float(p.get("metric_value")), current=_to_float(h.get("metric_value")), delta=d,
                     trend=t, importance_score=max(h.get("importance_score") or 0.0, p.get("importance_score") or 0.0))
        if t in ("improved", "regressed"):
            buckets[t].append(entry)
    for hid, p in prev_h.items():
        if hid not in cur_h:
            buckets["disappeared"].append(dict(p, trend="disappeared"))
    for b in buckets.values():
        b.sort(key=lambda x: abs(_to_float(x.get("delta")) or x.get("importance_score") or 0.0), reverse=True)
        del b[TOP_HOTSPOTS:]
    return {"baseline_run_id": previous.get("source_run_id"), "headline_metrics": head, "stall_breakdown": stalls,
            "source_hotspots": buckets}


def _delta_items(delta: Dict[str, Any]) -> List[Dict[str, Any]]:
    items = []
    for bucket in ("regressed", "new", "improved", "disappeared"):
        for it in (delta.get("source_hotspots") or {}).get(bucket, []):
            items.append(dict(it, bucket=bucket))
    items.sort(key=lambda x: abs(_to_float(x.get("delta")) or 0.0) + min(x.get("importance_score") or 0.0, 25.0),
               reverse=True)
    return items[:TOP_HOTSPOTS]


def build_node_b_handoff(bottlenecks: Sequence[Dict[str, Any]], hotspots: Sequence[Dict[str, Any]],
                         rules: Sequence[Dict[str, Any]], delta_summary: Dict[str, Any]) -> Dict[str, Any]:
    """What the diagnosis step reads: the top findings and the code regions to look at."""
    findings = [{"finding_id": f"finding::{c['class_id']}", "finding_type": "bottleneck_class", "summary": c["summary"],
                 "importance_score": c["severity_score"], "evidence": c["evidence"]} for c in bottlenecks[:4]]
    findings += [{"finding_id": f"finding::{h['hotspot_id']}", "finding_type": "source_hotspot",
                  "summary": h["explanation"], "importance_score": h["importance_score"],
                  "evidence": [_evidence("source_hotspot", h["hotspot_id"], h["metric_name"], h["metric_value"],
                                         h["explanation"])]} for h in hotspots[:2]]
    findings += [{"finding_id": f"finding::delta::{d.get('hotspot_id')}", "finding_type": "hotspot_delta",
                  "summary": f"{d['bucket']} hotspot at {d.get('scope_name') or d.get('location')}: "
                             f"{d.get('trend', 'changed')}.",
                  "importance_score": abs(_to_float(d.get("delta")) or 0.0) + min(d.get("importance_score") or 0.0, 25.0),
                  "evidence": [d]} for d in _delta_items(delta_summary)[:2]]
    seen, top = set(), []
    for f in sorted(findings, key=lambda x: x["importance_score"] or 0.0, reverse=True):
        if f["finding_id"] not in seen:
            seen.add(f["finding_id"])
            top.append(f)
    regions, keys = [], set()
    for h in hotspots[:TOP_HOTSPOTS]:
        key = str(h.get("location") or h.get("scope_name"))
        if key not in keys:
            keys.add(key)
            regions.append({"region_id": h["hotspot_id"], "scope_type": h["scope_type"], "scope_name": h["scope_name"],
                            "location": h.get("location"), "reason": h["explanation"]})
    for r in rules[:3]:
        key = str(r.get("location") or r["rule_name"])
        if key not in keys:
            keys.add(key)
            regions.append({"region_id": r["rule_id"], "scope_type": "rule", "scope_name": r["rule_name"],
                            "location": r.get("location"), "reason": r["message"]})
    return {"top_findings": top[:TOP_FINDINGS], "code_regions_to_investigate": regions[:TOP_HOTSPOTS]}


def build_node_c_handoff(headline_metrics: Dict[str, Any], bottlenecks: Sequence[Dict[str, Any]],
                         hotspots: Sequence[Dict[str, Any]], stall_breakdown: Sequence[Dict[str, Any]],
                         delta_summary: Dict[str, Any], tensor_core_utilization: Optional[Dict[str, Any]] = None,
                         memory_hierarchy: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """What the implementation step checks after its edit: target hotspots, metrics that must
    not regress (the tcgen05 pipe must not drop; DRAM bytes must not grow) and recheck points."""
    guard = []
    tc = tensor_core_utilization or {}
    if isinstance(tc.get("tensor_pipe_active_pct"), float):
        guard.append({"metric_name": tc.get("tensor_pipe_counter"), "current_value": tc["tensor_pipe_active_pct"],
                      "guardrail": "non_decreasing",
                      "reason": "The tcgen05 pipe's activity is the kernel's throughput; an edit must not lower it."})
    mem = memory_hierarchy or {}
    if isinstance(mem.get("dram_bytes"), float):
        guard.append({"metric_name": "dram__bytes_read.sum + dram__bytes_write.sum", "current_value": mem["dram_bytes"],
                      "guardrail": "non_increasing",
                      "reason": "DRAM traffic above the algorithmic bytes is operand re-reads; it must not grow."})
    for name, value in headline_metrics.items():
        if len(guard) >= 3:
            break
        if isinstance(value, float) and _direction(name) == "higher_better" and name not in [g["metric_name"] for g in guard]:
            guard.append({"metric_name": name, "current_value": value, "guardrail": "non_decreasing",
                          "reason": "Headline throughput metric of the current run."})
    for st in stall_breakdown[:1]:
        guard.append({"metric_name": st["metric_name"], "current_value": st["metric_value"],
                      "guardrail": "non_increasing", "reason": st["explanation"]})
    recheck = [{"scope_type": h["scope_type"], "scope_name": h["scope_name"], "location": h.get("location"),
                "metric_name": h["metric_name"], "reason": h["explanation"]} for h in hotspots[:4]]
    recheck += [{"scope_type": d.get("scope_type"), "scope_name": d.get("scope_name"), "location": d.get("location"),
                 "metric_name": d.get("metric_name"),
                 "reason": f"The previous run saw it {d.get('trend', 'changed')} ({d['bucket']})."}
                for d in _delta_items(delta_summary)[:2]]
    return {"target_hotspots": list(hotspots[:TOP_HOTSPOTS]), "guardrail_metrics": guard[:4],
            "expected_recheck_points": recheck[:TOP_HOTSPOTS]}


def _artifact(kind: str, path: Optional[Path], base: Path, missing: str, rc: Optional[int],
              reason: Optional[str] = None, best_effort: bool = False, alias: Optional[Path] = None) -> Dict[str, Any]:
    entry = {"artifact_kind": kind, "path": _rel(path, base),
             "status": "available" if path is not None and Path(path).exists() else missing,
             "return_code": rc, "best_effort": best_effort}
    if reason:
        entry["unavailable_reason"] = reason
    if alias is not None:
        entry["legacy_alias_path"] = _rel(alias, base)
    return entry


def analyze_run(*, run_dir: Path, source_run_id: str, headline_csv_path: Optional[Path],
                import_raw_path: Optional[Path], details_page_path: Optional[Path],
                source_csv_path: Optional[Path], rep_path: Optional[Path],
                wanted_headline_metrics: Sequence[str], previous_analysis_path: Optional[Path] = None,
                source_unavailable_reason: Optional[str] = None, details_unavailable_reason: Optional[str] = None,
                import_raw_unavailable_reason: Optional[str] = None, legacy_import_raw_alias: Optional[Path] = None,
                return_codes: Optional[Dict[str, Optional[int]]] = None) -> Dict[str, Any]:
    """The reference's analyze_run (scripts/ncu_analysis.py:1450) on gb100 exports: same
    keyword arguments, same schema (version 2), Blackwell reading of the counters."""
    run_dir = Path(run_dir)
    rcs = return_codes or {}
    head_records = parse_wide_csv_records(headline_csv_path) or long_csv_records(headline_csv_path)
    raw_records = parse_wide_csv_records(import_raw_path) or long_csv_records(import_raw_path)
    head_kv = parse_name_value_metrics(headline_csv_path)
    primary_head = select_primary_record(head_records)
    primary_raw = select_primary_record(raw_records)
    # The long (name/value) export has no per-launch header: treat it as one record.
    if primary_head is None and head_kv:
        primary_head = dict(head_kv)
    merged: Dict[str, Any] = dict(primary_raw or {})
    merged.update(primary_head or {})
    launch = build_launch(primary_head, primary_raw)
    kernel = launch.get("kernel_name")

    headline = filter_headline_metrics(merged, wanted_headline_metrics)
    details = [r for r in parse_generic_rows(details_page_path) if row_matches_kernel(r, kernel)]
    disassembly = source_page_is_disassembly(source_csv_path)
    source_rows = [] if disassembly else [r for r in parse_generic_rows(source_csv_path) if row_matches_kernel(r, kernel)]
    source_rows = [r for r in source_rows if _cell(r, ("Metric Name", "Metric"))]
    if source_csv_path is not None and Path(source_csv_path).exists() and not source_rows:
        source_unavailable_reason = source_unavailable_reason or (
            "source page holds disassembly only; hotspots come from the details page and the headline counters"
            if disassembly else "source page has no metric rows for the dominant kernel")

    stalls = build_stall_breakdown(merged)
    memory = build_memory_hierarchy(merged)
    occupancy = build_occupancy_latency(merged)
    tensor = build_tensor_core_utilization(merged)
    # Exports state sizes and times in display units (usecond, Mbyte, Kbyte/block ...): the
    # derived fields are put in ns and bytes so that the classes compare like with like.
    units = units_of(import_raw_path)
    units.update(units_of(headline_csv_path))

    def base_of(names, base):
        for name in names:
            val = _lookup(merged, (name,))
            if val is not None:
                return _in_base(val, units.get(name), base)
        return None

    launch["duration_ns"] = base_of(_DURATION, "ns")
    for key, names in (("shared_mem_per_block_allocated", ("launch__shared_mem_per_block_allocated",
                                                           "launch__shared_mem_per_block")),
                       ("dynamic_shared_mem_per_block", ("launch__shared_mem_per_block_dynamic",))):
        launch[key] = base_of(names, "byte")
    occupancy["shared_mem_per_block_allocated"] = launch["shared_mem_per_block_allocated"]
    rd = base_of(("dram__bytes_read.sum",), "byte")
    wr = base_of(("dram__bytes_write.sum",), "byte")
    memory["dram_bytes"] = rd + wr if rd is not None and wr is not None else None
    memory["tma_load_bytes"] = base_of(("l1tex__m_xbar2l1tex_read_bytes_mem_global_op_tma_ld.sum",
                                        "l1tex__m_xbar2l1tex_read_bytes.sum"), "byte")
    rules = build_rules(details, kernel)
    rows = source_rows or details
    hotspots = dedupe_hotspots([h for i, r in enumerate(rows) for h in [build_hotspot_from_row(r, index=i)] if h])
    if not source_rows:
        # Without source lines, the headline counters (tcgen05 pipe, L2 feed, DRAM, stalls) are
        # hotspots too, next to whatever the details page offers.
        hotspots = dedupe_hotspots(hotspots + _synthetic_hotspots(launch, tensor, memory, stalls))
    highlights = build_section_highlights(hotspots, rules, stalls)
    base = run_dir.parent
    artifacts = {
        "ncu_rep": _artifact("report", rep_path, base, "missing", rcs.get("rep")),
        "headline_csv": _artifact("headline_raw_page", headline_csv_path, base, "missing", rcs.get("headline_csv")),
        "import_raw_page": _artifact("import_raw_page", import_raw_path, base, "unavailable", rcs.get("import_raw"),
                                     import_raw_unavailable_reason, alias=legacy_import_raw_alias),
        "details_page": _artifact("details_page", details_page_path, base, "unavailable", rcs.get("details_page"),
                                  details_unavailable_reason),
        "source_page": _artifact("source_page", source_csv_path, base, "unavailable", rcs.get("source_page"),
                                 source_unavailable_reason, best_effort=True),
    }
    artifacts["source_page"]["structured_hotspots_available"] = bool(source_rows)
    analysis: Dict[str, Any] = {
        "schema_version": HANDOFF_SCHEMA_VERSION,
        "architecture": "gb100 (sm_100a): tcgen05 tensor pipe, TMA, TMEM",
        "status": "available" if (primary_head or primary_raw) else "missing",
        "source_run_id": source_run_id,
        "source_run_dir": _rel(run_dir, base),
        "launch": launch,
        "headline_metrics": headline,
        "stall_breakdown": stalls,
        "memory_hierarchy": memory,
        "occupancy_latency": occupancy,
        "tensor_core_utilization": tensor,
        "rules": rules,
        "section_highlights": highlights,
        "source_hotspots": hotspots[:TOP_HOTSPOTS],
        "artifacts": artifacts,
    }
    previous = None
    if previous_analysis_path is not None and Path(previous_analysis_path).exists():
        previous = json.loads(Path(previous_analysis_path).read_text(encoding="utf-8"))
    classes = classify_bottlenecks(launch, stalls, memory, occupancy, tensor, rules, highlights, hotspots)
    analysis["bottleneck_classes"] = classes
    analysis["delta_vs_previous_run"] = compute_delta_vs_previous_run(previous, analysis)
    analysis["handoff"] = {
        "node_b": build_node_b_handoff(classes, hotspots, rules, analysis["delta_vs_previous_run"]),
        "node_c": build_node_c_handoff(headline, classes, hotspots, stalls, analysis["delta_vs_previous_run"],
                                       tensor, memory),
    }
    return analysis


def render_analysis_md(analysis: Dict[str, Any]) -> str:
    """ncu_analysis.md next to ncu_analysis.json."""
    la = analysis.get("launch") or {}
    tc = analysis.get("tensor_core_utilization") or {}
    mem = analysis.get("memory_hierarchy") or {}
    out = ["# NCU analysis (gb100)", "",
           f"- schema version: `{analysis.get('schema_version')}`", f"- status: `{analysis.get('status')}`",
           f"- source run id: `{analysis.get('source_run_id')}`", "", "## Launch", ""]
    for key in ("kernel_name", "block_size", "grid_size", "cluster_size", "registers_per_thread",
                "shared_mem_per_block_allocated", "duration_ns"):
        out.append(f"- {key.replace('_', ' ')}: `{la.get(key)}`")
    out += ["", "## Tensor core and memory", "",
            f"- tcgen05 pipe active: `{tc.get('tensor_pipe_active_pct')}` ({tc.get('tensor_pipe_counter')})",
            f"- TMA pipe active: `{tc.get('tma_pipe_active_pct')}`",
            f"- L2 throughput: `{mem.get('lts_throughput_pct')}`, hit rate `{mem.get('l2_hit_rate_pct')}`",
            f"- DRAM throughput: `{mem.get('dram_throughput_pct')}`, bytes `{mem.get('dram_bytes')}`",
            "", "## Headline metrics", ""]
    out += [f"- `{k}`: `{v}`" for k, v in (analysis.get("headline_metrics") or {}).items()] or ["- none"]
    out += ["", "## Bottleneck classes", ""]
    out += [f"{c['rank']}. `{c['class_id']}` ({c['severity_score']}): {c['summary']}"
            for c in analysis.get("bottleneck_classes") or []] or ["- none"]
    out += ["", "## Stall breakdown", ""]
    out += [f"- `{s['stall_group']}` {s['share_pct']}%{' (by design)' if s['by_design'] else ''}"
            for s in (analysis.get("stall_breakdown") or [])[:6]] or ["- none"]
    out += ["", "## Top hotspots", ""]
    out += [f"- `{h['scope_name']}` @ `{h.get('location')}`: {h['explanation']}"
            for h in analysis.get("source_hotspots") or []] or ["- none"]
    delta = analysis.get("delta_vs_previous_run") or {}
    out += ["", "## Delta vs previous run", "", f"- baseline: `{delta.get('baseline_run_id')}`"]
    for name, d in list((delta.get("headline_metrics") or {}).items())[:8]:
        out.append(f"- `{name}`: {d.get('previous')} -> {d.get('current')} ({d.get('trend')})")
    node_b = (analysis.get("handoff") or {}).get("node_b") or {}
    out += ["", "## Handoff to node_b", ""]
    out += [f"- {f['finding_type']}: {f['summary']}" for f in node_b.get("top_findings") or []] or ["- none"]
    node_c = (analysis.get("handoff") or {}).get("node_c") or {}
    out += ["", "## Handoff to node_c", ""]
    out += [f"- guardrail `{g['metric_name']}` {g['guardrail']} (now {g['current_value']})"
            for g in node_c.get("guardrail_metrics") or []] or ["- none"]
    return "\n".join(out) + "\n"


def build_rich_summary_from_analysis(analysis: Dict[str, Any]) -> Dict[str, Any]:
    """The compact ncu summary eval_kernel.py stores in its run directory (reference :1683)."""
    la = analysis.get("launch") or {}
    art = analysis.get("artifacts") or {}
    delta = analysis.get("delta_vs_previous_run") or {}
    node_b = (analysis.get("handoff") or {}).get("node_b") or {}
    node_c = (analysis.get("handoff") or {}).get("node_c") or {}
    head_delta = sorted((delta.get("headline_metrics") or {}).items(),
                        key=lambda kv: abs((kv[1] or {}).get("delta") or 0.0), reverse=True)[:8]
    raw = art.get("import_raw_page") or {}
    return {
        "schema_version": HANDOFF_SCHEMA_VERSION,
        "status": analysis.get("status", "missing"),
        "source_run_id": analysis.get("source_run_id"),
        "source_run_dir": analysis.get("source_run_dir"),
        "analysis_path": None,
        "kernel_name": la.get("kernel_name"),
        "block_size": la.get("block_size"),
        "grid_size": la.get("grid_size"),
        "registers_per_thread": la.get("registers_per_thread"),
        "shared_mem_per_block_allocated": la.get("shared_mem_per_block_allocated"),
        "launch": la,
        "headline_metrics": analysis.get("headline_metrics") or {},
        "tensor_core_utilization": analysis.get("tensor_core_utilization") or {},
        "stall_breakdown": list((analysis.get("stall_breakdown") or [])[:6]),
        "bottleneck_classes": [{k: c.get(k) for k in ("class_id", "rank", "severity_score", "summary")}
                               | {"evidence": (c.get("evidence") or [])[:3]}
                               for c in (analysis.get("bottleneck_classes") or [])[:6]],
        "top_findings": list((node_b.get("top_findings") or [])[:TOP_FINDINGS]),
        "top_source_hotspots": list((analysis.get("source_hotspots") or [])[:TOP_HOTSPOTS]),
        "delta_vs_previous_run": {
            "baseline_run_id": delta.get("baseline_run_id"),
            "headline_metrics": dict(head_delta),
            "stall_breakdown": list((delta.get("stall_breakdown") or [])[:6]),
            "source_hotspots": {k: list(((delta.get("source_hotspots") or {}).get(k) or [])[:4])
                                for k in ("improved", "regressed", "new", "disappeared")},
        },
        "handoff": {
            "node_b": {"top_findings": list((node_b.get("top_findings") or [])[:TOP_FINDINGS]),
                       "code_regions_to_investigate": list((node_b.get("code_regions_to_investigate") or [])[:TOP_HOTSPOTS])},
            "node_c": {"target_hotspots": list((node_c.get("target_hotspots") or [])[:TOP_HOTSPOTS]),
                       "guardrail_metrics": list((node_c.get("guardrail_metrics") or [])[:6]),
                       "expected_recheck_points": list((node_c.get("expected_recheck_points") or [])[:TOP_HOTSPOTS])},
        },
        "raw_csv_path": (art.get("headline_csv") or {}).get("path"),
        "raw_rep_path": (art.get("ncu_rep") or {}).get("path"),
        "raw_details_csv_path": raw.get("legacy_alias_path") or raw.get("path"),
        "import_raw_csv_path": raw.get("path"),
        "details_page_csv_path": (art.get("details_page") or {}).get("path"),
        "source_csv_path": (art.get("source_page") or {}).get("path"),
        "artifacts": art,
    }


def write_analysis_outputs(*, run_dir: Path, analysis: Dict[str, Any]) -> Tuple[Path, Path]:
    """Writes ncu_analysis.json and ncu_analysis.md into the run directory (reference :1734)."""
    run_dir = Path(run_dir)
    json_path, md_path = run_dir / "ncu_analysis.json", run_dir / "ncu_analysis.md"
    json_path.write_text(json.dumps(analysis, indent=2) + "\n", encoding="utf-8")
    md_path.write_text(render_analysis_md(analysis), encoding="utf-8")
    return json_path, md_path


def _reference_cli(argv: Sequence[str]) -> None:
    """The reference's command line (scripts/ncu_analysis.py:1746-1781)."""
    ap = argparse.ArgumentParser(description="Normalise gb100 Nsight Compute exports into the analysis schema")
    ap.add_argument("--run-dir", type=Path, required=True)
    ap.add_argument("--source-run-id", required=True)
    for flag in ("--headline-csv", "--import-raw-csv", "--details-page-csv", "--source-csv", "--rep-path",
                 "--legacy-import-raw-alias", "--previous-analysis"):
        ap.add_argument(flag, type=Path, default=None)
    ap.add_argument("--headline-metric", action="append", default=[])
    for flag in ("--source-unavailable-reason", "--details-unavailable-reason", "--import-raw-unavailable-reason"):
        ap.add_argument(flag, default=None)
    a = ap.parse_args(argv)
    analysis = analyze_run(run_dir=a.run_dir, source_run_id=a.source_run_id, headline_csv_path=a.headline_csv,
                           import_raw_path=a.import_raw_csv, details_page_path=a.details_page_csv,
                           source_csv_path=a.source_csv, rep_path=a.rep_path, wanted_headline_metrics=a.headline_metric,
                           previous_analysis_path=a.previous_analysis,
                           source_unavailable_reason=a.source_unavailable_reason,
                           details_unavailable_reason=a.details_unavailable_reason,
                           import_raw_unavailable_reason=a.import_raw_unavailable_reason,
                           legacy_import_raw_alias=a.legacy_import_raw_alias)
    write_analysis_outputs(run_dir=a.run_dir, analysis=analysis)


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
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--run-dir" in argv:
        _reference_cli(argv)
        return
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
