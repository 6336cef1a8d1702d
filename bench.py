#!/usr/bin/env python3
"""Benchmark of the fixed BF16 GEMM (6464x7776x7232) on 1..N B200s; prints ONE JSON line.

One step = one C = A·B of the hero shape; with N GPUs the step is the
N-sharded GEMM: rank r computes the column slab r of C (A replicated, B slab contiguous on its
own GPU, width roundup16(ceil(7776/N))), no data-path collective.  Inputs are the reference's
seeded inputs (uniform [-1,1) -> BF16, seed 3407), generated on the host.

Timing (device, CUDA events on the launching stream, max over ranks):
  * W warm-up steps, then exactly K timed steps bracketed by barrier + synchronize;
  * L2 flushed before every step by a 256 MiB memset outside the per-step events (the
    reference protocol, src/runner/main.cpp:508-535); ms_per_step = mean of the K step events;
  * value = whole-job TFLOP/s = 2·M·N·K / ms_per_step (all ranks together);
  * e2e = the same metric through the C ABI from pinned HOST buffers (mo_gemm_from_host): H2D
    of A and the B slab, the GEMM, D2H of the C slab, all inside the per-step events; the
    library overlaps the copies with the GEMM in row bands;
  * roofline: the GEMM kernel's achieved TFLOP/s against MEASURED_PEAKS.json's burst cuBLAS
    BF16 figure; traffic from the committed ncu summary in profiles/;
  * clocks sampled by NVML every 2 ms during the timed region.

  * cublas: torch.matmul (cuBLAS) on the same slab, timed INTERLEAVED with this library's
    kernel (flush, ours, flush, cuBLAS, ... each launch bracketed by its own events), so both
    legs meet the same power and clock state;
  * workloads (N = 1 only, after the headline legs): the other BASELINE configs (square 8192,
    the LLM projection, the ragged M sweep, the 1000^3 cube) and the hero's 2/4/8-GPU column
    slabs, each with its own interleaved cuBLAS time and roofline fraction.

--impl reference runs the reference's CPU path (numpy float32 ``A_q @ B_q`` over all of A,
scripts/generate_fixed_bf16_dataset.py:122) on rank 0 with every host thread it may use (the
thread limit torchrun sets is lifted), on the same config as this arm.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M, N, K = 6464, 7776, 7232
SEED = 3407
METRIC = "TFLOP/s & ms, 6464x7776x7232 BF16 GEMM at 1/2/4/8 B200; % of tensor peak"
UNIFORM = {"name": "uniform", "low": -1.0, "high": 1.0}
DIST = UNIFORM
WORKLOAD = "fixed_bf16_gemm_v1"
# --workload: the hero shape is the default and the headline line; the other BASELINE configs
# are measured the same way when asked for (parity is their tests' job).
WORKLOADS = {
    "hero": (6464, 7776, 7232, UNIFORM, "fixed_bf16_gemm_v1"),
    "square8192": (8192, 8192, 8192, UNIFORM, "square_bf16_gemm_8192"),
    "llm": (4096, 28672, 8192, {"name": "normal", "std_a": 1.0, "std_b": 0.02, "seed_b": 9713},
            "llm_mlp_bf16_gemm_4096x28672x8192"),
    "m1": (1, 7776, 7232, UNIFORM, "ragged_bf16_gemm_m1"),
    "m16": (16, 7776, 7232, UNIFORM, "ragged_bf16_gemm_m16"),
    "m129": (129, 7776, 7232, UNIFORM, "ragged_bf16_gemm_m129"),
    "m1000": (1000, 7776, 7232, UNIFORM, "ragged_bf16_gemm_m1000"),
    "m3333": (3333, 7776, 7232, UNIFORM, "ragged_bf16_gemm_m3333"),
    "cube1000": (1000, 1000, 1000, UNIFORM, "cube_bf16_gemm_1000"),
    # One GPU's column slab of the hero at 2, 4 and 8 GPUs.
    "hero_slab2": (6464, 3888, 7232, UNIFORM, "fixed_bf16_gemm_v1 column slab at 2 GPUs"),
    "hero_slab4": (6464, 1952, 7232, UNIFORM, "fixed_bf16_gemm_v1 column slab at 4 GPUs"),
    "hero_slab8": (6464, 976, 7232, UNIFORM, "fixed_bf16_gemm_v1 column slab at 8 GPUs"),
}
# Measured after the headline legs of a 1-GPU run (the `workloads` object of the line).
SIDE_WORKLOADS = ["square8192", "llm", "m1", "m16", "m129", "m1000", "m3333", "cube1000",
                  "hero_slab2", "hero_slab4", "hero_slab8"]


def data_label() -> str:
    """The `data` field: how the current workload's inputs are drawn."""
    if DIST["name"] == "uniform":
        return f"synthetic: reference generator inputs (uniform [-1,1) -> bf16, seed {SEED})"
    return (f"synthetic: A ~ N(0, {DIST['std_a']}^2) seed {SEED}, B ~ N(0, {DIST['std_b']}^2) "
            f"seed {DIST['seed_b']}, both rounded to bf16")


def set_workload(name: str) -> None:
    global M, N, K, DIST, WORKLOAD, METRIC
    M, N, K, DIST, WORKLOAD = WORKLOADS[name]
    if name != "hero":
        METRIC = f"TFLOP/s & ms, {M}x{N}x{K} BF16 GEMM at 1/2/4/8 B200; % of roofline"
FLUSH_BYTES = 256 << 20
FALLBACK_PEAK_TFLOPS = 1590.0
# Committed ncu summaries, keyed by the per-GPU kernel shape (m, n, k), whose
# `dram_bytes_per_launch` line gives roofline.traffic.
TRAFFIC_SUMMARIES = {
    (6464, 7776, 7232): ROOT / "profiles" / "ncu_gemm_bf16_sm100_hero_6464x7776x7232.md",
    (16, 7776, 7232): ROOT / "profiles" / "ncu_gemm_bf16_sm100_m16_16x7776x7232.md",
    (129, 7776, 7232): ROOT / "profiles" / "ncu_gemm_bf16_sm100_m129_129x7776x7232.md",
    (6464, 976, 7232): ROOT / "profiles" / "ncu_gemm_bf16_sm100_hero_slab8_6464x976x7232.md",
    (6464, 3888, 7232): ROOT / "profiles" / "ncu_gemm_bf16_sm100_hero_slab2_6464x3888x7232.md",
    (6464, 1952, 7232): ROOT / "profiles" / "ncu_gemm_bf16_sm100_hero_slab4_6464x1952x7232.md",
}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["mo", "reference"], default="mo")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="hero",
                    help="BASELINE config to measure (default: the hero shape of the metric)")
    ap.add_argument("--no-workloads", action="store_true",
                    help="skip the other BASELINE configs measured after the headline (N = 1)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ----------------------------------------------------------------------------------------
# CPU legs (reference arm and cpu_baseline): the oracle restatement of the reference's CPU path
# ----------------------------------------------------------------------------------------
def host_threads() -> int:
    """Host threads this process may run on (its CPU affinity)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - not Linux
        return os.cpu_count() or 1


def use_all_host_threads() -> None:
    """Lets BLAS use every host thread of this process.  torchrun sets OMP_NUM_THREADS=1 for
    each rank; the CPU legs run on rank 0 alone, so they lift that limit (before numpy loads
    OpenBLAS, and again through threadpoolctl if it is loaded already)."""
    n = str(host_threads())
    for var in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = n
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=int(n), user_api="blas")
    except Exception:
        pass


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        info = [p for p in threadpool_info() if p.get("user_api") == "blas"]
        if info:
            return int(info[0]["num_threads"])
    except Exception:
        pass
    return os.cpu_count() or 1


def bench_config(world: int, widths) -> dict:
    """The workload of a bench line; both arms print the same dict."""
    return {"workload": f"{WORKLOAD} {M}x{N}x{K}" + (f", N-sharded x{world}" if world > 1 else ""),
            "m": M, "n": N, "k": K, "slab_n": list(widths),
            "l2": "flushed: 256 MiB memset before every step (GPU arm); "
                  "CPU arm: operands far larger than the host caches"}


def partition(n: int, g: int):
    """Column slabs of the N-shard (mo_shard_partition's arithmetic, for the CPU arm, which
    must not load the GPU library): w = roundup16(ceil(n / g))."""
    w = ((n + g - 1) // g + 15) // 16 * 16
    return [max(0, min(w, n - i * w)) for i in range(g)]


def cpu_reference_steps(steps: int, warmup: int, rows: int, min_seconds: float = 0.0):
    """Times numpy float32 A_q[rows] @ B_q on the host; returns per-step seconds and flops.
    Runs `steps` timed products, and more (up to 200) until they add up to `min_seconds`."""
    import numpy as np

    from oracle import bf16_oracle as orc

    if DIST["name"] == "uniform":
        case = orc.make_uniform_case(M, N, K, SEED)
    else:
        case = orc.make_normal_case(M, N, K, SEED, DIST["seed_b"], DIST["std_a"], DIST["std_b"])
    a = np.ascontiguousarray(orc.bf16_bits_to_float32(case.a_bits[:rows]))
    b = np.ascontiguousarray(orc.bf16_bits_to_float32(case.b_bits))
    times = []
    i = 0
    while i < warmup + steps or (sum(times) < min_seconds and len(times) < 200):
        t0 = time.perf_counter()
        c = a @ b
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
        del c
        i += 1
    return times, 2.0 * rows * N * K


def cpu_rows_for_budget(seconds_per_step: float) -> int:
    """Row band sized from a quick probe so one step takes about `seconds_per_step`."""
    import numpy as np

    probe_rows = 256
    a = np.random.default_rng(0).random((probe_rows, K), dtype=np.float32)
    b = np.random.default_rng(1).random((K, N), dtype=np.float32)
    a @ b
    t0 = time.perf_counter()
    a @ b
    dt = max(time.perf_counter() - t0, 1e-4)
    return int(max(64, min(M, probe_rows * seconds_per_step / dt)) // 64 * 64)


def run_reference_arm(args, rank: int, world: int) -> None:
    """The reference's own CPU path for this GEMM: numpy float32 ``A_q @ B_q`` over the whole
    problem (scripts/generate_fixed_bf16_dataset.py:122), every step the full M x N x K product,
    on every host thread.  Under torchrun rank 0 alone runs it."""
    if rank != 0:
        return
    use_all_host_threads()
    times, flops = cpu_reference_steps(args.steps, max(args.warmup, 1), M)
    mean_s = statistics.fmean(times)
    value = flops / mean_s / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(mean_s * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": data_label(),
        "config": bench_config(world, partition(N, world)),
        "path": "numpy float32 A_q @ B_q (scripts/generate_fixed_bf16_dataset.py:122), all of A per step",
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": blas_threads(),
                         "kind": "port", "sample": f"the whole {M}x{N}x{K} product per step, "
                                                   f"{args.steps} timed steps"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------
# Clocks (NVML, read-only)
# ----------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
        0x10: "sync_boost", 0x1: "gpu_idle",
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons = [], set()
        self.period = period_s
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _loop(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._loop, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst cuBLAS)"
    except Exception:
        return FALLBACK_PEAK_TFLOPS, "fallback (1.59 PFLOP/s)"


def measured_hbm():
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy)"
    except Exception:
        return 6650.0, "fallback (6.65 TB/s)"


def traffic_per_launch(shape):
    """DRAM bytes (read + write) per launch of the kernel on `shape` from its committed ncu
    summary, or None when there is none."""
    path = TRAFFIC_SUMMARIES.get(tuple(shape))
    if path is None:
        return None
    try:
        text = path.read_text()
    except OSError:
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", text)
    return float(m.group(1)) if m else None


# ----------------------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------------------
def interleaved_ms(torch, fn_a, fn_b, flush, stream, iters: int, dev, warmup: int = 3):
    """Mean device time of fn_a and fn_b launched alternately on `stream`, the L2 flushed
    before every launch, each launch between its own CUDA events."""
    for i in range(warmup):
        flush.fill_(i & 0xFF)
        fn_a()
        flush.fill_((i + 1) & 0xFF)
        fn_b()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(iters)]
    torch.cuda.synchronize(dev)
    for i in range(iters):
        flush.fill_((2 * i + 11) & 0xFF)
        ev[i][0].record(stream)
        fn_a()
        ev[i][1].record(stream)
        flush.fill_((2 * i + 12) & 0xFF)
        ev[i][2].record(stream)
        fn_b()
        ev[i][3].record(stream)
    torch.cuda.synchronize(dev)
    ms_a = statistics.fmean(e[0].elapsed_time(e[1]) for e in ev)
    ms_b = statistics.fmean(e[2].elapsed_time(e[3]) for e in ev)
    return ms_a, ms_b


def measure_workloads(torch, mo, dev, stream, flush, peak_tflops: float, hbm_gbs: float,
                      iters: int = 10) -> dict:
    """The other BASELINE configs on this GPU, each with the reference's seeded inputs: this
    library's kernel and cuBLAS (torch.matmul) interleaved, flush before every launch."""
    from matmul_optimizer_b200.dataset import draw_inputs

    out = {}
    for name in SIDE_WORKLOADS:
        m, n, k, dist, label = WORKLOADS[name]
        a_bits, b_bits = draw_inputs(m, n, k, SEED, dist)
        a = torch.from_numpy(a_bits.view("int16")).to(dev)
        b = torch.from_numpy(b_bits.view("int16")).to(dev)
        c = torch.empty((m, n), dtype=torch.int16, device=dev)
        del a_bits, b_bits

        def ours():
            rc = mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, stream)
            if rc != mo.MO_OK:
                raise RuntimeError(f"GEMM {name} failed: {mo.error_string(rc)}")

        a_bf, b_bf = a.view(torch.bfloat16), b.view(torch.bfloat16)
        ms, cb_ms = interleaved_ms(torch, ours, lambda: torch.matmul(a_bf, b_bf), flush, stream, iters, dev)
        flops = 2.0 * m * n * k
        nbytes = 2.0 * (m * k + k * n + m * n)
        tflops = flops / (ms * 1e-3) / 1e12
        hbm_bound = flops / nbytes < peak_tflops * 1e12 / (hbm_gbs * 1e9)
        plan = mo.select_plan(m, n, k, torch.cuda.get_device_properties(dev).multi_processor_count)
        out[name] = {
            "shape": [m, n, k], "config": label, "ms": round(ms, 4), "tflops": round(tflops, 2),
            "roofline": ({"bound": "hbm", "frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm_gbs, 4)} if hbm_bound
                         else {"bound": "tensor", "frac": round(tflops / peak_tflops, 4)}),
            "cublas_ms": round(cb_ms, 4), "mo_over_cublas": round(ms / cb_ms, 4),
            "plan": f"{plan['block_m']}x{plan['block_n']} cta_group::{plan['cta_group']}"
                    + (" stream-K" if plan["stream_k"] else "") + (" K-split" if plan["split"] else ""),
        }
        del a, b, c, a_bf, b_bf
        torch.cuda.empty_cache()
    watchdog = mo.read_watchdog(clear=True)
    if watchdog != 0:
        raise RuntimeError(f"device watchdog flag {watchdog} set during the workloads")
    return out


def run_mo(args, rank: int, world: int, local: int) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    import matmul_optimizer_b200 as mo
    from matmul_optimizer_b200.dataset import draw_inputs

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    mo.load_library()
    a_bits, b_bits = draw_inputs(M, N, K, SEED, DIST)
    begins, widths = mo.shard_partition(N, world)
    n0, ns = begins[rank], widths[rank]
    b_slab_bits = np.ascontiguousarray(b_bits[:, n0:n0 + ns])
    del b_bits

    stream = torch.cuda.current_stream(dev)
    a_h = torch.from_numpy(a_bits.view(np.int16)).pin_memory()
    b_h = torch.from_numpy(b_slab_bits.view(np.int16)).pin_memory()
    c_h = torch.empty((M, ns), dtype=torch.int16).pin_memory()
    a = a_h.to(dev)
    b = b_h.to(dev)
    c = torch.empty((M, ns), dtype=torch.int16, device=dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def gemm():
        rc = mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, ns, K, stream)
        if rc != mo.MO_OK:
            raise RuntimeError(f"GEMM launch failed: {mo.error_string(rc)}")

    # ---- warm-up
    for i in range(max(args.warmup, 3)):
        flush.fill_(i & 0xFF)
        gemm()
    torch.cuda.synchronize(dev)

    # ---- timed region: device-timed GEMM steps, L2 flushed between steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local)
    with sampler:
        for i in range(args.steps):
            flush.fill_((i + 7) & 0xFF)
            starts[i].record(stream)
            gemm()
            stops[i].record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, stops)]
    mean_ms = max_over_ranks(statistics.fmean(step_ms))
    median_ms = max_over_ranks(statistics.median(step_ms))
    flops_total = 2.0 * M * N * K
    value = flops_total / (mean_ms * 1e-3) / 1e12

    # ---- e2e through the C ABI from pinned host buffers.  One GPU: mo_gemm_from_host uploads A
    # and B, runs the GEMM and downloads C, the copies overlapped with slab GEMMs.  N GPUs: each
    # rank holds its row shard of A and its column slab of B in host memory; the shard goes up,
    # A is all-gathered over NVLink, then B's slab goes up and C's slab comes down around the
    # slab GEMMs (sharding.gemm_sharded_from_host).
    if world > 1:
        from matmul_optimizer_b200 import sharding

        r0, r1, shard_rows = sharding.row_shard(M, world, rank)
        a_rows_h = torch.zeros((shard_rows, K), dtype=torch.int16).pin_memory()
        a_rows_h[: r1 - r0].copy_(a_h[r0:r1])
        a_shard_d = torch.empty((shard_rows, K), dtype=torch.int16, device=dev)
        a_full_d = torch.empty((shard_rows * world, K), dtype=torch.int16, device=dev)
        h2d_step = (shard_rows * K + K * ns) * 2
    else:
        h2d_step = (M * K + K * ns) * 2
    d2h_step = M * ns * 2

    def gemm_host():
        if world > 1:
            rc = sharding.gemm_sharded_from_host(a_rows_h, a_shard_d, a_full_d, b_h, c_h, M, K, ns, stream)
        else:
            rc = mo.gemm_from_host(a_h.data_ptr(), b_h.data_ptr(), c_h.data_ptr(), M, ns, K, 0, stream)
        if rc != mo.MO_OK:
            raise RuntimeError(f"host-buffer GEMM failed: {mo.error_string(rc)}")

    e2e_steps = min(args.steps, 20)
    e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(e2e_steps)]
    e_stops = [torch.cuda.Event(enable_timing=True) for _ in range(e2e_steps)]
    for i in range(2):
        gemm_host()
    barrier()
    torch.cuda.synchronize(dev)
    for i in range(e2e_steps):
        e_starts[i].record(stream)
        gemm_host()
        e_stops[i].record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(statistics.fmean(s.elapsed_time(e) for s, e in zip(e_starts, e_stops)))
    e2e_value = flops_total / (e2e_ms * 1e-3) / 1e12
    # The last D2H copy is the step's result: it must equal the device result.
    if not torch.equal(c_h, c.cpu()):
        raise RuntimeError("e2e result mismatch between host copy and device buffer")

    # ---- same-box cuBLAS BF16 (torch.matmul) on the same slab, timed interleaved with this
    # library's kernel: flush, ours, flush, cuBLAS, ...; each launch between its own events.
    a_bf = a.view(torch.bfloat16)
    b_bf = b.view(torch.bfloat16)
    inter_mo_ms, cublas_ms = interleaved_ms(torch, gemm, lambda: torch.matmul(a_bf, b_bf), flush,
                                            stream, args.steps, dev)
    inter_mo_ms = max_over_ranks(inter_mo_ms)
    cublas_ms = max_over_ranks(cublas_ms)

    # ---- optional all-gather of C (N > 1), outside the timed region
    allgather = None
    if world > 1:
        w = widths[0]
        # NCCL has no 16-bit integer type; the BF16 view moves the same bytes.
        send = torch.zeros((M * w,), dtype=torch.bfloat16, device=dev)
        send[: M * ns].copy_(c.view(torch.bfloat16).view(-1))
        gathered = torch.empty((world * M * w,), dtype=torch.bfloat16, device=dev)
        full = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        times = []
        for i in range(6):
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            dist.all_gather_into_tensor(gathered, send)
            mo.unshard_columns(gathered.data_ptr(), full.data_ptr(), M, widths, M * w, stream)
            s1.record(stream)
            torch.cuda.synchronize(dev)
            if i >= 2:
                times.append(s0.elapsed_time(s1))
        allgather = {"ms": round(max_over_ranks(statistics.fmean(times)), 4),
                     "bytes_per_rank_received": (world - 1) * M * w * 2,
                     "how": "torch.distributed all_gather_into_tensor (NCCL) + mo_unshard_columns"}

    # Whole-job copy volume of the e2e step (every rank takes part in both reductions).
    h2d_total = int(sum_over_ranks(h2d_step))
    d2h_total = int(sum_over_ranks(d2h_step))

    watchdog = mo.read_watchdog(clear=True)
    if watchdog != 0:
        raise RuntimeError(f"device watchdog flag {watchdog} set during the benchmark")

    # ---- per-GPU roofline of the GEMM kernel
    peak, peak_src = measured_peak()
    kernel_flops = 2.0 * M * ns * K
    kernel_bytes = 2.0 * (M * K + K * ns + M * ns)
    kernel_ms = statistics.fmean(step_ms)
    kernel_ms_max = max_over_ranks(kernel_ms)
    achieved = kernel_flops / (kernel_ms_max * 1e-3) / 1e12
    hbm_peak, hbm_src = measured_hbm()
    # Ridge point: below peak_flops / peak_bytes FLOP per byte the kernel is HBM-bound.
    hbm_bound = kernel_flops / kernel_bytes < peak * 1e12 / (hbm_peak * 1e9)
    plan = mo.select_plan(M, ns, K, torch.cuda.get_device_properties(dev).multi_processor_count)
    kernel = (f"mo_sm100 {plan['block_m']}x{plan['block_n']}x{plan['block_k']} "
              f"cta_group::{plan['cta_group']} stages={plan['stages']} grid={plan['grid']}"
              + (" stream-K" if plan["stream_k"] else "") + (" K-split" if plan["split"] else ""))
    if os.environ.get("MATMUL_FIXED_MAIN_TILE_N") and (M, ns, K) == (6464, 7776, 7232):
        kernel += f" (MATMUL_FIXED_MAIN_TILE_N={os.environ['MATMUL_FIXED_MAIN_TILE_N']}: plan not shown)"
    clocks = sampler.summary()

    workloads = None
    if world == 1 and not args.no_workloads and WORKLOAD == WORKLOADS["hero"][4]:
        workloads = measure_workloads(torch, mo, dev, stream, flush, peak, hbm_peak)

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        use_all_host_threads()
        times, flops = cpu_reference_steps(3, 1, M, min_seconds=args.cpu_seconds)
        cpu_value = flops / statistics.fmean(times) / 1e12
        cpu_baseline = {"value": round(cpu_value, 4), "unit": "TFLOP/s", "cores": blas_threads(),
                        "kind": "port",
                        "sample": f"numpy float32 A_q @ B_q over all of A (generator.py:122), "
                                  f"{len(times)} runs, {sum(times):.1f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(mean_ms, 4),
            "ms_median": round(median_ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": data_label(),
            "config": bench_config(world, widths),
            "kernel": kernel,
            "tflops_per_gpu": round(achieved, 3),
            "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": h2d_total, "d2h_bytes_per_step": d2h_total,
                    "h2d_bytes_per_step_per_rank": h2d_step, "d2h_bytes_per_step_per_rank": d2h_step,
                    "path": ("mo_gemm_from_host (C ABI): pinned host A, B, C; uploads, slab GEMMs and downloads overlapped"
                             if world == 1 else
                             "per rank: pinned host A row shard + B slab + C slab; shard up, A all-gathered over NVLink "
                             "(NCCL), then mo_gemm_b_from_host (B slab up, slab GEMMs, C slab down, overlapped)")},
            "roofline": ({"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                          "frac": round(achieved / peak, 4), "peak_source": peak_src,
                          "traffic": traffic_per_launch((M, ns, K)),
                          "algorithmic_flops_per_launch": kernel_flops}
                         if not hbm_bound else
                         {"bound": "hbm", "achieved": round(kernel_bytes / (kernel_ms_max * 1e-3) / 1e9, 1),
                          "peak": hbm_peak, "unit": "GB/s",
                          "frac": round(kernel_bytes / (kernel_ms_max * 1e-3) / 1e9 / hbm_peak, 4),
                          "peak_source": hbm_src, "traffic": traffic_per_launch((M, ns, K)),
                          "algorithmic_bytes_per_launch": kernel_bytes}),
            "cublas": {"ms": round(cublas_ms, 4), "tflops": round(flops_total / (cublas_ms * 1e-3) / 1e12, 3),
                       "mo_ms_interleaved": round(inter_mo_ms, 4),
                       "mo_over_cublas": round(inter_mo_ms / cublas_ms, 4),
                       "how": "torch.matmul bf16 (cuBLAS) on the same slab, interleaved launch by launch "
                              "with this library's kernel (flush before each), max over ranks"},
            "cpu_baseline": cpu_baseline,
            "gpu_launches": args.steps * world,
            "gpu_launches_per_rank": args.steps,
            "clocks": clocks,
        }
        if allgather is not None:
            line["allgather"] = allgather
        if workloads is not None:
            line["workloads"] = workloads
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    set_workload(args.workload)
    rank, world, local = dist_env()
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        raise SystemExit(f"--gpus {args.gpus} does not match WORLD_SIZE {world}")
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.gpus > 1 and "WORLD_SIZE" not in os.environ:
        raise SystemExit("for --gpus N > 1 launch with torch.distributed.run (one process per GPU)")
    run_mo(args, rank, world, local)


if __name__ == "__main__":
    main()
