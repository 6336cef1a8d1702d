"""bench.py's reference arm (the reference's CPU path, no GPU needed) keeps the one-line JSON
contract: rank 0 prints exactly one line with the keys the driver reads, and any other rank
exits 0 without work or output."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def run_bench(extra_env, *args):
    env = dict(os.environ, **extra_env)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_json_line():
    proc = run_bench({"OPENBLAS_NUM_THREADS": "4"}, "--workload", "cube1000", "--steps", "2",
                     "--warmup", "1")
    assert proc.returncode == 0, proc.stderr
    lines = [l for l in proc.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, proc.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in line, key
    assert line["steps"] == 2 and line["warmup"] == 1 and line["value"] > 0
    assert line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "1000x1000x1000" in line["config"]["workload"]


def test_reference_arm_other_ranks_do_nothing():
    proc = run_bench({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--gpus", "2",
                     "--steps", "2", "--warmup", "1")
    assert proc.returncode == 0, proc.stderr
    assert proc.stdout.strip() == ""


def test_roofline_traffic_comes_from_committed_profiles():
    """Every shape with a committed ncu summary yields roofline.traffic: DRAM read + write bytes
    per launch, at least the launch's compulsory C write."""
    sys.path.insert(0, str(ROOT))
    import bench

    for shape, path in bench.TRAFFIC_SUMMARIES.items():
        assert path.is_file(), path
        m, n, _ = shape
        traffic = bench.traffic_per_launch(shape)
        assert traffic is not None and traffic >= 2 * m * n, (shape, traffic)
    assert bench.traffic_per_launch((7, 7, 7)) is None


def test_reference_arm_lifts_torchrun_thread_limit_and_matches_config():
    """Under torchrun (OMP_NUM_THREADS=1 per rank) rank 0 still runs the reference's CPU path on
    every host thread it may use, over the whole product, and prints the GPU arm's config."""
    proc = run_bench({"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0", "OMP_NUM_THREADS": "1",
                      "OPENBLAS_NUM_THREADS": "1"},
                     "--gpus", "2", "--workload", "cube1000", "--steps", "2", "--warmup", "1")
    assert proc.returncode == 0, proc.stderr
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    sys.path.insert(0, str(ROOT))
    import bench

    bench.set_workload("cube1000")
    assert line["config"] == bench.bench_config(2, bench.partition(1000, 2))
    assert line["config"]["slab_n"] == [512, 488]
    assert "whole 1000x1000x1000 product" in line["cpu_baseline"]["sample"]
