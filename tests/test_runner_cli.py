"""Runner executables fail the way the reference runner does (error JSON + exit code 1,
src/runner/main.cpp:541-550) on host-side errors; none of these reach a CUDA call."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from matmul_optimizer_b200 import build as nbuild

ROOT = Path(__file__).resolve().parent.parent

RUNNERS = [nbuild.RUNNER_PATH, nbuild.CUBLAS_RUNNER_PATH]


@pytest.mark.parametrize("exe", RUNNERS, ids=["custom", "cublas"])
def test_missing_case_gives_error_json(exe, tmp_path):
    assert exe.exists(), "build the runners first (python -m matmul_optimizer_b200.build)"
    out = tmp_path / "r.json"
    proc = subprocess.run([str(exe), "--dataset-dir", str(tmp_path), "--case-id", "nope",
                           "--mode", "perf", "--json-out", str(out)], capture_output=True, text=True)
    assert proc.returncode == 1
    res = json.loads(out.read_text())
    assert res == {"mode": "perf", "passed": False, "error": res["error"]}
    assert "case directory not found" in res["error"] and "[runner-error]" in proc.stderr


@pytest.mark.parametrize("args,msg", [
    (["--mode", "fast"], "unsupported --mode value"),
    (["--iters", "0"], "--iters must be > 0"),
    (["--warmup", "x"], "invalid integer"),
    (["--bogus"], "unknown argument"),
    (["--gpus", "0"], "--gpus must be in 1..64"),
])
def test_bad_arguments(args, msg, tmp_path):
    proc = subprocess.run([str(nbuild.RUNNER_PATH), "--dataset-dir", str(tmp_path), "--case-id", "c", *args],
                          capture_output=True, text=True)
    assert proc.returncode == 1 and msg in proc.stderr


def test_missing_required_flags():
    proc = subprocess.run([str(nbuild.RUNNER_PATH)], capture_output=True, text=True)
    assert proc.returncode == 1 and "--dataset-dir is required" in proc.stderr


def test_reference_eval_kernel_accepts_recorded_custom_runner_outputs(tmp_path, reference_root):
    """The reference's own scripts/eval_kernel.py, unmodified, run against custom_runner's outputs
    recorded on a B200 for the hero dataset (tests/golden/eval_kernel_hero, replayed with the argv
    check of replay_runner.py): three correctness cases pass and the perf run is reported."""
    ref = reference_root
    golden = Path(__file__).resolve().parent / "golden" / "eval_kernel_hero"
    (tmp_path / "datasets" / "fixed_bf16_gemm_v1").mkdir(parents=True)
    cmd = [sys.executable, str(ref / "scripts" / "eval_kernel.py"), "--runner", str(golden / "replay_runner.py"),
           "--kernel-tag", "mo_sm100", "--config", str(ROOT / "matmul_optimizer_b200" / "configs" / "fixed_bf16_gemm_v1.json"),
           "--dataset-root", str(tmp_path / "datasets"), "--runs-root", str(tmp_path / "runs"), "--skip-ncu"]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert proc.returncode == 0, proc.stderr
    (run_dir,) = list((tmp_path / "runs").iterdir())
    summary = json.loads((run_dir / "summary.json").read_text())
    assert [r["case_id"] for r in summary["correctness_runs"]] == [
        "case_00_seed_3407", "case_01_seed_9713", "case_02_seed_1729"]
    assert all(r["passed"] is True for r in summary["correctness_runs"]), summary["correctness_runs"]
    perf = summary["perf_run"]
    assert perf["passed"] is True and perf["mode"] == "perf" and perf["tflops"] > 400
    assert (run_dir / "summary.md").exists()
