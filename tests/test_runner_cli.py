"""Runner executables fail the way the reference runner does (error JSON + exit code 1,
src/runner/main.cpp:541-550) on host-side errors; none of these reach a CUDA call."""

import json
import subprocess

import pytest

from matmul_optimizer_b200 import build as nbuild

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
