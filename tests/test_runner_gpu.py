"""The runner executables keep the reference runner's CLI/JSON contract
(src/runner/main.cpp:119-155, :373-418) on a real GPU: correctness and perf modes for
custom_runner (libmo_gemm.so) and cublas_runner (cuBLASLt)."""

import json
import subprocess
from pathlib import Path

import pytest

from matmul_optimizer_b200 import build as nbuild
from matmul_optimizer_b200.dataset import generate

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_dataset(tmp_path_factory):
    root = tmp_path_factory.mktemp("datasets")
    config = {
        "dataset_id": "small_bf16_gemm", "description": "runner test",
        "gemm": {"m": 259, "n": 392, "k": 520},
        "distribution": {"name": "uniform", "low": -1.0, "high": 1.0},
        "correctness_policy": {"initial_rtol": 0.01, "initial_atol": 0.15},
        "cases": [{"case_id": "case_00_seed_3407", "seed": 3407}, {"case_id": "case_01_seed_9713", "seed": 9713}],
    }
    return Path(generate(config, root)["dataset_dir"])


def run_runner(exe, dataset_dir, case, mode, tmp_path, extra=()):
    out = tmp_path / f"{Path(exe).name}_{mode}_{case}.json"
    cmd = [str(exe), "--dataset-dir", str(dataset_dir), "--case-id", case, "--mode", mode,
           "--warmup", "2", "--iters", "5", "--flush-cache-mb", "256", "--json-out", str(out), *extra]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    return proc.returncode, json.loads(out.read_text()), proc.stderr


@pytest.mark.parametrize("exe", [nbuild.RUNNER_PATH, nbuild.CUBLAS_RUNNER_PATH], ids=["custom", "cublas"])
def test_runner_correctness_and_perf(cuda_device, small_dataset, tmp_path, exe):
    for case in ("case_00_seed_3407", "case_01_seed_9713"):
        rc, res, err = run_runner(exe, small_dataset, case, "correctness", tmp_path)
        assert rc == 0, err
        assert res["mode"] == "correctness" and res["passed"] is True
        corr = res["correctness"]
        assert set(corr) >= {"max_abs_err", "max_rel_err", "mean_abs_err", "bf16_exact_match", "atol", "rtol"}
        assert corr["atol"] == 0.15 and corr["rtol"] == 0.01
    rc, res, err = run_runner(exe, small_dataset, "case_00_seed_3407", "perf", tmp_path)
    assert rc == 0, err
    assert res["passed"] is True and res["runtime_ms"]["median"] > 0 and res["tflops"] > 0
    assert res["runtime_ms"]["p10"] <= res["runtime_ms"]["median"] <= res["runtime_ms"]["p90"]


def test_runner_reports_failure_json(cuda_device, small_dataset, tmp_path):
    rc, res, _ = run_runner(nbuild.RUNNER_PATH, small_dataset, "no_such_case", "correctness", tmp_path)
    assert rc == 1 and res["passed"] is False and "case directory not found" in res["error"]
