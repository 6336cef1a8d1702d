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


EVAL_KERNEL_POLICY = {"benchmark_case": "case_00_seed_3407",
                      "correctness_cases": ["case_00_seed_3407", "case_01_seed_9713", "case_02_seed_1729"],
                      "warmup": 10, "iters": 30, "flush_cache_mb": 256}


def eval_kernel_argv(exe, dataset_dir, case, mode, json_out):
    """The runner command scripts/eval_kernel.py builds (run_runner :316-340): correctness runs
    with warm-up 0 and 1 iteration, the perf run with the config's 10 and 30, flush 256 MiB."""
    warmup, iters = (0, 1) if mode == "correctness" else (EVAL_KERNEL_POLICY["warmup"], EVAL_KERNEL_POLICY["iters"])
    return [str(exe), "--dataset-dir", str(dataset_dir), "--case-id", case, "--mode", mode,
            "--warmup", str(warmup), "--iters", str(iters),
            "--flush-cache-mb", str(EVAL_KERNEL_POLICY["flush_cache_mb"]), "--json-out", str(json_out)]


def test_hero_dataset_through_eval_kernel_invocations(cuda_device, tmp_path):
    """custom_runner on the hero dataset (configs/fixed_bf16_gemm_v1.json, the reference's three
    seeds) exactly as scripts/eval_kernel.py invokes it: every correctness case passes the
    reference's rule and the perf run reports its timing.  With MO_EVK_RECORD=<dir> the JSON files
    and argv are kept, so that tests/golden/eval_kernel_hero can replay them through the reference's
    own eval_kernel.py on a machine that has the reference tree."""
    import os
    import shutil

    from matmul_optimizer_b200.dataset import CONFIG_DIR, load_config

    config = load_config(CONFIG_DIR / "fixed_bf16_gemm_v1.json")
    dataset_dir = Path(generate(config, tmp_path / "datasets")["dataset_dir"])
    record = os.environ.get("MO_EVK_RECORD")
    runs = [(case, "correctness") for case in EVAL_KERNEL_POLICY["correctness_cases"]]
    runs.append((EVAL_KERNEL_POLICY["benchmark_case"], "perf"))
    for case, mode in runs:
        out = tmp_path / f"{mode}_{case}.json"
        argv = eval_kernel_argv(nbuild.RUNNER_PATH, dataset_dir, case, mode, out)
        proc = subprocess.run(argv, capture_output=True, text=True, timeout=600)
        assert proc.returncode == 0, proc.stderr
        res = json.loads(out.read_text())
        assert res["mode"] == mode and res["passed"] is True, res
        if mode == "correctness":
            assert res["correctness"]["atol"] == 0.15 and res["correctness"]["rtol"] == 0.01
        else:
            assert 0 < res["runtime_ms"]["median"] < 2.0 and res["tflops"] > 400
        if record:
            Path(record).mkdir(parents=True, exist_ok=True)
            shutil.copy(out, Path(record) / out.name)
            flags = argv[1:]
            for path_flag in ("--dataset-dir", "--json-out"):  # machine paths are not part of the record
                flags[flags.index(path_flag) + 1] = "<" + path_flag[2:] + ">"
            (Path(record) / f"{mode}_{case}.argv.json").write_text(json.dumps(flags) + "\n")
