"""The committed integration patches (matmul_optimizer_b200/integration/) apply to a copy of the
reference's tree and do what INTEGRATION.md says: scripts/graph.py's build step configures for
sm_100a and hands the library location to CMake (graph.py:550-570), and the reference's
CMakeLists.txt then builds its own runner (src/runner/main.cpp) linked against libmo_gemm.so
instead of compiling src/kernels.  Runs on a machine with the reference checkout; the copy lives
in a temporary directory, nothing of the reference enters this repository."""

import py_compile
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PATCHES = ROOT / "matmul_optimizer_b200" / "integration"


@pytest.fixture()
def patched_tree(tmp_path, reference_root):
    tree = tmp_path / "ref"
    (tree / "scripts").mkdir(parents=True)
    (tree / "src").mkdir()
    shutil.copy(reference_root / "scripts" / "graph.py", tree / "scripts" / "graph.py")
    shutil.copy(reference_root / "CMakeLists.txt", tree / "CMakeLists.txt")
    shutil.copytree(reference_root / "src" / "runner", tree / "src" / "runner")
    shutil.copytree(reference_root / "include", tree / "include")
    for patch in sorted(PATCHES.glob("*.patch")):
        proc = subprocess.run(["patch", "-p1", "--forward", "-i", str(patch)], cwd=tree, capture_output=True, text=True)
        assert proc.returncode == 0, (patch.name, proc.stdout, proc.stderr)
    return tree


def test_graph_build_step_configures_sm100a(patched_tree):
    graph = patched_tree / "scripts" / "graph.py"
    py_compile.compile(str(graph), doraise=True)
    text = graph.read_text()
    assert "'-DCMAKE_CUDA_ARCHITECTURES=100a'" in text
    assert "-DMO_GEMM_ROOT=" in text and "libmo_gemm.so" in text


def test_reference_runner_builds_against_libmo_gemm(patched_tree, tmp_path):
    """cmake + the reference's runner source + this library: the executable links libmo_gemm.so,
    holds none of the reference's kernels, and answers a missing case with the reference's error
    JSON and exit code 1 (src/runner/main.cpp:541-550) without touching a GPU."""
    build = patched_tree / "build"
    cfg = subprocess.run(["cmake", "-S", str(patched_tree), "-B", str(build), "-DENABLE_CUTLASS_RUNNER=OFF",
                          "-DCMAKE_CUDA_ARCHITECTURES=100a", f"-DMO_GEMM_ROOT={ROOT}"],
                         capture_output=True, text=True, timeout=600)
    assert cfg.returncode == 0, cfg.stdout[-3000:] + cfg.stderr[-3000:]
    bld = subprocess.run(["cmake", "--build", str(build), "-j", "4"], capture_output=True, text=True, timeout=900)
    assert bld.returncode == 0, bld.stdout[-3000:] + bld.stderr[-3000:]
    exe = build / "custom_runner"
    assert exe.exists()
    dyn = subprocess.run(["readelf", "-d", str(exe)], capture_output=True, text=True).stdout
    assert "libmo_gemm.so" in dyn
    syms = subprocess.run(["nm", "-C", str(exe)], capture_output=True, text=True).stdout
    assert "bf16_gemm_v1_tensor_core" not in syms and "bf16_gemm_v1_fallback_kernel" not in syms
    out = tmp_path / "r.json"
    proc = subprocess.run([str(exe), "--dataset-dir", str(tmp_path), "--case-id", "none", "--mode", "correctness",
                           "--json-out", str(out)], capture_output=True, text=True, timeout=60)
    assert proc.returncode == 1
    assert "case directory not found" in out.read_text()
