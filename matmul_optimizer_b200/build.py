"""In-tree build of the native parts (nvcc / g++ only, no CMake):

* lib/libmo_gemm.so   - the sm_100a GEMM library: the C++ ABI of include/kernel_api.h and the
                        C ABI of include/mo_gemm.h (static cudart, driver API resolved at run
                        time, so the library loads on a machine without a GPU).
* bin/custom_runner   - the benchmark runner with the reference's CLI/JSON contract
                        (src/runner/main.cpp of the reference), linked to libmo_gemm.so.
* bin/cublas_runner   - the same runner driving cuBLASLt instead: the same-box library
                        baseline that replaces the reference's CUTLASS runner.

Every CUDA translation unit is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a).  Outputs stay inside the package directory so
they travel with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = PKG / "lib"
BIN_DIR = PKG / "bin"
LIB_PATH = LIB_DIR / "libmo_gemm.so"
RUNNER_PATH = BIN_DIR / "custom_runner"
CUBLAS_RUNNER_PATH = BIN_DIR / "cublas_runner"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_NVCC = ["-std=c++17", "-O3", "-lineinfo", "--expt-relaxed-constexpr",
               "-Xcompiler", "-fPIC", "-diag-suppress", "177"] + ARCH_FLAGS

LIB_SOURCES = [CSRC / "gemm_sm100.cu"]
LIB_HEADERS = [CSRC / "sm100_ptx.cuh", CSRC / "gemm_kernel.cuh", INCLUDE / "kernel_api.h", INCLUDE / "mo_gemm.h"]
RUNNER_SOURCES = [CSRC / "runner_main.cpp", CSRC / "runner_common.h"]
CUBLAS_RUNNER_SOURCES = [CSRC / "cublas_runner.cpp", CSRC / "runner_main.cpp", CSRC / "runner_common.h"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps if Path(d).exists())


def _run(cmd, verbose: bool) -> None:
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    proc = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... (exit {proc.returncode})")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, flush=True)


def build_library(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    LIB_DIR.mkdir(exist_ok=True)
    if force or _stale(LIB_PATH, LIB_SOURCES + LIB_HEADERS + [Path(__file__)]):
        cmd = [nvcc(), *COMMON_NVCC, "-shared", "-cudart", "static", f"-I{INCLUDE}",
               "-o", LIB_PATH, *LIB_SOURCES]
        if ptxas_verbose:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd, verbose or ptxas_verbose)
    return LIB_PATH


def build_runner(force: bool = False, verbose: bool = False) -> Path:
    BIN_DIR.mkdir(exist_ok=True)
    if force or _stale(RUNNER_PATH, RUNNER_SOURCES + [LIB_PATH, Path(__file__)]):
        cmd = [nvcc(), "-std=c++17", "-O2", *ARCH_FLAGS, f"-I{INCLUDE}", "-o", RUNNER_PATH,
               CSRC / "runner_main.cpp", f"-L{LIB_DIR}", "-lmo_gemm", "-lnccl",
               "-Xlinker", "-rpath=$ORIGIN/../lib"]
        _run(cmd, verbose)
    return RUNNER_PATH


def build_cublas_runner(force: bool = False, verbose: bool = False) -> Path:
    BIN_DIR.mkdir(exist_ok=True)
    if force or _stale(CUBLAS_RUNNER_PATH, CUBLAS_RUNNER_SOURCES + [Path(__file__)]):
        cmd = [nvcc(), "-std=c++17", "-O2", *ARCH_FLAGS, f"-I{INCLUDE}", "-DMO_RUNNER_CUBLAS",
               "-o", CUBLAS_RUNNER_PATH, CSRC / "runner_main.cpp", CSRC / "cublas_runner.cpp",
               "-lcublasLt", "-lnccl"]
        _run(cmd, verbose)
    return CUBLAS_RUNNER_PATH


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force, verbose)
    build_runner(force, verbose)
    build_cublas_runner(force, verbose)


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    build_library(a.force, a.verbose, a.ptxas_verbose)
    build_runner(a.force, a.verbose)
    build_cublas_runner(a.force, a.verbose)
