"""Shared pytest setup.

Markers: ``gpu`` - needs a CUDA B200 (run with ``-m gpu``); everything else runs on CPU.
The repository root is put on sys.path so tests import the package and the oracle directly.
"""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA sm_100 device")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "the GEMM library targets sm_100 (B200) only"
    return torch.device("cuda:0")


def find_reference_root():
    """The reference checkout when this machine has one (MO_REFERENCE_ROOT, else a directory named
    `reference` beside this repository), or None.  Tests that run the reference's own scripts
    skip without it; the GPU box never has it."""
    for cand in (os.environ.get("MO_REFERENCE_ROOT"), ROOT.parent / "reference"):
        if cand and (Path(cand) / "scripts" / "eval_kernel.py").exists():
            return Path(cand)
    return None


@pytest.fixture(scope="session")
def reference_root():
    root = find_reference_root()
    if root is None:
        pytest.skip("no reference checkout on this machine (set MO_REFERENCE_ROOT)")
    return root
