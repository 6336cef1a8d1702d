"""mo_launch_bf16_gemm_v1_noalloc: the GEMM for callers that cannot allocate device memory
during a call.  Examples are a plugin whose host application owns all device memory through
its own pool, and code that cannot afford cudaMalloc's synchronisation.  It keeps its K-split
partials in a fixed 32 MiB array inside the library instead of allocating a workspace.

This file is named to run last in a full GPU run.  Its tests also pass alone in a fresh
process: the entry point sets itself up on its first call on a device.  Each shape is called
twice in a row, with a call on other inputs of the same shape between them: the array then
holds partials that differ from the right ones, so a partial the split kernel failed to write
would show as a mismatch.  The results are compared with mo_launch_bf16_gemm_v1 through the C
ABI.  The algorithm makes them bit-identical, which is tighter than the tolerances of
tests/test_gemm_gpu.py, which are checked against the oracle too.  A subprocess that makes only
no-alloc calls checks the promise itself: the library's workspace pool is never created and the
device's free memory does not move.
"""

import json
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

import matmul_optimizer_b200 as mo
from oracle import bf16_oracle as orc
from tests.gpu_utils import to_device, to_host

pytestmark = pytest.mark.gpu


def _call(fn, a, b, m, n, k):
    c = torch.full((m, n), 0x7FC0, dtype=torch.int16, device=a.device)  # NaN fill: all must be written
    rc = fn(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream())
    torch.cuda.synchronize()
    return rc, to_host(c)


# (m, n, k): 4 K chunks at the hero K (the split path with scratch), a ragged M and N, a long K
# with many chunks, and a single-chunk K that needs no scratch.
SHAPES = [(16, 7776, 7232), (269, 7776, 7232), (129, 1000, 7232), (40, 520, 30000), (64, 264, 1024)]


@pytest.mark.parametrize("shape", SHAPES)
def test_noalloc_matches_regular_entry_point_twice(cuda_device, shape):
    m, n, k = shape
    case = orc.make_uniform_case(m, n, k, seed=7 * m + n + k)
    a, b = to_device(case.a_bits), to_device(case.b_bits)
    other = orc.make_uniform_case(m, n, k, seed=7 * m + n + k + 1)
    a2, b2 = to_device(other.a_bits), to_device(other.b_bits)
    rc, want = _call(mo.launch, a, b, m, n, k)
    assert rc == mo.MO_OK, mo.error_string(rc)
    rc, want2 = _call(mo.launch, a2, b2, m, n, k)
    assert rc == mo.MO_OK, mo.error_string(rc)
    for _ in range(2):
        rc, got = _call(mo.launch_noalloc, a, b, m, n, k)
        assert rc == mo.MO_OK, mo.error_string(rc)
        assert np.array_equal(got, want)
        # Other inputs in between leave other partials in the shared array.
        rc, got2 = _call(mo.launch_noalloc, a2, b2, m, n, k)
        assert rc == mo.MO_OK, mo.error_string(rc)
        assert np.array_equal(got2, want2)
    ref32 = orc.reference_gemm_fp32(case.a_bits, case.b_bits)
    assert orc.evaluate_correctness(got, ref32, orc.float32_to_bf16_bits(ref32))["passed"]
    assert mo.read_watchdog(clear=True) == 0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    m, n, k = 1024, 7776, 7232  # 4 chunks x 1024 x 7776 x 4 bytes = 121.5 MiB > 32 MiB
    a = torch.zeros((m, k), dtype=torch.int16, device="cuda:0")
    b = torch.zeros((k, n), dtype=torch.int16, device="cuda:0")
    c = torch.zeros((m, n), dtype=torch.int16, device="cuda:0")
    rc = mo.launch_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream())
    assert rc == mo.MO_ERR_SCRATCH_LIMIT
    assert "32 MiB" in mo.error_string(rc)
    torch.cuda.synchronize()
    assert torch.count_nonzero(c).item() == 0  # nothing was launched


_NO_ALLOC_PROBE = textwrap.dedent("""
    import json, sys
    import numpy as np
    import torch
    sys.path.insert(0, sys.argv[1])
    import matmul_optimizer_b200 as mo
    shapes = [(16, 7776, 7232), (269, 7776, 7232), (40, 520, 30000), (64, 264, 1024)]
    bufs = []
    for m, n, k in shapes:
        g = torch.Generator(device="cuda:0").manual_seed(m + n + k)
        a = torch.empty((m, k), dtype=torch.bfloat16, device="cuda:0").uniform_(-1, 1, generator=g)
        b = torch.empty((k, n), dtype=torch.bfloat16, device="cuda:0").uniform_(-1, 1, generator=g)
        c = torch.empty((m, n), dtype=torch.bfloat16, device="cuda:0")
        bufs.append((a, b, c, m, n, k))
    stream = torch.cuda.current_stream()
    def run_all():
        for a, b, c, m, n, k in bufs:
            rc = mo.launch_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, stream)
            assert rc == mo.MO_OK, mo.error_string(rc)
        torch.cuda.synchronize()
    run_all()  # first calls: set-up of the device state
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        run_all()
    free1 = torch.cuda.mem_get_info()[0]
    print(json.dumps({"free_before": free0, "free_after": free1,
                      "pool_bytes": mo.release_workspace(), "watchdog": mo.read_watchdog(clear=True)}))
""")


def test_noalloc_calls_allocate_nothing(cuda_device):
    """A fresh process that makes only no-alloc calls: the library's workspace pool is never
    created (mo_release_workspace reports 0 bytes held) and the device's free memory is the
    same before and after repeated calls on shapes that use the scratch array."""
    root = Path(__file__).resolve().parent.parent
    proc = subprocess.run([sys.executable, "-c", _NO_ALLOC_PROBE, str(root)], capture_output=True,
                          text=True, timeout=300, env=dict(os.environ))
    assert proc.returncode == 0, proc.stderr[-2000:]
    res = json.loads(proc.stdout.strip().splitlines()[-1])
    assert res["pool_bytes"] == 0, res
    assert res["free_after"] == res["free_before"], res
    assert res["watchdog"] == 0, res
