"""matmul_optimizer_b200: the fixed BF16 GEMM of YupengHan/matmul_optimizer, rebuilt for B200.

The product is the native library ``lib/libmo_gemm.so`` (sm_100a tcgen05/TMA kernel, C ABI in
include/mo_gemm.h, C++ ABI in include/kernel_api.h) and the runner executables under ``bin/``.
This module is the thin ctypes layer over the C ABI, mirroring the reference's kernel entry
``launch_bf16_gemm_v1`` (reference include/kernel_api.h:10-17): same argument meaning, device
pointers in, ``False`` on a null pointer, a non-positive dimension or a launch error.

There is no CPU or PyTorch fallback: every call goes through libmo_gemm.so, and a missing or
unloadable library raises ``LibraryNotBuilt``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import List, Optional, Sequence, Tuple

__all__ = [
    "LibraryNotBuilt", "MoGemmError", "library_path", "load_library", "launch_bf16_gemm_v1",
    "launch", "launch_noalloc", "gemm", "select_plan", "schedule", "SCHEDULE_FIELDS", "shard_partition", "gemm_nshard", "unshard_columns",
    "read_watchdog", "selftest_wait_timeout", "release_workspace", "gemm_from_host", "gemm_b_from_host",
    "error_string",
    "EXPORTED_SYMBOLS",
]

_PKG = Path(__file__).resolve().parent
_LIB = None

# Every function include/mo_gemm.h declares, plus the C++ ABI symbol of kernel_api.h.
EXPORTED_SYMBOLS = (
    "mo_error_string", "mo_version", "mo_launch_bf16_gemm_v1", "mo_gemm_select_plan",
    "mo_shard_partition", "mo_gemm_nshard", "mo_unshard_columns", "mo_read_device_watchdog",
    "mo_selftest_wait_timeout", "mo_launch_bf16_gemm_v1_noalloc", "mo_release_workspace",
    "mo_gemm_from_host", "mo_gemm_b_from_host", "mo_gemm_schedule",
)
CXX_SYMBOL = "_ZN16matmul_optimizer19launch_bf16_gemm_v1EPKtS1_PtiiiP11CUstream_st"

MO_OK = 0
MO_ERR_NULL_POINTER = -1
MO_ERR_BAD_DIMS = -2
MO_ERR_UNSUPPORTED = -3
MO_ERR_LAUNCH = -4
MO_ERR_DEVICE = -5
MO_ERR_BAD_ARGUMENT = -6
MO_ERR_DEVICE_TIMEOUT = -7
MO_ERR_SCRATCH_LIMIT = -8
MO_ERR_NO_MEMORY = -9


class LibraryNotBuilt(RuntimeError):
    """libmo_gemm.so is missing or cannot be loaded (run matmul_optimizer_b200.build)."""


class MoGemmError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        super().__init__(f"{what}: {error_string(code)} (code {code})" if what else error_string(code))


class _Plan(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in (
        "block_m", "block_n", "block_k", "stages", "cta_group", "num_tiles", "grid", "smem_bytes",
        "num_chunks", "split", "stream_k")]


def library_path() -> Path:
    return Path(os.environ.get("MO_GEMM_LIBRARY", _PKG / "lib" / "libmo_gemm.so"))


def load_library() -> ctypes.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not path.exists():
        raise LibraryNotBuilt(f"{path} not found; build it with `python -m matmul_optimizer_b200.build`")
    try:
        lib = ctypes.CDLL(str(path))
    except OSError as exc:  # pragma: no cover - depends on the machine
        raise LibraryNotBuilt(f"cannot load {path}: {exc}") from exc
    u16p = ctypes.c_void_p
    lib.mo_error_string.argtypes = [ctypes.c_int]
    lib.mo_error_string.restype = ctypes.c_char_p
    lib.mo_version.argtypes = []
    lib.mo_version.restype = ctypes.c_int
    lib.mo_launch_bf16_gemm_v1.argtypes = [u16p, u16p, u16p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_void_p]
    lib.mo_launch_bf16_gemm_v1.restype = ctypes.c_int
    lib.mo_launch_bf16_gemm_v1_noalloc.argtypes = lib.mo_launch_bf16_gemm_v1.argtypes
    lib.mo_launch_bf16_gemm_v1_noalloc.restype = ctypes.c_int
    lib.mo_gemm_select_plan.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(_Plan)]
    lib.mo_gemm_select_plan.restype = ctypes.c_int
    lib.mo_shard_partition.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                       ctypes.POINTER(ctypes.c_int)]
    lib.mo_shard_partition.restype = ctypes.c_int
    lib.mo_gemm_nshard.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                   ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                   ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                   ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_void_p)]
    lib.mo_gemm_nshard.restype = ctypes.c_int
    lib.mo_unshard_columns.argtypes = [u16p, u16p, ctypes.c_int, ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_int), ctypes.c_int64, ctypes.c_void_p]
    lib.mo_unshard_columns.restype = ctypes.c_int
    lib.mo_read_device_watchdog.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.mo_read_device_watchdog.restype = ctypes.c_int
    lib.mo_selftest_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_void_p]
    lib.mo_selftest_wait_timeout.restype = ctypes.c_int
    lib.mo_release_workspace.argtypes = [ctypes.POINTER(ctypes.c_int64)]
    lib.mo_release_workspace.restype = ctypes.c_int
    lib.mo_gemm_from_host.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p]
    lib.mo_gemm_from_host.restype = ctypes.c_int
    lib.mo_gemm_b_from_host.argtypes = lib.mo_gemm_from_host.argtypes
    lib.mo_gemm_schedule.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_int)]
    lib.mo_gemm_schedule.restype = ctypes.c_int
    lib.mo_gemm_b_from_host.restype = ctypes.c_int
    _LIB = lib
    return lib


def error_string(code: int) -> str:
    return load_library().mo_error_string(int(code)).decode()


def _stream_handle(stream) -> Optional[int]:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    handle = getattr(stream, "cuda_stream", None)  # torch.cuda.Stream
    if handle is None:
        raise TypeError(f"unsupported stream object {stream!r}")
    return int(handle)


def launch(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, stream=None) -> int:
    """C ABI call; returns the MO_* code."""
    return int(load_library().mo_launch_bf16_gemm_v1(a_ptr, b_ptr, c_ptr, m, n, k, _stream_handle(stream)))


def launch_noalloc(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, stream=None) -> int:
    """C ABI call of mo_launch_bf16_gemm_v1_noalloc: the same result as ``launch`` for callers
    that cannot allocate device memory during a call (a plugin inside a host application that
    owns all device memory, or code that cannot afford cudaMalloc's synchronisation).  Its
    scratch is a fixed 32 MiB array per GPU inside the library; calls that overlap on one GPU
    race on it.  Returns the MO_* code (MO_ERR_SCRATCH_LIMIT when the problem does not fit)."""
    return int(load_library().mo_launch_bf16_gemm_v1_noalloc(a_ptr, b_ptr, c_ptr, m, n, k,
                                                             _stream_handle(stream)))


def launch_bf16_gemm_v1(a_ptr: int, b_ptr: int, c_ptr: int, m: int, n: int, k: int, stream=None) -> bool:
    """Mirror of the reference's ``launch_bf16_gemm_v1``: device pointers to row-major BF16
    bits, asynchronous on ``stream``; True when the launch was issued."""
    return launch(a_ptr, b_ptr, c_ptr, m, n, k, stream) == MO_OK


def gemm(a, b, out=None, stream=None):
    """``out = a @ b`` for CUDA bf16 (or uint16 bit-pattern) tensors, row-major contiguous.

    Raises MoGemmError with the library's reason on failure.  Runs on ``stream`` (default:
    torch's current stream of the tensors' device)."""
    import torch

    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"shape mismatch {tuple(a.shape)} x {tuple(b.shape)}")
    for t in (a, b):
        if not t.is_cuda or t.dtype not in (torch.bfloat16, torch.uint16, torch.int16) or not t.is_contiguous():
            raise ValueError("operands must be contiguous CUDA bf16 (or 16-bit) tensors")
    m, k = a.shape
    n = b.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if stream is None:
        stream = torch.cuda.current_stream(a.device)
    with torch.cuda.device(a.device):
        rc = launch(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, stream)
    if rc != MO_OK:
        raise MoGemmError(rc, f"gemm {m}x{n}x{k}")
    return out


def select_plan(m: int, n: int, k: int, num_sms: int = 148) -> dict:
    plan = _Plan()
    rc = load_library().mo_gemm_select_plan(m, n, k, num_sms, ctypes.byref(plan))
    if rc != MO_OK:
        raise MoGemmError(rc, "select_plan")
    return {name: getattr(plan, name) for name, _ in _Plan._fields_}


SCHEDULE_FIELDS = ("cluster", "position", "m_block", "n_block", "chunk_begin", "chunk_end",
                   "sk_tile")


def schedule(m: int, n: int, k: int, num_sms: int = 148):
    """Work units of the plan for this shape (mo_gemm_schedule): an int32 array with one row per
    unit and the columns SCHEDULE_FIELDS, in each cluster's execution order.  Needs no GPU."""
    import numpy as np

    lib = load_library()
    count = ctypes.c_int(0)
    rc = lib.mo_gemm_schedule(m, n, k, num_sms, None, 0, ctypes.byref(count))
    if rc != MO_OK:
        raise MoGemmError(rc, "schedule")
    out = np.zeros((count.value, len(SCHEDULE_FIELDS)), dtype=np.int32)
    rc = lib.mo_gemm_schedule(m, n, k, num_sms, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                              count.value, ctypes.byref(count))
    if rc != MO_OK:
        raise MoGemmError(rc, "schedule")
    return out


def shard_partition(n: int, g: int) -> Tuple[List[int], List[int]]:
    begin = (ctypes.c_int * g)()
    width = (ctypes.c_int * g)()
    rc = load_library().mo_shard_partition(n, g, begin, width)
    if rc != MO_OK:
        raise MoGemmError(rc, "shard_partition")
    return list(begin), list(width)


def gemm_nshard(devices: Sequence[int], a_ptrs: Sequence[int], b_ptrs: Sequence[int],
                c_ptrs: Sequence[int], m: int, k: int, slab_n: Sequence[int],
                streams: Sequence[int]) -> None:
    g = len(devices)
    arr = lambda ctype, xs: (ctype * g)(*xs)  # noqa: E731
    rc = load_library().mo_gemm_nshard(
        g, arr(ctypes.c_int, devices), arr(ctypes.c_void_p, a_ptrs), arr(ctypes.c_void_p, b_ptrs),
        arr(ctypes.c_void_p, c_ptrs), m, k, arr(ctypes.c_int, slab_n),
        arr(ctypes.c_void_p, [_stream_handle(s) for s in streams]))
    if rc != MO_OK:
        raise MoGemmError(rc, "gemm_nshard")


def unshard_columns(gathered_ptr: int, c_ptr: int, m: int, slab_n: Sequence[int],
                    block_elems: int, stream=None) -> None:
    g = len(slab_n)
    rc = load_library().mo_unshard_columns(gathered_ptr, c_ptr, g, m, (ctypes.c_int * g)(*slab_n),
                                           block_elems, _stream_handle(stream))
    if rc != MO_OK:
        raise MoGemmError(rc, "unshard_columns")


def read_watchdog(clear: bool = True) -> int:
    flag = ctypes.c_int(0)
    rc = load_library().mo_read_device_watchdog(1 if clear else 0, ctypes.byref(flag))
    if rc != MO_OK:
        raise MoGemmError(rc, "read_watchdog")
    return flag.value


def gemm_from_host(a_host_ptr: int, b_host_ptr: int, c_host_ptr: int, m: int, n: int, k: int,
                   slabs: int = 0, stream=None) -> int:
    """C = A.B from host buffers (row-major BF16 bits; page-locked for overlap): uploads,
    column-slab GEMMs and downloads overlap on the library's own streams; `stream` waits for
    the result.  Returns the library's status code."""
    return load_library().mo_gemm_from_host(a_host_ptr, b_host_ptr, c_host_ptr, m, n, k, slabs,
                                            _stream_handle(stream))


def gemm_b_from_host(a_dev_ptr: int, b_host_ptr: int, c_host_ptr: int, m: int, n: int, k: int,
                     slabs: int = 0, stream=None) -> int:
    """gemm_from_host with A already on the device: only B goes up and C comes down."""
    return load_library().mo_gemm_b_from_host(a_dev_ptr, b_host_ptr, c_host_ptr, m, n, k, slabs,
                                              _stream_handle(stream))


def release_workspace() -> int:
    """Returns the library's pooled workspace memory on the current device; the bytes it held."""
    held = ctypes.c_int64(0)
    rc = load_library().mo_release_workspace(ctypes.byref(held))
    if rc != MO_OK:
        raise MoGemmError(rc, "release_workspace")
    return held.value


def selftest_wait_timeout(timeout_us: int, stream=None) -> None:
    rc = load_library().mo_selftest_wait_timeout(timeout_us, _stream_handle(stream))
    if rc != MO_OK:
        raise MoGemmError(rc, "selftest_wait_timeout")
