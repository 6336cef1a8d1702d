"""Helpers for the GPU tests: move BF16 bit matrices to the device and call the C ABI."""

from __future__ import annotations

import numpy as np
import torch

import matmul_optimizer_b200 as mo


def to_device(bits: np.ndarray, device="cuda:0") -> torch.Tensor:
    """uint16 BF16 bits -> int16 CUDA tensor with the same bytes."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(device)


def to_host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def run_gemm(a_bits: np.ndarray, b_bits: np.ndarray, device="cuda:0") -> np.ndarray:
    """C = A·B through mo_launch_bf16_gemm_v1 on the current stream; returns BF16 bits."""
    m, k = a_bits.shape
    n = b_bits.shape[1]
    a = to_device(a_bits, device)
    b = to_device(b_bits, device)
    c = torch.empty((m, n), dtype=torch.int16, device=device)
    rc = mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream())
    assert rc == mo.MO_OK, mo.error_string(rc)
    torch.cuda.synchronize()
    return to_host(c)


def gemm_dev(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    m, k = a.shape
    n = b.shape[1]
    c = torch.empty((m, n), dtype=torch.int16, device=a.device)
    rc = mo.launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream())
    assert rc == mo.MO_OK, mo.error_string(rc)
    return c
