"""Projections of the decode steps: ``y = x @ weight.T`` for few rows.

``gemm`` is the library's weight-streaming GEMM (``anemll_gemm``: 128 x 128 tcgen05 tiles fed by
TMA, split-K over a thread-block cluster whose partial tiles are summed through distributed shared
memory).  ``linear`` sends inputs of up to ``SKINNY_ROWS`` rows to it and everything else to torch's
GEMM.  ``SKINNY_ROWS`` is 0 for now: at batch 128 on a B200, torch's kernels stream the stack's
decode weights faster (4.4 TB/s for the 2048 x 12352 projection, 2.0 TB/s for 4096 x 2048) than
``anemll_gemm`` (2.9 and 1.2 TB/s; its TMA stream alone reaches 3.6 and 1.5 TB/s), so the decode
steps use torch's kernels until it overtakes them.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib

SKINNY_ROWS = 0  # rows up to which linear() uses anemll_gemm (see the module docstring)

__all__ = ["linear", "gemm", "gemm_device_error", "SKINNY_ROWS"]


def _fits(t):
    return t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0


def gemm(x2, weight, out=None):
    """``x2 [M, K] @ weight [N, K]^T`` through ``anemll_gemm`` (any M; fp16/bf16, rows 16-byte units)."""
    if not (x2.is_cuda and weight.is_cuda):
        raise RuntimeError("anemll_b200 ops take CUDA tensors (no CPU path)")
    if x2.dtype != weight.dtype or x2.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("gemm: x and weight must both be fp16 or both bf16")
    M, K = x2.shape
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise ValueError("gemm: inner dimensions differ")
    if not _fits(x2):
        x2 = x2.contiguous()
        if not _fits(x2):
            x2 = x2.clone()
    if not _fits(weight):
        raise ValueError("gemm: weight rows must be dense 16-byte units")
    y = out if out is not None else torch.empty(M, N, dtype=x2.dtype, device=x2.device)
    rc = _lib.load().anemll_gemm(_lib.ptr(x2), x2.stride(0), _lib.ptr(weight), weight.stride(0), _lib.ptr(y),
                                 y.stride(0), M, N, K, _lib.dtype_code(x2.dtype), _lib.stream_ptr(x2.device))
    _lib.check(rc, "anemll_gemm")
    return y


def linear(x, weight):
    """``F.linear(x, weight)`` (no bias) for x [..., K]: ``gemm`` for up to SKINNY_ROWS rows."""
    K = x.shape[-1]
    M = x.numel() // K if K else 0
    N = weight.shape[0]
    if (M == 0 or M > SKINNY_ROWS or not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16)
            or x.dtype != weight.dtype or N % 8 or K % 8 or not _fits(weight)):
        return F.linear(x, weight)
    return gemm(x.reshape(M, K), weight).view(*x.shape[:-1], N)


def gemm_device_error(reset=True) -> int:
    """Non-zero if a GEMM launch stopped on a bounded wait (synchronous)."""
    return int(_lib.load().anemll_gemm_error(int(bool(reset))))
