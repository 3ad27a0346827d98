"""Float32-faithful contractions of the GSQ step on CUDA tensors.

  mm_nt(A, B)  = alpha * A @ B.T     A [M, K], B [N, K]   (the forward residual X (W_bar - W)^T)
  mm_tn(A, B)  = alpha * A.T @ B     A [K, M], B [K, N]   (the weight gradient R^T X)
  sumsq(x)     = sum(x^2) in float64 (deterministic)
"""
from __future__ import annotations

import torch

from . import _lib


def _f32(t):
    if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
        raise ValueError("expected a contiguous CUDA float32 tensor")
    return t


def mm_nt(A, B, alpha=1.0, out=None):
    _f32(A), _f32(B)
    M, K = A.shape
    N, K2 = B.shape
    if K != K2:
        raise ValueError(f"inner dims differ: {K} vs {K2}")
    out = torch.empty(M, N, device=A.device, dtype=torch.float32) if out is None else _f32(out)
    _lib.call("gsq_gemm_f32", M, N, K, float(alpha), _lib.ptr(A), K, 1, _lib.ptr(B), 1, K, 0.0,
              _lib.ptr(out), N, _lib.stream_ptr())
    return out


def mm_tn(A, B, alpha=1.0, out=None):
    _f32(A), _f32(B)
    K, M = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"inner dims differ: {K} vs {K2}")
    out = torch.empty(M, N, device=A.device, dtype=torch.float32) if out is None else _f32(out)
    _lib.call("gsq_gemm_f32", M, N, K, float(alpha), _lib.ptr(A), 1, M, _lib.ptr(B), N, 1, 0.0,
              _lib.ptr(out), N, _lib.stream_ptr())
    return out


class SumSq:
    """Reusable float64 sum-of-squares accumulator (keeps its partials buffer)."""

    def __init__(self, device):
        self.partials = torch.empty(1024, device=device, dtype=torch.float64)

    def __call__(self, x, out):
        _f32(x)
        _lib.call("gsq_sumsq_f32", _lib.ptr(x), x.numel(), _lib.ptr(self.partials), _lib.ptr(out),
                  _lib.stream_ptr())
        return out
