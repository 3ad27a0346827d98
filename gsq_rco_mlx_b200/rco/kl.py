"""The RCO objective's KL head and straight-through dots on the GPU.

Reference: src/gsq_rco/common/evaluate.py:28-33,111-151 (tied-embedding logits, the chunked
KL(p_ref || p_q) value and its gradient w.r.t. the quantized hidden states) and
src/gsq_rco/rco/allocate.py:169-174 (the straight-through upstream <dL/dW_i, Delta_ik>).

Per chunk of rows, three tensor-core GEMMs and one row pass:
  zq = bf16(h_q E^T), zr = bf16(h_ref E^T)     gemm (one bf16 term each, bf16-chain epilogue)
  kl_rows, D = bf16(q - p)                      gsq_kl_rows (one CTA per row, f64 sums)
  g = bf16(D E)                                  gemm against E^T (K-major copy made once)
The logits of a chunk are two bf16 [chunk, V] buffers (V = 151936: 311 MB at 1024 rows); the
reference's chunk of 64 bounds MLX's lazy-graph memory, here the chunk only sets the buffer size.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _lib
from ..gemm import Terms, gemm, pad8

CHUNK = 1024


class KLHead:
    """The tied head E bf16 [V, H] on the GPU, its K-major transpose for the gradient GEMM,
    and the chunk buffers."""

    def __init__(self, E: torch.Tensor, chunk: int = CHUNK):
        if E.dtype != torch.bfloat16 or E.dim() != 2:
            raise ValueError("E must be a bf16 [V, H] tensor")
        self.E = E.contiguous()
        self.V, self.H = self.E.shape
        if self.V % 8:
            raise ValueError(f"vocabulary {self.V} must be a multiple of 8")
        dev = self.E.device
        self.dev = dev
        self.chunk = int(chunk)
        self.Et = Terms(self.V, self.H, 1, ld=self.H, tensors=[self.E])
        self.ET = Terms(self.H, self.V, 1, dev)
        _lib.call("gsq_transpose_bf16", _lib.ptr(self.E), self.V, self.H, self.H, 0,
                  _lib.ptr(self.ET.t[0]), self.ET.ld, 0, 1, 0, _lib.stream_ptr())
        c = self.chunk
        self.zq = torch.empty(c, self.V, device=dev, dtype=torch.bfloat16)
        self.zr = torch.empty(c, self.V, device=dev, dtype=torch.bfloat16)
        self.D = torch.empty(c, self.V, device=dev, dtype=torch.bfloat16)

    def _rows(self, x):
        return Terms(x.shape[0], x.shape[1], 1, ld=x.shape[1], tensors=[x])

    def logits(self, h, out):
        """out bf16 [m, V] = bf16(h E^T) (evaluate.py:28-33, before the float32 cast)."""
        gemm(self._rows(h), self.Et, epi=4, c_terms=self._rows(out))
        return out

    def kl_sum_and_grad(self, h_q, h_ref, grad=None):
        """Sum over rows of KL(p_ref || p_q) (float64 CUDA [1]) and its gradient w.r.t. h_q,
        bf16 [n, H] (unscaled: the sum's gradient), evaluate.py:111-124 per chunk."""
        n, H = h_q.shape
        if h_ref.shape != h_q.shape or H != self.H:
            raise ValueError(f"h_q {tuple(h_q.shape)} / h_ref {tuple(h_ref.shape)} vs H {self.H}")
        h_q, h_ref = h_q.contiguous(), h_ref.contiguous()
        grad = torch.empty(n, H, device=self.dev, dtype=torch.bfloat16) if grad is None else grad
        kl_rows = torch.empty(n, device=self.dev, dtype=torch.float64)
        st = _lib.stream_ptr()
        for a in range(0, n, self.chunk):
            m = min(self.chunk, n - a)
            zq, zr, D = self.zq[:m], self.zr[:m], self.D[:m]
            self.logits(h_q[a:a + m], zq)
            self.logits(h_ref[a:a + m], zr)
            _lib.call("gsq_kl_rows", _lib.ptr(zq), _lib.ptr(zr), m, self.V, self.V, _lib.ptr(D),
                      self.V, _lib.ptr(kl_rows[a:a + m]), None, st)
            gemm(self._rows(D), self.ET, epi=4, c_terms=self._rows(grad[a:a + m]))
        total = torch.empty(1, device=self.dev, dtype=torch.float64)
        _lib.call("gsq_sum_f64", _lib.ptr(kl_rows), n, _lib.ptr(total), st)
        return total, grad


def kl_value_and_grad_hidden(head: KLHead, h_q, h_ref):
    """Mean KL(p_ref || p_q) over the positions and its gradient w.r.t. h_q
    (evaluate.py:128-151): h_q, h_ref bf16 [..., H]. Returns (kl float, grad bf16 shaped like
    h_q) with grad = bf16(g / n) as the reference divides its bf16 gradient."""
    shape = h_q.shape
    n = int(np.prod(shape[:-1]))
    total, g = head.kl_sum_and_grad(h_q.reshape(n, shape[-1]), h_ref.reshape(n, shape[-1]))
    _lib.call("gsq_div_bf16", _lib.ptr(g), g.numel(), float(n), _lib.stream_ptr())
    return float(total.item()) / n, g.view(shape)


class DotsWorkspace:
    """Partial sums of ste_dots (one per device)."""

    def __init__(self, dev, max_blocks=4096, max_options=8):
        self.max_blocks = int(max_blocks)
        self.partials = torch.empty(self.max_blocks * max_options, device=dev,
                                    dtype=torch.float64)


def ste_dots(G, W_ref, cands, group_size=64, ws: DotsWorkspace = None, out=None):
    """allocate.py:169-174: <dL/dW, f32(bf16(dequant(db[i, k]))) - W_ref> for every option k.
    G float32 CUDA [out, in]; W_ref bf16 CUDA [out, in]; cands = [(codes uint8 CUDA [out, in],
    scales float32 CUDA [out, groups], bits)] for k = 0..K-1. Returns float64 CUDA [K]."""
    import ctypes as C
    out_f, in_f = W_ref.shape
    K = len(cands)
    if not 1 <= K <= 8:
        raise ValueError(f"1..8 options, got {K}")
    ws = ws or DotsWorkspace(G.device)
    codes = (C.c_void_p * K)(*[c[0].data_ptr() for c in cands])
    scales = (C.c_void_p * K)(*[c[1].data_ptr() for c in cands])
    bits = (C.c_int * K)(*[int(c[2]) for c in cands])
    out = torch.empty(K, device=G.device, dtype=torch.float64) if out is None else out
    _lib.call("ste_dots", _lib.ptr(G), _lib.ptr(W_ref), out_f, in_f, int(group_size), K, codes,
              scales, bits, _lib.ptr(ws.partials), ws.max_blocks, _lib.ptr(out),
              _lib.stream_ptr())
    return out
