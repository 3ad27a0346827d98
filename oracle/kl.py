"""CPU restatement of the RCO objective's KL head and straight-through dots (test
infrastructure: only tests/, the smoke check and the bench's CPU baseline use it).

kl_chunk_value_grad follows src/gsq_rco/common/evaluate.py:28-33,111-124 (tied-embedding logits
rounded to bf16, float32 softmax statistics, the logit gradient q - p rounded to bf16, then
bf16(D E)); kl_value_and_grad_hidden follows :128-151. ste_dots follows
src/gsq_rco/rco/allocate.py:169-174 with dequant of src/gsq_rco/rco/database.py:244-256 (and the
cast of the candidate to the model dtype, allocate.py:117). Sums in float64.
"""
from __future__ import annotations

import numpy as np
import torch

F32, F64 = torch.float32, torch.float64


def bf(x):
    return x.to(torch.bfloat16).to(x.dtype)


def logits(h, E):
    """bf16(h E^T) as float64 (float64 accumulation of exact bf16 products)."""
    return bf(h.to(F64) @ E.to(F64).T)


def kl_chunk_value_grad(hq, hr, E):
    """(sum over rows of KL(p_ref || p_q), dKL/dh_q bf16-valued float64 [n, H])."""
    zq, zr = logits(hq, E), logits(hr, E)
    lse_q = torch.logsumexp(zq, -1, keepdim=True).to(F32).to(F64)
    lse_r = torch.logsumexp(zr, -1, keepdim=True).to(F32).to(F64)
    q = torch.exp(zq - lse_q).to(F32)
    p = torch.exp(zr - lse_r).to(F32)
    value = float((p.to(F64) * ((zr - lse_r) - (zq - lse_q))).sum())
    D = bf((q - p).to(F64))
    grad = bf(D @ E.to(F64))
    return value, grad


def kl_value_and_grad_hidden(hq, hr, E, chunk=64):
    """Mean KL over positions and bf16(grad / n) (evaluate.py:128-151)."""
    n = hq.shape[0]
    total, grads = 0.0, []
    for a in range(0, n, chunk):
        v, g = kl_chunk_value_grad(hq[a:a + chunk], hr[a:a + chunk], E)
        total += v
        grads.append(g)
    grad = bf((torch.cat(grads) / n).to(F32).to(F64))
    return total / n, grad


def grid(bits):
    return (np.arange(2 ** bits) - 2 ** (bits - 1)).astype(np.float32)


def ste_dots(G, W_ref, cands, group_size=64):
    """[<G, f32(bf16(s grid[c])) - W_ref> for (codes, scales, bits) in cands] (float64)."""
    G = np.asarray(G, dtype=np.float32)
    W = np.asarray(W_ref, dtype=np.float32)
    out = []
    for codes, scales, bits in cands:
        vals = grid(bits)[np.asarray(codes).astype(np.int64)]
        s = np.repeat(np.asarray(scales, dtype=np.float32), group_size, axis=1)[:, :W.shape[1]]
        wq = torch.as_tensor((vals * s).astype(np.float32)).to(torch.bfloat16).float().numpy()
        out.append(float(np.sum((G * (wq - W)).astype(np.float64))))
    return np.array(out)
