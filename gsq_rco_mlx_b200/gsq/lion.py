"""Lion for the GSQ logits and group scales (reference src/gsq_rco/gsq/lion.py).

    u = sign(beta1 * m + (1 - beta1) * g)
    m <- beta2 * m + (1 - beta2) * g
    theta <- theta - lr * (u + wd * theta)

The stage optimiser applies this rule inside the fused soft-step kernel (gsq_soft_step:
soft backward, resample mean, Lion, next forward); ``lion_update`` is the stand-alone form of the reference API on CUDA
tensors, one launch per tensor.
"""
from __future__ import annotations

import torch

from .. import _lib

LR_LOGITS = 1e-4
LR_SCALES = 5e-5
WEIGHT_DECAY = 1.0
BETAS = (0.9, 0.95)
SCALE_LR_RULE = "frozen_above_3_bits"


def scale_lr(lr_scales: float, bits: int) -> float:
    """Group-scale step of a ``bits``-wide linear: frozen (0) above 3 bits (lion.py:27-41)."""
    return 0.0 if bits > 3 else lr_scales


def lion_update(P: dict, M: dict, G: dict, lr: dict, wd: float = WEIGHT_DECAY,
                betas: tuple = BETAS):
    """One Lion step on dicts of CUDA float32 tensors; returns (new params, new momentum).
    Pure in its inputs like the reference (lion.py:44-56): P and M are not modified."""
    b1, b2 = betas
    newP, newM = {}, {}
    for k in P:
        p = P[k].detach().to(torch.float32).contiguous().clone()
        m = M[k].detach().to(torch.float32).contiguous().clone()
        g = G[k].detach().to(device=p.device, dtype=torch.float32).contiguous()
        _lib.call("gsq_lion_f32", _lib.ptr(p), _lib.ptr(m), _lib.ptr(g), p.numel(),
                  float(lr[k]), float(wd), float(b1), float(b2), _lib.stream_ptr())
        newP[k], newM[k] = p, m
    return newP, newM
