"""GPTQ, RTN, Hessian and dequantization: CPU restatement in float64 (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows the reference egesabanci/gsq-rco-mlx src/gsq_rco/gsq/gptq.py:
  _encode                 :31-36   code = clip(rint(w / s), grid0, gridN) - grid0; s == 0 -> code of 0
  _group_scales           :43-51   |s| = f32(max|w| / max|grid|); sign -s iff err(-s) < err(s)
  dequantize              :63-73
  quantize_rtn            :76-86
  hessian_from_inputs     :89-101  H = 2 X^T X / M, streaming, float64
  quantize_gptq           :123-187 dead inputs, damping, U = upper Cholesky of Hd^-1,
                                   block-lazy column sweep, err = 1/2 tr(D H D^T)
The upper factor is formed here by the reverse-Cholesky identity (U = J chol(J Hd J)^-1 J,
J the exchange matrix), which equals the reference's chol(L^-T L^-1)^T up to rounding.
"""
from __future__ import annotations

import numpy as np

from .gsq import get_grid


def grid64(bits: int) -> np.ndarray:
    if not 1 <= bits <= 8:
        raise ValueError(f"bits must be in 1..8 (uint8 codes), got {bits}")
    return get_grid(bits).astype(np.float64)


def encode(x, s, grid):
    """gptq.py:31-36."""
    s_safe = np.where(s == 0, 1.0, s)
    q = np.clip(np.rint(x / s_safe), grid[0], grid[-1])
    return (q - grid[0]).astype(np.uint8)


def group_scales(Wg, grid, signed=True):
    """gptq.py:43-51 for grouped weights Wg [..., gs] -> float32 [...]."""
    s = (np.abs(Wg).max(axis=-1) / np.abs(grid).max()).astype(np.float32).astype(np.float64)
    if signed:
        def sq_err(sc):
            q = encode(Wg, sc[..., None], grid)
            return ((Wg - sc[..., None] * grid[q]) ** 2).sum(axis=-1)
        s = np.where(sq_err(-s) < sq_err(s), -s, s)
    return s.astype(np.float32)


def dequantize(codes, scales, bits, group_size=64):
    """gptq.py:63-73: w[:, c] = scales[:, c // gs] * grid[codes[:, c]], float32."""
    grid = get_grid(bits)
    codes = np.asarray(codes)
    out_f, in_f = codes.shape
    scales = np.asarray(scales, dtype=np.float32)
    if scales.shape != (out_f, -(-in_f // group_size)):
        raise ValueError(f"scales must be [{out_f}, {-(-in_f // group_size)}], got {scales.shape}")
    gid = np.arange(in_f) // group_size
    return (scales[:, gid] * grid[codes]).astype(np.float32)


def quantize_rtn(W, bits, group_size=64, signed_scale=True):
    """gptq.py:76-86."""
    grid = grid64(bits)
    W = np.asarray(W, dtype=np.float64)
    out_f, in_f = W.shape
    G = -(-in_f // group_size)
    Wp = np.zeros((out_f, G * group_size))
    Wp[:, :in_f] = W
    Wg = Wp.reshape(out_f, G, group_size)
    scales = group_scales(Wg, grid, signed_scale)
    codes = encode(Wg, scales.astype(np.float64)[..., None], grid).reshape(out_f, -1)[:, :in_f]
    codes = np.ascontiguousarray(codes)
    return {"codes": codes, "scales": scales, "w_q": dequantize(codes, scales, bits, group_size)}


def hessian_from_inputs(X, H=None, n=0):
    """gptq.py:89-101: streaming H = 2 X^T X / M in float64; returns (H, n + m)."""
    X = np.asarray(X, dtype=np.float64)
    total = n + X.shape[0]
    if H is None:
        H = np.zeros((X.shape[1], X.shape[1]))
    H *= n / total
    H += (2.0 / total) * (X.T @ X)
    return H, total


def upper_factor(H, damp=0.01):
    """Dead-input handling, damping and the upper factor U of Hd^-1 (gptq.py:143-157).
    Returns (U, dead column indices)."""
    Hd = np.array(H, dtype=np.float64)
    n = Hd.shape[0]
    dead = np.flatnonzero(np.diag(Hd) == 0)
    Hd[dead, dead] = 1.0
    Hd[np.arange(n), np.arange(n)] += damp * np.diag(Hd).mean()
    J = slice(None, None, -1)
    Lr = np.linalg.cholesky(Hd[J, J])          # J Hd J = Lr Lr^T
    Lr_inv = np.linalg.solve(Lr, np.eye(n))     # lower triangular inverse
    return np.ascontiguousarray(Lr_inv[J, J]), dead


def quantize_gptq(W, H, bits, group_size=64, damp=0.01, block_size=128, act_order=False,
                  signed_scale=True):
    """gptq.py:123-187, row-parallel: each output row is swept left to right independently."""
    if act_order:
        raise NotImplementedError("act_order is not implemented (as in the reference)")
    grid = grid64(bits)
    W0 = np.asarray(W, dtype=np.float64)
    H0 = np.asarray(H, dtype=np.float64)
    out_f, in_f = W0.shape
    if H0.shape != (in_f, in_f):
        raise ValueError(f"H must be [{in_f}, {in_f}], got {H0.shape}")
    U, dead = upper_factor(H0, damp)
    Wk = W0.copy()
    Wk[:, dead] = 0.0
    G = -(-in_f // group_size)
    codes = np.zeros((out_f, in_f), dtype=np.uint8)
    scales = np.zeros((out_f, G), dtype=np.float32)
    for i1 in range(0, in_f, block_size):
        i2 = min(i1 + block_size, in_f)
        W1 = Wk[:, i1:i2].copy()
        E = np.zeros((out_f, i2 - i1))
        for i in range(i2 - i1):
            j = i1 + i
            g = j // group_size
            if j % group_size == 0:
                e = min(j + group_size, in_f)
                # the group's current weights: lazy block updates are the in-block errors
                cur = Wk[:, j:e] - E[:, :i] @ U[i1:j, j:e]
                scales[:, g] = group_scales(cur, grid, signed_scale)
            s = scales[:, g].astype(np.float64)
            w = W1[:, i]
            c = encode(w, s, grid)
            codes[:, j] = c
            err = (w - s * grid[c]) / U[j, j]
            W1[:, i:] -= np.outer(err, U[j, j:i2])
            E[:, i] = err
        Wk[:, i2:] -= E @ U[i1:i2, i2:]
    w_q = dequantize(codes, scales, bits, group_size)
    D = w_q.astype(np.float64) - W0
    err_out = 0.5 * float(np.sum((D @ H0) * D))
    return {"codes": codes, "scales": scales, "w_q": w_q, "err": err_out}
