"""GPTQ, RTN, Hessian, dequantization and App-A logit inits (GPU for the array work).

Keeps the contract of the reference src/gsq_rco/gsq/gptq.py:
  quantize_rtn(W, bits, group_size, signed_scale)  -> {codes u8 [out,in], scales f32 [out,G], w_q f32}
  quantize_gptq(W, H, bits, ...)                   -> same dict + "err"
  hessian_from_inputs(X, H, n)                     -> (H, n), H = 2 X^T X / M in float64
  dequantize(codes, scales, bits, group_size)      -> f32 [out,in]
Inputs may be numpy arrays or torch tensors; results come back as numpy arrays (as in the
reference) unless ``device=True`` asks for CUDA tensors. The logit inits (gptq.py:192-232)
are tiny host-side numpy draws, as in the reference.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from .. import _lib
from .quant import get_grid

__all__ = ["quantize_gptq", "quantize_rtn", "hessian_from_inputs", "dequantize",
           "gptq_factor", "init_shift_logits", "init_logits_2bit_from_codes",
           "init_ternary_logits"]


def _grid_bits(bits: int):
    if not 1 <= int(bits) <= 8:
        raise ValueError(f"bits must be in 1..8 (uint8 codes), got {bits}")


def _dev(x, dtype):
    dev = _lib.device()
    if isinstance(x, torch.Tensor):
        return x.to(device=dev, dtype=dtype).contiguous()
    return torch.as_tensor(np.ascontiguousarray(x), device=dev).to(dtype).contiguous()


def _out(t, device):
    return t if device else t.cpu().numpy()


def dequantize(codes, scales, bits, group_size=64, device=False):
    """w_q[:, c] = scales[:, c // group_size] * grid[codes[:, c]] (float32)."""
    _grid_bits(bits)
    codes_t = _dev(codes, torch.uint8)
    out_f, in_f = codes_t.shape
    n_groups = -(-in_f // group_size)
    scales_t = _dev(scales, torch.float32)
    if tuple(scales_t.shape) != (out_f, n_groups):
        raise ValueError(f"scales must be [{out_f}, {n_groups}], got {tuple(scales_t.shape)}")
    wq = torch.empty(out_f, in_f, device=codes_t.device, dtype=torch.float32)
    _lib.call("gptq_dequant", _lib.ptr(codes_t), _lib.ptr(scales_t), out_f, in_f, int(bits),
              int(group_size), _lib.ptr(wq), _lib.stream_ptr())
    return _out(wq, device)


def hessian_from_inputs(X, H=None, n=0, device=False):
    """Streaming H = 2 X^T X / M in float64: feed (H, n) back with each batch X [m, in].
    A CUDA float64 H is updated in place (as the reference updates its numpy H)."""
    Xt = _dev(X, torch.float32)
    m, k = Xt.shape
    if H is None:
        Ht = torch.zeros(k, k, device=Xt.device, dtype=torch.float64)
        in_place = None
    elif isinstance(H, torch.Tensor) and H.is_cuda and H.dtype == torch.float64 and H.is_contiguous():
        Ht, in_place = H, None
    else:
        Ht = _dev(H, torch.float64)
        in_place = H
    _lib.call("hessian_accum", _lib.ptr(Xt), int(m), int(k), _lib.ptr(Ht), int(n),
              _lib.stream_ptr())
    total = int(n) + int(m)
    if isinstance(in_place, np.ndarray):
        in_place[...] = Ht.cpu().numpy()
        return in_place, total
    return (Ht if (device or isinstance(H, torch.Tensor)) else Ht.cpu().numpy()), total


def gptq_factor(H, damp=0.01):
    """(U, dead): U [n, n] float64 CUDA upper factor of (H + damp mean(diag H) I)^-1 = U^T U,
    dead [n] uint8 the inputs with H_ii == 0. Raises LinAlgError-like ValueError if the damped
    Hessian is not positive definite."""
    Ht = _dev(H, torch.float64)
    n = Ht.shape[0]
    if tuple(Ht.shape) != (n, n):
        raise ValueError(f"H must be square, got {tuple(Ht.shape)}")
    U = torch.empty(n, n, device=Ht.device, dtype=torch.float64)
    dead = torch.empty(n, device=Ht.device, dtype=torch.uint8)
    ws = torch.empty(2 * n * n + 64, device=Ht.device, dtype=torch.float64)
    info = torch.zeros(1, device=Ht.device, dtype=torch.int32)
    _lib.call("gptq_factor", _lib.ptr(Ht), n, float(damp), _lib.ptr(U), _lib.ptr(dead),
              _lib.ptr(ws), _lib.ptr(info), _lib.stream_ptr())
    bad = int(info.item())
    if bad:
        raise np.linalg.LinAlgError(f"damped Hessian is not positive definite (column {bad - 1})")
    return U, dead


def _sweep(Wt, U, dead, bits, group_size, block_size, signed_scale):
    out_f, in_f = Wt.shape
    G = -(-in_f // group_size)
    codes = torch.empty(out_f, in_f, device=Wt.device, dtype=torch.uint8)
    scales = torch.empty(out_f, G, device=Wt.device, dtype=torch.float32)
    work = torch.empty(out_f, in_f, device=Wt.device, dtype=torch.float64)
    _lib.call("gptq_sweep", _lib.ptr(Wt), _lib.ptr(U), _lib.ptr(dead), out_f, in_f, int(bits),
              int(group_size), int(block_size), int(bool(signed_scale)), _lib.ptr(codes),
              _lib.ptr(scales), _lib.ptr(work), _lib.stream_ptr())
    return codes, scales


def _err(wq, Wt, Ht):
    out_f, in_f = Wt.shape
    ws = torch.empty(2 * out_f * in_f + 1024, device=Wt.device, dtype=torch.float64)
    err = torch.empty(1, device=Wt.device, dtype=torch.float64)
    _lib.call("gptq_err", _lib.ptr(wq), _lib.ptr(Wt), _lib.ptr(Ht), out_f, in_f, _lib.ptr(err),
              _lib.ptr(ws), _lib.stream_ptr())
    return err


def quantize_gptq(W, H, bits, group_size=64, damp=0.01, block_size=128, act_order=False,
                  signed_scale=True, device=False, factor=None):
    """GPTQ on the grid, scales and codes of quantize_rtn (reference gptq.py:123-187).

    Minimises ||X (W_q - W)^T||^2 for H = 2 X^T X / M; the columns are swept left to right,
    each column's error pushed onto the later columns through the upper Cholesky factor of
    the damped inverse Hessian, lazily once per block_size columns. ``err`` = 1/2 tr(D H D^T).
    ``factor`` may pass a precomputed (U, dead) of the same H and damp (one factorization
    serves every linear and bit width that reads the same Hessian)."""
    if act_order:
        raise NotImplementedError("act_order needs a permuted static-group layout; not implemented")
    _grid_bits(bits)
    Wt = _dev(W, torch.float32)
    out_f, in_f = Wt.shape
    Ht = _dev(H, torch.float64)
    if tuple(Ht.shape) != (in_f, in_f):
        raise ValueError(f"H must be [{in_f}, {in_f}], got {tuple(Ht.shape)}")
    U, dead = factor if factor is not None else gptq_factor(Ht, damp)
    codes, scales = _sweep(Wt, U, dead, bits, group_size, block_size, signed_scale)
    wq = dequantize(codes, scales, bits, group_size, device=True)
    err = _err(wq, Wt, Ht)
    return {"codes": _out(codes, device), "scales": _out(scales, device), "w_q": _out(wq, device),
            "err": err if device else float(err.item())}


def quantize_rtn(W, bits, group_size=64, signed_scale=True, device=False):
    """Round-to-nearest with per-(row, group) signed scales (reference gptq.py:76-86): the
    GPTQ sweep with an identity factor, so no error is propagated."""
    _grid_bits(bits)
    Wt = _dev(W, torch.float32)
    out_f, in_f = Wt.shape
    U = torch.eye(in_f, device=Wt.device, dtype=torch.float64)
    dead = torch.zeros(in_f, device=Wt.device, dtype=torch.uint8)
    codes, scales = _sweep(Wt, U, dead, bits, group_size, 128, signed_scale)
    wq = dequantize(codes, scales, bits, group_size, device=True)
    return {"codes": _out(codes, device), "scales": _out(scales, device), "w_q": _out(wq, device)}


# ------------------------------------------------------------------ App-A inits (host) ---

def _app_a_logits(base, alpha, std, seed):
    """Eq. 4 of the GSQ paper's App. A: std (N(0, 1) + alpha (base - its mean over the
    candidates)), the normals one default_rng(seed) draw of base's shape; float32 [d, K]."""
    centred = base - base.mean(axis=-1, keepdims=True)
    normals = np.random.default_rng(seed).standard_normal(base.shape).astype(np.float32)
    return (std * (normals + alpha * centred)).astype(np.float32)


def init_logits_2bit_from_codes(codes, K, alpha=6.0, std=0.01, seed=0):
    """2-bit full grid (reference gptq.py:202-210): the base of weight i at grid level k is
    -(k - q_i)^2 / 2, peaked at its GPTQ code q_i. [d, K]."""
    q = np.asarray(codes).reshape(-1, 1).astype(np.float32)
    levels = np.arange(K, dtype=np.float32)[None, :]
    return _app_a_logits(-0.5 * np.square(levels - q), alpha, std, seed)


def init_shift_logits(numel, alpha=6.0, std=0.01, seed=0):
    """Local shift (reference gptq.py:213-219): every weight's base over the shifts -2..2 is
    -shift^2 / 2, peaked at the GPTQ code itself. [d, 5]."""
    shifts = np.arange(-2, 3, dtype=np.float32)
    base = np.broadcast_to(-0.5 * np.square(shifts), (int(numel), shifts.size))
    return _app_a_logits(base, alpha, std, seed)


def init_ternary_logits(q_gptq, alpha=3.0, std=0.01, seed=0):
    """Ternary mask and sign logits (reference gptq.py:222-232), each std (N(0,1) + alpha base):
    the mask base is +1 where the GPTQ value is kept and -1 where it is pruned, the sign base is
    sign(q); the mask's normals are drawn first. Returns (lm, lb), float32 [d]."""
    q = np.asarray(q_gptq).reshape(-1)
    rng = np.random.default_rng(seed)
    normals = [rng.standard_normal(q.shape).astype(np.float32) for _ in range(2)]
    bases = (np.where(q != 0, 1.0, -1.0), np.sign(q))
    return tuple((std * (e + alpha * b.astype(np.float32))).astype(np.float32)
                 for e, b in zip(normals, bases))
