"""CPU restatement of the packed-weight export format and the quantized-model eval (test
infrastructure only: tests/, the smoke check and the bench's CPU baseline use it).

pack_codes / unpack_codes follow src/gsq_rco/gsq/export.py:61-73 bit by bit: value j of a row
occupies stream bits [j b, (j + 1) b), least significant bit first, the stream read as
little-endian 32-bit words. Pinned to the reference's own pack_codes by golden vectors
(tests/golden/export.npz, made by tests/golden/make_golden.py). dequant follows export.py:13-19
and :85-91 (w = scale q + bias with bias = -2^(b-1) scale; ternary as 2-bit q = c + 1), rounded
to bf16: the dense weights of the bf16-dequantized model. model_nll follows
src/gsq_rco/common/evaluate.py:35-78 (windows fed as tokens[:-1], scored against tokens[1:],
logsumexp(z) - z[target] of the bf16 head logits) through oracle.block.block_hard, the
restatement of the reference block (src/gsq_rco/gsq/e2e.py:160-174) that stands in for mlx-lm's
Qwen2 forward. Sums in float64.
"""
from __future__ import annotations

import numpy as np
import torch

from .block import bf, block_hard, rmsnorm

F32, F64 = torch.float32, torch.float64


def grid(bits):
    """quant.get_grid (src/gsq_rco/gsq/quant.py:38-46): ternary [-1, 0, 1], else
    arange(2^b) - 2^(b-1)."""
    if bits == 1:
        return np.array([-1.0, 0.0, 1.0])
    return np.arange(1 << bits, dtype=np.float64) - (1 << (bits - 1))


def pack_codes(codes, bits):
    """uint8 [out, in] -> uint32 [out, in bits / 32], one stream bit at a time."""
    codes = np.asarray(codes, dtype=np.uint64)
    out_f, in_f = codes.shape
    if (in_f * bits) % 32:
        raise ValueError("not a whole number of words")
    words = np.zeros((out_f, in_f * bits // 32), dtype=np.uint64)
    for j in range(in_f):
        for t in range(bits):
            pos = j * bits + t
            words[:, pos // 32] |= ((codes[:, j] >> np.uint64(t)) & np.uint64(1)) << \
                np.uint64(pos % 32)
    return words.astype(np.uint32)


def unpack_codes(words, bits, in_f):
    """uint32 [out, in bits / 32] -> uint8 [out, in], one stream bit at a time."""
    w = np.asarray(words, dtype=np.uint64)
    out = np.zeros((w.shape[0], in_f), dtype=np.uint64)
    for j in range(in_f):
        for t in range(bits):
            pos = j * bits + t
            out[:, j] |= ((w[:, pos // 32] >> np.uint64(pos % 32)) & np.uint64(1)) << np.uint64(t)
    return out.astype(np.uint8)


def mlx_bits(bits):
    return 2 if bits == 1 else bits


def affine(codes, scales, bits, scale_dtype=torch.bfloat16):
    """(q, scale, bias) of the MLX affine form, scale / bias rounded to scale_dtype and returned
    as float64 values per group."""
    q = np.asarray(codes, dtype=np.int64) + (1 if bits == 1 else 0)
    s = torch.as_tensor(np.asarray(scales, dtype=np.float32))
    b = torch.as_tensor(np.float32(-(1 << (mlx_bits(bits) - 1))) * np.asarray(scales, np.float32))
    return q, s.to(scale_dtype).to(F64).numpy(), b.to(scale_dtype).to(F64).numpy()


def affine_weight(codes, scales, bits, group_size=64, scale_dtype=torch.bfloat16):
    """The unrounded weight scale q + bias (float64) with scale / bias in the export dtype: what
    MLX's quantized matrix-vector product multiplies by (export.py:13-19)."""
    q, s, b = affine(codes, scales, bits, scale_dtype)
    gid = np.arange(q.shape[1]) // group_size
    return torch.as_tensor(s[:, gid] * q + b[:, gid])


def dequant(codes, scales, bits, group_size=64, scale_dtype=torch.bfloat16):
    """Dense bf16 weight (float32 values) of native codes / scales after the affine export:
    bf16(scale q + bias) with scale / bias in the export dtype."""
    q, s, b = affine(codes, scales, bits, scale_dtype)
    gid = np.arange(q.shape[1]) // group_size
    w = s[:, gid] * q + b[:, gid]              # exact in float64
    return bf(torch.as_tensor(w).to(F32))


def nll_rows(z, targets):
    """logsumexp(z) - z[t] per row of float logits z [n, V] (float64); t < 0: 0."""
    z = torch.as_tensor(z).to(F64)
    t = torch.as_tensor(np.asarray(targets, dtype=np.int64))
    lse = torch.logsumexp(z, -1)
    picked = z.gather(1, t.clamp(min=0)[:, None])[:, 0]
    return torch.where(t >= 0, lse - picked, torch.zeros_like(lse))


def model_nll(embed, layers, norm, windows, n_heads, n_kv, eps=1e-6):
    """(summed NLL float64, tokens scored) of windows [N, S] under the dense bf16 model:
    embed bf16 [V, H], layers [{name: tensor}] (oracle.block.block_hard's keys), norm [H]."""
    E = embed.to(F32)
    total, n = 0.0, 0
    for win in np.asarray(windows):
        x = torch.as_tensor(win[:-1].astype(np.int64))
        h = E[x]
        for W in layers:
            h, _ = block_hard(h, W, n_heads, n_kv, eps)
        hn = rmsnorm(h, norm, eps)
        z = bf(hn.to(F64) @ E.to(F64).T)
        total += float(nll_rows(z, win[1:]).sum())
        n += len(win) - 1
    return total, n
