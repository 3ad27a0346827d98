"""Philox4x32-10 counter-based generator and the Gumbel noise built on it (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The reference draws Gumbel noise from MLX's key-split generator
(src/gsq_rco/gsq/staged.py:92-96, keys from staged.py:384 and :279-280). That bit
stream is not reproducible without MLX, so the B200 build draws from Philox4x32-10
(Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers: As Easy as 1, 2, 3", SC'11),
whose counters make the noise of weight i a pure function of (seed, linear, step,
resample, i). The noise transform is the reference's: u clipped to [1e-7, 1-1e-7],
g = -log(-log u) in float32 (staged.py:95-96).

Counter / key assignment (the CUDA kernels use the same):
  key     = (seed_lo32, seed_hi32 ^ linear_id)
  counter = (i, 0, step, resample)       one Philox call per weight and draw, x0..x3
  bits    = plane k < 4: x_k >> 8;  plane 4: (x0 & 255) | (x1 & 255) << 8 | (x2 & 255) << 16
  u       = (bits + 0.5) * 2^-24         (24 random bits, strictly inside (0, 1))
"""
from __future__ import annotations

import numpy as np

PHILOX_M0 = np.uint64(0xD2511F53)
PHILOX_M1 = np.uint64(0xCD9E8D57)
PHILOX_W0 = np.uint32(0x9E3779B9)
PHILOX_W1 = np.uint32(0xBB67AE85)
MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Ten Philox4x32 rounds on uint32 arrays (broadcastable). Returns four uint32 arrays."""
    c0 = np.asarray(c0, dtype=np.uint32)
    c1 = np.broadcast_to(np.asarray(c1, dtype=np.uint32), c0.shape).copy()
    c2 = np.broadcast_to(np.asarray(c2, dtype=np.uint32), c0.shape).copy()
    c3 = np.broadcast_to(np.asarray(c3, dtype=np.uint32), c0.shape).copy()
    c0 = c0.copy()
    k0 = np.uint32(k0)
    k1 = np.uint32(k1)
    with np.errstate(over="ignore"):
        for rnd in range(10):
            p0 = PHILOX_M0 * c0.astype(np.uint64)
            p1 = PHILOX_M1 * c2.astype(np.uint64)
            hi0 = (p0 >> np.uint64(32)).astype(np.uint32)
            lo0 = (p0 & MASK32).astype(np.uint32)
            hi1 = (p1 >> np.uint64(32)).astype(np.uint32)
            lo1 = (p1 & MASK32).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
            if rnd < 9:
                k0 = np.uint32(k0 + PHILOX_W0)
                k1 = np.uint32(k1 + PHILOX_W1)
    return c0, c1, c2, c3


def uniform_from_bits(x):
    """24-bit uniform in (0, 1), float32, from the high 24 bits: ((x >> 8) + 0.5) * 2^-24."""
    x = np.asarray(x, dtype=np.uint32)
    return uniform_from_24(x >> np.uint32(8))


def uniform_from_24(b):
    """(b + 0.5) * 2^-24 in float32 for 24-bit integers b."""
    return (np.asarray(b, dtype=np.uint32).astype(np.float32) + np.float32(0.5)) * \
        np.float32(2.0 ** -24)


def gumbel_from_uniform(u):
    """Reference transform (staged.py:95-96): clip to [1e-7, 1-1e-7], then -log(-log u), float32."""
    u = np.clip(np.asarray(u, dtype=np.float32), np.float32(1e-7), np.float32(1.0 - 1e-7))
    return -np.log(-np.log(u))


def gumbel_planes(seed: int, linear_id: int, step: int, resample: int, d: int, n_planes: int):
    """Gumbel noise [n_planes, d] float32 for one soft-weight draw (plane-major layout)."""
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    k0 = seed & 0xFFFFFFFF
    k1 = ((seed >> 32) ^ int(linear_id)) & 0xFFFFFFFF
    i = np.arange(d, dtype=np.uint32)
    out = np.empty((n_planes, d), dtype=np.float32)
    x = philox4x32_10(i, 0, step, resample, k0, k1)
    for k in range(min(4, n_planes)):
        out[k] = gumbel_from_uniform(uniform_from_bits(x[k]))
    if n_planes > 4:
        lo = (x[0] & np.uint32(255)) | ((x[1] & np.uint32(255)) << np.uint32(8)) | \
             ((x[2] & np.uint32(255)) << np.uint32(16))
        out[4] = gumbel_from_uniform(uniform_from_24(lo))
    return out
