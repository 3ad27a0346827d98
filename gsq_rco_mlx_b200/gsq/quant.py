"""Grid, schedules and local-shift helpers (host side, numpy).

Same contract as the reference src/gsq_rco/gsq/quant.py: get_grid (:38-46), gs_schedules
(:51-61), local_shift_indices (:75-83), local_shift_values (:86-108). These are tiny host
computations; the per-weight versions run inside the CUDA kernels.
"""
from __future__ import annotations

import numpy as np

TAU_START, TAU_END = 2.0, 0.05
KAPPA_START, KAPPA_END = 100.0, 500.0
SHIFT_DELTAS = (-2, -1, 0, 1, 2)
N_SHIFTS = len(SHIFT_DELTAS)


def get_grid(n_bits: int, kind: str = "uniform") -> np.ndarray:
    """Symmetric uniform grid: arange(2^b) - 2^(b-1); 1 bit is the ternary [-1, 0, 1]."""
    if n_bits == 1:
        return np.array([-1.0, 0.0, 1.0], dtype=np.float32)
    k = 2 ** n_bits
    return np.arange(k, dtype=np.float32) - (k // 2)


def linear_schedule(t: int, T: int, start: float, end: float) -> float:
    return start + (end - start) * min(1.0, t / max(1, T - 1))


def gs_schedules(t: int, T: int, tau=(TAU_START, TAU_END), kappa=(KAPPA_START, KAPPA_END)):
    """tau linear 2 -> 0.05 and kappa linear 100 -> 500 over T steps."""
    return (linear_schedule(t, T, tau[0], tau[1]), linear_schedule(t, T, kappa[0], kappa[1]))


def local_shift_indices(j0, shift_logits, n_levels: int):
    """j = clip(j0 + argmax_k l - 2, 0, n_levels - 1); shift_logits is [d, 5]."""
    delta = np.asarray(shift_logits).argmax(axis=-1) - 2
    return np.clip(np.asarray(j0) + delta, 0, n_levels - 1)


def local_shift_values(j0, grid):
    """Candidate table C[d, 5]: C[i, k] = grid[clip(j0[i] + k - 2)]."""
    g = np.asarray(grid, dtype=np.float32)
    jk = np.clip(np.asarray(j0)[:, None] + (np.arange(N_SHIFTS) - 2)[None, :], 0, len(g) - 1)
    return g[jk]
