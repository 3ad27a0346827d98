"""RCO budget manifold (host, float64) and the multiple-choice knapsack decode (GPU).

Same contract as the reference src/gsq_rco/rco/manifold.py. The continuous manifold math
(softmax, expected_cost Eq.1, normal_vector Eq.2, project_tangent, transport, retract by
bisection) works on [N, K] float64 arrays of a few hundred entries and stays on the host in
numpy, as in the reference. ``dp_knapsack`` validates on the host (the reference's exact
rules and messages) and runs the O(N K B') DP table in the CUDA kernel ``mckp_dp_f64``,
one CTA per instance; ``dp_knapsack_batch`` decodes several Gumbel samples in one launch.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _lib

RETRACT_TOL = 1e-8
RETRACT_MAX_SHIFT = 1e6
_DP_SMEM_BUDGET = 13823


# ------------------------------------------------------------------ continuous ops ---

def softmax(a):
    a = np.asarray(a, dtype=np.float64)
    e = np.exp(a - a.max(axis=1, keepdims=True))
    return e / e.sum(axis=1, keepdims=True)


def expected_cost(logits, costs, weights):
    """C(a) = sum_i w_i <softmax(a_i), c> (Eq.1)."""
    p = softmax(logits)
    c = np.asarray(costs, dtype=np.float64)
    w = np.asarray(weights, dtype=np.float64)
    return float((w[:, None] * p * c[None, :]).sum())


def normal_vector(logits, costs, weights):
    """n_ik = w_i p_ik (c_k - E_{p_i}[c]) (Eq.2)."""
    p = softmax(logits)
    c = np.asarray(costs, dtype=np.float64)
    w = np.asarray(weights, dtype=np.float64)
    mean_c = (p * c[None, :]).sum(axis=1, keepdims=True)
    return w[:, None] * p * (c[None, :] - mean_c)


def project_tangent(grad, normal):
    """g - (<g, n> / ||n||^2) n."""
    g = np.asarray(grad, dtype=np.float64)
    n = np.asarray(normal, dtype=np.float64)
    return g - (float((g * n).sum()) / (float((n * n).sum()) + 1e-12)) * n


def transport(m, normal_new):
    """First-moment transport onto the new tangent plane (projection)."""
    return project_tangent(m, normal_new)


def _feasible_range(costs, weights):
    c = np.asarray(costs, dtype=np.float64)
    w = np.asarray(weights, dtype=np.float64)
    return float(w.sum() * c.min()), float(w.sum() * c.max())


def _bracket(cost_at, budget, eps, lo, hi, max_shift):
    """Widen [lo, hi] geometrically until it brackets C(t) = B (C is nondecreasing in t)."""
    span = max(hi - lo, 1.0)
    while cost_at(lo) > budget + eps:
        hi, lo, span = lo, lo - 2.0 * span, 2.0 * span
        if abs(lo) > max_shift:
            raise ValueError(f"budget {budget} not bracketed for |t| <= {max_shift:g}")
    while cost_at(hi) < budget - eps:
        lo, hi, span = hi, hi + 2.0 * span, 2.0 * span
        if abs(hi) > max_shift:
            raise ValueError(f"budget {budget} not bracketed for |t| <= {max_shift:g}")
    return lo, hi


def retract(logits, costs, weights, budget, lo=-50.0, hi=50.0, iters=200, tol=None,
            max_shift=RETRACT_MAX_SHIFT):
    """Shift a -> a + t c with C(a + t c) = B by bisection (Prop.3), |C - B| <= tol (1e-8).
    Raises ValueError for an infeasible budget or an unbracketable root, RuntimeError if
    ``iters`` bisection steps do not reach the tolerance."""
    blo, bhi = _feasible_range(costs, weights)
    if not (blo - 1e-9 <= budget <= bhi + 1e-9):
        raise ValueError(f"budget {budget} outside feasible [{blo}, {bhi}] (sum w * min/max cost)")
    a = np.asarray(logits, dtype=np.float64)
    c = np.asarray(costs, dtype=np.float64)
    w = np.asarray(weights, dtype=np.float64)
    eps = RETRACT_TOL if tol is None else float(tol)

    def at(t):
        return expected_cost(a + t * c[None, :], c, w)

    lo_f, hi_f = _bracket(at, float(budget), eps, float(lo), float(hi), float(max_shift))
    res = float("inf")
    for _ in range(iters):
        mid = 0.5 * (lo_f + hi_f)
        if not lo_f < mid < hi_f:
            break
        cm = at(mid)
        res = abs(cm - float(budget))
        if res <= eps:
            return a + mid * c[None, :]
        if cm < budget:
            lo_f = mid
        else:
            hi_f = mid
    raise RuntimeError(f"retract: no shift reached |C-B| <= {eps:.3g} (best {res:.3g}) "
                       f"within {iters} steps or float resolution")


# ------------------------------------------------------------------ discrete decode ---

def assignment_value(z, scores) -> float:
    return float((np.asarray(z) * np.asarray(scores)).sum())


def assignment_cost(z, costs_int, weights_int) -> int:
    z = np.asarray(z)
    c = np.asarray(costs_int).reshape(-1)
    w = np.asarray(weights_int).reshape(-1)
    return int(((z * c[None, :]).sum(axis=1) * w).sum())


def _int_array(x, name):
    a = np.asarray(x).reshape(-1)
    if a.dtype.kind in "biu":
        return a.astype(np.int64)
    if a.dtype.kind != "f" or not np.all(np.isfinite(a)) or not np.all(a == np.round(a)):
        raise ValueError(f"{name} must be integer-valued, got {a.tolist()}")
    return a.astype(np.int64)


def _int_scalar(x, name):
    a = _int_array(x, name)
    if a.size != 1:
        raise ValueError(f"{name} must be a scalar, got {a.size} values")
    return int(a[0])


def topk_2option(scores, costs_int, weights_int, budget_int, exact_count=False):
    """Exact K = 2 decode with uniform weights: the n largest positive upgrade deltas."""
    s = np.asarray(scores, dtype=np.float64)
    if s.ndim != 2 or s.shape[1] != 2:
        raise ValueError(f"topk_2option needs scores [N,2], got {s.shape}")
    if not np.all(np.isfinite(s)):
        raise ValueError("scores must be finite")
    N = s.shape[0]
    c = _int_array(costs_int, "costs_int")
    w = _int_array(weights_int, "weights_int")
    B = _int_scalar(budget_int, "budget_int")
    if c.shape != (2,) or w.shape != (N,):
        raise ValueError("costs must be [2], weights [N]")
    if B < 0:
        raise ValueError("budget_int must be >= 0")
    if np.any(c < 0) or np.any(w < 0):
        raise ValueError("costs/weights must be nonneg ints")
    if np.any(w != w[0]):
        raise ValueError("topk_2option is exact only for uniform weights; use dp_knapsack")
    w0 = int(w[0])
    lo_k, hi_k = (0, 1) if c[0] <= c[1] else (1, 0)
    base = N * w0 * int(c[lo_k])
    if base > B:
        raise ValueError(f"infeasible: cheapest cost {base} > budget {B}")
    step = w0 * (int(c[hi_k]) - int(c[lo_k]))
    z = np.zeros((N, 2))
    if step == 0:
        if exact_count:
            raise ValueError("exact_count needs a nonzero cost step")
        z[np.arange(N), s.argmax(axis=1)] = 1.0
        return z
    n = min((B - base) // step, N)
    delta = s[:, hi_k] - s[:, lo_k]
    order = np.argsort(-delta, kind="stable")
    if not exact_count:
        order = order[delta[order] > 0]
    up = order[:n]
    z[:, lo_k] = 1.0
    z[up, lo_k] = 0.0
    z[up, hi_k] = 1.0
    return z


def _validate(scores, costs_int, weights_int, budget_int):
    s = np.asarray(scores, dtype=np.float64)
    if s.ndim != 2 or s.shape[0] < 1 or s.shape[1] < 1:
        raise ValueError(f"scores must be [N,K], got {s.shape}")
    if not np.all(np.isfinite(s)):
        raise ValueError("scores must be finite")
    N, K = s.shape
    if K > 255:
        raise ValueError("dp_knapsack supports at most 255 options per group")
    c = _int_array(costs_int, "costs_int")
    w = _int_array(weights_int, "weights_int")
    B = _int_scalar(budget_int, "budget_int")
    if c.shape != (K,) or w.shape != (N,):
        raise ValueError(f"costs must be [{K}], weights [{N}], got {c.shape}/{w.shape}")
    if B < 0:
        raise ValueError("budget_int must be >= 0")
    if np.any(c < 0) or np.any(w < 0):
        raise ValueError("costs/weights must be nonneg ints")
    cheapest = int((w * c.min()).sum())
    if cheapest > B:
        raise ValueError(f"infeasible: cheapest cost {cheapest} > budget {B}")
    return s, c, w, B


class DPWorkspace:
    """Device buffers of the DP (choice table, rows when they do not fit shared memory),
    grown on demand and reused across calls."""

    def __init__(self):
        self.choice = None
        self.rows = None

    def get(self, n_inst, N, B, dev):
        need = n_inst * N * (B + 1)
        if self.choice is None or self.choice.numel() < need or self.choice.device != dev:
            self.choice = torch.empty(need, device=dev, dtype=torch.uint8)
        rows = None
        if B > _DP_SMEM_BUDGET:
            need_r = n_inst * 2 * (B + 1)
            if self.rows is None or self.rows.numel() < need_r or self.rows.device != dev:
                self.rows = torch.empty(need_r, device=dev, dtype=torch.float64)
            rows = self.rows
        return self.choice, rows


_WS = DPWorkspace()


def mckp_dp_device(scores_t, step_t, budget, workspace=None):
    """DP on device tensors: scores [n_inst, N, K] float64, step [N, K] int64 -> int32 choice
    indices [n_inst, N] (CUDA tensor)."""
    n_inst, N, K = scores_t.shape
    ws = workspace or _WS
    choice, rows = ws.get(n_inst, N, int(budget), scores_t.device)
    z = torch.empty(n_inst, N, device=scores_t.device, dtype=torch.int32)
    _lib.call("mckp_dp_f64", _lib.ptr(scores_t), _lib.ptr(step_t), n_inst, N, K, int(budget),
              _lib.ptr(choice), _lib.ptr(rows), _lib.ptr(z), _lib.stream_ptr())
    return z


def dp_knapsack_batch(scores, costs_int, weights_int, budget_int):
    """DP decode of several score matrices [n_inst, N, K] sharing costs, weights and budget.
    Returns one-hot z [n_inst, N, K] (float64), as dp_knapsack per instance with the full DP."""
    S = np.asarray(scores, dtype=np.float64)
    if S.ndim != 3:
        raise ValueError(f"scores must be [n_inst, N, K], got {S.shape}")
    for s in S:
        _, c, w, B = _validate(s, costs_int, weights_int, budget_int)
    n_inst, N, K = S.shape
    if K == 1:
        return np.ones((n_inst, N, 1))
    dev = _lib.device()
    st = torch.as_tensor(np.ascontiguousarray(S), device=dev)
    step = torch.as_tensor(np.ascontiguousarray(w[:, None] * c[None, :]), device=dev)
    zi = mckp_dp_device(st, step, B).cpu().numpy()
    z = np.zeros((n_inst, N, K))
    np.put_along_axis(z, zi[..., None].astype(np.int64), 1.0, axis=2)
    return z


def dp_knapsack(scores, costs_int, weights_int, budget_int, use_topk=True):
    """Multiple-choice knapsack (Eq.4): one-hot z maximising sum z * s subject to
    sum_i w_i c_{k(i)} <= B'. Ties: the lowest option wins inside the DP, and the cheapest
    optimum is returned. K = 2 with uniform weights uses topk_2option (use_topk=True)."""
    s, c, w, B = _validate(scores, costs_int, weights_int, budget_int)
    N, K = s.shape
    if K == 1:
        return np.ones((N, 1))
    if use_topk and K == 2 and np.all(w == w[0]):
        return topk_2option(s, c, w, B)
    return dp_knapsack_batch(s[None], c, w, B)[0]
