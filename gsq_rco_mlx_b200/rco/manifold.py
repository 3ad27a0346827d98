"""RCO budget manifold (host, float64) and the multiple-choice knapsack decode (GPU).

The public functions keep the names, arguments, return values and exception types of the
reference module src/gsq_rco/rco/manifold.py; the code is this package's own.

Continuous part. For logits a [N, K], option costs c [K] and group weights w [N], the budget
manifold is {a : C(a) = B} with C(a) = sum_i w_i <softmax(a_i), c> (manifold.py:71-85, Eq. 1).
``Budget`` evaluates C, its normal and its slope along the cost direction for one (c, w); the
module functions wrap it. ``retract`` moves a along c onto the manifold. C(a + t c) is
nondecreasing in t with derivative sum_i w_i Var_{p_i(t)}[c], so the shift is found by Newton
steps on that derivative, kept inside a sign-change bracket (bisection whenever a Newton step
would leave it). Any shift with |C - B| <= tol is a valid retraction (manifold.py:146-207); this
one converges in a handful of cost evaluations instead of a long bisection.

Discrete part. ``dp_knapsack`` checks the problem on the host and solves the O(N K B') table in
the CUDA kernel ``mckp_dp_f64`` (one CTA per instance, bit-exact with manifold.py:304-334);
``dp_knapsack_batch`` decodes several score matrices in one launch; ``topk_2option`` is the
exact K = 2 decode for uniform weights (manifold.py:244-301).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _lib

RETRACT_TOL = 1e-8
RETRACT_MAX_SHIFT = 1e6
_DP_SMEM_BUDGET = 13823
_MAX_OPTIONS = 255


# ------------------------------------------------------------------ continuous ops ---

def softmax(a):
    """Row-wise softmax of a float64 [N, K] array."""
    x = np.asarray(a, dtype=np.float64)
    e = np.exp(x - np.max(x, axis=1, keepdims=True))
    return e / np.sum(e, axis=1, keepdims=True)


class Budget:
    """Costs c [K] and group weights w [N] of one budget manifold, in float64."""

    def __init__(self, costs, weights):
        self.c = np.asarray(costs, dtype=np.float64).reshape(-1)
        self.w = np.asarray(weights, dtype=np.float64).reshape(-1)

    def reachable(self):
        """(lowest, highest) expected cost: every group on its cheapest / dearest option."""
        total = float(np.sum(self.w))
        return total * float(np.min(self.c)), total * float(np.max(self.c))

    def _moments(self, a):
        p = softmax(a)
        mean = p @ self.c                       # E_{p_i}[c]
        return p, mean

    def cost(self, a) -> float:
        _, mean = self._moments(a)
        return float(np.dot(self.w, mean))

    def normal(self, a):
        """n_ik = w_i p_ik (c_k - E_{p_i}[c]) (Eq. 2)."""
        p, mean = self._moments(a)
        return self.w[:, None] * p * (self.c[None, :] - mean[:, None])

    def cost_and_slope(self, a):
        """C(a) and d/dt C(a + t c) at t = 0, i.e. sum_i w_i Var_{p_i}[c]."""
        p, mean = self._moments(a)
        second = p @ (self.c * self.c)
        var = np.maximum(second - mean * mean, 0.0)
        return float(np.dot(self.w, mean)), float(np.dot(self.w, var))


def expected_cost(logits, costs, weights):
    """C(a) = sum_i w_i <softmax(a_i), c> (Eq. 1), a Python float."""
    return Budget(costs, weights).cost(logits)


def normal_vector(logits, costs, weights):
    """Normal of the budget manifold at a: n_ik = w_i p_ik (c_k - E_{p_i}[c]) (Eq. 2)."""
    return Budget(costs, weights).normal(logits)


def project_tangent(grad, normal):
    """Remove the normal component: g - (<g, n> / (||n||^2 + 1e-12)) n."""
    g = np.asarray(grad, dtype=np.float64)
    n = np.asarray(normal, dtype=np.float64)
    coef = float(np.vdot(g, n)) / (float(np.vdot(n, n)) + 1e-12)
    return g - coef * n


def transport(m, normal_new):
    """Carry the first moment to the tangent plane at the new point (a projection)."""
    return project_tangent(m, normal_new)


def retract(logits, costs, weights, budget, lo=-50.0, hi=50.0, iters=200, tol=None,
            max_shift=RETRACT_MAX_SHIFT):
    """Return a + t c with |C(a + t c) - B| <= tol (default 1e-8).

    lo, hi: the first guesses of a bracket of t; it grows (doubling its reach) until the cost
    changes sign across it, up to |t| <= max_shift. Raises ValueError when B is outside the
    reachable costs or no bracket is found, RuntimeError when ``iters`` safeguarded Newton
    steps do not reach the tolerance."""
    bud = Budget(costs, weights)
    target = float(budget)
    low, high = bud.reachable()
    if target < low - 1e-9 or target > high + 1e-9:
        raise ValueError(f"retract: budget {target} cannot be met, the expected cost ranges "
                         f"over [{low}, {high}]")
    eps = RETRACT_TOL if tol is None else float(tol)
    a = np.asarray(logits, dtype=np.float64)

    def resid(t):
        cst, slope = bud.cost_and_slope(a + t * bud.c[None, :])
        return cst - target, slope

    t, (f, d) = 0.0, resid(0.0)
    if abs(f) <= eps:
        return a + 0.0 * bud.c[None, :]
    # a bracket [t_neg, t_pos] with resid(t_neg) <= 0 <= resid(t_pos), searched over
    # |t| <= max_shift with a reach that doubles from the first guess lo (or hi)
    limit = float(max_shift)
    if f > 0:
        t_pos, f_pos = 0.0, f
        reach = min(max(abs(float(lo)), 1.0), limit)
        while True:
            t_neg = -reach
            f_neg, _ = resid(t_neg)
            if f_neg <= 0:
                break
            if reach >= limit:
                raise ValueError(f"retract: no shift t >= -{limit:g} lowers the cost to "
                                 f"{target}")
            reach = min(2.0 * reach, limit)
    else:
        t_neg, f_neg = 0.0, f
        reach = min(max(abs(float(hi)), 1.0), limit)
        while True:
            t_pos = reach
            f_pos, _ = resid(t_pos)
            if f_pos >= 0:
                break
            if reach >= limit:
                raise ValueError(f"retract: no shift t <= {limit:g} raises the cost to "
                                 f"{target}")
            reach = min(2.0 * reach, limit)
    for end_t, end_f in ((t_neg, f_neg), (t_pos, f_pos)):
        if abs(end_f) <= eps:
            return a + end_t * bud.c[None, :]
    best = min(abs(f_neg), abs(f_pos))
    for _ in range(int(iters)):
        t_new = t - f / d if d > 0.0 else np.nan
        if not (t_neg < t_new < t_pos):
            t_new = 0.5 * (t_neg + t_pos)
            if not (t_neg < t_new < t_pos):
                break  # the bracket is one float wide
        t = t_new
        f, d = resid(t)
        best = min(best, abs(f))
        if abs(f) <= eps:
            return a + t * bud.c[None, :]
        if f < 0:
            t_neg = t
        else:
            t_pos = t
    raise RuntimeError(f"retract: |C - B| stayed above {eps:.3g} (closest {best:.3g}) after "
                       f"{iters} steps")


# ------------------------------------------------------------------ discrete decode ---

def assignment_value(z, scores) -> float:
    """sum_ik z_ik s_ik of a one-hot assignment."""
    return float(np.sum(np.asarray(z) * np.asarray(scores)))


def assignment_cost(z, costs_int, weights_int) -> int:
    """sum_i w_i c_{k(i)} of a one-hot assignment, an exact integer."""
    per_group = np.asarray(z) @ np.asarray(costs_int).reshape(-1)
    return int(np.rint(np.dot(per_group, np.asarray(weights_int).reshape(-1))))


def _as_ints(x, what):
    """int64 vector of x; floats are accepted only when they hold whole numbers."""
    v = np.asarray(x).reshape(-1)
    if v.dtype.kind in "biu":
        return v.astype(np.int64)
    whole = v.dtype.kind == "f" and bool(np.all(np.isfinite(v))) and bool(np.all(v == np.floor(v)))
    if not whole:
        raise ValueError(f"{what}: expected whole numbers (nothing is rounded), got {v.tolist()}")
    return v.astype(np.int64)


def _as_int(x, what):
    v = _as_ints(x, what)
    if v.size != 1:
        raise ValueError(f"{what}: expected one number, got {v.size}")
    return int(v[0])


def _problem(scores, costs_int, weights_int, budget_int, n_options=None):
    """Checked (scores [N, K] float64, costs [K], weights [N], budget) of one decode."""
    s = np.asarray(scores, dtype=np.float64)
    if s.ndim != 2 or 0 in s.shape:
        raise ValueError(f"scores: expected a non-empty [N, K] array, got shape {s.shape}")
    if n_options is not None and s.shape[1] != n_options:
        raise ValueError(f"scores: expected {n_options} options per group, got {s.shape[1]}")
    if not np.isfinite(s).all():
        raise ValueError("scores: every entry must be finite")
    n, k = s.shape
    if k > _MAX_OPTIONS:
        raise ValueError(f"scores: at most {_MAX_OPTIONS} options per group, got {k}")
    c = _as_ints(costs_int, "costs_int")
    w = _as_ints(weights_int, "weights_int")
    b = _as_int(budget_int, "budget_int")
    if c.shape != (k,):
        raise ValueError(f"costs_int: expected {k} costs, got {c.size}")
    if w.shape != (n,):
        raise ValueError(f"weights_int: expected {n} weights, got {w.size}")
    if b < 0 or (c < 0).any() or (w < 0).any():
        raise ValueError("costs_int, weights_int and budget_int must be >= 0")
    floor = int(np.sum(w) * np.min(c))
    if floor > b:
        raise ValueError(f"infeasible: even the cheapest assignment costs {floor}, "
                         f"above the budget {b}")
    return s, c, w, b


def topk_2option(scores, costs_int, weights_int, budget_int, exact_count=False):
    """Exact decode of K = 2 options with one weight for every group.

    Every group starts on its cheaper option; the budget left over pays for n upgrades of
    w (c_dear - c_cheap) each. The upgrades go to the largest score gains (ties to the lower
    group index), and only to positive gains unless ``exact_count`` asks for exactly n."""
    s, c, w, b = _problem(scores, costs_int, weights_int, budget_int, n_options=2)
    if (w != w[0]).any():
        raise ValueError("topk_2option: group weights differ; dp_knapsack handles that case")
    cheap = 0 if c[0] <= c[1] else 1
    dear = 1 - cheap
    n_groups = s.shape[0]
    z = np.zeros((n_groups, 2))
    upgrade = int(w[0]) * int(c[dear] - c[cheap])
    if upgrade == 0:
        if exact_count:
            raise ValueError("topk_2option: exact_count needs options of different cost")
        z[np.arange(n_groups), np.argmax(s, axis=1)] = 1.0
        return z
    spare = b - n_groups * int(w[0]) * int(c[cheap])
    n_up = min(spare // upgrade, n_groups)
    gain = s[:, dear] - s[:, cheap]
    rank = np.lexsort((np.arange(n_groups), -gain))   # by gain, then by group index
    if not exact_count:
        rank = rank[gain[rank] > 0]
    chosen = np.zeros(n_groups, dtype=bool)
    chosen[rank[:n_up]] = True
    z[:, cheap] = ~chosen
    z[:, dear] = chosen
    return z


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
    indices [n_inst, N] (CUDA tensor; -1 in every entry of an instance that has no feasible
    assignment or a negative step)."""
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
        raise ValueError(f"scores: expected [n_inst, N, K], got shape {S.shape}")
    for s in S:
        _, c, w, B = _problem(s, costs_int, weights_int, budget_int)
    n_inst, N, K = S.shape
    if K == 1:
        return np.ones((n_inst, N, 1))
    dev = _lib.device()
    st = torch.as_tensor(np.ascontiguousarray(S), device=dev)
    step = torch.as_tensor(np.ascontiguousarray(w[:, None] * c[None, :]), device=dev)
    zi = mckp_dp_device(st, step, B).cpu().numpy()
    if (zi < 0).any():
        raise RuntimeError("mckp_dp_f64 found no feasible assignment for a checked problem")
    z = np.zeros((n_inst, N, K))
    np.put_along_axis(z, zi[..., None].astype(np.int64), 1.0, axis=2)
    return z


def dp_knapsack(scores, costs_int, weights_int, budget_int, use_topk=True):
    """Multiple-choice knapsack (Eq. 4): one-hot z maximising sum z s subject to
    sum_i w_i c_{k(i)} <= B'. Ties: the lowest option wins inside the DP, and the cheapest
    optimum is returned. K = 2 with uniform weights uses topk_2option (use_topk=True)."""
    s, c, w, B = _problem(scores, costs_int, weights_int, budget_int)
    N, K = s.shape
    if K == 1:
        return np.ones((N, 1))
    if use_topk and K == 2 and (w == w[0]).all():
        return topk_2option(s, c, w, B)
    return dp_knapsack_batch(s[None], c, w, B)[0]
