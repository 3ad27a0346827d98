"""Exact multiple-choice knapsack DP and the RCO host math: CPU restatement (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows the reference egesabanci/gsq-rco-mlx src/gsq_rco/rco/manifold.py:
  _mckp_dp     :304-334  dp[b] = best value with cost <= b; strict '>' keeps the lowest option;
                         backtrack from the smallest budget that reaches dp[B]
  dp_knapsack  :337-380  validation, K == 1, and the K == 2 uniform-weight top-k shortcut
  topk_2option :244-301
The C restatement oracle/dp.c computes the same table with the same float64 operations and is
the timed CPU baseline of the DP.
"""
from __future__ import annotations

import numpy as np


def mckp_dp(s, step, budget):
    """manifold.py:304-334: s [N, K] float64 scores, step [N, K] integer costs, budget B."""
    s = np.asarray(s, dtype=np.float64)
    step = np.asarray(step, dtype=np.int64)
    N, K = s.shape
    B = int(budget)
    dp = np.zeros(B + 1)
    choice = np.zeros((N, B + 1), dtype=np.uint8)
    for i in range(N):
        new = np.full(B + 1, -np.inf)
        for k in range(K):
            c = int(step[i, k])
            if c > B:
                continue
            cand = dp[:B + 1 - c] + s[i, k]
            tgt = new[c:]
            better = cand > tgt
            tgt[better] = cand[better]
            choice[i, c:][better] = k
        dp = new
    b = int(np.argmax(dp >= dp[B]))
    z = np.zeros((N, K))
    for i in range(N - 1, -1, -1):
        k = int(choice[i, b])
        z[i, k] = 1.0
        b -= int(step[i, k])
    return z


def int_array(x, name):
    """manifold.py:226-234: integer-valued arrays only; rounding is refused."""
    a = np.asarray(x).reshape(-1)
    if a.dtype.kind in "biu":
        return a.astype(np.int64)
    if a.dtype.kind != "f" or not np.all(np.isfinite(a)) or not np.all(a == np.round(a)):
        raise ValueError(f"{name} must be integer-valued, got {a.tolist()}")
    return a.astype(np.int64)


def topk_2option(s, c, w, B):
    """manifold.py:244-301 with exact_count=False."""
    N = s.shape[0]
    w0 = int(w[0])
    lo_k, hi_k = (0, 1) if c[0] <= c[1] else (1, 0)
    base = N * w0 * int(c[lo_k])
    if base > B:
        raise ValueError(f"infeasible: cheapest cost {base} > budget {B}")
    step = w0 * (int(c[hi_k]) - int(c[lo_k]))
    z = np.zeros((N, 2))
    if step == 0:
        z[np.arange(N), s.argmax(axis=1)] = 1.0
        return z
    n = min((B - base) // step, N)
    delta = s[:, hi_k] - s[:, lo_k]
    order = np.argsort(-delta, kind="stable")
    order = order[delta[order] > 0]
    up = order[:n]
    z[:, lo_k] = 1.0
    z[up, lo_k] = 0.0
    z[up, hi_k] = 1.0
    return z


def dp_knapsack(scores, costs_int, weights_int, budget_int, use_topk=True):
    """manifold.py:337-380."""
    s = np.asarray(scores, dtype=np.float64)
    if s.ndim != 2 or s.shape[0] < 1 or s.shape[1] < 1:
        raise ValueError(f"scores must be [N,K], got {s.shape}")
    if not np.all(np.isfinite(s)):
        raise ValueError("scores must be finite")
    N, K = s.shape
    if K > 255:
        raise ValueError("dp_knapsack supports at most 255 options per group")
    c = int_array(costs_int, "costs_int")
    w = int_array(weights_int, "weights_int")
    B = int_array(budget_int, "budget_int")
    if B.size != 1:
        raise ValueError("budget_int must be a scalar")
    B = int(B[0])
    if c.shape != (K,) or w.shape != (N,):
        raise ValueError(f"costs must be [{K}], weights [{N}]")
    if B < 0:
        raise ValueError("budget_int must be >= 0")
    if np.any(c < 0) or np.any(w < 0):
        raise ValueError("costs/weights must be nonneg ints")
    if int((w * c.min()).sum()) > B:
        raise ValueError("infeasible: cheapest cost exceeds the budget")
    if K == 1:
        return np.ones((N, 1))
    if use_topk and K == 2 and np.all(w == w[0]):
        return topk_2option(s, c, w, B)
    return mckp_dp(s, w[:, None] * c[None, :], B)
