"""RCO loop (paper Alg.1) on the host, decoding on the GPU (reference src/gsq_rco/rco/loop.py).

One step: g Gumbel samples of the logits, h = (a + G) / tau, z = DP(h) (CUDA kernel), the
straight-through gradient p (v - <p, v>) / tau at the same perturbed softmax, projection on
the budget manifold's tangent plane, an Adam step, bisection retraction and momentum
transport. The [N, K] float64 state is a few hundred numbers and stays in numpy, as in the
reference; the random stream is the reference's numpy Generator, consumed in the same order
(Gumbel draw, then grad_fn).
"""
from __future__ import annotations

import numpy as np

from .manifold import (assignment_cost, assignment_value, dp_knapsack, expected_cost,
                       normal_vector, project_tangent, retract, softmax, transport)

TAU0, TAU_MIN = 1.0, 0.01
G_DEFAULT = 4
LR_DEFAULT = 0.1
ADAM_BETAS = (0.9, 0.999)
ADAM_EPS = 1e-8


def tau_schedule(t, T, tau0=TAU0, tau_min=TAU_MIN):
    """tau_t = max(tau_min, tau0 (tau_min / tau0)^(t / (T - 1)))."""
    if T <= 1:
        return float(tau_min)
    frac = min(max(t, 0), T - 1) / (T - 1)
    return max(float(tau_min), float(tau0) * (float(tau_min) / float(tau0)) ** frac)


def sample_gumbel(shape, rng=None, key=None):
    """Gumbel(0, 1) from the numpy Generator: -log(-log(clip(u, 1e-12, 1 - 1e-12)))."""
    r = rng or np.random.default_rng(0)
    u = r.random(tuple(shape)).astype(np.float64)
    return -np.log(-np.log(np.clip(u, 1e-12, 1 - 1e-12)))


def perturbed_logits(logits, gumbel, tau):
    return (logits + gumbel) / max(float(tau), 1e-6)


def soft_probs(h):
    return softmax(h)


def ste_grad(upstream, p, tau):
    """p (v - <p, v>) / tau, the softmax Jacobian applied to the upstream gradient."""
    tau = max(float(tau), 1e-6)
    up = np.asarray(upstream, dtype=np.float64)
    pp = np.asarray(p, dtype=np.float64)
    return (pp * (up - (pp * up).sum(axis=1, keepdims=True))) / tau


def to_int_grid(costs, weights, budget, ticks=1, allow_rounding=False):
    """Integer costs, weights and budget of the DP (fractional weights refused)."""
    c = np.asarray(costs, dtype=np.float64)
    w = np.asarray(weights, dtype=np.float64)
    wr = np.round(w)
    if not allow_rounding and not np.array_equal(wr, w):
        raise ValueError("to_int_grid: weights are not integer-valued; pass integer_weights(counts) "
                         "or allow_rounding=True (rounding changes the budget being enforced)")
    return (np.round(c * int(ticks)).astype(np.int64), wr.astype(np.int64),
            int(round(float(budget) * int(ticks))))


def integer_weights(counts):
    """(w_int, unit): parameter counts divided by their gcd."""
    raw = np.asarray(counts)
    if raw.size == 0:
        raise ValueError("counts must be non-empty")
    if raw.dtype.kind == "f":
        if not (np.all(np.isfinite(raw)) and np.all(raw == np.round(raw))):
            raise ValueError("counts must be integer-valued")
    elif raw.dtype.kind not in "iu":
        raise ValueError(f"counts must be numeric, got dtype {raw.dtype}")
    ints = raw.astype(np.int64)
    if np.any(ints < 0):
        raise ValueError("counts must be nonnegative")
    unit = int(np.gcd.reduce(ints.reshape(-1)))
    if unit == 0:
        raise ValueError("all counts are zero")
    return ints // unit, unit


def _unpack(out):
    if isinstance(out, tuple):
        return out[0], float(out[1])
    return out, None


def rco_loop(logits_init, costs, weights, budget, steps=10, g=G_DEFAULT, lr=LR_DEFAULT, seed=0,
             tau0=TAU0, tau_min=TAU_MIN, beta1=ADAM_BETAS[0], beta2=ADAM_BETAS[1], eps=ADAM_EPS,
             grad_fn=None, use_mx=False, ticks=1, callback=None):
    """RCO (Alg.1). grad_fn(z, p, step, sample, rng) returns dL/dy at y = z, or (dL/dy, loss).
    Returns the dict of the reference (logits, momentum, velocity, history, z_final, ...)."""
    if grad_fn is None:
        raise ValueError("rco_loop needs grad_fn(z, p, step, sample, rng) returning dL/dy "
                         "(or (dL/dy, loss)); there is no silent random default")
    if use_mx:
        raise NotImplementedError("the MLX backend is not part of this build")
    c_np = np.asarray(costs, dtype=np.float64)
    w_np = np.asarray(weights, dtype=np.float64)
    B = float(budget)
    ci, wi, Bi = to_int_grid(c_np, w_np, B, ticks)
    rng = np.random.default_rng(seed)
    a = retract(np.asarray(logits_init, dtype=np.float64).copy(), c_np, w_np, B)
    m = np.zeros_like(a)
    v = np.zeros_like(a)
    history = []
    for t in range(steps):
        tau = tau_schedule(t, steps, tau0, tau_min)
        losses = []
        g_acc = np.zeros_like(a)
        for j in range(g):
            h = perturbed_logits(a, sample_gumbel(a.shape, rng=rng), tau)
            z = dp_knapsack(h, ci, wi, Bi)
            p = soft_probs(h)
            up, loss = _unpack(grad_fn(z, p, t, j, rng))
            if loss is not None:
                losses.append(loss)
            g_acc = g_acc + ste_grad(up, p, tau)
        gp = project_tangent(g_acc / g, normal_vector(a, c_np, w_np))
        m = beta1 * m + (1 - beta1) * gp
        v = beta2 * v + (1 - beta2) * gp * gp
        mhat = m / (1 - beta1 ** (t + 1))
        vhat = v / (1 - beta2 ** (t + 1))
        a = retract(a - lr * mhat / (np.sqrt(vhat) + eps), c_np, w_np, B)
        m = transport(m, normal_vector(a, c_np, w_np))
        if losses and len(losses) != g:
            raise ValueError("grad_fn returned a loss for some samples only")
        rec = {"t": t, "tau": tau, "cost": expected_cost(a, c_np, w_np)}
        if losses:
            rec["loss"] = float(np.mean(losses))
        history.append(rec)
        if callback is not None:
            callback(t, a, rec)
    z_final = dp_knapsack(a, ci, wi, Bi)
    return {"logits": a, "momentum": m, "velocity": v, "history": history, "z_final": z_final,
            "decoded_cost": assignment_cost(z_final, ci, wi),
            "decoded_value": assignment_value(z_final, a), "budget": B, "budget_int": Bi,
            "costs_int": ci, "weights_int": wi}
