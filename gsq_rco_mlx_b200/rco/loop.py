"""RCO loop (paper Alg. 1) on the host, decoding on the GPU.

The public functions keep the names, arguments, return values and exception types of the
reference module src/gsq_rco/rco/loop.py; the code is this package's own. ``RcoOptimizer``
holds the state of one allocation run (logits, Adam moments, the numpy random stream) and
advances it one step at a time; ``rco_loop`` runs it for ``steps`` steps and returns the
reference's result dictionary.

One step t (loop.py:224-279 numpy path):
  * tau_t from the exponential anneal;
  * for each of the g samples: Gumbel noise G from the run's numpy Generator, perturbed logits
    h = (a + G) / tau, z = exact knapsack decode of h (CUDA kernel), p = softmax(h), the
    caller's upstream dL/dy at y = z, and the straight-through gradient p (v - <p, v>) / tau;
    the Gumbel draw of a sample comes before its grad_fn call, which may draw from the same
    Generator (the KL objective draws its windows there), so the stream order is the
    reference's;
  * the mean over samples is projected on the tangent plane at a, Adam (bias-corrected) steps
    a, the retraction puts a back on the budget manifold and the first moment is carried to
    the new tangent plane.
The [N, K] float64 state is a few hundred numbers and stays in numpy.
"""
from __future__ import annotations

import numpy as np

from . import manifold as mf

TAU0, TAU_MIN = 1.0, 0.01
G_DEFAULT = 4
LR_DEFAULT = 0.1
ADAM_BETAS = (0.9, 0.999)
ADAM_EPS = 1e-8


def tau_schedule(t, T, tau0=TAU0, tau_min=TAU_MIN):
    """Exponential anneal from tau0 at t = 0 to tau_min at t = T - 1 (floored at tau_min)."""
    if T <= 1:
        return float(tau_min)
    frac = min(max(t, 0), T - 1) / (T - 1)
    return max(float(tau_min), float(tau0) * (float(tau_min) / float(tau0)) ** frac)


def sample_gumbel(shape, rng=None, key=None):
    """Standard Gumbel noise -log(-log(u)), u = rng.random(shape) clipped to [1e-12, 1 - 1e-12]
    (a fresh default_rng(0) when no Generator is given)."""
    gen = np.random.default_rng(0) if rng is None else rng
    u = np.clip(gen.random(tuple(shape)).astype(np.float64), 1e-12, 1.0 - 1e-12)
    return -np.log(-np.log(u))


def perturbed_logits(logits, gumbel, tau):
    """h = (a + G) / tau, tau floored at 1e-6."""
    return (logits + gumbel) / max(float(tau), 1e-6)


def soft_probs(h):
    """Softmax of the perturbed logits that produced the decode."""
    return mf.softmax(h)


def ste_grad(upstream, p, tau):
    """Straight-through backward: the softmax Jacobian at p applied to the upstream v,
    p (v - <p, v>) / tau (tau floored at 1e-6)."""
    v = np.asarray(upstream, dtype=np.float64)
    q = np.asarray(p, dtype=np.float64)
    centred = v - np.einsum("ik,ik->i", q, v)[:, None]
    return q * centred / max(float(tau), 1e-6)


def to_int_grid(costs, weights, budget, ticks=1, allow_rounding=False):
    """Costs and budget scaled by ``ticks`` and rounded to the DP's integer grid; weights must
    already be whole numbers (build them with integer_weights) unless ``allow_rounding``.
    Returns (costs_int int64 [K], weights_int int64 [N], budget_int)."""
    scale = int(ticks)
    w = np.asarray(weights, dtype=np.float64)
    w_int = np.round(w)
    if not allow_rounding and (w_int != w).any():
        raise ValueError("to_int_grid: group weights must be whole numbers; rounding them would "
                         "change the enforced budget (use integer_weights, or allow_rounding)")
    c_int = np.round(np.asarray(costs, dtype=np.float64) * scale).astype(np.int64)
    return c_int, w_int.astype(np.int64), int(round(float(budget) * scale))


def integer_weights(counts):
    """Group weights as the smallest whole numbers in the ratio of ``counts``:
    (counts // unit, unit) with unit = gcd(counts). Raises ValueError for empty, negative,
    fractional, non-numeric or all-zero counts."""
    x = np.asarray(counts)
    if x.size == 0:
        raise ValueError("integer_weights: no counts given")
    if x.dtype.kind == "f":
        if not np.isfinite(x).all() or (np.floor(x) != x).any():
            raise ValueError("integer_weights: counts must be whole numbers")
    elif x.dtype.kind not in "iu":
        raise ValueError(f"integer_weights: counts must be numbers, not {x.dtype}")
    n = x.astype(np.int64).reshape(-1)
    if (n < 0).any():
        raise ValueError("integer_weights: counts must be >= 0")
    unit = int(np.gcd.reduce(n))
    if unit == 0:
        raise ValueError("integer_weights: every count is zero")
    return x.astype(np.int64) // unit, unit


class RcoOptimizer:
    """State and step of one RCO run on the budget manifold of (costs, weights, budget).

    ``decode(h, costs_int, weights_int, budget_int)`` returns the one-hot decode of a score
    matrix; it defaults to the exact knapsack on the GPU (manifold.dp_knapsack)."""

    def __init__(self, logits_init, costs, weights, budget, *, steps, g=G_DEFAULT,
                 lr=LR_DEFAULT, seed=0, tau0=TAU0, tau_min=TAU_MIN, betas=ADAM_BETAS,
                 eps=ADAM_EPS, ticks=1, decode=None):
        self.costs = np.asarray(costs, dtype=np.float64)
        self.weights = np.asarray(weights, dtype=np.float64)
        self.budget = float(budget)
        self.grid = to_int_grid(self.costs, self.weights, self.budget, ticks)
        self.steps, self.g, self.lr = int(steps), int(g), float(lr)
        self.tau0, self.tau_min = float(tau0), float(tau_min)
        self.b1, self.b2 = (float(b) for b in betas)
        self.eps = float(eps)
        self.decode = decode or mf.dp_knapsack
        self.rng = np.random.default_rng(seed)
        self.logits = self._onto_manifold(np.array(logits_init, dtype=np.float64))
        self.m = np.zeros_like(self.logits)
        self.v = np.zeros_like(self.logits)
        self.t = 0

    def _onto_manifold(self, a):
        return mf.retract(a, self.costs, self.weights, self.budget)

    def _normal(self, a):
        return mf.normal_vector(a, self.costs, self.weights)

    def sample_gradient(self, grad_fn, tau, sample):
        """One Gumbel sample: decode, upstream, straight-through gradient. Returns
        (gradient [N, K], loss or None)."""
        h = perturbed_logits(self.logits, sample_gumbel(self.logits.shape, rng=self.rng), tau)
        z = self.decode(h, *self.grid)
        p = soft_probs(h)
        out = grad_fn(z, p, self.t, sample, self.rng)
        up, loss = (out[0], float(out[1])) if isinstance(out, tuple) else (out, None)
        return ste_grad(up, p, tau), loss

    def step(self, grad_fn):
        """Advance one step; returns the step's record {t, tau, cost[, loss]}."""
        tau = tau_schedule(self.t, self.steps, self.tau0, self.tau_min)
        total = np.zeros_like(self.logits)
        losses = []
        for j in range(self.g):
            grad, loss = self.sample_gradient(grad_fn, tau, j)
            total += grad
            if loss is not None:
                losses.append(loss)
        if losses and len(losses) != self.g:
            raise ValueError("rco_loop: grad_fn must return a loss for every sample or for none")
        gt = mf.project_tangent(total / self.g, self._normal(self.logits))
        k = self.t + 1
        self.m = self.b1 * self.m + (1.0 - self.b1) * gt
        self.v = self.b2 * self.v + (1.0 - self.b2) * gt * gt
        m_hat = self.m / (1.0 - self.b1 ** k)
        v_hat = self.v / (1.0 - self.b2 ** k)
        self.logits = self._onto_manifold(self.logits - self.lr * m_hat /
                                          (np.sqrt(v_hat) + self.eps))
        self.m = mf.transport(self.m, self._normal(self.logits))
        rec = {"t": self.t, "tau": tau,
               "cost": mf.expected_cost(self.logits, self.costs, self.weights)}
        if losses:
            rec["loss"] = float(np.mean(losses))
        self.t = k
        return rec

    def result(self, history):
        ci, wi, bi = self.grid
        z = self.decode(self.logits, ci, wi, bi)
        return {"logits": self.logits, "momentum": self.m, "velocity": self.v,
                "history": history, "z_final": z,
                "decoded_cost": mf.assignment_cost(z, ci, wi),
                "decoded_value": mf.assignment_value(z, self.logits), "budget": self.budget,
                "budget_int": bi, "costs_int": ci, "weights_int": wi}


def rco_loop(logits_init, costs, weights, budget, steps=10, g=G_DEFAULT, lr=LR_DEFAULT, seed=0,
             tau0=TAU0, tau_min=TAU_MIN, beta1=ADAM_BETAS[0], beta2=ADAM_BETAS[1], eps=ADAM_EPS,
             grad_fn=None, use_mx=False, ticks=1, callback=None, decode=None):
    """RCO (Alg. 1). grad_fn(z, p, step, sample, rng) returns dL/dy at y = z, or (dL/dy, loss).
    callback(t, logits, record) runs after every step. Returns {logits, momentum, velocity,
    history, z_final, decoded_cost, decoded_value, budget, budget_int, costs_int,
    weights_int}. ``decode`` replaces the GPU knapsack decode (same arguments as
    manifold.dp_knapsack)."""
    if grad_fn is None:
        raise ValueError("rco_loop: grad_fn(z, p, step, sample, rng) is required; it gives the "
                         "upstream gradient of the objective")
    if use_mx:
        raise NotImplementedError("rco_loop: the MLX backend is not part of this package")
    opt = RcoOptimizer(logits_init, costs, weights, budget, steps=steps, g=g, lr=lr, seed=seed,
                       tau0=tau0, tau_min=tau_min, betas=(beta1, beta2), eps=eps, ticks=ticks,
                       decode=decode)
    history = []
    for _ in range(int(steps)):
        rec = opt.step(grad_fn)
        history.append(rec)
        if callback is not None:
            callback(rec["t"], opt.logits, rec)
    return opt.result(history)
