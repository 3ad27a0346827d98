"""GSQ soft-quantized linear, its gradients and Lion: CPU restatement (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows the reference egesabanci/gsq-rco-mlx:
  grid / schedules / local shift   src/gsq_rco/gsq/quant.py:38-46, 51-61, 75-108
  App-A logit inits                src/gsq_rco/gsq/gptq.py:192-232 (ternary :222-232)
  Gumbel-softmax soft weight       src/gsq_rco/gsq/staged.py:82-106, 271-298
  ternary (1-bit) soft weight      src/gsq_rco/gsq/staged.py:87-89, 109-115, 251-253, 305-308
                                   (tests/oracles.py:92-103, 126-160)
  qk stage loss                    src/gsq_rco/gsq/staged.py:322-329
  analytic gradients               tests/oracles.py:311-347 (full grid), extended here to the
                                   5-neighbour local shift: u_k = s * G * C_k
  Lion                             src/gsq_rco/gsq/lion.py:44-56 (and tests/oracles.py:185-213)
  scale_lr                         src/gsq_rco/gsq/lion.py:27-41
  stage optimiser step             src/gsq_rco/gsq/staged.py:357-400

Elementwise math is float32 like the reference's MLX arrays; contractions are float64
(more exact than the reference's float32 GEMMs). Randomness is an input: Gumbel planes
are passed in (host-supplied noise), or drawn from oracle.philox with the counters the
CUDA kernels use.

Device layout shared with the CUDA path: logits and their momentum are plane-major
[K, d] (K = 5 local-shift candidates, 4 grid values at 2 bits, or the mask and sign logits of
ternary weights, whose draws take 4 Gumbel planes); d = out * in, weight i = row * in + col;
scales [out, G] with G = ceil(in / group_size).
"""
from __future__ import annotations

import numpy as np

from .philox import gumbel_planes

_BACKEND = "numpy"


def set_backend(name: str) -> str:
    """Select the elementwise passes of the training loops: "numpy" (this file, pinned to the
    reference's golden vectors) or "c" (oracle/gsq_c.c, the same arithmetic split over the
    host's cores, checked against numpy). Returns the previous backend."""
    global _BACKEND
    if name not in ("numpy", "c"):
        raise ValueError(name)
    prev, _BACKEND = _BACKEND, name
    return prev


def fast() -> bool:
    return _BACKEND == "c"

TAU_START, TAU_END = 2.0, 0.05        # quant.py:22-23
KAPPA_START, KAPPA_END = 100.0, 500.0  # quant.py:24
LR_LOGITS = 1e-4                       # lion.py:18
LR_SCALES = 5e-5                       # lion.py:19
WEIGHT_DECAY = 1.0                     # lion.py:20
BETAS = (0.9, 0.95)                    # lion.py:21
ALPHA_SCALAR = 6.0                     # staged.py:52
INIT_STD = 0.01                        # staged.py:53


# ------------------------------------------------------------------ grid ---

def get_grid(bits: int) -> np.ndarray:
    """quant.py:38-46: arange(2^b) - 2^(b-1) (2-bit [-2,-1,0,1]); 1-bit is ternary [-1,0,1]."""
    if bits == 1:
        return np.array([-1.0, 0.0, 1.0], dtype=np.float32)
    k = 2 ** bits
    return np.arange(k, dtype=np.float32) - (k // 2)


def linear_schedule(t: int, T: int, start: float, end: float) -> float:
    """quant.py:51-52."""
    return start + (end - start) * min(1.0, t / max(1, T - 1))


def gs_schedules(t: int, T: int):
    """quant.py:55-61: tau linear 2 -> 0.05, kappa linear 100 -> 500."""
    return (linear_schedule(t, T, TAU_START, TAU_END),
            linear_schedule(t, T, KAPPA_START, KAPPA_END))


def local_shift_values(j0, grid) -> np.ndarray:
    """quant.py:86-108 (numpy branch): C[i, k] = grid[clip(j0[i] + k - 2, 0, K-1)], [d, 5]."""
    jj = np.asarray(j0).astype(np.int64)
    g = np.asarray(grid, dtype=np.float32)
    jk = np.clip(jj[:, None] + (np.arange(5) - 2)[None, :], 0, len(g) - 1)
    return g[jk]


def local_shift_indices(j0, logits_dk, n_levels: int) -> np.ndarray:
    """quant.py:75-83: j = clip(j0 + argmax_k l - 2, 0, K-1). logits_dk is [d, 5]."""
    delta = np.asarray(logits_dk).argmax(axis=-1) - 2
    return np.clip(np.asarray(j0).astype(np.int64) + delta, 0, n_levels - 1)


def candidate_values(bits: int, j0) -> np.ndarray:
    """Candidate grid values per weight, plane-major [K, d]: the local shift for 3..7 bits
    (staged.py:263-266), the full grid for 2 bits (staged.py:255-257); None for ternary
    weights, whose value is the product of a mask and a sign draw."""
    if bits == 1:
        return None
    grid = get_grid(bits)
    j0 = np.asarray(j0).reshape(-1)
    if bits == 2:
        return np.repeat(grid[:, None], j0.size, axis=1).astype(np.float32)
    if 3 <= bits <= 7:
        return np.ascontiguousarray(local_shift_values(j0, grid).T)
    raise ValueError(f"GSQ soft weights cover 2..7 bits, got {bits}")


# ----------------------------------------------------------------- inits ---

def noisy_alpha_init(base, alpha, std, seed):
    """gptq.py:192-199: l = std * (eps + alpha * (base - mean_k base)), eps ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    b = base - base.mean(axis=-1, keepdims=True)
    eps = rng.standard_normal(base.shape).astype(np.float32)
    return (std * (eps + alpha * b)).astype(np.float32)


def init_shift_logits(numel, alpha=ALPHA_SCALAR, std=INIT_STD, seed=0):
    """gptq.py:213-219: base_k = -(k-2)^2 / 2 for k = 0..4, then the Eq.4 noise. [d, 5]."""
    c = np.array([-2, -1, 0, 1, 2], dtype=np.float32)
    base = np.tile(-(c ** 2) / 2.0, (int(numel), 1))
    return noisy_alpha_init(base, alpha, std, seed)


def init_logits_2bit_from_codes(codes, K, alpha=ALPHA_SCALAR, std=INIT_STD, seed=0):
    """gptq.py:202-210: base_k = -(k - q_i)^2 / 2 over the K grid levels. [d, K]."""
    kk = np.arange(K, dtype=np.float32)
    base = -((kk[None, :] - np.asarray(codes).reshape(-1)[:, None].astype(np.float32)) ** 2) / 2.0
    return noisy_alpha_init(base.astype(np.float32), alpha, std, seed)


def init_ternary_logits(q, alpha=3.0, std=INIT_STD, seed=0):
    """gptq.py:222-232: mask logits std (N(0,1) + alpha (+1 if q != 0 else -1)) and sign logits
    std (N(0,1) + alpha sign(q)), the mask's normals drawn first. [2, d] float32."""
    q = np.asarray(q).reshape(-1)
    rng = np.random.default_rng(seed)
    eps = [rng.standard_normal(q.shape).astype(np.float32) for _ in range(2)]
    base = [np.where(q != 0, 1.0, -1.0), np.sign(q)]
    return np.stack([(std * (e + alpha * b.astype(np.float32))).astype(np.float32)
                     for e, b in zip(eps, base)])


def init_logits(bits, codes, seed):
    """Initial logits of one linear, plane-major [K, d] float32 (staged.py:250-266)."""
    codes = np.asarray(codes)
    if bits == 1:
        return init_ternary_logits(get_grid(1)[codes.reshape(-1)], seed=seed)
    if bits == 2:
        l = init_logits_2bit_from_codes(codes, 4, seed=seed)
    else:
        l = init_shift_logits(codes.size, seed=seed)
    return np.ascontiguousarray(l.T)


def scale_lr(lr_scales: float, bits: int) -> float:
    """lion.py:27-41: group scales above 3 bits are frozen."""
    return 0.0 if bits > 3 else lr_scales


# ----------------------------------------------------------- soft weight ---

def gs_probs(logits_kd, noise_kd, tau, kappa):
    """staged.py:82-84: p = softmax((kappa * l + g) / tau) over the candidate axis, float32.
    The division by tau and by the sum are multiplications by the float32 reciprocals, the
    order of operations of the CUDA kernels."""
    inv_tau = np.float32(1.0) / np.float32(tau)
    kappa = np.float32(kappa)
    y = (kappa * logits_kd.astype(np.float32) + noise_kd.astype(np.float32)) * inv_tau
    y = y - y.max(axis=0, keepdims=True)
    e = np.exp(y)
    inv = np.float32(1.0) / e.sum(axis=0, keepdims=True)
    return e * inv


def _sigmoid32(z):
    one = np.float32(1.0)
    with np.errstate(over="ignore"):
        return one / (one + np.exp(-z))


def ternary_probs(logits_2d, noise_4d, tau, kappa):
    """staged.py:87-89 and 109-115 in float32: the mask probability
    m = sigmoid((2 kappa lm + (g1 - g0)) / tau) and the sign probability
    v = sigmoid((2 kappa lb + (g3 - g2)) / tau); the division by tau a multiplication by its
    float32 reciprocal (the CUDA kernels' order). Returns [2, d] = (m, v)."""
    inv_tau = np.float32(1.0) / np.float32(tau)
    k2 = np.float32(2.0) * np.float32(kappa)
    l = np.asarray(logits_2d, dtype=np.float32)
    g = np.asarray(noise_4d, dtype=np.float32)
    m = _sigmoid32((k2 * l[0] + (g[1] - g[0])) * inv_tau)
    v = _sigmoid32((k2 * l[1] + (g[3] - g[2])) * inv_tau)
    return np.stack([m, v]).astype(np.float32)


def ternary_value(p):
    """c = m (2 v - 1) (staged.py:113-115), float32."""
    return (p[0] * (np.float32(2.0) * p[1] - np.float32(1.0))).astype(np.float32)


def ternary_backward(G, p, c, scales, group_size, tau, kappa):
    """Gradients of the ternary soft weight w = s m (2 v - 1) given G = dL/dw, float64:
    dL/dlm = (2 kappa / tau) s G (2 v - 1) m (1 - m), dL/dlb = (2 kappa / tau) s G m 2 v (1 - v)
    (the sigmoid's derivative through z = (2 kappa l + g' - g) / tau), dL/ds = group_sum(G c)."""
    out_f, in_f = G.shape
    sG = (expand_scales(scales, in_f, group_size).astype(np.float64) * G).reshape(-1)
    m, v = p[0].astype(np.float64), p[1].astype(np.float64)
    kt2 = 2.0 * kappa / tau
    glog = np.stack([kt2 * sG * (2.0 * v - 1.0) * m * (1.0 - m),
                     kt2 * sG * m * 2.0 * v * (1.0 - v)])
    return glog, group_sum(G * c.astype(np.float64), group_size)


def ternary_hard_codes(logits_2d):
    """staged.py:305-308: m = lm >= 0, b = lb >= 0, code = m (2 b - 1) + 1 (grid [-1, 0, 1])."""
    m = (np.asarray(logits_2d[0]) >= 0).astype(np.int64)
    b = (np.asarray(logits_2d[1]) >= 0).astype(np.int64)
    return (m * (2 * b - 1) + 1).astype(np.uint8)


def expand_scales(scales, in_f, group_size):
    """Per-(row, group) scales -> per-weight [out, in] (staged.py:298 mx.take over gid)."""
    return np.repeat(np.asarray(scales, dtype=np.float32), group_size, axis=1)[:, :in_f]


def group_sum(A, group_size):
    """Sum A [out, in] over each (row, group) -> [out, G] (tests/oracles.py:294-300)."""
    out_f, in_f = A.shape
    G = -(-in_f // group_size)
    Ap = np.zeros((out_f, G * group_size), dtype=np.float64)
    Ap[:, :in_f] = A
    return Ap.reshape(out_f, G, group_size).sum(axis=-1)


def soft_weight(logits_kd, noise_kd, Ckd, scales, shape, group_size, tau, kappa):
    """staged.py:271-298: w_bar = s[:, col // gs] * sum_k p_k C_k, float32 [out, in].
    Returns (w_bar, p [K, d], c [out, in]). Ckd None: ternary weights (c = m (2 v - 1))."""
    if Ckd is None:
        p = ternary_probs(logits_kd, noise_kd, tau, kappa)
        c = ternary_value(p).reshape(shape)
        w = expand_scales(scales, shape[1], group_size) * c
        return w.astype(np.float32), p, c
    if fast():
        from . import gsq_fast
        return gsq_fast.soft_weight(logits_kd, noise_kd, Ckd, scales, shape, group_size, tau,
                                    kappa)
    p = gs_probs(logits_kd, noise_kd, tau, kappa)
    c = (p * Ckd).sum(axis=0).astype(np.float32).reshape(shape)
    w = expand_scales(scales, shape[1], group_size) * c
    return w.astype(np.float32), p, c


def soft_backward(G, p, Ckd, c, scales, group_size, tau, kappa):
    """Gradients of the loss w.r.t. logits [K, d] and scales [out, G] given G = dL/dw_bar.

    tests/oracles.py:340-344 for the full grid; the local shift replaces grid_k by C_k:
      u_k = s * G * C_k,   dL/dl = (kappa / tau) * p * (u - <p, u>),   dL/ds = group_sum(G * c).
    Ckd None: the ternary gradients (ternary_backward).
    """
    if Ckd is None:
        return ternary_backward(G, p, c, scales, group_size, tau, kappa)
    out_f, in_f = G.shape
    sG = (expand_scales(scales, in_f, group_size).astype(np.float64) * G).reshape(-1)
    u = sG[None, :] * Ckd.astype(np.float64)
    pd = p.astype(np.float64)
    glog = (kappa / tau) * pd * (u - (pd * u).sum(axis=0, keepdims=True))
    gs = group_sum(G * c.astype(np.float64), group_size)
    return glog, gs


def backward_accumulate(acc, G, p, Ckd, c, scales, group_size, tau, kappa):
    """Add one draw's float32 logit and scale gradients to acc = [glog, gscale] (None entries
    start the sums), the resample accumulation of staged.py:386."""
    if fast() and Ckd is not None:
        from . import gsq_fast
        if acc[0] is None:
            acc[0] = np.zeros(p.shape, dtype=np.float32)
            acc[1] = np.zeros((G.shape[0], -(-G.shape[1] // group_size)), dtype=np.float32)
        gsq_fast.soft_backward_acc(G, p, Ckd, c, scales, group_size, tau, kappa, acc[0], acc[1])
        return acc
    glog, gs = soft_backward(G, p, Ckd, c, scales, group_size, tau, kappa)
    glog, gs = glog.astype(np.float32), gs.astype(np.float32)
    acc[0] = glog if acc[0] is None else acc[0] + glog
    acc[1] = gs if acc[1] is None else acc[1] + gs
    return acc


def lion(P, M, G, lr, wd=WEIGHT_DECAY, betas=BETAS):
    """lion.py:44-56 in float32: u = sign(b1 m + (1-b1) g); m <- b2 m + (1-b2) g;
    p <- p - lr (u + wd p)."""
    b1, b2 = betas
    P = np.asarray(P, dtype=np.float32)
    M = np.asarray(M, dtype=np.float32)
    G = np.asarray(G, dtype=np.float32)
    f = np.float32
    newP = P - f(lr) * (np.sign(f(b1) * M + f(1 - b1) * G) + f(wd) * P)
    newM = f(b2) * M + f(1 - b2) * G
    return newP.astype(np.float32), newM.astype(np.float32)


# ------------------------------------------------------------ qk stage ---

def linear_loss_and_grads(X, W, logits_kd, Ckd, scales, noises, group_size, tau, kappa,
                          gemm_dtype=np.float64):
    """qk-stage loss of one linear (staged.py:322-329), averaged over the resamples in
    ``noises`` (staged.py:383-390): mean((X (w_bar - W)^T)^2), its logit and scale grads.

    X [M, in], W [out, in], noises: list of [K, d] Gumbel planes, one per resample.
    Returns (mean loss, glog [K, d], gscale [out, G], list of G_r = dL/dw_bar).
    """
    X = np.asarray(X, dtype=gemm_dtype)
    Wd = np.asarray(W, dtype=gemm_dtype)
    M = X.shape[0]
    out_f = Wd.shape[0]
    acc_l = 0.0
    acc = [None, None]
    Gs = []
    for noise in noises:
        w, p, c = soft_weight(logits_kd, noise, Ckd, scales, Wd.shape, group_size, tau, kappa)
        R = X @ (w.astype(gemm_dtype) - Wd).T
        acc_l += float((R * R).mean(dtype=np.float64))
        G = ((2.0 / (M * out_f)) * (R.T @ X)).astype(np.float64)
        Gs.append(G)
        # the reference accumulates float32 gradients (staged.py:386), then divides by R
        backward_accumulate(acc, G, p, Ckd, c, scales, group_size, tau, kappa)
    n = np.float32(len(noises))
    return acc_l / len(noises), acc[0] / n, acc[1] / n, Gs


class LinearState:
    """Training state of one soft linear (the arrays of staged.py:_Linear.P plus momentum)."""

    def __init__(self, bits, codes, scales16, group_size, seed, linear_id=0):
        self.bits = int(bits)
        self.codes0 = np.asarray(codes, dtype=np.uint8)
        self.shape = self.codes0.shape
        self.group_size = int(group_size)
        self.Ckd = candidate_values(self.bits, self.codes0.reshape(-1))
        self.logits = init_logits(self.bits, self.codes0, seed)
        self.scales = np.asarray(scales16, dtype=np.float32).copy()
        self.mom_logits = np.zeros_like(self.logits)
        self.mom_scales = np.zeros_like(self.scales)
        self.linear_id = int(linear_id)

    @property
    def K(self):
        return self.logits.shape[0]

    @property
    def n_noise(self):
        """Gumbel planes per draw: four for ternary weights, else one per candidate."""
        return 4 if self.bits == 1 else self.K

    def hard_codes(self):
        """staged.py:300-314: argmax decode (local shift clipped to the grid; 2-bit argmax;
        ternary: the mask and sign logits' signs)."""
        if self.bits == 1:
            return ternary_hard_codes(self.logits).reshape(self.shape)
        if self.bits == 2:
            return self.logits.argmax(axis=0).astype(np.uint8).reshape(self.shape)
        j = local_shift_indices(self.codes0.reshape(-1), self.logits.T, 2 ** self.bits)
        return j.astype(np.uint8).reshape(self.shape)

    def stored_scales(self):
        """staged.py:316-317: float32 -> float16."""
        return self.scales.astype(np.float16)

    def noise(self, seed, step, resample):
        if fast():
            from . import gsq_fast
            return gsq_fast.gumbel_planes(seed, self.linear_id, step, resample,
                                          self.codes0.size, self.n_noise)
        return gumbel_planes(seed, self.linear_id, step, resample, self.codes0.size,
                             self.n_noise)


def lion_step(state: LinearState, glog, gs, lr_logits=LR_LOGITS, lr_scales=LR_SCALES):
    """One Lion step on logits and scales (staged.py:389-392; scale lr per lion.py:27-41)."""
    if fast():
        from . import gsq_fast
        gsq_fast.lion_(state.logits, state.mom_logits, glog, lr_logits, WEIGHT_DECAY, BETAS)
        gsq_fast.lion_(state.scales, state.mom_scales, gs, scale_lr(lr_scales, state.bits),
                       WEIGHT_DECAY, BETAS)
        return
    state.logits, state.mom_logits = lion(state.logits, state.mom_logits, glog, lr_logits)
    state.scales, state.mom_scales = lion(state.scales, state.mom_scales, gs,
                                          scale_lr(lr_scales, state.bits))


def train_linear(state: LinearState, X_rows_of, W, n_seqs, steps, micro_batch=2, resamples=2,
                 seed=0, noise_seed=None, noise_fn=None, lr_logits=LR_LOGITS,
                 lr_scales=LR_SCALES, perturb=None):
    """qk-stage optimiser on one linear (staged.py:357-400 with one linear in lins).

    X_rows_of(idx) returns the [M, in] rows of the sorted sequence ids idx (positions 1.. only,
    staged.py:128-130). The micro-batch draw is the reference's numpy stream
    (staged.py:373,380). noise_fn(t, r) returns the [K, d] Gumbel planes of resample r at step
    t; by default they come from oracle.philox with ``noise_seed``. ``perturb`` (tests only)
    maps each G_r to a perturbed copy, to measure how the trajectory reacts to GEMM rounding.
    Returns the per-step mean soft loss.
    """
    rng = np.random.default_rng(seed)
    m = min(micro_batch, n_seqs)
    noise_seed = seed if noise_seed is None else noise_seed
    hist = []
    for t in range(steps):
        tau, kappa = gs_schedules(t, steps)
        idx = np.sort(rng.choice(n_seqs, size=m, replace=False))
        X = X_rows_of(idx)
        if noise_fn is None:
            noises = [state.noise(noise_seed, t, r) for r in range(resamples)]
        else:
            noises = [noise_fn(t, r) for r in range(resamples)]
        if perturb is None:
            loss, glog, gs, _ = linear_loss_and_grads(X, W, state.logits, state.Ckd, state.scales,
                                                      noises, state.group_size, tau, kappa)
        else:
            loss, glog, gs = perturbed_grads(X, W, state, noises, tau, kappa, perturb)
        lion_step(state, glog, gs, lr_logits, lr_scales)
        hist.append(loss)
    return hist


def perturbed_grads(X, W, state, noises, tau, kappa, perturb):
    """linear_loss_and_grads with each G_r passed through ``perturb`` (sensitivity studies)."""
    X = np.asarray(X, dtype=np.float64)
    Wd = np.asarray(W, dtype=np.float64)
    M, out_f = X.shape[0], Wd.shape[0]
    acc_l, acc_glog, acc_gs = 0.0, None, None
    for noise in noises:
        w, p, c = soft_weight(state.logits, noise, state.Ckd, state.scales, Wd.shape,
                              state.group_size, tau, kappa)
        R = X @ (w.astype(np.float64) - Wd).T
        acc_l += float((R * R).mean())
        G = perturb((2.0 / (M * out_f)) * (R.T @ X))
        glog, gs = soft_backward(G, p, state.Ckd, c, state.scales, state.group_size, tau, kappa)
        glog, gs = glog.astype(np.float32), gs.astype(np.float32)
        acc_glog = glog if acc_glog is None else acc_glog + glog
        acc_gs = gs if acc_gs is None else acc_gs + gs
    n = np.float32(len(noises))
    return acc_l / len(noises), acc_glog / n, acc_gs / n
