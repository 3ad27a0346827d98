"""GSQ stage optimiser on the GPU (reference src/gsq_rco/gsq/staged.py).

``SoftLinear`` is the device-resident training state of one linear (staged.py:230-317):
plane-major logits and their Lion momentum, group scales and their momentum, and the GPTQ
codes j0. Its ``soft`` builds one Gumbel-softmax soft weight (staged.py:271-298) and stores
the draw's probabilities; its ``step`` is one fused pass: the soft backward from the stored
probabilities, the resample mean and Lion (staged.py:383-392 with lion.py:44-56), and the next
step's soft weights.

``train_linears`` is the qk-stage optimiser (staged.py:357-400 with the linear loss of
:322-329): per step the schedules, a sorted micro-batch draw from the numpy stream, the
micro-batch Gram matrix X^T X, R resamples of (weight gradient D X^T X, loss sum D * G), then
one fused step launch per linear. ``train_stage`` runs the vo / mlp stage steps (``VOStep``,
``MLPStep``) the same way; every stage step repeats its GEMMs as prepared plans.

Gumbel noise: Philox4x32-10 keyed by (stage seed, linear id) with counter (weight, block,
step, resample), drawn inside the kernels, or host-supplied planes for parity runs.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch

from .. import _lib
from ..gemm import PlanCache, Terms, check_err, err_flag, gemm, gemm_tc, pad8
from .gptq import init_logits_2bit_from_codes, init_shift_logits, init_ternary_logits
from .lion import BETAS, LR_LOGITS, LR_SCALES, WEIGHT_DECAY, scale_lr
from .quant import get_grid, gs_schedules

ALPHA_SCALAR = 6.0
ALPHA_TERNARY = 3.0
INIT_STD = 0.01
STAGES = ("qk", "vo", "mlp")
STAGE_LAYERS = {"qk": ("q_proj", "k_proj"), "vo": ("v_proj", "o_proj"),
                "mlp": ("gate_proj", "up_proj", "down_proj")}


@dataclass(frozen=True)
class BlockOpts:
    """Optimisation settings of one block (reference staged.py:65-77)."""
    group_size: int = 64
    damp: float = 0.01
    block_size: int = 128
    steps: int = 200
    micro_batch: int = 2
    resamples: int = 2
    lr_logits: float = LR_LOGITS
    lr_scales: float = LR_SCALES
    seed: int = 0


def _shift_init_t(d, seed):
    """init_shift_logits(d, seed) transposed to the plane-major [K, d] layout."""
    return np.ascontiguousarray(
        init_shift_logits(d, alpha=ALPHA_SCALAR, std=INIT_STD, seed=seed).T)


class ShiftInitPool:
    """The initial local-shift logits of a block's soft linears, drawn on host threads while
    the GPU runs the Hessian passes and the earlier stages. The draws are the reference's
    (numpy default_rng(seed) normals, gptq.py:192-219), which are sequential per linear; the
    linears run in parallel (numpy releases the GIL in its generators and ufunc loops)."""

    def __init__(self, jobs):
        from concurrent.futures import ThreadPoolExecutor
        self._ex = ThreadPoolExecutor(max_workers=max(1, min(8, len(jobs))))
        self._fut = {name: self._ex.submit(_shift_init_t, d, seed)
                     for name, (d, seed) in jobs.items()}

    def take(self, name):
        fut = self._fut.pop(name, None)
        return None if fut is None else fut.result()

    def close(self):
        self._ex.shutdown(wait=True, cancel_futures=True)


class SoftLinear:
    """One linear under the stage optimiser: GPTQ codes and scales plus trainable logits."""

    def __init__(self, name, bits, codes, scales16, group_size, seed, linear_id=0, logits0=None):
        """logits0: the initial logits [K, d] float32 (init_shift_logits of (d, seed),
        transposed) when computed ahead, e.g. by ShiftInitPool. bits 1 is ternary: two logit
        planes per weight (mask, sign; staged.py:251-253) and four Gumbel planes per draw."""
        self.name, self.bits = name, int(bits)
        if not 1 <= self.bits <= 7:
            raise NotImplementedError(
                f"{name}: soft weights cover 1..7 bits (8-bit linears are GPTQ only)")
        codes = np.asarray(codes, dtype=np.uint8)
        self.shape = codes.shape
        self.out_f, self.in_f = self.shape
        self.group_size = int(group_size)
        self.linear_id = int(linear_id)
        self.codes0 = codes
        dev = _lib.device()
        self.j0 = torch.as_tensor(codes.reshape(-1), device=dev)
        d = codes.size
        if logits0 is not None:
            lt = np.asarray(logits0, dtype=np.float32)
            if self.bits <= 2 or lt.shape[1] != d:
                raise ValueError(f"{name}: precomputed logits {lt.shape} do not fit {d} weights")
        elif self.bits == 1:
            lt = np.stack(init_ternary_logits(get_grid(1)[codes.reshape(-1)],
                                              alpha=ALPHA_TERNARY, std=INIT_STD, seed=seed))
        elif self.bits == 2:
            lt = init_logits_2bit_from_codes(codes, 4, alpha=ALPHA_SCALAR, std=INIT_STD,
                                             seed=seed).T
        else:
            lt = _shift_init_t(d, seed)
        self.K = lt.shape[0]
        self.n_noise = 4 if self.bits == 1 else self.K   # Gumbel planes per draw
        self.logits = torch.as_tensor(np.ascontiguousarray(lt), device=dev)
        self.mom = torch.zeros_like(self.logits)
        self.scales = torch.as_tensor(np.asarray(scales16, dtype=np.float32), device=dev).contiguous()
        self.mom_s = torch.zeros_like(self.scales)

    @property
    def d(self):
        return self.out_f * self.in_f

    def soft(self, tau, kappa, step, resample, seed, w_ref=None, out=None, noise=None,
             terms=None, probs=None):
        """w_bar (or w_bar - w_ref) of one Gumbel draw: float32 [out, in] into ``out``, and/or
        three bf16 terms into ``terms`` (a [3, out, in] tensor, the residual GEMM's B operand);
        ``probs`` ([K, d] float32) receives the draw's probabilities for the backward (ternary:
        the mask and sign probabilities). noise: host Gumbel planes [n_noise, d] or None."""
        if out is None and terms is None and probs is None:
            out = torch.empty(self.shape, device=self.logits.device, dtype=torch.float32)
        _lib.call("gsq_soft_fwd", _lib.ptr(self.logits), _lib.ptr(self.j0), _lib.ptr(self.scales),
                  _lib.ptr(noise), int(seed) & (2 ** 64 - 1), self.linear_id, int(step),
                  int(resample), self.out_f, self.in_f, self.group_size, self.bits, float(tau),
                  float(kappa), _lib.ptr(w_ref), _lib.ptr(out), _lib.ptr(terms), _lib.ptr(probs),
                  _lib.stream_ptr())
        return out

    def step(self, probs, grad_w, tau, kappa, lr_logits=LR_LOGITS, lr_scales=LR_SCALES,
             nxt=None):
        """Fused backward of this step (stored probs [R, K, d], grad_w [R, out, in]), resample
        mean and Lion; with nxt = dict(step, tau, kappa, seed, w_ref, terms | out, noise) also
        the next step's forward (probs updated in place, soft weights written; noise
        [R, n_noise, d] or None)."""
        R = grad_w.shape[0]
        n = nxt or {}
        _lib.call("gsq_soft_step", _lib.ptr(self.logits), _lib.ptr(self.mom), _lib.ptr(self.j0),
                  _lib.ptr(self.scales), _lib.ptr(self.mom_s), _lib.ptr(probs), _lib.ptr(grad_w),
                  int(R), self.out_f, self.in_f, self.group_size, self.bits, float(tau),
                  float(kappa), float(lr_logits), float(scale_lr(lr_scales, self.bits)),
                  float(WEIGHT_DECAY), float(BETAS[0]), float(BETAS[1]), int(nxt is not None),
                  _lib.ptr(n.get("noise")), int(n.get("seed", 0)) & (2 ** 64 - 1), self.linear_id,
                  int(n.get("step", 0)), float(n.get("tau", 1.0)), float(n.get("kappa", 1.0)),
                  _lib.ptr(n.get("w_ref")), _lib.ptr(n.get("out")), _lib.ptr(n.get("terms")),
                  _lib.stream_ptr())

    def hard_codes(self) -> np.ndarray:
        """Argmax codes of the learned logits; ternary: the signs of the mask and sign logits
        (staged.py:300-314)."""
        codes = torch.empty(self.shape, device=self.logits.device, dtype=torch.uint8)
        _lib.call("gsq_harden", _lib.ptr(self.logits), _lib.ptr(self.j0), self.out_f, self.in_f,
                  self.bits, _lib.ptr(codes), _lib.stream_ptr())
        return codes.cpu().numpy()

    def stored_scales(self) -> np.ndarray:
        """Learned scales rounded to float16, the stored form (staged.py:316-317)."""
        return self.scales.cpu().numpy().astype(np.float16)

    def logits_dk(self) -> np.ndarray:
        """Logits in the reference layout [d, K]."""
        return self.logits.T.cpu().numpy()


class LinearStep:
    """The qk-stage step of the linears that read the same rows X [M, in] (staged.py:322-329).

    A linear's loss is mean((X D^T)^2) with D = w_bar - W, and its weight gradient is
    2 / (M out) (X D^T)^T X = 2 / (M out) D (X^T X): both see X only through the micro-batch
    Gram matrix Hm = X^T X [in, in]. Per step one tensor-core GEMM forms Hm (X read MN-major,
    shared by every linear and resample; summed over the ranks under data parallelism); then
    per linear and resample G_r = 2 / (M out) D_r Hm (D_r: the three bf16 terms the soft step
    writes) and the loss sum D_r * (D_r Hm) = (M out / 2) sum D_r * G_r. At the qk shapes
    (M = 4094 rows, in = 896) that is a third of the FLOPs of forming R = X D^T and R^T X. One
    fused pass per linear then runs the backward, the resample mean, Lion, and the next step's
    soft weights and probabilities. All GEMM operands are bf16 terms (three for float32 data,
    one for exactly-bf16 rows)."""

    def __init__(self, lins, M, in_f, resamples, x_terms=3, M_total=None):
        """M: rows of this rank's micro-batch share; M_total: rows of the whole micro-batch (the
        loss normalisation), M when one process runs the stage."""
        dev = lins[0].logits.device
        self.lins, self.M, self.in_f, self.R = lins, int(M), int(in_f), int(resamples)
        self.M_total = int(M if M_total is None else M_total)
        self.nx = int(x_terms)
        self.X = Terms(M, in_f, self.nx, dev)   # read MN-major (as X^T) on both sides of Hm
        R = self.R
        self.Dbuf = {l.name: torch.zeros(R, 3, l.out_f, l.in_f, device=dev, dtype=torch.bfloat16)
                     for l in lins}
        self.D = {l.name: [Terms(l.out_f, l.in_f, 3, ld=l.in_f, tensors=self.Dbuf[l.name][r])
                           for r in range(R)] for l in lins}
        self.probs = {l.name: torch.zeros(R, l.K, l.d, device=dev, dtype=torch.float32)
                      for l in lins}
        self.Hf = torch.empty(in_f, in_f, device=dev, dtype=torch.float32)
        self.Hm = Terms(in_f, in_f, 3, dev)
        self.gflat, views = _flat_views(dev, [(R,) + l.shape for l in lins])
        self.grads = {l.name: v for l, v in zip(lins, views)}
        self.partials = torch.zeros(1024, device=dev, dtype=torch.float64)
        self.loss = torch.zeros(len(lins) * R, device=dev, dtype=torch.float64)
        self.seq = SeqIds(dev)
        self.dev = dev
        self.plans = PlanCache()

    def stage(self, x_all, seq_ids, per_seq, seq_stride, offset):
        """Gather rows of x_all (float32 [n_rows, in]) into the X operand terms."""
        ids = self.seq(seq_ids)
        rows = len(ids) * per_seq
        if rows != self.M:
            raise ValueError(f"micro-batch has {rows} rows, step expects {self.M}")
        _lib.call("gsq_gather_split", _lib.ptr(x_all), int(x_all.dtype == torch.bfloat16),
                  x_all.shape[-1], _lib.ptr(ids),
                  int(per_seq), int(seq_stride), int(offset), self.M, self.in_f, self.nx,
                  self.X.ptrs(), self.X.ld, None, 0, _lib.stream_ptr())

    def first_forward(self, targets, t, tau, kappa, noise_seed, noise_of=None):
        """Soft weights and probabilities of the first step of the stage."""
        for lin in self.lins:
            for r in range(self.R):
                noise = None if noise_of is None else noise_of(t, r, lin)
                lin.soft(tau, kappa, t, r, noise_seed, w_ref=targets[lin.name], noise=noise,
                         terms=self.Dbuf[lin.name][r], probs=self.probs[lin.name][r])

    def contract(self, dp=None):
        """Gram matrix of the micro-batch (summed over the ranks of ``dp``), then the weight
        gradients and losses of every linear and resample (global: no further reduction)."""
        from ..gemm import split_into
        st = _lib.stream_ptr()
        self.plans.run("gram", self.X, self.X, M=self.in_f, N=self.in_f, K=self.M, C=self.Hf,
                       a_major=1, b_major=1)
        if dp is not None:
            dp.allreduce(self.Hf)
        split_into(self.Hf, self.Hm)
        for li, lin in enumerate(self.lins):
            G = self.grads[lin.name]
            norm = self.M_total * lin.out_f
            for r in range(self.R):
                self.plans.run(("grad", li, r), self.D[lin.name][r], self.Hm, alpha=2.0 / norm,
                               C=G[r])
                t = self.D[lin.name][r].t
                slot = self.loss[li * self.R + r:li * self.R + r + 1]
                _lib.call("gsq_dot_terms", _lib.ptr(t[0]), _lib.ptr(t[1]), _lib.ptr(t[2]),
                          lin.in_f, _lib.ptr(G[r]), lin.in_f, lin.out_f, lin.in_f, norm / 2.0,
                          _lib.ptr(self.partials), _lib.ptr(slot), st)

    def update(self, targets, t, tau, kappa, opts, noise_seed, nxt=None, noise_of=None):
        """Fused backward + Lion of step t; nxt = (t1, tau1, kappa1) also runs step t1's forward."""
        for lin in self.lins:
            n = None
            if nxt is not None:
                t1, tau1, kappa1 = nxt
                noise = None
                if noise_of is not None:
                    noise = torch.stack([noise_of(t1, r, lin) for r in range(self.R)]).contiguous()
                n = {"step": t1, "tau": tau1, "kappa": kappa1, "seed": noise_seed,
                     "w_ref": targets[lin.name], "terms": self.Dbuf[lin.name], "noise": noise}
            lin.step(self.probs[lin.name], self.grads[lin.name], tau, kappa, opts.lr_logits,
                     opts.lr_scales, nxt=n)

    def mean_loss(self):
        """sum over linears of mean R^2, averaged over resamples (staged.py:386-394)."""
        la = self.loss.view(len(self.lins), self.R).cpu().numpy()
        denom = np.array([self.M_total * lin.out_f for lin in self.lins],
                         dtype=np.float64)[:, None]
        return float((la / denom).sum(axis=0).sum() / self.R)


def train_linears(lins, x_all, targets, n_seqs, opts: BlockOpts, seed, noise_of=None,
                  noise_seed=None, exact_bf16_rows=False, timer=None, name="qk", dp=None):
    """qk-stage optimiser: loss = sum over linears of mean ||X (W_bar - W)^T||^2.

    x_all: float32 CUDA tensor [n_seqs, T, in] of the linears' inputs; each step draws a sorted
    micro-batch of sequences from the reference's numpy stream (staged.py:373,380) and uses
    their positions 1..T-1. targets[name] is the float32 CUDA weight W. noise_of(t, r, lin),
    if given, returns host-supplied Gumbel planes [K, d] (parity runs); otherwise the kernels
    draw Philox noise keyed by ``noise_seed`` (default: seed). exact_bf16_rows declares the
    rows exactly representable in bf16 (one operand term instead of three).
    Returns (history, median_ms)."""
    if not lins or opts.steps == 0:
        return [], None
    rng = np.random.default_rng(seed)
    n_seq, T, in_f = x_all.shape
    noise_seed = seed if noise_seed is None else noise_seed
    dp = dp or DataParallel()
    m = min(opts.micro_batch, n_seqs // dp.total(1))
    p0, p1 = dp.window(1, T)
    step = LinearStep(lins, m * (p1 - p0), in_f, opts.resamples, 1 if exact_bf16_rows else 3,
                      M_total=dp.total(m) * (T - 1))
    flat = x_all.view(n_seq * T, in_f)
    err_flag(step.dev).zero_()
    hist = torch.zeros(opts.steps, len(lins) * step.R, device=step.dev, dtype=torch.float64)
    timer = timer or StageTimer(min(3, opts.steps - 1))
    tau, kappa = gs_schedules(0, opts.steps)
    step.first_forward(targets, 0, tau, kappa, noise_seed, noise_of)
    for t in range(opts.steps):
        timer.begin(name, t)
        tau, kappa = gs_schedules(t, opts.steps)
        idx = dp.draw(rng, n_seqs, m)
        step.stage(flat, idx, p1 - p0, T, p0)
        step.contract(dp)
        nxt = (t + 1, *gs_schedules(t + 1, opts.steps)) if t + 1 < opts.steps else None
        step.update(targets, t, tau, kappa, opts, noise_seed, nxt=nxt, noise_of=noise_of)
        hist[t].copy_(step.loss)  # a device copy; summed on the host at the end
        timer.end(name, t, t == opts.steps - 1)
    check_err(step.dev)
    denom = torch.tensor([step.M_total * lin.out_f for lin in lins], device=step.dev,
                         dtype=torch.float64)
    per_lin = hist.view(opts.steps, len(lins), step.R).sum(2)
    history = ((per_lin / denom).sum(1) / step.R).cpu().tolist()
    return history, (round(timer.ms[name], 4) if name in timer.ms else None)


# ------------------------------------------------------------------------- block stages ---

class DataParallel:
    """Data parallelism of the GSQ stages over calibration tokens, one of two splits:

    * "sequences" (weak scaling): every rank draws the same global micro-batch of
      m x world sequences from the replicated numpy stream (the reference's sorted draw,
      staged.py:373,380) and takes its own m of them; the loss is the mean over the whole
      global micro-batch, so one rank's gradients are a share of the global ones.
    * "positions" (strong scaling): every rank draws the same m sequences and takes one
      window of positions of each.

    The default is "positions": the reference's step (micro-batch 2) at any number of ranks;
    "sequences" trains on a global micro-batch of m x world sequences per step.

    Either way each rank computes dL/dw_bar of every resample on its rows, one all-reduce per
    step sums the weight gradients (4 B per weight per resample: the logit and scale
    gradients are linear maps of them) and the loss partials, and every rank runs the
    identical fused Lion update, so the soft-weight states stay bit-identical across ranks. A
    single process is world 1, where both splits are the reference's step."""

    def __init__(self, group=None, split="positions"):
        import torch.distributed as dist
        if split not in ("sequences", "positions"):
            raise ValueError(f"split must be 'sequences' or 'positions', got {split!r}")
        on = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
        self.dist = dist if on else None
        self.group = group
        self.world = dist.get_world_size(group) if on else 1
        self.rank = dist.get_rank(group) if on else 0
        self.split = split

    def window(self, lo, hi):
        """This rank's contiguous share [a, b) of the positions [lo, hi) (all of them when
        the ranks split sequences)."""
        if self.split == "sequences":
            return lo, hi
        return self.share(lo, hi)

    def share(self, lo, hi):
        """This rank's contiguous share [a, b) of the range [lo, hi)."""
        base, extra = divmod(hi - lo, self.world)
        a = lo + self.rank * base + min(self.rank, extra)
        return a, a + base + (1 if self.rank < extra else 0)

    def total(self, m):
        """Sequences of the global micro-batch when each rank takes m."""
        return m * self.world if self.split == "sequences" else m

    def draw(self, rng, n_seqs, m):
        """This rank's sorted sequence ids of one step's micro-batch (m of them)."""
        g = self.total(m)
        if g > n_seqs:
            raise ValueError(f"a global micro-batch of {g} sequences needs at least {g} "
                             f"calibration sequences, got {n_seqs}")
        idx = np.sort(rng.choice(n_seqs, size=g, replace=False))
        if self.split == "sequences":
            return idx[self.rank * m:(self.rank + 1) * m]
        return idx

    def allreduce(self, *tensors):
        if self.dist is not None:
            for t in tensors:
                self.dist.all_reduce(t, group=self.group)


def _flat_views(dev, shapes):
    """One float32 buffer with contiguous views of the given shapes (one all-reduce per step)."""
    sizes = [int(np.prod(sh)) for sh in shapes]
    flat = torch.empty(sum(sizes), device=dev, dtype=torch.float32)
    views, off = [], 0
    for sh, n in zip(shapes, sizes):
        views.append(flat[off:off + n].view(sh))
        off += n
    return flat, views


class SeqIds:
    """A step's micro-batch sequence ids on the device without stalling the host: the ids go
    through a ring of pinned host slots (a copy from pageable memory would wait for the stream
    to drain, so the host could never launch ahead of the GPU). A host slot is rewritten only
    after its previous copy has completed (one CUDA event per slot); the device slots are
    reused in stream order."""

    def __init__(self, dev, n=64, slots=4):
        self.host = torch.empty(slots, n, dtype=torch.int32).pin_memory()
        self.dev = torch.zeros(slots, n, dtype=torch.int32, device=dev)
        self.events = [None] * slots
        self.k = 0

    def __call__(self, ids):
        k = self.k
        self.k = (k + 1) % len(self.events)
        if self.events[k] is not None:
            self.events[k].synchronize()
        a = np.asarray(ids, dtype=np.int32)
        self.host[k, :a.size] = torch.from_numpy(a)
        d = self.dev[k, :a.size]
        d.copy_(self.host[k, :a.size], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.events[k] = ev
        return d


def _gather(src, ids_t, per_seq, stride, offset, rows, cols, n_terms, row_terms=None,
            col_terms=None):
    """Rows seq * stride + offset + r (r < per_seq) of src into operand terms."""
    _lib.call("gsq_gather_split", _lib.ptr(src), int(src.dtype == torch.bfloat16), src.shape[-1],
              _lib.ptr(ids_t), int(per_seq), int(stride), int(offset), int(rows), int(cols),
              int(n_terms), None if row_terms is None else row_terms.ptrs(),
              0 if row_terms is None else row_terms.ld,
              None if col_terms is None else col_terms.ptrs(),
              0 if col_terms is None else col_terms.ld, _lib.stream_ptr())


def _col_terms(base: Terms, col0: int, cols: int) -> Terms:
    """Columns [col0, col0 + cols) of a Terms operand as a Terms view (same rows and ld)."""
    v = Terms.__new__(Terms)
    v.rows, v.cols, v.n, v.ld = base.rows, int(cols), base.n, base.ld
    v.t = [t[:, col0:] for t in base.t]
    return v


def _bf16_rows(x):
    """A bf16 tensor [rows, cols] as a one-term operand."""
    return Terms(x.shape[0], x.shape[1], 1, ld=x.shape[1], tensors=[x])


class _StageBase:
    """Soft-weight buffers and the fused update shared by the vo and mlp stage steps."""

    def _init_soft(self, lins, R, dev):
        self.lins, self.R, self.dev = lins, int(R), dev
        self.plans = PlanCache()
        self.seq = SeqIds(dev)
        self.Dbuf = {l.name: torch.zeros(R, 3, l.out_f, l.in_f, device=dev, dtype=torch.bfloat16)
                     for l in lins}
        self.D = {l.name: [Terms(l.out_f, l.in_f, 3, ld=l.in_f, tensors=self.Dbuf[l.name][r])
                           for r in range(R)] for l in lins}
        self.probs = {l.name: torch.zeros(R, l.K, l.d, device=dev, dtype=torch.float32)
                      for l in lins}
        self.loss = torch.zeros(R, device=dev, dtype=torch.float64)

    def first_forward(self, t, tau, kappa, noise_seed, noise_of=None):
        for lin in self.lins:
            for r in range(self.R):
                noise = None if noise_of is None else noise_of(t, r, lin)
                lin.soft(tau, kappa, t, r, noise_seed, noise=noise, terms=self.Dbuf[lin.name][r],
                         probs=self.probs[lin.name][r])

    def update(self, t, tau, kappa, opts, noise_seed, nxt=None, noise_of=None):
        for lin in self.lins:
            n = None
            if nxt is not None:
                t1, tau1, kappa1 = nxt
                noise = None
                if noise_of is not None:
                    noise = torch.stack([noise_of(t1, r, lin) for r in range(self.R)]).contiguous()
                n = {"step": t1, "tau": tau1, "kappa": kappa1, "seed": noise_seed,
                     "terms": self.Dbuf[lin.name], "noise": noise}
            lin.step(self.probs[lin.name], self.grad_of(lin), tau, kappa, opts.lr_logits,
                     opts.lr_scales, nxt=n)

    def mean_loss(self):
        return float(self.loss.sum().item() / (self.R * self.count))


class MLPStep(_StageBase):
    """The mlp stage step (staged.py:345-354): Y = h1 + (silu(mn Wg^T) * (mn Wu^T)) Wd^T with soft
    gate / up / down, loss mean((Y - Y_fp)^2) over positions 1.. of the micro-batch. The
    attention is hard, so its outputs h1 and mn = rmsnorm(h1) are fixed per sequence and come
    from a cache. Per resample, five tensor-core GEMMs with fused epilogues:
      F1  gate | up = mn [Wg|Wu]^T       SwiGLU epilogue: g, u (float32), d = silu(g) u as terms
      F3  r = h1 + d Wd^T - Y_fp         residual-loss epilogue: loss partials, dR = 2 r / count
      B1  dL/dWd = dR^T d                dR and d read MN-major (row-major, as their transposes)
      B2  dd = dR Wd                     Wd read MN-major; SwiGLU-backward epilogue: dL/dg and
                                         dL/du as row-major terms [dg | du]
      B3  dL/dWg = dg^T mn, dL/dWu = du^T mn    [dg | du] and mn read MN-major
    No operand is transposed in memory: every reduction over the micro-batch rows reads the
    row-major activations through MN-major tensor-core operands.
    """

    def __init__(self, lins, cfg, m, T, R, window=None, m_total=None):
        """window: this rank's positions [p0, p1) of each sequence (default all of 1..T-1);
        m_total: sequences of the global micro-batch (the loss normalisation; default m)."""
        gate, up, down = lins
        dev = gate.logits.device
        self._init_soft(lins, R, dev)
        H, I = cfg.hidden, cfg.inter
        self.p0, p1 = window or (1, T)
        self.w = p1 - self.p0
        M = m * self.w
        self.m_total = int(m if m_total is None else m_total)
        self.cfg, self.m, self.T, self.M = cfg, m, T, M
        self.count = self.m_total * (T - 1) * H
        bf = torch.bfloat16
        self.MN = Terms(M, H, 1, dev)
        self.H1 = Terms(M, H, 1, dev)
        self.Y = Terms(M, H, 1, dev)
        self.g = torch.empty(M, I, device=dev, dtype=torch.float32)
        self.u = torch.empty(M, I, device=dev, dtype=torch.float32)
        self.DIN = Terms(M, I, 3, dev)
        self.DR = Terms(M, H, 3, dev)
        self.DGU = Terms(M, 2 * I, 3, dev)
        self.DG, self.DU = _col_terms(self.DGU, 0, I), _col_terms(self.DGU, I, I)
        self.gflat, (self.grad_gu, self.grad_d) = _flat_views(dev, [(2, R, I, H), (R, H, I)])
        tiles = ((M + 127) // 128) * ((H + 127) // 128)
        self.sq = torch.zeros(tiles, device=dev, dtype=torch.float64)
        self.names = (gate.name, up.name, down.name)

    def grad_of(self, lin):
        g, u, d = self.names
        return self.grad_gu[0] if lin.name == g else (self.grad_gu[1] if lin.name == u else self.grad_d)

    def stage(self, mn_all, h1_all, y_all, seq_ids):
        """Positions 1.. of the chosen sequences of the caches (bf16 [N*T, H])."""
        H, T = self.cfg.hidden, self.T
        ids = self.seq(seq_ids)
        _gather(mn_all, ids, self.w, T, self.p0, self.M, H, 1, self.MN)
        _gather(h1_all, ids, self.w, T, self.p0, self.M, H, 1, self.H1)
        _gather(y_all, ids, self.w, T, self.p0, self.M, H, 1, self.Y)

    def contract(self):
        H, I, M = self.cfg.hidden, self.cfg.inter, self.M
        gname, uname, dname = self.names
        tiles = self.sq.numel()
        for r in range(self.R):
            run = lambda name, *a, **k: self.plans.run((name, r), *a, **k)
            run("F1", self.MN, self.D[gname][r], B2=self.D[uname][r], epi=2, aux0=self.g,
                aux1=self.u, c_terms=self.DIN)
            run("F3", self.DIN, self.D[dname][r], epi=1, resid=self.H1.t[0], target=self.Y.t[0],
                ld_rt=self.H1.ld, out_scale=2.0 / self.count, sq_partial=self.sq,
                c_terms=self.DR)
            _lib.call("gsq_sum_f64", _lib.ptr(self.sq), tiles, _lib.ptr(self.loss[r:r + 1]),
                      _lib.stream_ptr())
            run("B1", self.DR, self.DIN, C=self.grad_d[r], a_major=1, b_major=1)
            run("B2", self.DR, self.D[dname][r], b_major=1, epi=3, aux0=self.g, aux1=self.u,
                c_terms=self.DGU, ct_up_rows=I)
            run("B3g", self.DG, self.MN, C=self.grad_gu[0, r], ldc=H, a_major=1, b_major=1)
            run("B3u", self.DU, self.MN, C=self.grad_gu[1, r], ldc=H, a_major=1, b_major=1)


class VOStep(_StageBase):
    """The vo stage step (staged.py:332-342): A = (P v) Wo^T with soft v / o, loss
    mean((A - A_fp)^2) over positions 1.. per sequence, averaged over the micro-batch. q and k
    are hard, so the probabilities P come from the cached q / k of the chosen sequences. This
    rank takes the query positions [q0, q1) of every micro-batch sequence (all of them in one
    process) and the keys 0..q1-1 they see. Per resample:
      V     v^T = (hn Wv^T + bv)^T per sequence (keys)      bias epilogue, transposed terms
      PV    o = P v per (sequence, head)                    causal k-range when q0 = 0
      Y     r = o Wo^T - A_fp (0 at position 0)             residual-loss epilogue: dY = 2 r / n
      Go    dL/dWo = dY^T o                                 dY, o read MN-major
      dO    dO^T = (dY Wo)^T per sequence
      dV    P^T dO per (sequence, head), summed over the heads of each kv head (P MN-major)
      Gv    dL/dWv = dV^T hn
    """

    def __init__(self, lins, cfg, m, T, R, v_bias, window=None, m_total=None):
        """window: this rank's query positions [q0, q1) (default all); m_total: sequences of the
        global micro-batch (the loss normalisation; default m)."""
        v, o = lins
        dev = v.logits.device
        self._init_soft(lins, R, dev)
        c = cfg
        H, nh, nkv, hd = c.hidden, c.n_heads, c.n_kv, c.head_dim
        self.q0, q1 = window or (0, T)
        self.Tq, self.Tk = q1 - self.q0, q1
        Tq, Tk = self.Tq, self.Tk
        self.m_total = int(m if m_total is None else m_total)
        self.cfg, self.m, self.T = cfg, m, T
        self.count = self.m_total * (T - 1) * H
        self.HN, self.HNT = Terms(m * Tk, H, 1, dev), Terms(H, m * Tk, 1, dev)
        self.A = Terms(m * Tq, H, 1, dev)
        self.QK = torch.empty(m * Tk, (nh + nkv) * hd, device=dev, dtype=torch.bfloat16)
        self.q_rot = Terms(m * nh * Tk, hd, 3, dev)
        self.k_rot = Terms(m * nkv * Tk, hd, 3, dev)
        self.scores = torch.empty(m * nh, Tq, Tk, device=dev, dtype=torch.float32)
        self.P = Terms(m * nh * Tq, Tk, 1, dev)
        # dV = P^T dO reads P as an MN-major operand when the query window is whole k-blocks;
        # otherwise through a transposed copy
        self.PT = None if Tq % 64 == 0 else Terms(m * nh * Tk, Tq, 1, dev)
        self.VT = Terms(m * nkv * hd, Tk, 3, dev)
        self.O = Terms(m * Tq, H, 3, dev)
        self.DY = Terms(m * Tq, H, 3, dev)
        self.DoT = Terms(H, H, 3, dev)
        self.DOT = Terms(m * H, Tq, 3, dev)
        self.dv = torch.empty(m * nh, Tk, hd, device=dev, dtype=torch.float32)
        self.DVT = Terms(nkv * hd, m * Tk, 3, dev)
        self.gflat, (self.grad_v, self.grad_o) = _flat_views(dev, [(R, nkv * hd, H), (R, H, H)])
        tiles = ((m * Tq + 127) // 128) * ((H + 127) // 128)
        self.sq = torch.zeros(tiles, device=dev, dtype=torch.float64)
        self.v_bias = v_bias.float().contiguous()
        self.names = (v.name, o.name)
        from .e2e import rope_tables
        cos, sin = rope_tables(T, hd, c.theta)
        self.cos = torch.as_tensor(cos, device=dev)
        self.sin = torch.as_tensor(sin, device=dev)

    def grad_of(self, lin):
        return self.grad_v if lin.name == self.names[0] else self.grad_o

    def stage(self, hn_all, a_all, qk_all, seq_ids):
        """Positions 0..q1-1 of the chosen sequences: hn and the hard q|k rows; the target A_fp
        of the query positions q0..q1-1; then the causal probabilities P of the query rows over
        their keys (and P^T)."""
        c, T, m = self.cfg, self.T, self.m
        H, Tq, Tk, q0 = c.hidden, self.Tq, self.Tk, self.q0
        ids = self.seq(seq_ids)
        _gather(hn_all, ids, Tk, T, 0, m * Tk, H, 1, self.HN, self.HNT)
        _gather(a_all, ids, Tq, T, q0, m * Tq, H, 1, self.A)
        qkw = qk_all.shape[1]
        QKt = Terms(m * Tk, qkw, 1, ld=qkw, tensors=[self.QK])
        _gather(qk_all, ids, Tk, T, 0, m * Tk, qkw, 1, QKt)
        st = _lib.stream_ptr()
        qd = c.n_heads * c.head_dim
        t = self.q_rot.t
        _lib.call("gsq_rope_split", _lib.ptr(self.QK), qkw, m, Tk, c.n_heads, _lib.ptr(self.cos),
                  _lib.ptr(self.sin), _lib.ptr(t[0]), _lib.ptr(t[1]), _lib.ptr(t[2]), st)
        t = self.k_rot.t
        from .e2e import C_ptr
        _lib.call("gsq_rope_split", C_ptr(self.QK[:, qd:]), qkw, m, Tk, c.n_kv, _lib.ptr(self.cos),
                  _lib.ptr(self.sin), _lib.ptr(t[0]), _lib.ptr(t[1]), _lib.ptr(t[2]), st)
        B = m * c.n_heads
        if q0 == 0:   # square: tiles above the diagonal are never read
            self.plans.run("scores", self.q_rot, self.k_rot, M=Tk, N=Tk, K=c.head_dim, batch=B,
                           alpha=1.0 / 8.0, C=self.scores, ldc=Tk, a_off=(1, Tk, 0),
                           b_off=(c.rep, Tk, 0), c_off=(1, Tk * Tk, 0), skip_upper=True)
        else:         # the query rows q0.. of each (sequence, head) block of q_rot
            qv = Terms(self.q_rot.rows - q0, c.head_dim, 3, ld=self.q_rot.ld,
                       tensors=[x[q0:] for x in self.q_rot.t])
            self.plans.run("scores", qv, self.k_rot, M=Tq, N=Tk, K=c.head_dim, batch=B,
                           alpha=1.0 / 8.0, C=self.scores, ldc=Tk, a_off=(1, Tk, 0),
                           b_off=(c.rep, Tk, 0), c_off=(1, Tq * Tk, 0))
        _lib.call("gsq_softmax_causal_rows", _lib.ptr(self.scores), B, Tq, Tk, Tk, q0,
                  _lib.ptr(self.P.t[0]), self.P.ld, st)
        if self.PT is not None:
            # P^T feeds the causal dV GEMM when q0 = 0: the transposes of P's zero tiles are unread
            _lib.call("gsq_transpose_bf16", _lib.ptr(self.P.t[0]), Tq, Tk, self.P.ld,
                      Tq * self.P.ld, _lib.ptr(self.PT.t[0]), self.PT.ld, Tk * self.PT.ld, B,
                      int(q0 == 0), st)

    def contract(self):
        c, m = self.cfg, self.m
        H, nh, hd = c.hidden, c.n_heads, c.head_dim
        Tq, Tk, q0 = self.Tq, self.Tk, self.q0
        nkvd = c.n_kv * hd
        vname, oname = self.names
        tiles = self.sq.numel()
        st = _lib.stream_ptr()
        B = m * nh
        for r in range(self.R):
            run = lambda name, *a, **k: self.plans.run((name, r), *a, **k)
            # 128 x 64 tiles: 2 x 16 x 2 = 64 CTAs for the two 64-wide kv heads of 2 sequences
            run("V", self.HN, self.D[vname][r], M=Tk, batch=m, bias=self.v_bias, a_off=(1, Tk, 0),
                ct_terms=self.VT, t_off=(1, nkvd, 0, 0, 0), bn=64)
            run("PV", self.P, self.VT, M=Tq, N=hd, K=Tk, batch=B, bn=64, causal=int(q0 == 0),
                 a_off=(1, Tq, 0), b_off=(c.rep, hd, 0), c_off=(nh, Tq * H, hd),
                 c_terms=self.O)
            run("Y", self.O, self.D[oname][r], epi=1, target=self.A.t[0], ld_rt=self.A.ld,
                 row_period=Tq if q0 == 0 else 0, out_scale=2.0 / self.count,
                 sq_partial=self.sq, c_terms=self.DY)
            _lib.call("gsq_sum_f64", _lib.ptr(self.sq), tiles, _lib.ptr(self.loss[r:r + 1]), st)
            run("dWo", self.DY, self.O, M=H, N=H, K=m * Tq, C=self.grad_o[r], a_major=1, b_major=1)
            for i in range(3):
                _lib.call("gsq_transpose_bf16", _lib.ptr(self.Dbuf[oname][r][i]), H, H, H, 0,
                          _lib.ptr(self.DoT.t[i]), self.DoT.ld, 0, 1, 0, st)
            run("dO", self.DY, self.DoT, M=Tq, batch=m, a_off=(1, Tq, 0), ct_terms=self.DOT,
                 t_off=(1, H, 0, 0, 0))
            if self.PT is None:
                run("dV", self.P, self.DOT, M=Tk, N=hd, K=Tq, batch=B, bn=64,
                     causal=2 if q0 == 0 else 0, a_off=(1, Tq, 0), b_off=(1, hd, 0), C=self.dv,
                     ldc=hd, c_off=(1, Tk * hd, 0), a_major=1)
            else:
                run("dV", self.PT, self.DOT, M=Tk, N=hd, K=Tq, batch=B, bn=64,
                     causal=2 if q0 == 0 else 0, a_off=(1, Tk, 0), b_off=(1, hd, 0), C=self.dv,
                     ldc=hd, c_off=(1, Tk * hd, 0))
            t = self.DVT.t
            _lib.call("gsq_head_group_sum_t", _lib.ptr(self.dv), m, nh, c.rep, Tk, _lib.ptr(t[0]),
                      _lib.ptr(t[1]), _lib.ptr(t[2]), self.DVT.ld, st)
            run("dWv", self.DVT, self.HNT, C=self.grad_v[r])


class StageTimer:
    """CUDA-event timing of the steps after the first `warmup` of each stage: ms[name]. With
    nvtx=True the timed steps of every stage also form an NVTX range "gsq_steps" (a profiler
    filter for the launch list of the steps alone). With a gemm.LaunchLog, the log records the
    GEMM launches of the timed steps only, tagged with the stage name."""

    def __init__(self, warmup=3, nvtx=False, launch_log=None):
        self.warmup = int(warmup)
        self.nvtx = bool(nvtx)
        self.launch_log = launch_log
        self.ms = {}
        self.launches = {}  # our kernel launches inside each stage's timed steps
        self._ev = {}
        self._n0 = {}

    def begin(self, name, t):
        """At the start of step t."""
        if t == self.warmup:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._ev[name] = e
            self._n0[name] = _lib.Launches.n
            if self.nvtx:
                torch.cuda.nvtx.range_push("gsq_steps")
            if self.launch_log is not None:
                from ..gemm import LaunchLog
                self.launch_log.tag = name
                LaunchLog.active = self.launch_log

    def end(self, name, t, last):
        """After step t; last closes the timed range: ms[name] = mean over steps warmup..t."""
        if last and name in self._ev:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.launches[name] = _lib.Launches.n - self._n0[name]
            if self.launch_log is not None:
                from ..gemm import LaunchLog
                LaunchLog.active = None
            if self.nvtx:
                torch.cuda.nvtx.range_pop()
            e.synchronize()
            n = t + 1 - self.warmup
            self.ms[name] = self._ev[name].elapsed_time(e) / max(n, 1)


def train_stage(step, stage_args_of, n_seqs, opts: BlockOpts, seed, noise_seed=None,
                noise_of=None, timer=None, name="stage", dp=None):
    """The stage optimiser loop (staged.py:357-400) around a vo / mlp step: schedules, the
    sorted micro-batch draw of the numpy stream, contractions, the fused update with the next
    step's forward. stage_args_of(idx) returns the arguments of step.stage for sequence ids idx.
    The per-step mean soft loss stays on the device until the end. Returns (history, ms/step)."""
    if opts.steps == 0:
        return [], None
    rng = np.random.default_rng(seed)
    m = step.m
    noise_seed = seed if noise_seed is None else noise_seed
    draw = (dp or DataParallel()).draw
    err_flag(step.dev).zero_()
    tau, kappa = gs_schedules(0, opts.steps)
    step.first_forward(0, tau, kappa, noise_seed, noise_of)
    hist = torch.zeros(opts.steps, step.R, device=step.dev, dtype=torch.float64)
    timer = timer or StageTimer(min(3, opts.steps - 1))
    for t in range(opts.steps):
        timer.begin(name, t)
        tau, kappa = gs_schedules(t, opts.steps)
        idx = draw(rng, n_seqs, m)
        step.stage(*stage_args_of(idx))
        step.contract()
        if dp is not None:
            dp.allreduce(step.gflat, step.loss)
        nxt = (t + 1, *gs_schedules(t + 1, opts.steps)) if t + 1 < opts.steps else None
        step.update(t, tau, kappa, opts, noise_seed, nxt=nxt, noise_of=noise_of)
        hist[t].copy_(step.loss.view(-1))  # a device copy; summed on the host at the end
        timer.end(name, t, t == opts.steps - 1)
    check_err(step.dev)
    history = (hist.sum(1) / (step.R * step.count)).cpu().tolist()
    return history, (round(timer.ms[name], 4) if name in timer.ms else None)


# --------------------------------------------------------------------- block quantizer ---

def _hard_bf16(codes_t, scales16, bits, group_size):
    """Stored form (uint8 codes, fp16 scales) -> the bf16 weight the stream uses
    (staged.py:194-196): dequantize with the fp16-rounded scales, cast to bf16."""
    from .gptq import dequantize
    w = dequantize(codes_t, torch.as_tensor(np.asarray(scales16, dtype=np.float32)), bits,
                   group_size, device=True)
    return w.to(torch.bfloat16)


def quantize_block(h, W: dict, bits: dict, opts: BlockOpts, layer: int, cfg=None, T=None,
                   chunk_seqs=8, log=print, noise_of=None, timer=None, dp=None, record=None):
    """Quantize the seven linears of one block on the calibration stream (staged.py:405-522).

    h: bf16 CUDA [N*T, H], the block inputs of the N calibration sequences (the quantized
    prefix). W: bf16 CUDA block weights (linears, q/k/v biases, in_norm, post_norm).
    Returns (shard, stats, Wq): shard[name] = {"codes" uint8 [out, in], "scales" float16, "bits"},
    Wq the bf16 hard weights of the block. Each stage: GPTQ warm start from the Hessian of its
    real input, Lion training of logits and group scales, hardening (argmax codes, fp16 scales).
    dp: a DataParallel over the ranks of a process group (each rank computes its position
    window of every micro-batch sequence; the stage gradients are summed over the ranks); the
    Hessian passes and GPTQ run on every rank alike, so every rank returns the same result.
    record: a dict that receives record["warm_start"][name] = {"codes", "scales"}, the GPTQ
    warm start of each linear (host arrays).
    """
    from .e2e import BlockConfig, BlockWeights, LIN_ORDER, Qwen2Block
    from .gptq import gptq_factor, quantize_gptq
    cfg = cfg or BlockConfig()
    H = cfg.hidden
    N = h.shape[0] // T
    dev = h.device
    gs = opts.group_size
    seed = opts.seed * 1_000_003 + layer * 1_009
    cs = min(chunk_seqs, N)
    eng = Qwen2Block(cfg, cs, T, dev)
    W_fp = BlockWeights(W)
    Wf = {name: W[name].float().contiguous() for name in LIN_ORDER}
    Wcur = dict(W)
    shard, stats = {}, {"stages": {}, "linears": {}}
    factors = {}
    pos_of = {name: i for i, name in enumerate(LIN_ORDER)}
    inits = ShiftInitPool({name: (W[name].numel(), seed + 10 * pos_of[name])
                           for name in LIN_ORDER if 3 <= bits[name] <= 7})

    def chunks():
        for a in range(0, N, cs):
            yield a, min(cs, N - a)

    def hessian(site, Wb, extra=None, mn_src=None):
        """Hessian of the input of `site` over positions 1.., under block weights Wb; the
        forward ends at the site (and starts at the MLP from cached rows mn_src)."""
        width = cfg.inter if site == "d_in" else H
        Hs = torch.zeros(width, width, device=dev, dtype=torch.float64)
        n = 0
        for a, s in chunks():
            rows = slice(a * T, (a + s) * T)
            if mn_src is not None:
                eng.forward(None, Wb, S=s, taps=(site,), upto=site, mn=mn_src[rows])
            else:
                eng.forward(h[rows], Wb, S=s, taps=(site,), upto=site)
            n = eng.hessian_add(site, Hs, n, S=s)
            if extra:
                extra(a, s)
        return Hs

    def gptq(name, Hs, pos):
        key = id(Hs)
        if key not in factors:
            factors[key] = gptq_factor(Hs, opts.damp)
        g = quantize_gptq(Wf[name], Hs, bits[name], gs, opts.damp, opts.block_size, device=True,
                          factor=factors[key])
        s16 = g["scales"].cpu().numpy().astype(np.float16)
        codes = g["codes"].cpu().numpy()
        Wcur[name] = _hard_bf16(g["codes"], s16, bits[name], gs)
        stats["linears"].setdefault(name, {"bits": bits[name]})["err_gptq"] = float(g["err"].item())
        if record is not None:
            record.setdefault("warm_start", {})[name] = {"codes": codes, "scales": s16}
        if bits[name] == 8:
            shard[name] = {"codes": codes, "scales": s16, "bits": 8}
            return None
        return SoftLinear(name, bits[name], codes, s16, gs, seed=seed + 10 * pos,
                          linear_id=layer * 8 + pos, logits0=inits.take(name))

    def harden(lin):
        codes = lin.hard_codes()
        s16 = lin.stored_scales()
        Wcur[lin.name] = _hard_bf16(torch.as_tensor(codes, device=dev), s16, lin.bits, gs)
        shard[lin.name] = {"codes": codes, "scales": s16, "bits": lin.bits}
        stats["linears"][lin.name]["flip_frac"] = float(np.mean(codes != lin.codes0))

    def stage_done(stage, t0, hist, ms):
        stats["stages"][stage] = {"seconds": round(time.perf_counter() - t0, 3), "steps": len(hist),
                                  "ms_per_step": ms,
                                  "soft_loss_first": hist[0] if hist else None,
                                  "soft_loss_last": hist[-1] if hist else None}
        log(f"    stage {stage}: {len(hist)} steps, {ms} ms/step, "
            f"{stats['stages'][stage]['seconds']:.2f} s")

    # ---- qk: linear reconstruction on hn rows -------------------------------------------
    t0 = time.perf_counter()
    hn_all = torch.empty(N * T, H, device=dev, dtype=torch.bfloat16)

    def keep_hn(a, s):
        hn_all[a * T:(a + s) * T].copy_(eng.hn[:s * T])
    H_hn = hessian("hn", W_fp, keep_hn)
    qk = [gptq(n, H_hn, i) for i, n in enumerate(STAGE_LAYERS["qk"])]
    qk_lins = [l for l in qk if l is not None]
    dp = dp or DataParallel()
    hist, ms = train_linears(qk_lins, hn_all.view(N, T, H), Wf, N, opts, seed + 1, dp=dp,
                             exact_bf16_rows=True, noise_of=noise_of, timer=timer,
                             name="qk") if qk_lins else ([], None)
    for lin in qk_lins:
        harden(lin)
    stage_done("qk", t0, hist, ms)

    # ---- vo: attention output, q and k hard -----------------------------------------------
    t0 = time.perf_counter()
    v_lin = gptq("v_proj", H_hn, 2)
    H_o = hessian("o", BlockWeights(Wcur))
    o_lin = gptq("o_proj", H_o, 3)
    vo_lins = [l for l in (v_lin, o_lin) if l is not None]
    A_all = torch.empty(N * T, H, device=dev, dtype=torch.bfloat16)
    Y_all = torch.empty(N * T, H, device=dev, dtype=torch.bfloat16)
    qkw = (cfg.n_heads + cfg.n_kv) * cfg.head_dim
    qk_all = torch.empty(N * T, qkw, device=dev, dtype=torch.bfloat16)
    Wc = BlockWeights(Wcur)
    from .e2e import wterms
    for a, s in chunks():
        # full-precision targets: the attention output (vo stage) and the block output (mlp
        # stage) from one pass
        eng.forward(h[a * T:(a + s) * T], W_fp, S=s, attn_out=A_all[a * T:(a + s) * T],
                    out=Y_all[a * T:(a + s) * T])
        # hard q|k rows under the trained q / k (the vo stage's fixed attention pattern)
        gemm(_bf16_rows(hn_all[a * T:(a + s) * T]), wterms(Wc.qk), epi=4, bias=Wc.qk_bias,
             c_terms=_bf16_rows(qk_all[a * T:(a + s) * T]))
    if len(vo_lins) == 2:
        m = min(opts.micro_batch, N // dp.total(1))
        vstep = VOStep(vo_lins, cfg, m, T, opts.resamples, W["v_bias"],
                       window=dp.window(0, T), m_total=dp.total(m))
        hist, ms = train_stage(vstep, lambda idx: (hn_all, A_all, qk_all, idx), N, opts,
                               seed + 2, noise_of=noise_of, timer=timer, name="vo", dp=dp)
    else:
        hist, ms = [], None  # an 8-bit v or o keeps its GPTQ values (not trained here)
    for lin in vo_lins:
        harden(lin)
    stage_done("vo", t0, hist, ms)
    del A_all, qk_all

    # ---- mlp: block output, attention hard -------------------------------------------------
    t0 = time.perf_counter()
    mn_all = torch.empty(N * T, H, device=dev, dtype=torch.bfloat16)
    h1_all = torch.empty(N * T, H, device=dev, dtype=torch.bfloat16)

    def keep_mn(a, s):
        mn_all[a * T:(a + s) * T].copy_(eng.mn[:s * T])
        h1_all[a * T:(a + s) * T].copy_(eng.h1[:s * T])
    H_gu = hessian("mn", BlockWeights(Wcur), keep_mn)
    gate, up = gptq("gate_proj", H_gu, 4), gptq("up_proj", H_gu, 5)
    H_d = hessian("d_in", BlockWeights(Wcur), mn_src=mn_all)
    down = gptq("down_proj", H_d, 6)
    mlp_lins = [l for l in (gate, up, down) if l is not None]
    if len(mlp_lins) == 3:
        m = min(opts.micro_batch, N // dp.total(1))
        mstep = MLPStep(mlp_lins, cfg, m, T, opts.resamples, window=dp.window(1, T),
                        m_total=dp.total(m))
        hist, ms = train_stage(mstep, lambda idx: (mn_all, h1_all, Y_all, idx), N, opts,
                               seed + 3, noise_of=noise_of, timer=timer, name="mlp", dp=dp)
    else:
        hist, ms = [], None
    for lin in mlp_lins:
        harden(lin)
    stage_done("mlp", t0, hist, ms)
    inits.close()
    return shard, stats, Wcur
