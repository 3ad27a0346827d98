"""GSQ stage optimiser on the GPU (reference src/gsq_rco/gsq/staged.py).

``SoftLinear`` is the device-resident training state of one linear (staged.py:230-317):
plane-major logits and their Lion momentum, group scales and their momentum, and the GPTQ
codes j0. Its ``soft`` builds one Gumbel-softmax soft weight (staged.py:271-298) and stores
the draw's probabilities; its ``step`` is one fused pass: the soft backward from the stored
probabilities, the resample mean and Lion (staged.py:383-392 with lion.py:44-56), and the next
step's soft weights.

``train_linears`` is the qk-stage optimiser (staged.py:357-400 with the linear loss of
:322-329): per step the schedules, a sorted micro-batch draw from the numpy stream, R
resamples of (residual GEMM with the loss in its epilogue, weight-gradient GEMM), then one
fused step launch per linear.

Gumbel noise: Philox4x32-10 keyed by (stage seed, linear id) with counter (weight, block,
step, resample), drawn inside the kernels, or host-supplied planes for parity runs.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch

from .. import _lib
from ..gemm import Terms, err_flag, check_err, gemm_tc, pad8
from .gptq import init_logits_2bit_from_codes, init_shift_logits
from .lion import BETAS, LR_LOGITS, LR_SCALES, WEIGHT_DECAY, scale_lr
from .quant import gs_schedules

ALPHA_SCALAR = 6.0
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


class SoftLinear:
    """One linear under the stage optimiser: GPTQ codes and scales plus trainable logits."""

    def __init__(self, name, bits, codes, scales16, group_size, seed, linear_id=0):
        self.name, self.bits = name, int(bits)
        if not 2 <= self.bits <= 7:
            raise NotImplementedError(
                f"{name}: soft weights cover 2..7 bits (8-bit linears are GPTQ only)")
        codes = np.asarray(codes, dtype=np.uint8)
        self.shape = codes.shape
        self.out_f, self.in_f = self.shape
        self.group_size = int(group_size)
        self.linear_id = int(linear_id)
        self.codes0 = codes
        dev = _lib.device()
        self.j0 = torch.as_tensor(codes.reshape(-1), device=dev)
        d = codes.size
        if self.bits == 2:
            l0 = init_logits_2bit_from_codes(codes, 4, alpha=ALPHA_SCALAR, std=INIT_STD, seed=seed)
        else:
            l0 = init_shift_logits(d, alpha=ALPHA_SCALAR, std=INIT_STD, seed=seed)
        self.K = l0.shape[1]
        self.logits = torch.as_tensor(np.ascontiguousarray(l0.T), device=dev)
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
        ``probs`` ([K, d] float32) receives the draw's probabilities for the backward."""
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
        the next step's forward (probs updated in place, soft weights written)."""
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
        """Argmax codes of the learned logits (staged.py:300-314)."""
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
    Per resample r: R_r = X (w_bar_r - W)^T on the tensor cores (epilogue: loss partials and
    R_r^T as bf16 terms), then G_r = 2 / (M out) R_r^T X. One fused pass per linear then runs
    the backward, the resample mean, Lion, and the next step's soft weights and probabilities.
    All GEMM operands are bf16 terms (three for float32 data, one for exactly-bf16 rows)."""

    def __init__(self, lins, M, in_f, resamples, x_terms=3):
        dev = lins[0].logits.device
        self.lins, self.M, self.in_f, self.R = lins, int(M), int(in_f), int(resamples)
        self.nx = int(x_terms)
        self.X = Terms(M, in_f, self.nx, dev)        # A of the residual GEMM
        self.XT = Terms(in_f, M, self.nx, dev)       # B of the weight-gradient GEMM
        R = self.R
        self.Dbuf = {l.name: torch.zeros(R, 3, l.out_f, l.in_f, device=dev, dtype=torch.bfloat16)
                     for l in lins}
        self.D = {l.name: [Terms(l.out_f, l.in_f, 3, ld=l.in_f, tensors=self.Dbuf[l.name][r])
                           for r in range(R)] for l in lins}
        self.probs = {l.name: torch.zeros(R, l.K, l.d, device=dev, dtype=torch.float32)
                      for l in lins}
        self.RT = {l.name: Terms(l.out_f, M, 3, dev) for l in lins}
        self.grads = {l.name: torch.empty((R,) + l.shape, device=dev, dtype=torch.float32)
                      for l in lins}
        tiles = max(((M + 127) // 128) * ((l.out_f + 127) // 128) for l in lins)
        self.sq = torch.zeros(tiles, device=dev, dtype=torch.float64)
        self.loss = torch.zeros(len(lins) * R, device=dev, dtype=torch.float64)
        self.seq = torch.zeros(64, device=dev, dtype=torch.int32)
        self.dev = dev

    def stage(self, x_all, seq_ids, per_seq, seq_stride, offset):
        """Gather rows of x_all (float32 [n_rows, in]) into the X and X^T operand terms."""
        ids = torch.as_tensor(np.asarray(seq_ids, dtype=np.int32))
        self.seq[:len(ids)].copy_(ids, non_blocking=True)
        rows = len(ids) * per_seq
        if rows != self.M:
            raise ValueError(f"micro-batch has {rows} rows, step expects {self.M}")
        _lib.call("gsq_gather_split", _lib.ptr(x_all), int(x_all.dtype == torch.bfloat16),
                  x_all.shape[-1], _lib.ptr(self.seq),
                  int(per_seq), int(seq_stride), int(offset), self.M, self.in_f, self.nx,
                  self.X.ptrs(), self.X.ld, self.XT.ptrs(), self.XT.ld, _lib.stream_ptr())

    def first_forward(self, targets, t, tau, kappa, noise_seed, noise_of=None):
        """Soft weights and probabilities of the first step of the stage."""
        for lin in self.lins:
            for r in range(self.R):
                noise = None if noise_of is None else noise_of(t, r, lin)
                lin.soft(tau, kappa, t, r, noise_seed, w_ref=targets[lin.name], noise=noise,
                         terms=self.Dbuf[lin.name][r], probs=self.probs[lin.name][r])

    def contract(self):
        """Residuals, losses and weight gradients of every linear and resample."""
        for li, lin in enumerate(self.lins):
            RT, G = self.RT[lin.name], self.grads[lin.name]
            tiles = ((self.M + 127) // 128) * ((lin.out_f + 127) // 128)
            for r in range(self.R):
                gemm_tc(self.X, self.D[lin.name][r], ct_terms=RT, sq_partial=self.sq)
                slot = self.loss[li * self.R + r:li * self.R + r + 1]
                _lib.call("gsq_sum_f64", _lib.ptr(self.sq), tiles, _lib.ptr(slot),
                          _lib.stream_ptr())
                gemm_tc(RT, self.XT, alpha=2.0 / (self.M * lin.out_f), C=G[r])

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
        denom = np.array([self.M * lin.out_f for lin in self.lins], dtype=np.float64)[:, None]
        return float((la / denom).sum(axis=0).sum() / self.R)


def train_linears(lins, x_all, targets, n_seqs, opts: BlockOpts, seed, noise_of=None,
                  noise_seed=None, exact_bf16_rows=False, sync_timing=True):
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
    m = min(opts.micro_batch, n_seqs)
    n_seq, T, in_f = x_all.shape
    noise_seed = seed if noise_seed is None else noise_seed
    step = LinearStep(lins, m * (T - 1), in_f, opts.resamples, 1 if exact_bf16_rows else 3)
    flat = x_all.view(n_seq * T, in_f)
    err_flag(step.dev).zero_()
    history, step_s = [], []
    tau, kappa = gs_schedules(0, opts.steps)
    step.first_forward(targets, 0, tau, kappa, noise_seed, noise_of)
    for t in range(opts.steps):
        t0 = time.perf_counter()
        tau, kappa = gs_schedules(t, opts.steps)
        idx = np.sort(rng.choice(n_seqs, size=m, replace=False))
        step.stage(flat, idx, T - 1, T, 1)
        step.contract()
        nxt = (t + 1, *gs_schedules(t + 1, opts.steps)) if t + 1 < opts.steps else None
        step.update(targets, t, tau, kappa, opts, noise_seed, nxt=nxt, noise_of=noise_of)
        history.append(step.mean_loss())
        if sync_timing:
            torch.cuda.synchronize()
        step_s.append(time.perf_counter() - t0)
    check_err(step.dev)
    return history, round(1000 * float(np.median(step_s[3:] or step_s)), 1)
