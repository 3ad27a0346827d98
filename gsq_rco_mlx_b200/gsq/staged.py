"""GSQ stage optimiser on the GPU (reference src/gsq_rco/gsq/staged.py).

``SoftLinear`` is the device-resident training state of one linear (staged.py:230-317):
plane-major logits and their Lion momentum, group scales and their momentum, and the GPTQ
codes j0. Its ``soft`` builds one Gumbel-softmax soft weight (staged.py:271-298) and its
``backward_lion`` runs the fused soft backward + resample average + Lion
(staged.py:383-392 with lion.py:44-56), both as single CUDA launches.

``train_linears`` is the qk-stage optimiser (staged.py:357-400 with the linear loss of
:322-329): per step the schedules, a sorted micro-batch draw from the numpy stream, R
resamples of (soft weight, residual GEMM, loss, weight-gradient GEMM), then one fused
backward + Lion launch per linear.

Gumbel noise: Philox4x32-10 keyed by (stage seed, linear id) with counter (weight, block,
step, resample), drawn inside the kernels, or host-supplied planes for parity runs.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch

from .. import _lib
from ..gemm import SumSq, mm_nt, mm_tn
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

    def soft(self, tau, kappa, step, resample, seed, w_ref=None, out=None, noise=None):
        """w_bar (or w_bar - w_ref) float32 [out, in] of one Gumbel draw."""
        out = torch.empty(self.shape, device=self.logits.device, dtype=torch.float32) \
            if out is None else out
        _lib.call("gsq_soft_fwd", _lib.ptr(self.logits), _lib.ptr(self.j0), _lib.ptr(self.scales),
                  _lib.ptr(noise), int(seed) & (2 ** 64 - 1), self.linear_id, int(step),
                  int(resample), self.out_f, self.in_f, self.group_size, self.bits, float(tau),
                  float(kappa), _lib.ptr(w_ref), _lib.ptr(out), None, None, None, _lib.stream_ptr())
        return out

    def backward_lion(self, grad_w, tau, kappa, step, seed, lr_logits=LR_LOGITS,
                      lr_scales=LR_SCALES, noise=None):
        """Fused soft backward over grad_w [R, out, in], resample mean and Lion step."""
        R = grad_w.shape[0]
        _lib.call("gsq_soft_bwd_lion", _lib.ptr(self.logits), _lib.ptr(self.mom), _lib.ptr(self.j0),
                  _lib.ptr(self.scales), _lib.ptr(self.mom_s), _lib.ptr(grad_w), _lib.ptr(noise),
                  int(seed) & (2 ** 64 - 1), self.linear_id, int(step), int(R), self.out_f,
                  self.in_f, self.group_size, self.bits, float(tau), float(kappa),
                  float(lr_logits), float(scale_lr(lr_scales, self.bits)), float(WEIGHT_DECAY),
                  float(BETAS[0]), float(BETAS[1]), _lib.stream_ptr())

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


def train_linears(lins, rows_of, targets, n_seqs, opts: BlockOpts, seed, noise_of=None,
                  noise_seed=None, sync_timing=True):
    """qk-stage optimiser: loss = sum over linears of mean ||X (W_bar - W)^T||^2.

    rows_of(idx) returns the device float32 rows X [M, in] of the sorted sequence ids idx;
    targets[name] is the float32 CUDA weight W of each linear. noise_of(t, r, lin), if given,
    returns host-supplied Gumbel planes [K, d] (parity runs); otherwise the kernels draw
    Philox noise keyed by ``noise_seed`` (default: seed). Returns (history, median_ms)."""
    if not lins or opts.steps == 0:
        return [], None
    rng = np.random.default_rng(seed)
    m = min(opts.micro_batch, n_seqs)
    R = opts.resamples
    noise_seed = seed if noise_seed is None else noise_seed
    dev = lins[0].logits.device
    sumsq = SumSq(dev)
    loss_acc = torch.zeros(len(lins) * R, device=dev, dtype=torch.float64)
    grads = {lin.name: torch.empty((R,) + lin.shape, device=dev, dtype=torch.float32)
             for lin in lins}
    history, step_s = [], []
    for t in range(opts.steps):
        t0 = time.perf_counter()
        tau, kappa = gs_schedules(t, opts.steps)
        idx = np.sort(rng.choice(n_seqs, size=m, replace=False))
        X = rows_of(idx)
        M = X.shape[0]
        for li, lin in enumerate(lins):
            for r in range(R):
                noise = None if noise_of is None else noise_of(t, r, lin)
                D = lin.soft(tau, kappa, t, r, noise_seed, w_ref=targets[lin.name], noise=noise)
                Rm = mm_nt(X, D)
                sumsq(Rm, loss_acc[li * R + r:li * R + r + 1])
                mm_tn(Rm, X, alpha=2.0 / (M * lin.out_f), out=grads[lin.name][r])
            stacked = None
            if noise_of is not None:
                stacked = torch.stack([noise_of(t, r, lin) for r in range(R)]).contiguous()
            lin.backward_lion(grads[lin.name], tau, kappa, t, noise_seed, opts.lr_logits,
                              opts.lr_scales, noise=stacked)
        la = loss_acc.view(len(lins), R).cpu().numpy()
        denom = np.array([M * lin.out_f for lin in lins], dtype=np.float64)[:, None]
        history.append(float((la / denom).sum(axis=0).sum() / R))
        if sync_timing:
            torch.cuda.synchronize()
        step_s.append(time.perf_counter() - t0)
    return history, round(1000 * float(np.median(step_s[3:] or step_s)), 1)
