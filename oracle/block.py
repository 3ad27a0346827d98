"""Qwen2 decoder block and the GSQ vo / mlp stage losses: CPU restatement (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). A floating-point reference, written with
torch on the CPU: bf16 storage is emulated by rounding float32 values to bf16 at the points where
the reference's MLX arrays are bf16, products are float64 (more exact than the reference's
float32 GEMMs), and the stage gradients come from torch autograd in float64.

Follows the reference egesabanci/gsq-rco-mlx:
  rmsnorm / rope / silu           src/gsq_rco/gsq/e2e.py:90-112
  attn_core / block                src/gsq_rco/gsq/e2e.py:123-174
  _rows (positions 1..)            src/gsq_rco/gsq/staged.py:128-130
  _loss_attn (vo stage)            src/gsq_rco/gsq/staged.py:332-342
  _loss_block (mlp stage)          src/gsq_rco/gsq/staged.py:345-354
Rounding choices shared with the CUDA kernels where the reference leaves them open: the RMS
mean is a float64 sum rounded to float32; the softmax sum is float64; 1 / x is a rounded
reciprocal; sigmoid(x) = 1 / (1 + exp(-x)).
"""
from __future__ import annotations

import numpy as np
import torch

F32, F64 = torch.float32, torch.float64


def bf(x):
    """Round float values to bf16 (kept as float32)."""
    return x.to(torch.bfloat16).to(F32)


def rope_tables(T, head_dim=64, theta=1e6):
    """cos / sin [T, head_dim / 2] float32 (e2e.py:96-100), numpy float32 arithmetic."""
    ex = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    freq = (np.float32(1.0) / (np.float32(theta) ** ex)).astype(np.float32)
    ang = np.arange(T, dtype=np.float32)[:, None] * freq[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rmsnorm(x, w, eps=1e-6):
    """e2e.py:90-93 for bf16 x: bf16((x * 1/sqrt(mean x^2 + eps)) * w)."""
    xf = x.to(F32)
    var = ((xf * xf).to(F64).sum(-1, keepdim=True) / xf.shape[-1]).to(F32)
    inv = torch.reciprocal(torch.sqrt(var + eps))
    return bf((xf * inv) * w.to(F32))


def rope(x, cos, sin):
    """e2e.py:103-108, half split, float32: x [..., T, 64] bf16 values."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h].to(F32), x[..., h:].to(F32)
    c, s = torch.as_tensor(cos), torch.as_tensor(sin)
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


def sigmoid(x):
    return torch.reciprocal(1.0 + torch.exp(-x))


def attention_probs(hn, W, n_heads=14, n_kv=2, theta=1e6):
    """Causal softmax probabilities of one sequence under hard (bf16) q / k: bf16 [nh, T, T]
    (e2e.py:132-154)."""
    T = hn.shape[0]
    hd = W["q_proj"].shape[0] // n_heads
    q = bf(bf(hn.to(F64) @ W["q_proj"].to(F64).T).to(F32) + W["q_bias"])
    k = bf(bf(hn.to(F64) @ W["k_proj"].to(F64).T).to(F32) + W["k_bias"])
    cos, sin = rope_tables(T, hd, theta)
    q = rope(q.view(T, n_heads, hd).transpose(0, 1), cos, sin)          # [nh, T, hd] f32
    k = rope(k.view(T, n_kv, hd).transpose(0, 1), cos, sin)
    k = k.repeat_interleave(n_heads // n_kv, dim=0)
    sc = (q.to(F64) @ k.to(F64).transpose(1, 2)).to(F32) * np.float32(1.0 / np.sqrt(hd))
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool), 1)
    sc = sc.masked_fill(mask, -torch.inf)
    m = sc.max(-1, keepdim=True).values
    e = torch.exp(sc - m)
    tot = e.to(F64).sum(-1, keepdim=True).to(F32)
    return bf(e * torch.reciprocal(tot))


def attn_core_hard(hn, W, n_heads=14, n_kv=2):
    """e2e.py:123-158 with bf16 weights: o bf16 [T, nh * hd], and the probabilities."""
    T = hn.shape[0]
    hd = W["q_proj"].shape[0] // n_heads
    P = attention_probs(hn, W, n_heads, n_kv)
    v = bf(bf(hn.to(F64) @ W["v_proj"].to(F64).T).to(F32) + W["v_bias"])
    v = v.view(T, n_kv, hd).transpose(0, 1).repeat_interleave(n_heads // n_kv, dim=0)
    o = bf((P.to(F64) @ v.to(F64)).to(F32))
    return o.transpose(0, 1).reshape(T, n_heads * hd), P


def block_hard(h, W, n_heads=14, n_kv=2, eps=1e-6):
    """e2e.py:160-174 with bf16 weights on one sequence h [T, H]; returns (out, taps) where taps
    holds the inputs of every linear (hn, o, mn, d_in), h1 and the attention probabilities."""
    hn = rmsnorm(h, W["in_norm"], eps)
    o, P = attn_core_hard(hn, W, n_heads, n_kv)
    h1 = bf(h + bf(o.to(F64) @ W["o_proj"].to(F64).T))
    mn = rmsnorm(h1, W["post_norm"], eps)
    g = bf(mn.to(F64) @ W["gate_proj"].to(F64).T)
    u = bf(mn.to(F64) @ W["up_proj"].to(F64).T)
    d_in = bf(bf(g * bf(sigmoid(g))) * u)
    out = bf(h1 + bf(d_in.to(F64) @ W["down_proj"].to(F64).T))
    return out, {"hn": hn, "o": o, "h1": h1, "mn": mn, "d_in": d_in, "P": P}


def attn_out_hard(hn, W, n_heads=14, n_kv=2):
    """The vo-stage target: bf16(attn_core(hn) @ Wo^T) (staged.py:483-484)."""
    o, _ = attn_core_hard(hn, W, n_heads, n_kv)
    return bf(o.to(F64) @ W["o_proj"].to(F64).T)


# ------------------------------------------------------------- stage losses ---

def mlp_loss_and_grads(mn, h1, Y, Wg, Wu, Wd):
    """mlp stage (staged.py:345-354) on the micro-batch rows (positions 1..): mn, h1, Y bf16
    [M, H]; soft float32 weights. Returns (loss, dL/dWg, dL/dWu, dL/dWd) in float64."""
    wg = torch.as_tensor(Wg, dtype=F64).requires_grad_()
    wu = torch.as_tensor(Wu, dtype=F64).requires_grad_()
    wd = torch.as_tensor(Wd, dtype=F64).requires_grad_()
    x = mn.to(F64)
    g = x @ wg.T
    u = x @ wu.T
    d_in = g * torch.sigmoid(g) * u
    r = h1.to(F64) + d_in @ wd.T - Y.to(F64)
    loss = (r * r).mean()
    loss.backward()
    return float(loss.detach()), wg.grad.numpy(), wu.grad.numpy(), wd.grad.numpy()


def vo_loss_and_grads(hn_seqs, A_seqs, P_seqs, Wv, bv, Wo, n_heads=14, n_kv=2):
    """vo stage (staged.py:332-342): per sequence R = (P v) Wo^T - A over positions 1..,
    v = hn Wv^T + bv (float32, soft Wv), P the bf16 probabilities of the hard q / k.
    Returns (loss averaged over sequences, dL/dWv, dL/dWo) in float64."""
    wv = torch.as_tensor(Wv, dtype=F64).requires_grad_()
    wo = torch.as_tensor(Wo, dtype=F64).requires_grad_()
    total = 0.0
    S = len(hn_seqs)
    for hn, A, P in zip(hn_seqs, A_seqs, P_seqs):
        T = hn.shape[0]
        hd = wv.shape[0] // n_kv
        v = hn.to(F64) @ wv.T + bv.to(F64)
        v = v.view(T, n_kv, hd).transpose(0, 1).repeat_interleave(n_heads // n_kv, dim=0)
        o = (P.to(F64) @ v).transpose(0, 1).reshape(T, n_heads * hd)
        r = (o @ wo.T - A.to(F64))[1:]
        total = total + (r * r).mean()
    loss = total / S
    loss.backward()
    return float(loss.detach()), wv.grad.numpy(), wo.grad.numpy()


# ------------------------------------------------------------- stage optimisers ---

def _soft(state, t, r, noise_seed, tau, kappa):
    from .gsq import soft_weight
    noise = state.noise(noise_seed, t, r)
    w, p, c = soft_weight(state.logits, noise, state.Ckd, state.scales, state.shape,
                          state.group_size, tau, kappa)
    return w, p, c


def _apply(states, grads_per_r, soft_per_r, tau, kappa, lr_logits, lr_scales):
    """Resample mean of the soft backward and one Lion step per linear (staged.py:383-392)."""
    from .gsq import lion_step, soft_backward
    R = len(grads_per_r)
    for j, st in enumerate(states):
        acc_g, acc_s = None, None
        for r in range(R):
            _, p, c = soft_per_r[r][j]
            gl, gsc = soft_backward(grads_per_r[r][j], p, st.Ckd, c, st.scales, st.group_size,
                                    tau, kappa)
            gl, gsc = gl.astype(np.float32), gsc.astype(np.float32)
            acc_g = gl if acc_g is None else acc_g + gl
            acc_s = gsc if acc_s is None else acc_s + gsc
        lion_step(st, acc_g / np.float32(R), acc_s / np.float32(R), lr_logits, lr_scales)


def train_mlp(states, mn_seqs, h1_seqs, Y_seqs, steps, micro_batch=2, resamples=2, seed=0,
              noise_seed=0, lr_logits=1e-4, lr_scales=5e-5):
    """mlp-stage optimiser (staged.py:357-400 with _loss_block): states = gate, up, down
    LinearStates; per-sequence bf16 caches [T, H]. Returns the loss history."""
    from .gsq import gs_schedules
    rng = np.random.default_rng(seed)
    n = len(mn_seqs)
    m = min(micro_batch, n)
    hist = []
    for t in range(steps):
        tau, kappa = gs_schedules(t, steps)
        idx = np.sort(rng.choice(n, size=m, replace=False))
        mn = torch.cat([mn_seqs[i][1:] for i in idx])
        h1 = torch.cat([h1_seqs[i][1:] for i in idx])
        Y = torch.cat([Y_seqs[i][1:] for i in idx])
        grads, softs, loss = [], [], 0.0
        for r in range(resamples):
            sw = [_soft(st, t, r, noise_seed, tau, kappa) for st in states]
            l, gg, gu, gd = mlp_loss_and_grads(mn, h1, Y, sw[0][0], sw[1][0], sw[2][0])
            loss += l
            grads.append([gg, gu, gd])
            softs.append(sw)
        _apply(states, grads, softs, tau, kappa, lr_logits, lr_scales)
        hist.append(loss / resamples)
    return hist


def train_vo(states, hn_seqs, A_seqs, P_of, bv, steps, n_heads, n_kv, micro_batch=2,
             resamples=2, seed=0, noise_seed=0, lr_logits=1e-4, lr_scales=5e-5):
    """vo-stage optimiser (staged.py:357-400 with _loss_attn): states = v, o LinearStates;
    P_of(t, idx) returns the bf16 probabilities [nh, T, T] of each chosen sequence."""
    from .gsq import gs_schedules
    rng = np.random.default_rng(seed)
    n = len(hn_seqs)
    m = min(micro_batch, n)
    hist = []
    for t in range(steps):
        tau, kappa = gs_schedules(t, steps)
        idx = np.sort(rng.choice(n, size=m, replace=False))
        Ps = P_of(t, idx)
        grads, softs, loss = [], [], 0.0
        for r in range(resamples):
            sw = [_soft(st, t, r, noise_seed, tau, kappa) for st in states]
            l, gv, go = vo_loss_and_grads([hn_seqs[i] for i in idx], [A_seqs[i] for i in idx],
                                          Ps, sw[0][0], bv, sw[1][0], n_heads, n_kv)
            loss += l
            grads.append([gv, go])
            softs.append(sw)
        _apply(states, grads, softs, tau, kappa, lr_logits, lr_scales)
        hist.append(loss / resamples)
    return hist
