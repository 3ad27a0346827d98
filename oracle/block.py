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

def mlp_loss_and_grads(mn, h1, Y, Wg, Wu, Wd, dtype=F64):
    """mlp stage (staged.py:345-354) on the micro-batch rows (positions 1..): mn, h1, Y bf16
    [M, H]; soft float32 weights. Returns (loss, dL/dWg, dL/dWu, dL/dWd), computed in
    ``dtype`` (float64 for parity; float32 is the reference's own arithmetic)."""
    wg = torch.as_tensor(Wg, dtype=dtype).requires_grad_()
    wu = torch.as_tensor(Wu, dtype=dtype).requires_grad_()
    wd = torch.as_tensor(Wd, dtype=dtype).requires_grad_()
    x = mn.to(dtype)
    g = x @ wg.T
    u = x @ wu.T
    d_in = g * torch.sigmoid(g) * u
    r = h1.to(dtype) + d_in @ wd.T - Y.to(dtype)
    loss = (r * r).mean()
    loss.backward()
    return (float(loss.detach()), wg.grad.double().numpy(), wu.grad.double().numpy(),
            wd.grad.double().numpy())


def vo_loss_and_grads(hn_seqs, A_seqs, P_seqs, Wv, bv, Wo, n_heads=14, n_kv=2, dtype=F64):
    """vo stage (staged.py:332-342): per sequence R = (P v) Wo^T - A over positions 1..,
    v = hn Wv^T + bv (float32, soft Wv), P the bf16 probabilities of the hard q / k.
    Returns (loss averaged over sequences, dL/dWv, dL/dWo) in float64."""
    wv = torch.as_tensor(Wv, dtype=dtype).requires_grad_()
    wo = torch.as_tensor(Wo, dtype=dtype).requires_grad_()
    total = 0.0
    S = len(hn_seqs)
    for hn, A, P in zip(hn_seqs, A_seqs, P_seqs):
        T = hn.shape[0]
        hd = wv.shape[0] // n_kv
        v = hn.to(dtype) @ wv.T + bv.to(dtype)
        v = v.view(T, n_kv, hd).transpose(0, 1).repeat_interleave(n_heads // n_kv, dim=0)
        o = (P.to(dtype) @ v).transpose(0, 1).reshape(T, n_heads * hd)
        r = (o @ wo.T - A.to(dtype))[1:]
        total = total + (r * r).mean()
    loss = total / S
    loss.backward()
    return float(loss.detach()), wv.grad.double().numpy(), wo.grad.double().numpy()


# ------------------------------------------------------------- stage optimisers ---

def _soft(state, t, r, noise_seed, tau, kappa):
    from .gsq import soft_weight
    noise = state.noise(noise_seed, t, r)
    w, p, c = soft_weight(state.logits, noise, state.Ckd, state.scales, state.shape,
                          state.group_size, tau, kappa)
    return w, p, c


def _jitter(grads, grad_noise):
    """grads times (1 + amp N(0, 1)) with grad_noise = (amp, numpy Generator): float32-level
    perturbations for measuring how far rounding alone moves a trajectory."""
    if grad_noise is None:
        return grads
    amp, rng = grad_noise
    return [g * (1.0 + amp * rng.standard_normal(g.shape)) for g in grads]


def _apply(states, grads_per_r, soft_per_r, tau, kappa, lr_logits, lr_scales):
    """Resample mean of the soft backward and one Lion step per linear (staged.py:383-392)."""
    from .gsq import backward_accumulate, lion_step
    R = len(grads_per_r)
    for j, st in enumerate(states):
        acc = [None, None]
        for r in range(R):
            _, p, c = soft_per_r[r][j]
            backward_accumulate(acc, grads_per_r[r][j], p, st.Ckd, c, st.scales,
                                st.group_size, tau, kappa)
        lion_step(st, acc[0] / np.float32(R), acc[1] / np.float32(R), lr_logits, lr_scales)


def train_mlp(states, mn_seqs, h1_seqs, Y_seqs, steps, micro_batch=2, resamples=2, seed=0,
              noise_seed=0, lr_logits=1e-4, lr_scales=5e-5, dtype=F64, grad_noise=None):
    """mlp-stage optimiser (staged.py:357-400 with _loss_block): states = gate, up, down
    LinearStates; per-sequence bf16 caches [T, H]. grad_noise = (amp, Generator) perturbs every
    weight gradient by a relative amp (sensitivity measurements). Returns the loss history."""
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
            l, gg, gu, gd = mlp_loss_and_grads(mn, h1, Y, sw[0][0], sw[1][0], sw[2][0], dtype)
            loss += l
            grads.append(_jitter([gg, gu, gd], grad_noise))
            softs.append(sw)
        _apply(states, grads, softs, tau, kappa, lr_logits, lr_scales)
        hist.append(loss / resamples)
    return hist


def train_vo(states, hn_seqs, A_seqs, P_of, bv, steps, n_heads, n_kv, micro_batch=2,
             resamples=2, seed=0, noise_seed=0, lr_logits=1e-4, lr_scales=5e-5, dtype=F64,
             grad_noise=None):
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
                                          Ps, sw[0][0], bv, sw[1][0], n_heads, n_kv, dtype)
            loss += l
            grads.append(_jitter([gv, go], grad_noise))
            softs.append(sw)
        _apply(states, grads, softs, tau, kappa, lr_logits, lr_scales)
        hist.append(loss / resamples)
    return hist


# ------------------------------------------------------------- block quantizer chain ---

STAGE_LINEARS = {"qk": ("q_proj", "k_proj"), "vo": ("v_proj", "o_proj"),
                 "mlp": ("gate_proj", "up_proj", "down_proj")}
LIN_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def _hessian(rows):
    """Running-mean Hessian 2 X^T X / n over the rows (positions 1..) of every sequence
    (staged.py:143-163), float64."""
    from .gptq import hessian_from_inputs
    H, n = None, 0
    for x in rows:
        H, n = hessian_from_inputs(x.to(F64).numpy(), H, n)
    return H


def _hard_weight(codes, s16, bits, group_size):
    """staged.py:194-196: dequantized with the fp16 scales, stored as bf16."""
    from .gptq import dequantize
    w = dequantize(codes, np.asarray(s16, dtype=np.float32), bits, group_size)
    return torch.as_tensor(np.asarray(w, dtype=np.float32)).bfloat16()


def recon_error(W, codes, s16, bits, group_size, H):
    """The GPTQ objective tr((W - Q) H (W - Q)^T) of codes with float16 scales under the
    Hessian H (gptq.py:123-187 minimises it column by column), float64."""
    from .gptq import dequantize
    Q = dequantize(codes, np.asarray(s16, dtype=np.float32), bits, group_size)
    D = np.asarray(W, dtype=np.float64) - np.asarray(Q, dtype=np.float64)
    return float(np.einsum("ij,ij->", D @ np.asarray(H, dtype=np.float64), D))


def quantize_block(h_seqs, W, bits, steps, layer=0, opt_seed=0, n_heads=14, n_kv=2,
                   group_size=64, damp=0.01, block_size=128, micro_batch=2, resamples=2,
                   eps=1e-6, warm_start=None, follow=None):
    """The block quantizer of staged.py:405-522 on the CPU: for each stage, Hessians of the
    linears' inputs under the weights hardened so far, GPTQ warm starts (fp16 scales), 200
    Lion steps with Philox noise keyed as the CUDA path keys it, hardening (argmax codes, fp16
    scales). h_seqs: bf16 [T, H] inputs of the calibration sequences; W: bf16 block weights.
    warm_start {name: {codes, scales}}: continue from these GPTQ results instead of this chain's
    own (which are still computed and returned), so that a comparison of the training stages
    does not count a GPTQ near-tie twice. follow {name: {codes, scales}}: after each stage,
    record this chain's hardened result but continue from these (another run's hardened
    weights), so that every stage starts from the same weights as that run's.
    Returns (shard {name: {codes, scales, bits}}, {stage: loss history},
    {name: this chain's own GPTQ (codes, float16 scales, {"own": its objective under this
    chain's Hessian, "warm": the warm start's objective under the same Hessian or None})})."""
    from .gptq import quantize_gptq
    from .gsq import LinearState, train_linear
    Wf = {k: v.float() for k, v in W.items()}
    Wcur = {k: v.clone() for k, v in W.items()}
    seed = opt_seed * 1_000_003 + layer * 1_009
    shard, hist, gptq_codes = {}, {}, {}
    states = {}

    def gptq(name, H, pos):
        w = Wf[name].numpy()
        g = quantize_gptq(w, H, bits[name], group_size, damp, block_size)
        codes, s16 = g["codes"], g["scales"].astype(np.float16)
        errs = {"own": recon_error(w, codes, s16, bits[name], group_size, H), "warm": None}
        gptq_codes[name] = (codes, s16, errs)
        if warm_start is not None:
            codes = np.asarray(warm_start[name]["codes"], dtype=np.uint8)
            s16 = np.asarray(warm_start[name]["scales"], dtype=np.float16)
            errs["warm"] = recon_error(w, codes, s16, bits[name], group_size, H)
        Wcur[name] = _hard_weight(codes, s16, bits[name], group_size)
        states[name] = LinearState(bits[name], codes, s16, group_size, seed=seed + 10 * pos,
                                   linear_id=layer * 8 + pos)
        return states[name]

    def harden(name):
        st = states[name]
        codes, s16 = st.hard_codes(), st.stored_scales()
        shard[name] = {"codes": codes, "scales": s16, "bits": st.bits}
        if follow is not None:
            codes = np.asarray(follow[name]["codes"], dtype=np.uint8)
            s16 = np.asarray(follow[name]["scales"], dtype=np.float16)
        Wcur[name] = _hard_weight(codes, s16, st.bits, group_size)

    def fwd(Wb):
        return [block_hard(h, {k: v.float() for k, v in Wb.items()}, n_heads, n_kv, eps)
                for h in h_seqs]

    n = len(h_seqs)
    # qk: linear reconstruction on hn rows (positions 1..)
    hn = [rmsnorm(h, Wf["in_norm"], eps) for h in h_seqs]
    H_hn = _hessian([x[1:] for x in hn])
    qk = [gptq(name, H_hn, i) for i, name in enumerate(STAGE_LINEARS["qk"])]
    Xs = torch.stack([x[1:] for x in hn]).numpy()
    in_f = Xs.shape[-1]
    per = []
    for st, name in zip(qk, STAGE_LINEARS["qk"]):
        per.append(train_linear(st, lambda idx: Xs[idx].reshape(-1, in_f), Wf[name].numpy(), n,
                                steps, micro_batch, resamples, seed=seed + 1,
                                noise_seed=seed + 1))
    hist["qk"] = list(np.sum(per, axis=0))
    for name in STAGE_LINEARS["qk"]:
        harden(name)
    # vo: attention output with q and k hard
    v_st = gptq("v_proj", H_hn, 2)
    taps = fwd(Wcur)
    H_o = _hessian([tp["o"][1:] for _, tp in taps])
    o_st = gptq("o_proj", H_o, 3)
    A = [attn_out_hard(x, Wf, n_heads, n_kv) for x in hn]
    Ps = [attention_probs(x, {k: v.float() for k, v in Wcur.items()}, n_heads, n_kv) for x in hn]
    hist["vo"] = train_vo([v_st, o_st], hn, A, lambda t, idx: [Ps[i] for i in idx],
                          Wf["v_bias"], steps, n_heads, n_kv, micro_batch, resamples,
                          seed=seed + 2, noise_seed=seed + 2)
    for name in STAGE_LINEARS["vo"]:
        harden(name)
    # mlp: block output with the attention hard
    taps = fwd(Wcur)
    H_gu = _hessian([tp["mn"][1:] for _, tp in taps])
    g_st, u_st = gptq("gate_proj", H_gu, 4), gptq("up_proj", H_gu, 5)
    taps_d = fwd(Wcur)
    H_d = _hessian([tp["d_in"][1:] for _, tp in taps_d])
    d_st = gptq("down_proj", H_d, 6)
    Y = [block_hard(h, Wf, n_heads, n_kv, eps)[0] for h in h_seqs]
    hist["mlp"] = train_mlp([g_st, u_st, d_st], [tp["mn"] for _, tp in taps],
                            [tp["h1"] for _, tp in taps], Y, steps, micro_batch, resamples,
                            seed=seed + 3, noise_seed=seed + 3)
    for name in STAGE_LINEARS["mlp"]:
        harden(name)
    return shard, hist, gptq_codes
