"""CPU restatement of the Qwen2 block's vector-Jacobian product (test infrastructure only).

The RCO objective (src/gsq_rco/rco/allocate.py:156-167, _layer_vjp) takes the vjp of one
decoder block with MLX autodiff: the cotangent of the block input and the gradients of its seven
linear weights under a cotangent of the block output. MLX's bf16 autodiff rounding cannot be
reproduced without MLX, so the backward here is defined as: float32/float64 math on the bf16
forward values of oracle.block.block_hard (e2e.py:160-174), every cotangent rounded to bf16
where the forward tensor is bf16 (hn, q, k, v, P, o, h1, mn, g, u, the SwiGLU intermediates, the
block input), the casts passing cotangents through unchanged, the weight gradients in float32.
Scores S and the RoPE'd q / k are float32 in the forward, so their cotangents stay float32.
"""
from __future__ import annotations

import torch

from .block import F32, F64, bf, rope, rope_tables, sigmoid


def _ident(x):
    return x.to(F32)


def _rmsnorm(x, w, eps, rnd):
    """oracle.block.rmsnorm with the final rounding given (bf16 or none)."""
    xf = x.to(F32)
    var = ((xf * xf).to(F64).sum(-1, keepdim=True) / xf.shape[-1]).to(F32)
    inv = torch.reciprocal(torch.sqrt(var + eps))
    return rnd((xf * inv) * w.to(F32))


def forward_keep(h, W, n_heads=14, n_kv=2, eps=1e-6, theta=1e6, rounding=True):
    """block_hard's forward on one sequence h [T, H], keeping every intermediate. rounding=False
    drops every bf16 rounding (the smooth function whose exact gradients check the formulas)."""
    bf = globals()["bf"] if rounding else _ident
    rmsnorm = lambda x_, w_, e_: _rmsnorm(x_, w_, e_, bf)
    T, H = h.shape
    hd = W["q_proj"].shape[0] // n_heads
    x = {"h": h.to(F32)}
    hn = rmsnorm(h, W["in_norm"], eps)
    q = bf(bf(hn.to(F64) @ W["q_proj"].to(F64).T).to(F32) + W["q_bias"].to(F32))
    k = bf(bf(hn.to(F64) @ W["k_proj"].to(F64).T).to(F32) + W["k_bias"].to(F32))
    v = bf(bf(hn.to(F64) @ W["v_proj"].to(F64).T).to(F32) + W["v_bias"].to(F32))
    cos, sin = rope_tables(T, hd, theta)
    qh = q.view(T, n_heads, hd).transpose(0, 1)           # [nh, T, hd]
    kh = k.view(T, n_kv, hd).transpose(0, 1)
    vh = v.view(T, n_kv, hd).transpose(0, 1)
    qr, kr = rope(qh, cos, sin), rope(kh, cos, sin)        # float32
    rep = n_heads // n_kv
    krr, vrr = kr.repeat_interleave(rep, 0), vh.repeat_interleave(rep, 0)
    S = (qr.to(F64) @ krr.to(F64).transpose(1, 2)).to(F32) * torch.tensor(0.125, dtype=F32)
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool), 1)
    S = S.masked_fill(mask, -torch.inf)
    m = S.max(-1, keepdim=True).values
    e = torch.exp(S - m)
    tot = e.to(F64).sum(-1, keepdim=True).to(F32)
    Pf = e * torch.reciprocal(tot)                         # float32 softmax
    P = bf(Pf)
    oh = bf((P.to(F64) @ vrr.to(F64)).to(F32))             # [nh, T, hd]
    o = oh.transpose(0, 1).reshape(T, n_heads * hd)
    h1 = bf(x["h"] + bf(o.to(F64) @ W["o_proj"].to(F64).T).to(F32))
    mn = rmsnorm(h1, W["post_norm"], eps)
    g = bf(mn.to(F64) @ W["gate_proj"].to(F64).T).to(F32)
    u = bf(mn.to(F64) @ W["up_proj"].to(F64).T).to(F32)
    s = bf(sigmoid(g))
    a = bf(g * s)
    d = bf(a * u)
    out = bf(h1 + bf(d.to(F64) @ W["down_proj"].to(F64).T).to(F32))
    x.update(hn=hn, q=q, k=k, v=v, qr=qr, kr=kr, krr=krr, vrr=vrr, Pf=Pf, P=P, o=o, h1=h1, mn=mn,
             g=g, u=u, s=s, a=a, d=d, out=out, cos=cos, sin=sin, mask=mask)
    return out, x


def rmsnorm_bwd(x, w, dy, eps=1e-6):
    """Cotangent of x for y = (x inv) w, inv = 1 / sqrt(mean x^2 + eps), float64."""
    x, w, dy = x.to(F64), w.to(F64), dy.to(F64)
    Hn = x.shape[-1]
    var = (x * x).sum(-1, keepdim=True) / Hn
    inv = 1.0 / torch.sqrt(var + eps)
    dot = (x * w * dy).sum(-1, keepdim=True)
    return inv * w * dy - (inv ** 3 / Hn) * x * dot


def rope_bwd(dy, cos, sin):
    """Cotangent of x for the half-split rotation y = rope(x)."""
    h = dy.shape[-1] // 2
    c, s = torch.as_tensor(cos).to(dy.dtype), torch.as_tensor(sin).to(dy.dtype)
    d1, d2 = dy[..., :h], dy[..., h:]
    return torch.cat([d1 * c + d2 * s, -d1 * s + d2 * c], dim=-1)


def block_vjp(h, W, cot, n_heads=14, n_kv=2, eps=1e-6, rounding=True):
    """(dh bf16-valued float32 [T, H], {name: dW float32}) of one sequence."""
    _, x = forward_keep(h, W, n_heads, n_kv, eps, rounding=rounding)
    bf = globals()["bf"] if rounding else _ident
    T, H = h.shape
    hd = W["q_proj"].shape[0] // n_heads
    rep = n_heads // n_kv
    W64 = {k: v.to(F64) for k, v in W.items()}
    dout = cot.to(F64)
    grads = {}
    # out = h1 + bf(d Wd^T)
    dd = bf(dout @ W64["down_proj"])
    grads["down_proj"] = (dout.T @ x["d"].to(F64)).to(F32)
    # d = bf(a u), a = bf(g s), s = bf(sigmoid(g))
    g, u, s, a = x["g"].to(F64), x["u"].to(F64), x["s"].to(F64), x["a"].to(F64)
    dd64 = dd.to(F64)
    du = bf(dd64 * a)
    da = bf(dd64 * u).to(F64)
    ds = bf(da * g).to(F64)
    sf = torch.sigmoid(g)
    dg = bf(da * s + ds * sf * (1.0 - sf))
    dmn = bf(dg.to(F64) @ W64["gate_proj"] + du.to(F64) @ W64["up_proj"])
    grads["gate_proj"] = (dg.to(F64).T @ x["mn"].to(F64)).to(F32)
    grads["up_proj"] = (du.to(F64).T @ x["mn"].to(F64)).to(F32)
    dh1 = bf(dout + bf(rmsnorm_bwd(x["h1"], W["post_norm"], dmn, eps)).to(F64))
    # h1 = h + bf(o Wo^T)
    dh1_64 = dh1.to(F64)
    do = bf(dh1_64 @ W64["o_proj"])
    grads["o_proj"] = (dh1_64.T @ x["o"].to(F64)).to(F32)
    # attention, per head
    doh = do.view(T, n_heads, hd).transpose(0, 1).to(F64)          # [nh, T, hd]
    P, Pf = x["P"].to(F64), x["Pf"].to(F64)
    dP = bf(doh @ x["vrr"].to(F64).transpose(1, 2)).to(F64)
    dv_h = P.transpose(1, 2) @ doh                                   # [nh, T, hd]
    dv = bf(dv_h.view(n_kv, rep, T, hd).sum(1))                       # [nkv, T, hd]
    dS = Pf * (dP - (dP * Pf).sum(-1, keepdim=True))
    dS = dS.masked_fill(x["mask"], 0.0) * 0.125
    dqr = dS @ x["krr"].to(F64)                                       # [nh, T, hd]
    dkr = (dS.transpose(1, 2) @ x["qr"].to(F64)).view(n_kv, rep, T, hd).sum(1)
    dq = bf(rope_bwd(dqr, x["cos"], x["sin"]))                        # [nh, T, hd]
    dk = bf(rope_bwd(dkr, x["cos"], x["sin"]))
    dq = dq.transpose(0, 1).reshape(T, n_heads * hd).to(F64)
    dk = dk.transpose(0, 1).reshape(T, n_kv * hd).to(F64)
    dv = dv.transpose(0, 1).reshape(T, n_kv * hd).to(F64)
    hn = x["hn"].to(F64)
    dhn = bf(dq @ W64["q_proj"] + dk @ W64["k_proj"] + dv @ W64["v_proj"])
    grads["q_proj"] = (dq.T @ hn).to(F32)
    grads["k_proj"] = (dk.T @ hn).to(F32)
    grads["v_proj"] = (dv.T @ hn).to(F32)
    dh = bf(dh1_64 + bf(rmsnorm_bwd(x["h"], W["in_norm"], dhn, eps)).to(F64))
    return dh.to(F32), grads
