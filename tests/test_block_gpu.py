"""The GPU decoder block (hard bf16 forward, Hessian taps) vs the torch-CPU oracle of the
reference block (src/gsq_rco/gsq/e2e.py): bf16 outputs equal up to rare last-bit rounding
differences, Hessians within float32 accuracy."""
import numpy as np
import pytest
import torch

from oracle import block as ob

pytestmark = pytest.mark.gpu
DEV = "cuda"


def small_block(seed=0, H=128, nh=2, nkv=1, inter=256, scale=0.05):
    g = torch.Generator().manual_seed(seed)
    hd = 64
    def w(*shape):
        return (scale * torch.randn(*shape, generator=g)).bfloat16()
    W = {"q_proj": w(nh * hd, H), "k_proj": w(nkv * hd, H), "v_proj": w(nkv * hd, H),
         "o_proj": w(H, nh * hd), "gate_proj": w(inter, H), "up_proj": w(inter, H),
         "down_proj": w(H, inter), "q_bias": w(nh * hd), "k_bias": w(nkv * hd),
         "v_bias": w(nkv * hd), "in_norm": (1 + 0.1 * torch.randn(H, generator=g)).bfloat16(),
         "post_norm": (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()}
    return W


def frac_diff(a, b):
    """Fraction of elements off by more than a few bf16 ulps of themselves plus a fraction of
    the tensor's RMS (chains of bf16 roundings near zero), and the fraction exactly equal."""
    a, b = a.float().cpu(), b.float().cpu()
    d = (a - b).abs()
    tol = 2.0 ** -6 * b.abs() + 2.0 ** -8 * b.pow(2).mean().sqrt()
    return float((d > tol).float().mean()), float((a == b).float().mean())


@pytest.mark.parametrize("dims", [dict(H=128, nh=2, nkv=1, inter=256, T=128, S=2),
                                  dict(H=896, nh=14, nkv=2, inter=4864, T=256, S=2)])
def test_hard_forward_matches_oracle(dims):
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig, BlockWeights, Qwen2Block
    T, S = dims.pop("T"), dims.pop("S")
    cfg = BlockConfig(hidden=dims["H"], n_heads=dims["nh"], n_kv=dims["nkv"], inter=dims["inter"])
    W = small_block(H=dims["H"], nh=dims["nh"], nkv=dims["nkv"], inter=dims["inter"])
    g = torch.Generator().manual_seed(5)
    h = (0.5 * torch.randn(S * T, cfg.hidden, generator=g)).bfloat16()
    blk = Qwen2Block(cfg, S, T)
    Wd = BlockWeights({k: v.to(DEV) for k, v in W.items()})
    out = blk.forward(h.to(DEV), Wd, taps=("hn", "o", "mn", "d_in"))
    torch.cuda.synchronize()
    from gsq_rco_mlx_b200.gemm import check_err
    check_err(torch.device(DEV))
    Wf = {k: v.float() for k, v in W.items()}
    F64 = torch.float64
    for s in range(S):
        sl = slice(s * T, (s + 1) * T)
        hs = h[sl].float()
        g_hn, g_o, g_h1 = blk.hn[sl].float().cpu(), blk.o[sl].float().cpu(), blk.h1[sl].float().cpu()
        g_mn, g_d, g_out = blk.mn[sl].float().cpu(), blk.d_in[sl].float().cpu(), out[sl].float().cpu()
        # each stage against the oracle fed the GPU's own input to that stage
        stages = [
            ("hn", g_hn, ob.rmsnorm(hs, Wf["in_norm"])),
            ("o", g_o, ob.attn_core_hard(g_hn, Wf, cfg.n_heads, cfg.n_kv)[0]),
            ("h1", g_h1, ob.bf(hs + ob.bf(g_o.to(F64) @ Wf["o_proj"].to(F64).T))),
            ("mn", g_mn, ob.rmsnorm(g_h1, Wf["post_norm"])),
        ]
        gg = ob.bf(g_mn.to(F64) @ Wf["gate_proj"].to(F64).T)
        uu = ob.bf(g_mn.to(F64) @ Wf["up_proj"].to(F64).T)
        stages.append(("d_in", g_d, ob.bf(ob.bf(gg * ob.bf(ob.sigmoid(gg))) * uu)))
        stages.append(("out", g_out, ob.bf(g_h1 + ob.bf(g_d.to(F64) @ Wf["down_proj"].to(F64).T))))
        for name, got, ref in stages:
            bad, eq = frac_diff(got, ref)
            assert bad < 2e-3 and eq > 0.97, (name, bad, eq)
        # end to end (bf16 rounding differences propagate through the chain)
        ref_out, _ = ob.block_hard(hs, Wf, cfg.n_heads, cfg.n_kv)
        e2e = ((g_out - ref_out).norm() / ref_out.norm()).item()
        assert e2e < 1e-2, e2e
        # transposed taps: position 0 zeroed, the rest equal to the row-major values
        tp = blk.tap("hn").t[0][:, sl].float().cpu()
        assert torch.all(tp[:, 0] == 0)
        assert torch.equal(tp[:, 1:], g_hn[1:].T)
    # Hessian of the q/k/v input over positions 1.. of both sequences
    H64 = torch.zeros(cfg.hidden, cfg.hidden, device=DEV, dtype=torch.float64)
    n = blk.hessian_add("hn", H64, 0)
    X = torch.cat([blk.hn[s * T + 1:(s + 1) * T].double() for s in range(S)]).cpu()
    Href = 2.0 * X.T @ X / X.shape[0]
    assert n == S * (T - 1)
    assert ((H64.cpu() - Href).norm() / Href.norm()).item() < 1e-6


def test_attention_output_target():
    """attn_out = bf16(attn_core(hn) Wo^T), the vo-stage target (staged.py:483-484)."""
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig, BlockWeights, Qwen2Block
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    W = small_block()
    T, S = 128, 2
    h = (0.5 * torch.randn(S * T, cfg.hidden, generator=torch.Generator().manual_seed(2))).bfloat16()
    blk = Qwen2Block(cfg, S, T)
    A = torch.empty(S * T, cfg.hidden, device=DEV, dtype=torch.bfloat16)
    blk.forward(h.to(DEV), BlockWeights({k: v.to(DEV) for k, v in W.items()}), attn_out=A)
    Wf = {k: v.float() for k, v in W.items()}
    for s in range(S):
        hn = ob.rmsnorm(h[s * T:(s + 1) * T].float(), Wf["in_norm"])
        bad, eq = frac_diff(A[s * T:(s + 1) * T], ob.attn_out_hard(hn, Wf, 2, 1))
        assert bad < 2e-3 and eq > 0.95, (bad, eq)


@pytest.mark.parametrize("T", [128, 384, 2048])
def test_causal_softmax_vector_rows(T):
    """gsq_softmax_causal (the vectorised row kernel when no transpose is asked) against the
    oracle's float32 softmax with a float64 sum: P equal up to rare last-bit differences on keys
    <= query, zeros from the query to the end of its 128-key block; the transposed-output form
    (the reference kernel over whole rows) agrees on that region."""
    from gsq_rco_mlx_b200 import _lib
    B = 3
    g = torch.Generator().manual_seed(T)
    S = (4 * torch.randn(B, T, T, generator=g)).float()
    Sd = S.to(DEV)
    P = torch.full((B * T, T), 7.0, device=DEV, dtype=torch.bfloat16)
    P2 = torch.empty(B * T, T, device=DEV, dtype=torch.bfloat16)
    PT = torch.empty(B, T, T, device=DEV, dtype=torch.bfloat16)
    st = _lib.stream_ptr()
    _lib.call("gsq_softmax_causal", _lib.ptr(Sd), B, T, _lib.ptr(P), None, st)
    _lib.call("gsq_softmax_causal", _lib.ptr(Sd), B, T, _lib.ptr(P2), _lib.ptr(PT), st)
    torch.cuda.synchronize()
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool), 1)
    Sm = S.masked_fill(mask, -torch.inf)
    m = Sm.max(-1, keepdim=True).values
    e = torch.exp(Sm - m)
    ref = ob.bf(e * torch.reciprocal(e.double().sum(-1, keepdim=True).float()))
    got = P.float().cpu().view(B, T, T)
    t = torch.arange(T)[:, None]
    k = torch.arange(T)[None, :]
    inside = (k // 128) <= (t // 128)                 # the written region
    assert torch.all(got[:, ~inside] == 7.0)           # beyond the block: untouched
    region = inside.expand(B, T, T)
    assert float((got[region] != ref[region]).float().mean()) < 1e-3
    assert torch.equal(got[region], P2.float().cpu().view(B, T, T)[region])
    assert torch.equal(PT.float().cpu(), P2.float().cpu().view(B, T, T).transpose(1, 2))


@pytest.mark.parametrize("row0,rows,cols", [(0, 384, 384), (256, 128, 384), (1000, 1048, 2048)])
def test_causal_softmax_row_window(row0, rows, cols):
    """gsq_softmax_causal_rows (query rows row0 .. row0 + rows - 1 over cols keys) against the
    oracle's float32 softmax with a float64 sum: equal up to rare last-bit differences on keys
    <= query; masked keys are zero up to the end of the query's 128-key block when row0 == 0 (a
    square causal block, whose consumers read no further) and up to cols otherwise."""
    from gsq_rco_mlx_b200 import _lib
    B = 2
    g = torch.Generator().manual_seed(row0 + rows + cols)
    S = (4 * torch.randn(B, rows, cols, generator=g)).float()
    P = torch.full((B * rows, cols), 7.0, device=DEV, dtype=torch.bfloat16)
    _lib.call("gsq_softmax_causal_rows", _lib.ptr(S.to(DEV)), B, rows, cols, cols, row0,
              _lib.ptr(P), cols, _lib.stream_ptr())
    torch.cuda.synchronize()
    t = row0 + torch.arange(rows)[:, None]
    k = torch.arange(cols)[None, :]
    Sm = S.masked_fill(k > t, -torch.inf)
    m = Sm.max(-1, keepdim=True).values
    e = torch.exp(Sm - m)
    ref = ob.bf(e * torch.reciprocal(e.double().sum(-1, keepdim=True).float()))
    got = P.float().cpu().view(B, rows, cols)
    inside = (k // 128) <= (t // 128) if row0 == 0 else torch.ones(rows, cols, dtype=torch.bool)
    assert torch.all(got[:, ~inside] == 7.0)
    region = inside.expand(B, rows, cols)
    assert float((got[region] != ref[region]).float().mean()) < 1e-3
    assert torch.all(got[:, (k > t) & inside] == 0)
