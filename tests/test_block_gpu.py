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
    a, b = a.float().cpu(), b.float().cpu()
    d = (a - b).abs()
    tol = 2.0 ** -7 * b.abs() + 1e-6
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
    for s in range(S):
        hs = h[s * T:(s + 1) * T].float()
        ref, taps = ob.block_hard(hs, Wf, cfg.n_heads, cfg.n_kv)
        sl = slice(s * T, (s + 1) * T)
        for name, got in [("hn", blk.hn[sl]), ("o", blk.o[sl]), ("h1", blk.h1[sl]),
                          ("mn", blk.mn[sl]), ("d_in", blk.d_in[sl]), ("out", out[sl])]:
            bad, eq = frac_diff(got, taps.get(name, ref))
            assert bad < 2e-3 and eq > 0.95, (name, bad, eq)
        # transposed taps: position 0 zeroed, the rest equal to the row-major values
        tp = blk.tap("hn").t[0][:, sl].float().cpu()
        assert torch.all(tp[:, 0] == 0)
        assert torch.equal(tp[:, 1:], blk.hn[sl][1:].float().cpu().T)
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
