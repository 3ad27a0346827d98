"""The decoder block's vjp on the GPU (the RCO objective's per-layer backward) against the
explicit-formula oracle (oracle/block_vjp.py, itself checked against float64 autograd): the
input cotangent (bf16) and the seven float32 weight gradients, summed over the sequences."""
import pytest
import torch

from oracle import block_vjp as ov

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("dims", [dict(H=128, nh=2, nkv=1, inter=256, T=128, S=2),
                                  dict(H=896, nh=14, nkv=2, inter=4864, T=256, S=2)])
def test_block_vjp_matches_oracle(dims):
    from tests.test_block_gpu import small_block
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig, BlockWeights, LIN_ORDER, Qwen2Block
    T, S = dims.pop("T"), dims.pop("S")
    cfg = BlockConfig(hidden=dims["H"], n_heads=dims["nh"], n_kv=dims["nkv"],
                      inter=dims["inter"])
    W = small_block(7, dims["H"], dims["nh"], dims["nkv"], dims["inter"])
    g = torch.Generator().manual_seed(8)
    h = torch.randn(S * T, cfg.hidden, generator=g).bfloat16()
    cot = (0.01 * torch.randn(S * T, cfg.hidden, generator=g)).bfloat16()
    eng = Qwen2Block(cfg, S, T, torch.device(DEV))
    Wd = BlockWeights({k: v.to(DEV) for k, v in W.items()})
    dh, grads = eng.vjp(h.to(DEV), Wd, cot.to(DEV))
    from gsq_rco_mlx_b200.gemm import check_err
    check_err(torch.device(DEV))
    Wf = {k: v.float() for k, v in W.items()}
    dh_ref, g_ref = [], {}
    for s in range(S):
        rows = slice(s * T, (s + 1) * T)
        d, gr = ov.block_vjp(h[rows].float(), Wf, cot[rows].float(), cfg.n_heads, cfg.n_kv)
        dh_ref.append(d)
        for k, v in gr.items():
            g_ref[k] = g_ref.get(k, 0) + v
    dh_ref = torch.cat(dh_ref)
    r = _rel(dh, dh_ref)
    assert r < 2e-2, r
    for name in LIN_ORDER:
        rg = _rel(grads[name], g_ref[name])
        assert rg < 2e-2, (name, rg)
    # accumulation over chunks: a second call with accumulate adds the same gradients
    dh2, grads2 = eng.vjp(h.to(DEV), Wd, cot.to(DEV), grads={k: v.clone() for k, v in
                                                              grads.items()} | {
        "_gu": torch.cat([grads["gate_proj"], grads["up_proj"]]),
        "_qkv": torch.cat([grads["q_proj"], grads["k_proj"], grads["v_proj"]])},
        accumulate=True)
    torch.cuda.synchronize()
    assert _rel(grads2["_gu"], 2 * torch.cat([grads["gate_proj"], grads["up_proj"]])) < 1e-6
