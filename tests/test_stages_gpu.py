"""The vo and mlp stage optimisers on the GPU vs the oracle (torch-CPU float64 autograd of the
reference stage losses, staged.py:332-354), fed the same caches and the same Gumbel noise:
logits and scales within 1e-3 relative after the run, hard codes equal on >= 99.9 %."""
import numpy as np
import pytest
import torch

from oracle import block as ob
from oracle import gptq as og
from oracle import gsq as ogsq

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _weights(seed, H=128, nh=2, nkv=1, inter=256):
    from tests.test_block_gpu import small_block
    return small_block(seed, H, nh, nkv, inter)


def _pair(name, W, bits, pos, seed=0):
    from gsq_rco_mlx_b200.gsq.staged import SoftLinear
    r = og.quantize_rtn(W, bits, 64)
    s16 = r["scales"].astype(np.float16)
    lin = SoftLinear(name, bits, r["codes"], s16, 64, seed=seed + pos, linear_id=pos)
    st = ogsq.LinearState(bits, r["codes"], s16, 64, seed=seed + pos, linear_id=pos)
    return lin, st


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_mlp_stage_matches_oracle():
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig, BlockWeights, Qwen2Block
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, MLPStep, train_stage
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    W = _weights(1)
    N, T, steps = 6, 64, 25
    h = (0.5 * torch.randn(N * T, cfg.hidden, generator=torch.Generator().manual_seed(3))).bfloat16()
    blk = Qwen2Block(cfg, N, T)
    Wd = BlockWeights({k: v.to(DEV) for k, v in W.items()})
    Y = blk.forward(h.to(DEV), Wd).clone()
    mn, h1 = blk.mn.clone(), blk.h1.clone()
    pairs = [_pair(n, W[n].float().numpy(), 3, i + 4) for i, n in
             enumerate(("gate_proj", "up_proj", "down_proj"))]
    opts = BlockOpts(steps=steps)
    step = MLPStep([p[0] for p in pairs], cfg, 2, T, 2)
    hist = train_stage(step, lambda idx: (mn, h1, Y, idx), N, opts, seed=5, noise_seed=9)[0]
    seqs = lambda x: [x[i * T:(i + 1) * T].float().cpu() for i in range(N)]
    hist_o = ob.train_mlp([p[1] for p in pairs], seqs(mn), seqs(h1), seqs(Y), steps, seed=5,
                          noise_seed=9)
    for lin, st in pairs:
        rl = _rel(lin.logits.cpu().numpy(), st.logits)
        rs = _rel(lin.scales.cpu().numpy(), st.scales)
        assert rl <= 1e-3 and rs <= 1e-3, (lin.name, rl, rs)
        assert (lin.hard_codes() == st.hard_codes()).mean() >= 0.999
    assert abs(hist[-1] - hist_o[-1]) <= 1e-3 * hist_o[-1]


def test_vo_stage_matches_oracle():
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig, BlockWeights, Qwen2Block, wterms
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, VOStep, train_stage, _bf16_rows
    from gsq_rco_mlx_b200.gemm import gemm
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    W = _weights(2)
    N, T, steps = 6, 64, 25
    h = (0.5 * torch.randn(N * T, cfg.hidden, generator=torch.Generator().manual_seed(4))).bfloat16()
    blk = Qwen2Block(cfg, N, T)
    Wd = BlockWeights({k: v.to(DEV) for k, v in W.items()})
    A = torch.empty(N * T, cfg.hidden, device=DEV, dtype=torch.bfloat16)
    blk.forward(h.to(DEV), Wd, attn_out=A)
    hn = blk.hn.clone()
    qk = torch.empty(N * T, 3 * 64, device=DEV, dtype=torch.bfloat16)
    gemm(_bf16_rows(hn), wterms(Wd.qk), epi=4, bias=Wd.qk_bias, c_terms=_bf16_rows(qk))
    pairs = [_pair(n, W[n].float().numpy(), 3, i + 2) for i, n in enumerate(("v_proj", "o_proj"))]
    opts = BlockOpts(steps=steps)
    step = VOStep([p[0] for p in pairs], cfg, 2, T, 2, Wd.W["v_bias"])
    # record the micro-batch probabilities the GPU step uses, to feed the oracle the same P
    Ps = {}
    orig_stage = step.stage

    def stage_and_keep(hn_all, a_all, qk_all, idx):
        orig_stage(hn_all, a_all, qk_all, idx)
        Pm = step.P.t[0].float().cpu().view(2, cfg.n_heads, T, T)
        Ps[len(Ps)] = [Pm[j] for j in range(2)]
    step.stage = stage_and_keep
    hist = train_stage(step, lambda idx: (hn, A, qk, idx), N, opts, seed=6, noise_seed=11)[0]
    seqs = lambda x: [x[i * T:(i + 1) * T].float().cpu() for i in range(N)]
    hist_o = ob.train_vo([p[1] for p in pairs], seqs(hn), seqs(A), lambda t, idx: Ps[t],
                         W["v_bias"].float(), steps, cfg.n_heads, cfg.n_kv, seed=6, noise_seed=11)
    for lin, st in pairs:
        rl = _rel(lin.logits.cpu().numpy(), st.logits)
        rs = _rel(lin.scales.cpu().numpy(), st.scales)
        assert rl <= 1e-3 and rs <= 1e-3, (lin.name, rl, rs)
        assert (lin.hard_codes() == st.hard_codes()).mean() >= 0.999
    assert abs(hist[-1] - hist_o[-1]) <= 1e-3 * hist_o[-1]
    # the probabilities of the micro-batch equal the oracle's from the same hn (bf16; rare
    # last-bit flips from the float32 scores)
    rng = np.random.default_rng(6)
    i0 = int(np.sort(rng.choice(N, size=2, replace=False))[0])
    P_ref = ob.attention_probs(hn[i0 * T:(i0 + 1) * T].float().cpu(),
                               {k: v.float() for k, v in W.items()}, 2, 1)
    assert float((Ps[0][0] == P_ref).float().mean()) >= 0.97


def test_quantize_block_runs_small():
    """The whole block quantizer on a small block: shapes, code ranges, finite statistics."""
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig, LIN_ORDER
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, quantize_block
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    W = {k: v.to(DEV) for k, v in _weights(3).items()}
    N, T = 4, 64
    h = (0.5 * torch.randn(N * T, cfg.hidden, generator=torch.Generator().manual_seed(5))).bfloat16().to(DEV)
    bits = {n: 3 for n in LIN_ORDER}
    shard, stats, Wq = quantize_block(h, W, bits, BlockOpts(steps=8), layer=0, cfg=cfg, T=T,
                                      chunk_seqs=2, log=lambda *a: None)
    for n in LIN_ORDER:
        assert shard[n]["codes"].shape == tuple(W[n].shape) and shard[n]["codes"].max() < 8
        assert shard[n]["scales"].dtype == np.float16
        assert Wq[n].dtype == torch.bfloat16
    for s in ("qk", "vo", "mlp"):
        assert stats["stages"][s]["steps"] == 8
        assert np.isfinite(stats["stages"][s]["soft_loss_last"])
