"""App-H scale fine-tune (reference src/gsq_rco/gsq/staged.py:555-634) on the GPU: the group-
scale gradient kernel against a numpy reduction, and the first step's scale gradients of a small
quantized stack against float64 autograd of the CPU restatement (oracle.block) through
W = bf16(s grid[code]), the final norm and the tied-head KL."""
import numpy as np
import pytest
import torch

from oracle import block as ob

pytestmark = pytest.mark.gpu
DEV = "cuda"
F64 = torch.float64


def test_scale_grad_kernel():
    from gsq_rco_mlx_b200 import _lib
    rng = np.random.default_rng(0)
    out_f, in_f, gs = 40, 200, 64
    for bits in (1, 2, 3, 4):
        nlev = 3 if bits == 1 else 1 << bits
        G = rng.standard_normal((out_f, in_f)).astype(np.float32)
        codes = rng.integers(0, nlev, size=(out_f, in_f)).astype(np.uint8)
        grid = np.array([-1, 0, 1]) if bits == 1 else np.arange(nlev) - nlev // 2
        out = torch.empty(out_f, (in_f + gs - 1) // gs, device=DEV)
        Gd, cd = torch.as_tensor(G).to(DEV), torch.as_tensor(codes).to(DEV)
        _lib.call("gsq_scale_grad", _lib.ptr(Gd), _lib.ptr(cd), out_f, in_f, bits, gs,
                  _lib.ptr(out), _lib.stream_ptr())
        torch.cuda.synchronize()
        prod = G.astype(np.float64) * grid[codes]
        ref = np.stack([prod[:, a:a + gs].sum(1) for a in range(0, in_f, gs)], 1)
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-6, atol=1e-5)


def _setup():
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig, LIN_ORDER
    from gsq_rco_mlx_b200.rco.database import random_model
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    model = random_model(n_layers=2, seed=7, device=DEV, cfg=cfg, vocab=512)
    rng = np.random.default_rng(3)
    qblocks = {}
    for L, W in enumerate(model.layers):
        qblocks[L] = {}
        for name in LIN_ORDER:
            w = W[name].float().cpu().numpy()
            N, K = w.shape
            s = (np.abs(w).reshape(N, K // 64, 64).max(-1) / 4 + 1e-3).astype(np.float16)
            c = np.clip(np.rint(w / np.repeat(s.astype(np.float32), 64, 1)) + 4, 0, 7)
            qblocks[L][name] = {"codes": c.astype(np.uint8), "scales": s, "bits": 3}
    tokens = rng.integers(0, 512, size=(2, 64))
    return cfg, model, qblocks, tokens


def test_first_step_gradients_match_autograd():
    from gsq_rco_mlx_b200.gsq.e2e import LIN_ORDER
    from gsq_rco_mlx_b200.gsq.finetune import ScaleFinetune
    cfg, model, qblocks, tokens = _setup()
    ft = ScaleFinetune(model, qblocks, tokens)
    kl0 = ft.step(0)
    torch.cuda.synchronize()
    # oracle: float64 autograd of the restated forward through W = bf16(s grid[code])
    E = model.embed.float().cpu()
    norm = model.norm.float().cpu()
    tok = torch.as_tensor(tokens[0].astype(np.int64))
    S = {}
    layers = []
    for L, Wd in enumerate(model.layers):
        W = {k: v.float().cpu() for k, v in Wd.items()}
        for name in LIN_ORDER:
            q = qblocks[L][name]
            s = torch.tensor(q["scales"].astype(np.float64), requires_grad=True)
            S[(L, name)] = s
            grid = torch.as_tensor(q["codes"].astype(np.float64) - 4)
            W[name] = ob.bf(s.repeat_interleave(64, 1) * grid)
        layers.append(W)

    def final(h, Ws):
        for W in Ws:
            h, _ = ob.block_hard(h, W, cfg.n_heads, cfg.n_kv, cfg.eps)
        return ob.rmsnorm(h, norm, cfg.eps)

    with torch.no_grad():
        Wfp = [{k: v.float().cpu() for k, v in Wd.items()} for Wd in model.layers]
        href = final(E[tok], Wfp)
        zr = ob.bf(href.to(F64) @ E.to(F64).T)
        lr = torch.log_softmax(zr, -1)
    hq = final(E[tok], layers)
    zq = ob.bf(hq.to(F64) @ E.to(F64).T)
    lq = torch.log_softmax(zq, -1)
    kl = (lr.exp() * (lr - lq)).sum() / len(tok)
    kl.backward()
    assert abs(kl0 - float(kl)) <= 2e-2 * abs(float(kl)) + 1e-6, (kl0, float(kl))
    for key, s in S.items():
        gpu = ft.q[key]["grad"].double().cpu()
        ref = s.grad
        cos = float((gpu * ref).sum() / (gpu.norm() * ref.norm() + 1e-30))
        rel = float((gpu - ref).norm() / (ref.norm() + 1e-30))
        assert cos > 0.99 and rel < 0.1, (key, cos, rel)


def test_finetune_runs_and_reduces_kl():
    from gsq_rco_mlx_b200.gsq.finetune import scale_finetune
    cfg, model, qblocks, tokens = _setup()
    scales, kls = scale_finetune(model, qblocks, tokens[:1], steps=30, lr=2e-4, log=lambda *a: None)
    assert len(kls) == 30 and all(np.isfinite(kls))
    assert np.mean(kls[-5:]) < kls[0]
    assert scales[0]["q_proj"].dtype == np.float16
    assert scales[1]["down_proj"].shape == qblocks[1]["down_proj"]["scales"].shape


def test_finetune_shards_rewrites_scales(tmp_path):
    from gsq_rco_mlx_b200.gsq import pipeline as pl
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts
    cfg, model, qblocks, tokens = _setup()
    fp = pl.fingerprint(BlockOpts(), 2, 64)
    for L, lins in qblocks.items():
        pl.save_shard(str(tmp_path / f"layer_{L:02d}.npz"), L, lins,
                      {n: 3 for n in lins}, fp, {"seconds": 0})
    res = pl.finetune_shards(model, str(tmp_path), [0, 1], tokens, steps=4, log=lambda *a: None)
    assert res["steps"] == 4 and np.isfinite(res["kl_last"])
    meta, stats, lins = pl.load_shard(str(tmp_path / "layer_01.npz"))
    assert stats["scale_finetune"]["steps"] == 4 and meta["fingerprint"] == fp
    assert not np.array_equal(lins["up_proj"]["scales"], qblocks[1]["up_proj"]["scales"])
    assert np.array_equal(lins["up_proj"]["codes"], qblocks[1]["up_proj"]["codes"])
