"""Packed quantized-model eval on the GPU against the CPU oracle (oracle/evaluate.py):
the dequant of MLX-affine packed words (bit-exact), the packed GEMV / GEMM (float32 accumulation,
one output rounding), the NLL row pass, and the perplexity of a small mixed-bit model against
the NLL of the bf16-dequantized dense model (reference src/gsq_rco/common/evaluate.py:35-78,
src/gsq_rco/gsq/export.py)."""
import numpy as np
import pytest
import torch

from oracle import evaluate as oe

pytestmark = pytest.mark.gpu
DEV = "cuda"
DT = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _linear(N, K, bits, gs, scale_dtype, seed, unrounded=False):
    from gsq_rco_mlx_b200.common.evaluate import PackedLinear
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, len(oe.grid(bits)), size=(N, K), dtype=np.uint8)
    codes[0] = 0
    codes[1] = len(oe.grid(bits)) - 1
    s = (0.02 * rng.standard_normal((N, K // gs))).astype(np.float32)
    lin = PackedLinear.from_native(codes, s, bits, gs, scale_dtype, device=DEV)
    if unrounded:
        return lin, oe.affine_weight(codes, s, bits, gs, DT[scale_dtype])
    return lin, oe.dequant(codes, s, bits, gs, DT[scale_dtype])


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 5, 6, 8])
@pytest.mark.parametrize("scale_dtype,gs", [("bfloat16", 64), ("float16", 32),
                                            ("float32", 128)])
def test_dequant_is_bit_exact(bits, scale_dtype, gs):
    lin, ref = _linear(96, 384, bits, gs, scale_dtype, seed=bits)
    out = torch.empty(96, 384, device=DEV, dtype=torch.bfloat16)
    lin.dequant(out)
    torch.cuda.synchronize()
    assert torch.equal(out.float().cpu(), ref)


@pytest.mark.parametrize("M", [1, 3, 8, 9, 200])
@pytest.mark.parametrize("bits", [2, 3, 4, 6])
def test_packed_matmul_matches_dense(M, bits):
    """M <= 8: the fused matrix-vector form multiplies by the unrounded weight s q + bias (MLX's
    quantized matrix-vector product); M > 8: the tensor-core GEMM on the bf16-dequantized
    weight."""
    from gsq_rco_mlx_b200.gemm import check_err
    N, K = 320, 896
    lin, Wd = _linear(N, K, bits, 64, "float16", seed=10 + bits, unrounded=M <= 8)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).bfloat16()
    ref = x.double() @ Wd.double().T
    mag = x.double().abs() @ Wd.double().abs().T
    y32 = lin(x.to(DEV), y_f32=True)
    yb = lin(x.to(DEV))
    torch.cuda.synchronize()
    check_err(torch.device(DEV))
    d32 = (y32.double().cpu() - ref).abs()
    assert float((d32 - 4e-5 * mag).max()) <= 0.0
    # bf16 output: one rounding of the float32 sum
    db = (yb.double().cpu() - ref).abs()
    assert float((db - (2.0 ** -8 * ref.abs() + 4e-5 * mag)).max()) <= 0.0


def test_nll_rows():
    from gsq_rco_mlx_b200 import _lib
    n, V = 37, 1000
    g = torch.Generator().manual_seed(2)
    z = (3 * torch.randn(n, V, generator=g)).bfloat16()
    t = torch.randint(0, V, (n,), generator=g, dtype=torch.int32)
    t[5] = -1
    out = torch.empty(n, device=DEV, dtype=torch.float64)
    zd, td = z.to(DEV), t.to(DEV)
    _lib.call("gsq_nll_rows", _lib.ptr(zd), n, V, V, _lib.ptr(td), _lib.ptr(out),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    ref = oe.nll_rows(z.float(), t.numpy())
    np.testing.assert_allclose(out.cpu().numpy(), ref.numpy(), rtol=1e-6, atol=1e-5)
    assert float(out[5]) == 0.0


def _small_model(layers=2, seed=0):
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig
    from gsq_rco_mlx_b200.rco.database import random_model
    cfg = BlockConfig(hidden=256, n_heads=4, n_kv=2, inter=512)
    return random_model(n_layers=layers, seed=seed, device=DEV, cfg=cfg, vocab=1024)


def _mixed_quantized(model, seed=0):
    from gsq_rco_mlx_b200.gsq.e2e import LIN_ORDER
    from gsq_rco_mlx_b200.gsq.export import module_path
    rng = np.random.default_rng(seed)
    q = {}
    for L, W in enumerate(model.layers):
        for j, name in enumerate(LIN_ORDER):
            N, K = W[name].shape
            bits = (2, 3, 4)[(L * 7 + j) % 3]
            # codes near the dense weight so the model stays close to its dense activations
            s = (W[name].float().cpu().numpy().reshape(N, K // 64, 64).std(-1) + 1e-3) \
                .astype(np.float32)
            w = W[name].float().cpu().numpy()
            c = np.rint(w / np.repeat(s, 64, 1)) + (1 << (bits - 1))
            c = np.clip(c + rng.integers(-1, 2, size=c.shape), 0, (1 << bits) - 1)
            q[module_path(L, name)] = dict(codes=c.astype(np.uint8), scales=s, bits=bits,
                                           group_size=64)
    return q


def test_perplexity_matches_dense_oracle(tmp_path):
    from gsq_rco_mlx_b200.common.evaluate import PackedModel, perplexity
    from gsq_rco_mlx_b200.gsq import export as ex
    from gsq_rco_mlx_b200.gsq.e2e import LIN_ORDER
    model = _small_model()
    q = _mixed_quantized(model)
    pm = PackedModel.from_quantized(model, q, scale_dtype="float16")
    rng = np.random.default_rng(4)
    windows = rng.integers(0, 1024, size=(5, 128))
    r = perplexity(pm, windows, chunk_seqs=2)
    torch.cuda.synchronize()
    assert r["n_tokens"] == 5 * 127 and r["seq_len"] == 128 and r["n_windows"] == 5
    # the oracle on the bf16-dequantized dense weights (windows fed as tokens[:-1])
    layers = []
    for L, W in enumerate(model.layers):
        d = {k: v.float().cpu() for k, v in W.items()}
        for name in LIN_ORDER:
            qq = q[ex.module_path(L, name)]
            d[name] = oe.dequant(qq["codes"], qq["scales"], qq["bits"], 64, torch.float16)
        layers.append(d)
    tot, n = oe.model_nll(model.embed.float().cpu(), layers, model.norm.float().cpu(), windows,
                          model.cfg.n_heads, model.cfg.n_kv, model.cfg.eps)
    assert n == r["n_tokens"]
    assert abs(r["nll_per_token"] - tot / n) <= 1e-3, (r["nll_per_token"], tot / n)
    # the exported checkpoint loads back to the same packed model: identical NLL
    base, out = tmp_path / "base", tmp_path / "q"
    ex.save_base_checkpoint(model, str(base))
    ex.export_mlx_lm(str(out), q, str(base), scale_dtype="float16")
    pm2 = PackedModel.load(str(out), device=DEV)
    r2 = perplexity(pm2, windows, chunk_seqs=3)
    assert r2["nll_per_token"] == pytest.approx(r["nll_per_token"], rel=1e-12)


def test_packed_linear_rejects_bad_shapes():
    from gsq_rco_mlx_b200.common.evaluate import PackedLinear
    lin, _ = _linear(64, 256, 3, 64, "bfloat16", seed=1)
    with pytest.raises(ValueError):
        lin(torch.zeros(4, 128, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        PackedLinear(lin.words, lin.scales, lin.biases, 3, 64, 512)
