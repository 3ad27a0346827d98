"""The block-by-block quantization driver on the GPU (reference src/gsq_rco/gsq/pipeline.py:
120-174): shards written for every quantized block, a resumed run that replays the finished
blocks from their shards reproduces the remaining shards bit for bit (the replayed stream equals
the trained one), and the shards export to an mlx-lm checkpoint that the packed eval loads."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _model():
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig
    from gsq_rco_mlx_b200.rco.database import random_model
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    return random_model(n_layers=2, seed=4, device=DEV, cfg=cfg, vocab=512)


def test_quantize_model_resume_and_export(tmp_path):
    from gsq_rco_mlx_b200.common.evaluate import PackedModel, perplexity
    from gsq_rco_mlx_b200.gsq import export as ex
    from gsq_rco_mlx_b200.gsq import pipeline as pl
    from gsq_rco_mlx_b200.gsq.e2e import LIN_ORDER
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts
    model = _model()
    cal = np.random.default_rng(1).integers(0, 512, size=(4, 64))
    bits = pl.load_bits([0, 1], alloc={"per_layer_bits": {"0": 3, "1": 2}})
    opts = BlockOpts(steps=4)
    out = str(tmp_path / "q")
    res = pl.quantize_model(model, cal, bits, opts, out, log=lambda *a: None)
    torch.cuda.synchronize()
    assert sorted(res["layers"]) == [0, 1]
    first = {i: pl.load_shard(os.path.join(out, f"layer_{i:02d}.npz")) for i in (0, 1)}
    for i in (0, 1):
        meta, stats, lins = first[i]
        assert meta["layer"] == i and meta["bits"] == bits[i]
        for n in LIN_ORDER:
            assert lins[n]["codes"].shape == tuple(model.layers[i][n].shape)
            assert int(lins[n]["codes"].max()) < (1 << bits[i][n])
    with pytest.raises(FileExistsError):
        pl.quantize_model(model, cal, bits, opts, out, log=lambda *a: None)
    # drop the last shard and resume: block 0 replays from its shard, block 1 trains again
    os.remove(os.path.join(out, "layer_01.npz"))
    pl.quantize_model(model, cal, bits, opts, out, resume=True, log=lambda *a: None)
    _, _, again = pl.load_shard(os.path.join(out, "layer_01.npz"))
    for n in LIN_ORDER:
        assert np.array_equal(again[n]["codes"], first[1][2][n]["codes"]), n
        assert np.array_equal(again[n]["scales"], first[1][2][n]["scales"]), n
    with pytest.raises(ValueError):   # other settings than the shards were made with
        pl.quantize_model(model, cal, bits, BlockOpts(steps=5), out, resume=True,
                          log=lambda *a: None)
    # export the shards next to a base checkpoint and evaluate the packed model
    base = str(tmp_path / "base")
    ex.save_base_checkpoint(model, base)
    path = pl.export_quantized(out, base, [0, 1])
    assert os.path.exists(path)
    pm = PackedModel.load(os.path.join(out, "mlx"), device=DEV)
    r = perplexity(pm, np.random.default_rng(2).integers(0, 512, size=(2, 64)), chunk_seqs=2)
    assert np.isfinite(r["nll_per_token"]) and r["n_tokens"] == 2 * 63
