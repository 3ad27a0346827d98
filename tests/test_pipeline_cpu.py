"""Host side of the block-by-block quantization driver (reference src/gsq_rco/gsq/pipeline.py):
bit allocations, the layer_XX.npz shard format and its round trip."""
import json

import numpy as np
import pytest

from gsq_rco_mlx_b200.gsq import pipeline as pl
from gsq_rco_mlx_b200.gsq.e2e import LIN_ORDER
from gsq_rco_mlx_b200.gsq.staged import BlockOpts


def test_load_bits_forms():
    u = pl.load_bits([0, 1], uniform_bits=3)
    assert u == {i: {n: 3 for n in LIN_ORDER} for i in (0, 1)}
    per_layer = pl.load_bits([0, 1], alloc={"per_layer_bits": {"0": 2, "1": 4}})
    assert per_layer[0]["down_proj"] == 2 and per_layer[1]["q_proj"] == 4
    alloc = {"per_linear_bits": {f"{i}.{n}": 2 + (i + j) % 3 for i in (0, 1)
                                 for j, n in enumerate(LIN_ORDER)}}
    per_lin = pl.load_bits([0, 1], alloc=alloc)
    assert per_lin[1]["k_proj"] == 2 + (1 + 1) % 3
    with pytest.raises(ValueError):
        pl.load_bits([0], alloc=alloc, uniform_bits=3)
    with pytest.raises(ValueError):
        pl.load_bits([2], alloc=alloc)                       # layer without bits
    with pytest.raises(ValueError):
        pl.load_bits([0], uniform_bits=9)


def test_shard_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    lins = {n: {"codes": rng.integers(0, 8, size=(64, 128), dtype=np.uint8),
                "scales": (0.01 * rng.standard_normal((64, 2))).astype(np.float16), "bits": 3}
            for n in LIN_ORDER}
    fp = pl.fingerprint(BlockOpts(steps=5), 4, 128)
    bits = {n: 3 for n in LIN_ORDER}
    path = str(tmp_path / "layer_03.npz")
    pl.save_shard(path, 3, lins, bits, fp, {"seconds": 1.5})
    with np.load(path) as z:                     # the reference's keys and dtypes
        keys = set(z.files)
        assert {"meta", "stats"} <= keys
        for n in LIN_ORDER:
            assert z[f"{n}.codes"].dtype == np.uint8 and z[f"{n}.scales"].dtype == np.float16
            assert int(z[f"{n}.bits"]) == 3
        assert json.loads(str(z["meta"])) == {"layer": 3, "fingerprint": fp, "bits": bits}
    meta, stats, back = pl.load_shard(path)
    assert stats == {"seconds": 1.5} and meta["layer"] == 3
    for n in LIN_ORDER:
        assert np.array_equal(back[n]["codes"], lins[n]["codes"])
        assert np.array_equal(back[n]["scales"], lins[n]["scales"])
