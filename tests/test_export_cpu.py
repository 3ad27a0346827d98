"""MLX affine export format (host side, no GPU): packed words against the reference's own
pack_codes (golden vectors), the bit-by-bit oracle, the affine scales / biases, the bit
accounting, and the safetensors checkpoint written by export_mlx_lm (reference
src/gsq_rco/gsq/export.py, tests/test_export.py:92-150)."""
import json
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from gsq_rco_mlx_b200.gsq import export as ex
from gsq_rco_mlx_b200.gsq.e2e import BlockConfig
from oracle import evaluate as oe

GOLD = np.load(Path(__file__).parent / "golden" / "export.npz")


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_pack_codes_matches_reference_words(bits):
    codes, words = GOLD[f"codes{bits}"], GOLD[f"words{bits}"]
    assert words.dtype == np.uint32
    np.testing.assert_array_equal(ex.pack_codes(codes, bits), words)
    np.testing.assert_array_equal(oe.pack_codes(codes, bits), words)
    np.testing.assert_array_equal(ex.unpack_codes(words, bits, codes.shape[1]), codes)
    np.testing.assert_array_equal(oe.unpack_codes(words, bits, codes.shape[1]), codes)


def test_ternary_is_stored_as_two_bit():
    codes = GOLD["codes_t"]
    packed, sc, bi = ex.to_mlx_affine(codes, np.ones((codes.shape[0], 2), np.float32), 1, 64)
    np.testing.assert_array_equal(packed, GOLD["words_t"])
    assert [ex.mlx_bits(b) for b in (1, 2, 3, 4, 5, 6, 8)] == list(GOLD["mlx_bits"])
    assert torch.equal(bi, -2 * sc)
    with pytest.raises(ValueError):
        ex.mlx_bits(7)


def test_ragged_whole_word_rows():
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 256, size=(3, 4), dtype=np.uint8)       # 4 x 8 bits = 1 word
    np.testing.assert_array_equal(ex.pack_codes(codes, 8), oe.pack_codes(codes, 8))
    with pytest.raises(ValueError):
        ex.pack_codes(codes[:, :3], 3)                                  # 9 bits


@pytest.mark.parametrize("scale_dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("bits", [1, 2, 3, 4, 8])
def test_affine_values_equal_native_dequant(bits, scale_dtype):
    """scale q + bias equals scale grid[c] exactly (bias = -2^(b-1) scale in every dtype); with
    16-bit scales the loaded weight is within 2^-7 relative of the float32 native weight
    (export.py:16-20, test_export.py:107-111)."""
    rng = np.random.default_rng(bits)
    codes = rng.integers(0, len(oe.grid(bits)), size=(8, 256), dtype=np.uint8)
    s = (rng.standard_normal((8, 4)) * 0.1).astype(np.float32)
    packed, sc, bi = ex.to_mlx_affine(codes, s, bits, 64, scale_dtype)
    q = ex.unpack_codes(packed, ex.mlx_bits(bits), 256).astype(np.float64)
    gid = np.arange(256) // 64
    w = sc.double().numpy()[:, gid] * q + bi.double().numpy()[:, gid]
    np.testing.assert_array_equal(w, sc.double().numpy()[:, gid] * oe.grid(bits)[codes])
    ref = s.astype(np.float64)[:, gid] * oe.grid(bits)[codes]
    if scale_dtype == "float32":
        np.testing.assert_array_equal(w, ref)
    else:
        assert np.all(np.abs(w - ref) <= 2.0 ** -7 * np.abs(ref))
    # the oracle's dense weight is the bf16 rounding of the same values
    dt = ex.SCALE_DTYPES[scale_dtype][0]
    np.testing.assert_array_equal(oe.dequant(codes, s, bits, 64, dt).numpy(),
                                  torch.as_tensor(w).float().bfloat16().float().numpy())


def test_to_mlx_affine_rejects_bad_inputs():
    with pytest.raises(ValueError):
        ex.to_mlx_affine(np.full((2, 64), 4, np.uint8), np.ones((2, 1), np.float32), 2)
    with pytest.raises(ValueError):
        ex.to_mlx_affine(np.zeros((2, 64), np.uint8), np.ones((2, 1), np.float32), 2, 48)
    with pytest.raises(ValueError):
        ex.to_mlx_affine(np.zeros((2, 128), np.uint8), np.ones((2, 1), np.float32), 2, 64)


def test_bits_report_hand_case():
    hand = {"a": dict(codes=np.zeros((4, 128), np.uint8), scales=np.ones((4, 2), np.float16),
                      bits=2, group_size=64),
            "b": dict(codes=np.zeros((2, 64), np.uint8), scales=np.ones((2, 1), np.float16),
                      bits=1, group_size=64)}
    rep = ex.bits_report(hand, 640)
    for k in ("code_bpp", "native_bpp", "mlx_bpp", "shard_bpp"):
        assert rep[k] == pytest.approx(float(GOLD[f"report_{k}"]), rel=1e-15)
    with pytest.raises(ValueError):
        ex.bits_report(hand, 641)


def _tiny_model():
    from gsq_rco_mlx_b200.rco.database import random_model
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    return random_model(n_layers=2, seed=3, device="cpu", cfg=cfg, vocab=512)


def test_safetensors_round_trip(tmp_path):
    t = {"a": torch.randn(3, 5).bfloat16(), "b": torch.arange(6, dtype=torch.int32),
         "c": np.arange(8, dtype=np.uint32).reshape(2, 4), "d": torch.randn(4).half()}
    path = tmp_path / "x.safetensors"
    ex.write_safetensors(str(path), t, {"format": "mlx"})
    st = ex.SafetensorsFile(str(path))
    assert st.names() == ["a", "b", "c", "d"]
    assert st.metadata == {"format": "mlx"}
    assert torch.equal(st.tensor("a"), t["a"])
    assert torch.equal(st.tensor("b"), t["b"])
    assert st.tensor("c").numpy().view(np.uint32).tolist() == t["c"].tolist()
    assert torch.equal(st.tensor("d"), t["d"])
    np.testing.assert_array_equal(st.tensor_f32("a"), t["a"].float().numpy())


def test_export_mlx_lm_checkpoint(tmp_path):
    model = _tiny_model()
    base = tmp_path / "base"
    ex.save_base_checkpoint(model, str(base))
    rng = np.random.default_rng(0)
    quantized = {}
    for L in range(2):
        for j, name in enumerate(("q_proj", "up_proj", "down_proj")):
            W = model.layers[L][name]
            bits = (2, 3, 4)[(L + j) % 3]
            quantized[ex.module_path(L, name)] = dict(
                codes=rng.integers(0, 1 << bits, size=tuple(W.shape), dtype=np.uint8),
                scales=(0.01 * rng.standard_normal((W.shape[0], W.shape[1] // 64))).astype(
                    np.float32), bits=bits, group_size=64)
    out = tmp_path / "out"
    ex.export_mlx_lm(str(out), quantized, str(base), scale_dtype="float16")
    bst = ex.SafetensorsFile(str(base / "model.safetensors"))
    qst = ex.SafetensorsFile(str(out / "model.safetensors"))
    conf = json.loads((out / "config.json").read_text())
    for name in bst.names():
        path = name[:-len(".weight")] if name.endswith(".weight") else None
        if path in quantized:
            q = quantized[path]
            assert qst.dtype(name) == "U32"
            np.testing.assert_array_equal(qst.tensor(name).numpy().view(np.uint32),
                                          oe.pack_codes(q["codes"], q["bits"]))
            assert qst.dtype(path + ".scales") == "F16"
            sc = qst.tensor(path + ".scales").float().numpy()
            np.testing.assert_array_equal(sc, q["scales"].astype(np.float16).astype(np.float32))
            # the bias is cast from -2^(b-1) s in float32 (export.py:88), so it keeps digits
            # the float16 scale loses where s is subnormal in float16
            np.testing.assert_array_equal(
                qst.tensor(path + ".biases").float().numpy(),
                (np.float32(-(1 << (q["bits"] - 1))) * q["scales"]).astype(np.float16)
                .astype(np.float32))
            assert conf["quantization"][path] == {"group_size": 64, "bits": q["bits"]}
        else:
            assert qst.read_bytes(name) == bst.read_bytes(name), name
    with pytest.raises(ValueError):
        ex.export_mlx_lm(str(out), {"model.layers.9.mlp.up_proj": quantized[
            ex.module_path(0, "up_proj")]}, str(base))
    with pytest.raises(ValueError):
        ex.export_mlx_lm(str(out), {}, str(base))
