"""The 24-layer database builder (reference src/gsq_rco/rco/database.py:158-241) on a short
stack: full-precision forward with four taps per layer, float64 Hessians, GPTQ per (linear,
option), against the torch-CPU block oracle and the numpy GPTQ oracle.

Two levels: (1) the builder's own Hessians against the oracle Hessian of the same taps, and the
oracle GPTQ on those Hessians (the parity bar: codes >= 99.9 %, sensitivity within 1e-3);
(2) the whole chain against the oracle forward, whose bf16 chains round the same way per
operation but drift apart over two blocks in rare last bits (bounded agreement)."""
import numpy as np
import pytest
import torch

from oracle import block as ob
from oracle import gptq as og

pytestmark = pytest.mark.gpu
DEV = "cuda"

SITE_TAP = {"qkv": "hn", "o": "o", "gate_up": "mn", "down": "d_in"}
SITE_OF = {"q_proj": "qkv", "k_proj": "qkv", "v_proj": "qkv", "o_proj": "o",
           "gate_proj": "gate_up", "up_proj": "gate_up", "down_proj": "down"}
NAMES = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


def oracle_hessians(model, tokens, n_layers):
    """Per layer: the oracle block on every window (bf16), Hessians of positions 1.. (float64)."""
    E = model.embed.cpu()
    hs = [E[torch.as_tensor(t, dtype=torch.long)] for t in tokens]
    out_H = []
    for L in range(n_layers):
        Wc = {k: v.cpu() for k, v in model.layers[L].items()}
        acc = {s: (None, 0) for s in SITE_TAP}
        outs = []
        for h in hs:
            out, taps = ob.block_hard(h, Wc)
            outs.append(out)
            for s, tap in SITE_TAP.items():
                acc[s] = og.hessian_from_inputs(taps[tap][1:].double().numpy(), *acc[s])
        hs = outs
        out_H.append({s: acc[s][0] for s in SITE_TAP})
    return out_H


def rel(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def built(tmp_path_factory):
    from gsq_rco_mlx_b200.rco.database import DBSpec, build_database, random_model
    model = random_model(n_layers=2, seed=3, device=torch.device(DEV), vocab=2048)
    tokens = np.random.default_rng(1).integers(0, 2048, size=(3, 160)).astype(np.int32)
    db = tmp_path_factory.mktemp("db")
    Hs = {}
    man, res = build_database(model, tokens, DBSpec(options=(2, 3), n_layers=2), db_dir=db,
                              log=lambda *a: None, chunk_windows=2, hessians_out=Hs)
    return model, tokens, db, man, res, {k: v.cpu().numpy() for k, v in Hs.items()}


def test_database_files_and_manifest(built):
    model, tokens, db, man, res, _ = built
    assert (db / "manifest.json").exists() and (db / "sensitivity.npy").exists()
    c0 = np.load(db / "L01.down_proj.b3.codes.npy")
    s0 = np.load(db / "L01.down_proj.b3.scales.npy")
    assert c0.dtype == np.uint8 and c0.shape == (896, 4864)
    assert s0.dtype == np.float32 and s0.shape == (896, 76)
    assert np.array_equal(c0, res[(1, "down_proj", 3)][0])
    assert man["calibration"]["hessian_rows"] == 3 * 159
    assert np.array_equal(np.load(db / "sensitivity.npy"), man["sensitivity"])
    assert man["groups"][:2] == ["0.q_proj", "0.k_proj"] and len(man["counts"]) == 14


def test_gptq_on_builder_hessians_matches_oracle(built):
    """The parity bar on the builder's own Hessians: codes >= 99.9 %, err within 1e-3."""
    model, tokens, db, man, res, Hs = built
    sens = man["sensitivity"]
    for L in range(2):
        for name in NAMES:
            W = model.layers[L][name].float().cpu().numpy()
            for k, b in enumerate((2, 3)):
                r = og.quantize_gptq(W, Hs[(L, SITE_OF[name])], b, 64, 0.01)
                agree = float(np.mean(res[(L, name, b)][0] == r["codes"]))
                assert agree >= 0.999, (L, name, b, agree)
                i = L * 7 + NAMES.index(name)
                assert abs(sens[i, k] - r["err"]) <= 1e-3 * abs(r["err"]), (L, name, b)


def test_builder_hessians_match_oracle_forward(built):
    """Layer 0 Hessians against the oracle forward: float32-accumulation accuracy; layer 1 (after
    one block of bf16 chains on both sides) within rare-last-bit drift."""
    model, tokens, db, man, res, Hs = built
    ref = oracle_hessians(model, tokens, 2)
    for site in SITE_TAP:
        r0 = rel(Hs[(0, site)], ref[0][site])
        assert r0 < 2e-3, (site, r0)
        r1 = rel(Hs[(1, site)], ref[1][site])
        assert r1 < 2e-2, (site, r1)
    # on the qkv site of layer 0 (the embedding rows, no upstream block): float32 exactness
    assert rel(Hs[(0, "qkv")], ref[0]["qkv"]) < 1e-5
