"""MCKP DP on the GPU: bit-exact against the reference's decodes (golden vectors)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_dp_golden_bit_exact():
    from gsq_rco_mlx_b200.rco import manifold
    z = np.load(os.path.join(GOLD, "dp.npz"))
    for n in range(int(z["dp_n"])):
        s, c, w, B = z[f"dp{n}_s"], z[f"dp{n}_c"], z[f"dp{n}_w"], int(z[f"dp{n}_B"])
        use_topk = True
        if n < 60:
            use_topk = False  # the reference ran these with the full DP
        got = manifold.dp_knapsack(s, c, w, B, use_topk=use_topk)
        assert np.array_equal(got, z[f"dp{n}_z"]), n


def test_dp_batch_equals_single():
    from gsq_rco_mlx_b200.rco import manifold
    z = np.load(os.path.join(GOLD, "dp.npz"))
    w = z["qwen_w_int"]
    rng = np.random.default_rng(4)
    S = rng.standard_normal((8, 168, 3))
    zb = manifold.dp_knapsack_batch(S, np.array([2, 3, 4]), w, 3 * int(w.sum()))
    from oracle import dp as odp
    for j in range(8):
        assert np.array_equal(zb[j], odp.dp_knapsack(S[j], np.array([2, 3, 4]), w, 3 * int(w.sum())))


def test_rco_loop_linear_objective_matches_reference():
    from gsq_rco_mlx_b200.rco import loop
    z = np.load(os.path.join(GOLD, "rco_host.npz"))
    target = z["lin_target"]

    def grad_fn(zz, p, t, j, rng):
        return -target, float(-(zz * target).sum())
    res = loop.rco_loop(np.zeros((12, 3)), np.array([2.0, 3.0, 4.0]), z["lin_w"], 3.0 * z["lin_w"].sum(),
                        steps=15, g=4, lr=0.1, seed=3, grad_fn=grad_fn)
    np.testing.assert_allclose(res["logits"], z["lin_logits"], rtol=1e-12, atol=1e-12)
    assert np.array_equal(res["z_final"], z["lin_z"])
    np.testing.assert_allclose([h["cost"] for h in res["history"]], z["lin_cost"], rtol=1e-13)
    np.testing.assert_allclose([h["loss"] for h in res["history"]], z["lin_loss"], rtol=1e-13)
