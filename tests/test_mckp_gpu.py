"""MCKP DP on the GPU: bit-exact against the reference's decodes (golden vectors), batched
decodes, the RCO loop with the GPU decode, and the kernel's refusal of problems that have no
feasible assignment or a negative step (z = -1, no out-of-table access)."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_dp_golden_bit_exact():
    from gsq_rco_mlx_b200.rco import manifold
    z = np.load(os.path.join(GOLD, "dp.npz"))
    for n in range(int(z["dp_n"])):
        s, c, w, B = z[f"dp{n}_s"], z[f"dp{n}_c"], z[f"dp{n}_w"], int(z[f"dp{n}_B"])
        # the first 60 cases are the reference's full-DP decodes (random non-uniform weights)
        got = manifold.dp_knapsack(s, c, w, B, use_topk=n >= 60)
        assert np.array_equal(got, z[f"dp{n}_z"]), n


def test_dp_batch_equals_oracle():
    from gsq_rco_mlx_b200.rco import manifold
    from oracle import dp as odp
    z = np.load(os.path.join(GOLD, "dp.npz"))
    w = z["qwen_w_int"]
    rng = np.random.default_rng(4)
    S = rng.standard_normal((8, 168, 3))
    costs = np.array([2, 3, 4])
    zb = manifold.dp_knapsack_batch(S, costs, w, 3 * int(w.sum()))
    for j in range(8):
        assert np.array_equal(zb[j], odp.dp_knapsack(S[j], costs, w, 3 * int(w.sum())))


def test_rco_loop_with_gpu_decode_matches_reference():
    from gsq_rco_mlx_b200.rco import loop
    z = np.load(os.path.join(GOLD, "rco_host.npz"))
    target = z["lin_target"]

    def grad_fn(zz, p, t, j, rng):
        return -target, float(-(zz * target).sum())
    res = loop.rco_loop(np.zeros((12, 3)), np.array([2.0, 3.0, 4.0]), z["lin_w"],
                        3.0 * z["lin_w"].sum(), steps=15, g=4, lr=0.1, seed=3, grad_fn=grad_fn)
    np.testing.assert_allclose(res["logits"], z["lin_logits"], rtol=1e-6, atol=1e-8)
    assert np.array_equal(res["z_final"], z["lin_z"])
    np.testing.assert_array_equal([h["loss"] for h in res["history"]], z["lin_loss"])


def _raw_dp(S, step, B):
    """mckp_dp_f64 through the C ABI on device copies of S [n_inst, N, K] and step [N, K]."""
    from gsq_rco_mlx_b200 import _lib
    lib = _lib.lib()
    dev = torch.device("cuda", 0)
    n_inst, N, K = S.shape
    s_t = torch.as_tensor(np.ascontiguousarray(S), device=dev)
    st_t = torch.as_tensor(np.ascontiguousarray(step, dtype=np.int64), device=dev)
    ch = torch.empty(n_inst * N * (B + 1), device=dev, dtype=torch.uint8)
    rows = torch.empty(n_inst * 2 * (B + 1), device=dev, dtype=torch.float64)
    z = torch.full((n_inst, N), 7, device=dev, dtype=torch.int32)
    rc = lib.mckp_dp_f64(C.c_void_p(s_t.data_ptr()), C.c_void_p(st_t.data_ptr()), n_inst, N, K,
                         B, C.c_void_p(ch.data_ptr()), C.c_void_p(rows.data_ptr()),
                         C.c_void_p(z.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    torch.cuda.synchronize()
    return z.cpu().numpy()


def test_infeasible_and_negative_steps_give_minus_one():
    """The C entry point is also called without the Python checks. An instance whose cheapest
    assignment exceeds the budget, or whose step table holds a negative entry, gets z = -1 in
    every group; the other instances of the same launch decode normally."""
    from oracle import dp as odp
    rng = np.random.default_rng(7)
    w = np.array([3, 1, 2, 5, 4])
    costs = np.array([2, 3, 4])
    step = w[:, None] * costs[None, :]
    S = rng.standard_normal((2, 5, 3))
    cheapest = int(step.min(axis=1).sum())             # 30
    z = _raw_dp(S, step, cheapest - 1)
    assert np.all(z == -1)
    B = cheapest + 7
    z = _raw_dp(S, step, B)
    for j in range(2):
        assert np.array_equal(z[j], odp.dp_knapsack(S[j], costs, w, B).argmax(axis=1))
    bad = step.copy()
    bad[2, 1] = -3
    assert np.all(_raw_dp(S, bad, B) == -1)


def test_rows_in_global_memory_for_large_budgets():
    """Budgets above the shared-memory rows (B' > 13823) use the caller's row workspace."""
    from gsq_rco_mlx_b200.rco import manifold
    from oracle import dp as odp
    rng = np.random.default_rng(9)
    w = rng.integers(1, 40, size=60)
    costs = np.array([2, 3, 4, 6])
    B = 3 * int(w.sum()) * 8                           # well above 13823 with 8 ticks
    costs8 = costs * 8
    assert B > 13823
    S = rng.standard_normal((60, 4))
    got = manifold.dp_knapsack(S, costs8, w, B)
    assert np.array_equal(got, odp.dp_knapsack(S, costs8, w, B))
