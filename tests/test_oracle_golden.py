"""Pins the CPU oracle to golden vectors produced by the reference's own numpy code
(tests/golden/make_golden.py). CPU only."""
import ctypes
import os

import numpy as np
import pytest

from oracle import dp as odp
from oracle import gptq as og
from oracle import gsq as ogsq
from oracle.philox import gumbel_planes, philox4x32_10

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def test_philox_known_answers():
    """Random123 known-answer vectors for Philox4x32-10."""
    cases = [((0, 0, 0, 0), (0, 0), "6627e8d5 e169c58d bc57ac4c 9b00dbd8"),
             ((0xffffffff,) * 4, (0xffffffff,) * 2, "408f276d 41c83b0e a20bc7c6 6d5451fd"),
             ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
              "d16cfe09 94fdcceb 5001e420 24126ea1")]
    for c, k, want in cases:
        r = philox4x32_10(np.array([c[0]], dtype=np.uint32), c[1], c[2], c[3], k[0], k[1])
        assert " ".join("%08x" % int(x[0]) for x in r) == want


def test_gumbel_moments():
    """Gumbel(0,1): mean 0.5772, variance pi^2/6 (reference tests/test_gsq_pipeline.py:139-142)."""
    g = gumbel_planes(7, 3, 0, 1, 200_000, 5)
    assert abs(g.mean() - 0.5772) < 0.01 and abs(g.var() - np.pi ** 2 / 6) < 0.03


def test_grid_schedule_local_shift_inits():
    z = load("gsq.npz")
    for b in range(1, 9):
        assert np.array_equal(ogsq.get_grid(b), z[f"grid{b}"])
    sch = np.array([ogsq.gs_schedules(t, 200) for t in range(200)])
    assert np.array_equal(sch, z["sched"])
    assert np.array_equal(ogsq.local_shift_values(z["ls_j0"], ogsq.get_grid(3)), z["ls_C"])
    assert np.array_equal(ogsq.local_shift_indices(z["ls_j0"], z["ls_logits"], 8), z["ls_idx"])
    edge = ogsq.local_shift_indices(np.array([0, 7]), np.array(
        [[-99., -99., -99., -99., 99.], [99., -99., -99., -99., -99.]], dtype=np.float32), 8)
    assert list(edge) == [2, 5] and np.array_equal(edge, z["ls_edge"])
    assert np.array_equal(ogsq.init_shift_logits(300, 6.0, 0.01, seed=5), z["init_shift"])
    assert np.array_equal(ogsq.init_logits_2bit_from_codes(z["init2_codes"], 4, 6.0, 0.01, seed=6),
                          z["init2"])


def test_product_inits_match_reference():
    """The product's App-A logit inits (host numpy, gsq/gptq.py) against the reference's own
    outputs: the same normals and float32 arithmetic, bit for bit."""
    from gsq_rco_mlx_b200.gsq import gptq as pg
    z = load("gsq.npz")
    assert np.array_equal(pg.init_shift_logits(300, 6.0, 0.01, seed=5), z["init_shift"])
    assert np.array_equal(pg.init_logits_2bit_from_codes(z["init2_codes"], 4, 6.0, 0.01, seed=6),
                          z["init2"])


def test_linear_grads_match_reference_oracle_2bit():
    """The restated loss/gradients equal tests/oracles.py:311-347 on the same Gumbel draws."""
    z = load("gsq.npz")
    W, X = z["lg_W"], z["lg_X"]
    bits, gs = 2, 16
    Ckd = ogsq.candidate_values(bits, z["lg_codes"].reshape(-1))
    logits_kd = np.ascontiguousarray(z["lg_logits"].T)
    noises = [np.ascontiguousarray(n.T) for n in z["lg_noise"]]
    tau, kappa = float(z["lg_tau"]), float(z["lg_kappa"])
    # the reference oracle runs the softmax in float64: compare in float64 here
    acc_l, acc_g, acc_s = 0.0, 0.0, 0.0
    for nz in noises:
        y = (kappa * logits_kd + nz.astype(np.float64)) / tau
        y -= y.max(axis=0, keepdims=True)
        p = np.exp(y); p /= p.sum(axis=0, keepdims=True)
        c = (p * Ckd).sum(axis=0).reshape(W.shape)
        sel = ogsq.expand_scales(z["lg_scales"], W.shape[1], gs).astype(np.float64)
        R = X @ (sel * c - W).T
        acc_l += (R * R).mean()
        G = (2.0 / (X.shape[0] * W.shape[0])) * (R.T @ X)
        gl, gsc = ogsq.soft_backward(G, p, Ckd, c, z["lg_scales"], gs, tau, kappa)
        acc_g = acc_g + gl
        acc_s = acc_s + gsc
    n = len(noises)
    assert abs(acc_l / n - float(z["lg_loss"])) <= 1e-12 * float(z["lg_loss"])
    np.testing.assert_allclose(acc_g.T / n, z["lg_glog"], rtol=1e-9, atol=1e-14)
    np.testing.assert_allclose(acc_s / n, z["lg_gscale"], rtol=1e-9, atol=1e-14)


def test_local_shift_grads_finite_differences():
    """Local-shift logit and scale gradients vs central differences (the reference checks the
    full grid the same way, tests/test_gsq_phase1.py:148-174)."""
    rng = np.random.default_rng(3)
    out_f, in_f, gs = 8, 64, 32
    W = 0.02 * rng.standard_normal((out_f, in_f))
    X = rng.standard_normal((40, in_f))
    r = og.quantize_rtn(W, 3, gs)
    Ckd = ogsq.candidate_values(3, r["codes"].reshape(-1)).astype(np.float64)
    lg = ogsq.init_logits(3, r["codes"], seed=1).astype(np.float64)
    sc = r["scales"].astype(np.float64)
    noise = gumbel_planes(1, 0, 0, 0, W.size, 5).astype(np.float64)
    tau, kappa = 2.0, 20.0  # unsaturated softmax, so every logit carries gradient

    def loss(lg_, sc_):
        y = (kappa * lg_ + noise) / tau
        y -= y.max(axis=0, keepdims=True)
        p = np.exp(y); p /= p.sum(axis=0, keepdims=True)
        c = (p * Ckd).sum(axis=0).reshape(W.shape)
        R = X @ (np.repeat(sc_, gs, axis=1) * c - W).T
        return (R * R).mean(), p, c, R

    L0, p, c, R = loss(lg, sc)
    G = (2.0 / (X.shape[0] * out_f)) * (R.T @ X)
    gl, gsc = ogsq.soft_backward(G, p, Ckd, c, sc, gs, tau, kappa)
    h = 1e-7
    for (k, i) in [(0, 3), (2, 100), (4, 511), (1, 257)]:
        e = np.zeros_like(lg); e[k, i] = h
        fd = (loss(lg + e, sc)[0] - loss(lg - e, sc)[0]) / (2 * h)
        assert abs(fd - gl[k, i]) <= 1e-4 * max(abs(fd), 1e-12)
    for (o, g) in [(0, 0), (5, 1), (7, 1)]:
        e = np.zeros_like(sc); e[o, g] = 1e-7
        fd = (loss(lg, sc + e)[0] - loss(lg, sc - e)[0]) / 2e-7
        assert abs(fd - gsc[o, g]) <= 1e-6 * max(abs(fd), 1e-12) + 1e-14


def test_ternary_matches_reference_oracle():
    """Ternary (1-bit) soft weights: the mask / sign logit init against gsq/gptq.py:222-232 and
    the soft / hard weight against the reference test oracle (tests/oracles.py:126-160) from the
    same Gumbel draws. The reference oracle divides by tau and clips the sigmoid's argument to
    +-50; the restatement multiplies by 1 / tau in float32: equal to a few float32 ulps of m and
    v (an absolute 1e-6 s where 2 v - 1 nearly cancels)."""
    from gsq_rco_mlx_b200.gsq.gptq import init_ternary_logits
    z = load("ternary.npz")
    q = z["init_q"]
    lm, lb = init_ternary_logits(q, alpha=3.0, std=0.01, seed=4)
    assert np.array_equal(lm, z["init_lm"]) and np.array_equal(lb, z["init_lb"])
    assert np.array_equal(ogsq.init_ternary_logits(q, alpha=3.0, seed=4),
                          np.stack([z["init_lm"], z["init_lb"]]))
    L = np.stack([z["lm"], z["lb"]])
    for j in range(2):
        tau, kappa = float(z[f"tau{j}"]), float(z[f"kappa{j}"])
        p = ogsq.ternary_probs(L, z["noise"], tau, kappa)
        w = np.float32(z["scale"]) * ogsq.ternary_value(p)
        np.testing.assert_allclose(w, z[f"soft{j}"], rtol=2e-6, atol=1e-6 * float(z["scale"]))
    codes = ogsq.ternary_hard_codes(L)
    np.testing.assert_array_equal(np.float32(z["scale"]) * ogsq.get_grid(1)[codes], z["hard"])
    np.testing.assert_array_equal(codes != 1, z["hard_m"] != 0)


def test_ternary_grads_finite_differences():
    """Ternary mask / sign logit and scale gradients vs central differences of the qk-stage loss
    through w = s m (2 v - 1) (float64)."""
    rng = np.random.default_rng(4)
    out_f, in_f, gs = 8, 64, 32
    W = 0.02 * rng.standard_normal((out_f, in_f))
    X = rng.standard_normal((40, in_f))
    r = og.quantize_rtn(W, 1, gs)
    lg = ogsq.init_logits(1, r["codes"], seed=2).astype(np.float64) + \
        0.3 * rng.standard_normal((2, W.size))
    sc = r["scales"].astype(np.float64)
    noise = gumbel_planes(1, 0, 0, 0, W.size, 4).astype(np.float64)
    tau, kappa = 2.0, 3.0
    sig = lambda x: 1.0 / (1.0 + np.exp(-x))

    def loss(lg_, sc_):
        m = sig((2 * kappa * lg_[0] + noise[1] - noise[0]) / tau)
        v = sig((2 * kappa * lg_[1] + noise[3] - noise[2]) / tau)
        c = (m * (2 * v - 1)).reshape(W.shape)
        R = X @ (np.repeat(sc_, gs, axis=1) * c - W).T
        return (R * R).mean(), np.stack([m, v]), c, R

    L0, p, c, R = loss(lg, sc)
    G = (2.0 / (X.shape[0] * out_f)) * (R.T @ X)
    gl, gsc = ogsq.soft_backward(G, p, None, c, sc, gs, tau, kappa)
    h = 1e-7
    for (k, i) in [(0, 3), (1, 100), (0, 511), (1, 257)]:
        e = np.zeros_like(lg); e[k, i] = h
        fd = (loss(lg + e, sc)[0] - loss(lg - e, sc)[0]) / (2 * h)
        assert abs(fd - gl[k, i]) <= 1e-4 * max(abs(fd), 1e-12) + 1e-15
    for (o, g) in [(0, 0), (5, 1), (7, 1)]:
        e = np.zeros_like(sc); e[o, g] = 1e-7
        fd = (loss(lg, sc + e)[0] - loss(lg, sc - e)[0]) / 2e-7
        assert abs(fd - gsc[o, g]) <= 1e-6 * max(abs(fd), 1e-12) + 1e-14


def test_lion_matches_reference_oracle():
    z = load("gsq.npz")
    P = z["lion_traj"][0]
    M = np.zeros_like(P)
    for t in range(3):
        P, M = ogsq.lion(P, M, z["lion_G"][t], 1e-2)
        np.testing.assert_array_equal(P, z["lion_traj"][t + 1])


def test_gptq_matches_reference():
    z = load("gptq.npz")
    for ci in range(int(z["gptq_n"])):
        r = og.quantize_gptq(z[f"gptq{ci}_W"], z[f"gptq{ci}_H"], int(z[f"gptq{ci}_bits"]),
                             int(z[f"gptq{ci}_gs"]), 0.01, int(z[f"gptq{ci}_block"]))
        agree = (r["codes"] == z[f"gptq{ci}_codes"]).mean()
        assert agree >= 0.999, (ci, agree)
        assert abs(r["err"] - float(z[f"gptq{ci}_err"])) <= 1e-6 * float(z[f"gptq{ci}_err"])
        np.testing.assert_allclose(r["scales"], z[f"gptq{ci}_scales"], rtol=1e-5)
    for bits in (1, 2, 3, 4, 8):
        r = og.quantize_rtn(z["rtn_W"], bits, 64)
        assert np.array_equal(r["codes"], z[f"rtn{bits}_codes"])
        assert np.array_equal(r["scales"], z[f"rtn{bits}_scales"])
        assert np.array_equal(r["w_q"], z[f"rtn{bits}_wq"])
    assert np.array_equal(og.quantize_gptq(z["rtn_W"], np.eye(100), 3, 64)["codes"],
                          z["gptq_eye_codes"])
    c96 = og.quantize_gptq(z["blk_W"], z["blk_H"], 2, 24, block_size=96)["codes"]
    c16 = og.quantize_gptq(z["blk_W"], z["blk_H"], 2, 24, block_size=16)["codes"]
    assert np.array_equal(c96, z["blk_codes96"]) and np.array_equal(c16, z["blk_codes16"])
    X = z["hess_X"]
    Ha, na = og.hessian_from_inputs(X[:200])
    Hab, nab = og.hessian_from_inputs(X[200:], Ha, na)
    assert nab == int(z["hess_n"])
    np.testing.assert_allclose(Hab, z["hess_H"], rtol=1e-12, atol=1e-12)
    with pytest.raises(NotImplementedError):
        og.quantize_gptq(z["blk_W"], z["blk_H"], 2, 24, act_order=True)
    with pytest.raises(ValueError):
        og.quantize_rtn(z["rtn_W"], 9, 64)


def _dp_cases():
    z = load("dp.npz")
    return [(z[f"dp{n}_s"], z[f"dp{n}_c"], z[f"dp{n}_w"], int(z[f"dp{n}_B"]), z[f"dp{n}_z"])
            for n in range(int(z["dp_n"]))]


def test_dp_numpy_matches_reference():
    for s, c, w, B, zref in _dp_cases():
        assert np.array_equal(odp.dp_knapsack(s, c, w, B), zref)


def test_dp_c_matches_reference():
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    so = os.path.join(here, "oracle", "_build", "libdp_oracle.so")
    if not os.path.exists(so):
        import subprocess
        subprocess.run(["make", "-C", os.path.join(here, "oracle")], check=True)
    lib = ctypes.CDLL(so)
    for s, c, w, B, zref in _dp_cases():
        if len(c) == 2 and np.all(w == w[0]):
            continue  # the K = 2 top-k shortcut is host logic, not the DP table
        N, K = s.shape
        step = np.ascontiguousarray((w[:, None] * c[None, :]).astype(np.int64))
        sv = np.ascontiguousarray(s, dtype=np.float64)
        choice = np.zeros(N * (B + 1), dtype=np.uint8)
        zi = np.zeros(N, dtype=np.int32)
        rc = lib.oracle_mckp_dp(sv.ctypes.data_as(ctypes.c_void_p), step.ctypes.data_as(ctypes.c_void_p),
                                N, K, ctypes.c_int64(B), choice.ctypes.data_as(ctypes.c_void_p),
                                zi.ctypes.data_as(ctypes.c_void_p))
        assert rc == 0
        assert np.array_equal(zref.argmax(axis=1), zi)


@pytest.mark.parametrize("bits", [2, 3])
def test_c_backend_matches_numpy_oracle(bits):
    """The C backend of the GSQ oracle (oracle/gsq_c.c, used by the full-size parity runs)
    against the numpy restatement that the golden vectors pin: the Philox noise, soft weight,
    backward and Lion agree to float32 rounding, and a short training run stays together."""
    from oracle import gsq as ogsq
    from oracle import gsq_fast
    from oracle.philox import gumbel_planes
    rng = np.random.default_rng(bits)
    out_f, in_f = 48, 200                       # ragged last group
    codes = rng.integers(0, 2 ** bits, size=(out_f, in_f)).astype(np.uint8)
    s16 = (0.01 + 0.02 * rng.random((out_f, 4))).astype(np.float16)
    st = ogsq.LinearState(bits, codes, s16, 64, seed=1, linear_id=3)
    d, K = codes.size, st.K
    nz = gumbel_planes(5, 3, 7, 1, d, K)
    nz_c = gsq_fast.gumbel_planes(5, 3, 7, 1, d, K)
    assert np.abs(nz_c - nz).max() <= 4e-7 * np.abs(nz).max()
    w, p, c = ogsq.soft_weight(st.logits, nz, st.Ckd, st.scales, (out_f, in_f), 64, 0.7, 180.0)
    w2, p2, c2 = gsq_fast.soft_weight(st.logits, nz, st.Ckd, st.scales, (out_f, in_f), 64,
                                      0.7, 180.0)
    np.testing.assert_allclose(p2, p, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(w2, w, rtol=2e-6, atol=1e-8)
    G = rng.standard_normal((out_f, in_f)) * 1e-3
    gl, gsc = ogsq.soft_backward(G, p, st.Ckd, c, st.scales, 64, 0.7, 180.0)
    acc = [np.zeros((K, d), np.float32), np.zeros((out_f, 4), np.float32)]
    gsq_fast.soft_backward_acc(G, p, st.Ckd, c, st.scales, 64, 0.7, 180.0, acc[0], acc[1])
    np.testing.assert_array_equal(acc[0], gl.astype(np.float32))
    np.testing.assert_allclose(acc[1], gsc.astype(np.float32), rtol=1e-6, atol=1e-12)
    P, M = st.logits.copy(), (0.1 * rng.standard_normal(st.logits.shape)).astype(np.float32)
    Pn, Mn = ogsq.lion(P, M, gl, 1e-4)
    gsq_fast.lion_(P, M, gl, 1e-4, ogsq.WEIGHT_DECAY, ogsq.BETAS)
    np.testing.assert_array_equal(P, Pn)
    np.testing.assert_array_equal(M, Mn)
    # a short qk-stage run with each backend
    X = rng.standard_normal((8 * 33, in_f)).astype(np.float32)
    Wf = (0.02 * rng.standard_normal((out_f, in_f))).astype(np.float32)
    Xs = X.reshape(8, 33, in_f)[:, 1:]
    runs = []
    for backend in ("numpy", "c"):
        prev = ogsq.set_backend(backend)
        try:
            s = ogsq.LinearState(bits, codes, s16, 64, seed=1, linear_id=3)
            h = ogsq.train_linear(s, lambda idx: Xs[idx].reshape(-1, in_f), Wf, 8, 6, seed=2,
                                  noise_seed=9)
            runs.append((s.logits.copy(), s.scales.copy(), h))
        finally:
            ogsq.set_backend(prev)
    (l0, s0, h0), (l1, s1, h1) = runs
    assert np.linalg.norm(l1 - l0) <= 1e-5 * np.linalg.norm(l0)
    assert np.linalg.norm(s1 - s0) <= 1e-5 * np.linalg.norm(s0)
    np.testing.assert_allclose(h1, h0, rtol=1e-5)
