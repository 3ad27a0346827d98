"""GSQ soft linear on the GPU vs the oracle: soft weight, in-kernel Philox noise, fused
backward + Lion, argmax decode, and the 200-step qk-stage trajectory (the parity bar:
logits, scales and loss within 1e-3 relative, final codes equal on >= 99.9% of weights)."""
import numpy as np
import pytest
import torch

from oracle import gptq as og
from oracle import gsq as ogsq
from oracle.philox import gumbel_planes

pytestmark = pytest.mark.gpu

DEV = "cuda"


def make_linear(out_f=96, in_f=256, bits=3, gs=64, seed=0):
    from gsq_rco_mlx_b200.gsq.staged import SoftLinear
    rng = np.random.default_rng(seed)
    W = (0.02 * rng.standard_normal((out_f, in_f))).astype(np.float32)
    r = og.quantize_rtn(W, bits, gs)
    s16 = r["scales"].astype(np.float16)
    lin = SoftLinear("up_proj", bits, r["codes"], s16, gs, seed=seed + 7, linear_id=5)
    st = ogsq.LinearState(bits, r["codes"], s16, gs, seed=seed + 7, linear_id=5)
    return W, lin, st


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_soft_weight_host_noise(bits):
    W, lin, st = make_linear(bits=bits)
    noise = gumbel_planes(11, 5, 3, 1, W.size, st.K)
    tau, kappa = ogsq.gs_schedules(37, 200)
    w_o, _, _ = ogsq.soft_weight(st.logits, noise, st.Ckd, st.scales, W.shape, 64, tau, kappa)
    got = lin.soft(tau, kappa, 3, 1, 11, noise=torch.as_tensor(noise, device=DEV)).cpu().numpy()
    np.testing.assert_allclose(got, w_o, rtol=2e-6, atol=1e-6 * np.abs(w_o).max())
    # residual against the FP weight
    Wt = torch.as_tensor(W, device=DEV)
    got_r = lin.soft(tau, kappa, 3, 1, 11, w_ref=Wt, noise=torch.as_tensor(noise, device=DEV))
    np.testing.assert_allclose(got_r.cpu().numpy(), w_o - W, rtol=1e-5, atol=1e-6 * np.abs(w_o).max())


def test_philox_noise_in_kernel_matches_oracle():
    W, lin, st = make_linear()
    tau, kappa = 0.9, 300.0
    for (seed, step, r) in [(0, 0, 0), (123456789012, 17, 1)]:
        noise = gumbel_planes(seed, 5, step, r, W.size, 5)
        w_o, _, _ = ogsq.soft_weight(st.logits, noise, st.Ckd, st.scales, W.shape, 64, tau, kappa)
        got = lin.soft(tau, kappa, step, r, seed).cpu().numpy()
        np.testing.assert_allclose(got, w_o, rtol=1e-5, atol=1e-6 * np.abs(w_o).max())


def test_backward_lion_one_step():
    W, lin, st = make_linear()
    rng = np.random.default_rng(3)
    tau, kappa = ogsq.gs_schedules(5, 200)
    Gs = [(1e-3 * rng.standard_normal(W.shape)).astype(np.float32) for _ in range(2)]
    noises = [gumbel_planes(9, 5, 5, r, W.size, 5) for r in range(2)]
    acc_g, acc_s = None, None
    for G, nz in zip(Gs, noises):
        _, p, c = ogsq.soft_weight(st.logits, nz, st.Ckd, st.scales, W.shape, 64, tau, kappa)
        gl, gsc = ogsq.soft_backward(G.astype(np.float64), p, st.Ckd, c, st.scales, 64, tau, kappa)
        gl, gsc = gl.astype(np.float32), gsc.astype(np.float32)
        acc_g = gl if acc_g is None else acc_g + gl
        acc_s = gsc if acc_s is None else acc_s + gsc
    ogsq.lion_step(st, acc_g / np.float32(2), acc_s / np.float32(2))
    grads = torch.as_tensor(np.stack(Gs), device=DEV)
    P = torch.empty(2, 5, W.size, device=DEV)
    for r in range(2):
        lin.soft(tau, kappa, 5, r, 9, probs=P[r])
    lin.step(P, grads, tau, kappa)
    lg, mm = lin.logits.cpu().numpy(), lin.mom.cpu().numpy()
    # Lion moves by +-lr: a sign decided by rounding differs by 2 lr on a handful of entries
    diff = np.abs(lg - st.logits)
    assert (diff > 1e-7).mean() < 1e-3 and diff.max() <= 2.5e-4
    np.testing.assert_allclose(mm, st.mom_logits, rtol=1e-4, atol=1e-9)
    np.testing.assert_allclose(lin.scales.cpu().numpy(), st.scales, rtol=0, atol=2.5e-4)
    np.testing.assert_allclose(lin.mom_s.cpu().numpy(), st.mom_scales, rtol=1e-4, atol=1e-12)


def test_gradient_matches_reference_oracle_2bit():
    """dL/dlogits and dL/dscales of the reference test oracle (tests/oracles.py:311-347,
    2-bit full grid, 3 resamples), read back through the Lion momentum with lr = 0."""
    import os
    from gsq_rco_mlx_b200.gsq.staged import SoftLinear
    from gsq_rco_mlx_b200.gemm import mm_nt, mm_tn
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "gsq.npz"))
    W, X = z["lg_W"], z["lg_X"].astype(np.float32)
    lin = SoftLinear("q", 2, z["lg_codes"], z["lg_scales"].astype(np.float16), 16, seed=0)
    lin.logits.copy_(torch.as_tensor(np.ascontiguousarray(z["lg_logits"].T), device=DEV))
    lin.scales.copy_(torch.as_tensor(z["lg_scales"], device=DEV))
    tau, kappa = float(z["lg_tau"]), float(z["lg_kappa"])
    noises = torch.as_tensor(np.ascontiguousarray(z["lg_noise"].transpose(0, 2, 1)), device=DEV)
    Xt, Wt = torch.as_tensor(X, device=DEV), torch.as_tensor(W, device=DEV)
    grads = torch.empty(3, *W.shape, device=DEV)
    P = torch.empty(3, 4, W.size, device=DEV)
    loss = 0.0
    for r in range(3):
        D = lin.soft(tau, kappa, 0, r, 0, w_ref=Wt, noise=noises[r].contiguous(),
                     out=torch.empty(W.shape, device=DEV), probs=P[r])
        Rm = mm_nt(Xt, D)
        loss += float((Rm.double() ** 2).mean())
        mm_tn(Rm, Xt, alpha=2.0 / (X.shape[0] * W.shape[0]), out=grads[r])
    lin.step(P, grads, tau, kappa, lr_logits=0.0, lr_scales=0.0)
    g_log = lin.mom.cpu().numpy().T / np.float32(0.05)
    g_sc = lin.mom_s.cpu().numpy() / np.float32(0.05)
    assert abs(loss / 3 - float(z["lg_loss"])) <= 1e-5 * float(z["lg_loss"])
    np.testing.assert_allclose(g_log, z["lg_glog"], rtol=2e-3, atol=2e-4 * np.abs(z["lg_glog"]).max())
    np.testing.assert_allclose(g_sc, z["lg_gscale"], rtol=2e-3, atol=2e-4 * np.abs(z["lg_gscale"]).max())


def test_fused_step_forward_equals_fresh_forward():
    """The next-step forward inside the fused pass equals a separate soft() of the updated
    state: same probabilities and the same bf16 terms."""
    W, lin, st = make_linear()
    rng = np.random.default_rng(8)
    tau, kappa = ogsq.gs_schedules(10, 200)
    tau1, kappa1 = ogsq.gs_schedules(11, 200)
    Wt = torch.as_tensor(W, device=DEV)
    P = torch.empty(2, 5, W.size, device=DEV)
    for r in range(2):
        lin.soft(tau, kappa, 10, r, 4, w_ref=Wt, probs=P[r])
    grads = torch.as_tensor((1e-3 * rng.standard_normal((2,) + W.shape)).astype(np.float32), device=DEV)
    terms = torch.zeros(2, 3, *W.shape, device=DEV, dtype=torch.bfloat16)
    lin.step(P, grads, tau, kappa, nxt={"step": 11, "tau": tau1, "kappa": kappa1, "seed": 4,
                                        "w_ref": Wt, "terms": terms})
    for r in range(2):
        Pf = torch.empty(5, W.size, device=DEV)
        Tf = torch.zeros(3, *W.shape, device=DEV, dtype=torch.bfloat16)
        lin.soft(tau1, kappa1, 11, r, 4, w_ref=Wt, terms=Tf, probs=Pf)
        assert torch.equal(Pf, P[r])
        assert torch.equal(Tf, terms[r])
    # the terms reconstruct w_bar - W to float32 precision
    wf = lin.soft(tau1, kappa1, 11, 0, 4, w_ref=Wt)
    rec = terms[0].float().sum(0)
    assert torch.equal(rec, wf) or (rec - wf).abs().max() <= 1e-7 * wf.abs().max()


def test_harden_matches_oracle():
    W, lin, st = make_linear(bits=3)
    rng = np.random.default_rng(5)
    lg = rng.standard_normal(st.logits.shape).astype(np.float32)
    lg[:, :3] = 0.0  # exact ties: the first maximum wins
    st.logits = lg
    lin.logits.copy_(torch.as_tensor(lg, device=DEV))
    assert np.array_equal(lin.hard_codes(), st.hard_codes())
    W2, lin2, st2 = make_linear(bits=2)
    lg2 = rng.standard_normal(st2.logits.shape).astype(np.float32)
    st2.logits = lg2
    lin2.logits.copy_(torch.as_tensor(lg2, device=DEV))
    assert np.array_equal(lin2.hard_codes(), st2.hard_codes())


def _qk_parity(host_noise: bool):
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, SoftLinear, train_linears
    rng = np.random.default_rng(0)
    out_f, in_f, n_seq, T = 128, 512, 32, 512
    W = (0.02 * rng.standard_normal((out_f, in_f))).astype(np.float32)
    sch = np.exp(rng.standard_normal(in_f)).astype(np.float32)
    X = (rng.standard_normal((n_seq * T, in_f)).astype(np.float32) * sch)
    H, _ = og.hessian_from_inputs(X)
    g = og.quantize_gptq(W, H, 3, 64)
    codes, s16 = g["codes"], g["scales"].astype(np.float16)
    Xs = X.reshape(n_seq, T, in_f)[:, 1:]
    st = ogsq.LinearState(3, codes, s16, 64, seed=0, linear_id=1)
    hist_o = ogsq.train_linear(st, lambda idx: Xs[idx].reshape(-1, in_f), W, n_seq, 200, seed=1,
                               noise_seed=77)
    lin = SoftLinear("q_proj", 3, codes, s16, 64, seed=0, linear_id=1)
    Xd = torch.as_tensor(X.reshape(n_seq, T, in_f), device=DEV)
    noise_of = None
    if host_noise:
        noise_of = lambda t, r, l: torch.as_tensor(gumbel_planes(77, 1, t, r, W.size, 5), device=DEV)
    hist, _ = train_linears([lin], Xd, {"q_proj": torch.as_tensor(W, device=DEV)}, n_seq,
                            BlockOpts(steps=200), seed=1, noise_of=noise_of, noise_seed=77)
    rl = np.linalg.norm(lin.logits.cpu().numpy() - st.logits) / np.linalg.norm(st.logits)
    rs = np.linalg.norm(lin.scales.cpu().numpy() - st.scales) / np.linalg.norm(st.scales)
    rloss = abs(hist[-1] - hist_o[-1]) / hist_o[-1]
    codes_eq = (lin.hard_codes() == st.hard_codes()).mean()
    return rl, rs, rloss, codes_eq


@pytest.mark.parametrize("host_noise", [True, False])
def test_qk_stage_200_steps_parity(host_noise):
    """200 Lion steps of the qk stage, tensor-core contractions, vs the oracle (float64 GEMMs)."""
    rl, rs, rloss, codes_eq = _qk_parity(host_noise)
    print(f"parity: logits {rl:.2e} scales {rs:.2e} loss {rloss:.2e} codes {codes_eq:.6f}")
    assert rl <= 1e-3 and rs <= 1e-3 and rloss <= 1e-3, (rl, rs, rloss)
    assert codes_eq >= 0.999, codes_eq


def test_qk_stage_exact_bf16_rows():
    """Rows that are exactly bf16 (normed block inputs) use one operand term: same result."""
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, SoftLinear, train_linears
    rng = np.random.default_rng(2)
    out_f, in_f, n_seq, T = 64, 256, 8, 129
    W = (0.02 * rng.standard_normal((out_f, in_f))).astype(np.float32)
    X = torch.as_tensor(rng.standard_normal((n_seq, T, in_f)).astype(np.float32)).bfloat16().float()
    r = og.quantize_rtn(W, 3, 64)
    res = []
    for exact in (False, True):
        lin = SoftLinear("k_proj", 3, r["codes"], r["scales"].astype(np.float16), 64, seed=0)
        train_linears([lin], X.to(DEV), {"k_proj": torch.as_tensor(W, device=DEV)}, n_seq,
                      BlockOpts(steps=20), seed=3, exact_bf16_rows=exact)
        res.append(lin.logits.cpu().numpy())
    assert np.linalg.norm(res[0] - res[1]) / np.linalg.norm(res[0]) < 1e-4


@pytest.mark.parametrize("src", ["bf16", "f32"])
@pytest.mark.parametrize("n_terms", [1, 3])
def test_gather_rows_vector_path_equals_tiled_path(src, n_terms):
    """gsq_gather_split with row terms only (the 16-byte row kernel) writes the same bf16 terms
    as the tiled kernel that also writes the transposed copy, and the terms are split3 of the
    gathered rows (positions `offset ..` of the chosen sequences)."""
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.gemm import Terms
    T, N, H, per, off = 64, 5, 96, 40, 3
    g = torch.Generator().manual_seed(n_terms + (src == "f32"))
    x = torch.randn(N * T, H, generator=g) * 0.5
    x = x.bfloat16() if src == "bf16" else x
    xd = x.to(DEV)
    seq = torch.tensor([4, 0, 2], dtype=torch.int32, device=DEV)
    rows = 3 * per
    A, B, BT = Terms(rows, H, n_terms, DEV), Terms(rows, H, n_terms, DEV), Terms(H, rows, n_terms, DEV)
    st = _lib.stream_ptr()
    args = (_lib.ptr(xd), int(src == "bf16"), H, _lib.ptr(seq), per, T, off, rows, H, n_terms)
    _lib.call("gsq_gather_split", *args, A.ptrs(), A.ld, None, 0, st)
    _lib.call("gsq_gather_split", *args, B.ptrs(), B.ld, BT.ptrs(), BT.ld, st)
    torch.cuda.synchronize()
    idx = torch.cat([s * T + off + torch.arange(per) for s in (4, 0, 2)])
    want = x.float()[idx].double()
    got = sum(A.t[i][:, :H].double().cpu() for i in range(n_terms))
    for i in range(n_terms):
        assert torch.equal(A.t[i][:, :H].cpu(), B.t[i][:, :H].cpu())
        assert torch.equal(BT.t[i][:, :rows].cpu(), B.t[i][:, :H].cpu().T)
    tol = 0.0 if (src == "bf16" or n_terms == 3) else 2.0 ** -8
    assert float(((got - want).abs() / want.abs().clamp_min(1e-30)).max()) <= tol
