"""Ternary (1-bit) soft weights on the GPU vs the oracle (reference staged.py:87-89, 109-115,
251-253, 305-308): the soft weight from host and Philox Gumbel planes, the fused backward + Lion
+ next forward, the sign decode, and 200 qk-stage Lion steps."""
import numpy as np
import pytest
import torch

from oracle import gptq as og
from oracle import gsq as ogsq
from oracle.philox import gumbel_planes

pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_ternary(out_f=96, in_f=256, gs=64, seed=0):
    from gsq_rco_mlx_b200.gsq.staged import SoftLinear
    rng = np.random.default_rng(seed)
    W = (0.02 * rng.standard_normal((out_f, in_f))).astype(np.float32)
    r = og.quantize_rtn(W, 1, gs)
    s16 = r["scales"].astype(np.float16)
    lin = SoftLinear("up_proj", 1, r["codes"], s16, gs, seed=seed + 3, linear_id=2)
    st = ogsq.LinearState(1, r["codes"], s16, gs, seed=seed + 3, linear_id=2)
    assert np.array_equal(lin.logits.cpu().numpy(), st.logits)
    return W, lin, st


@pytest.mark.parametrize("host_noise", [True, False])
def test_ternary_soft_weight(host_noise):
    W, lin, st = make_ternary()
    # logits spread so that m and v cover the whole (0, 1) range
    lg = (0.3 * np.random.default_rng(1).standard_normal(st.logits.shape)).astype(np.float32)
    st.logits = lg
    lin.logits.copy_(torch.as_tensor(lg, device=DEV))
    for (tau, kappa, step, r) in [(1.5, 4.0, 3, 1), (0.6, 150.0, 17, 0)]:
        noise = gumbel_planes(11, 2, step, r, W.size, 4)
        w_o, p_o, _ = ogsq.soft_weight(st.logits, noise, None, st.scales, W.shape, 64, tau, kappa)
        P = torch.empty(2, W.size, device=DEV)
        nz = torch.as_tensor(noise, device=DEV) if host_noise else None
        got = lin.soft(tau, kappa, step, r, 11, noise=nz, probs=P,
                       out=torch.empty(W.shape, device=DEV)).cpu().numpy()
        s = np.abs(w_o).max()
        np.testing.assert_allclose(got, w_o, rtol=2e-6, atol=2e-6 * s)
        # probabilities to float32 accuracy in absolute terms: the in-kernel Gumbel transform
        # uses the hardware base-2 logarithm, a few ulps from the oracle's, which moves a
        # saturated sigmoid (m ~ 1e-9) by more than its own relative precision
        np.testing.assert_allclose(P.cpu().numpy(), p_o, rtol=2e-6, atol=2e-7)


def test_ternary_step_and_next_forward():
    """One fused step from the stored (m, v) of two draws: Lion on the mask / sign logits and the
    scales against the oracle's gradients; the step's next forward equals a fresh soft()."""
    W, lin, st = make_ternary()
    rng = np.random.default_rng(3)
    tau, kappa = ogsq.gs_schedules(5, 200)
    tau1, kappa1 = ogsq.gs_schedules(6, 200)
    Gs = [(1e-3 * rng.standard_normal(W.shape)).astype(np.float32) for _ in range(2)]
    acc = [None, None]
    P = torch.empty(2, 2, W.size, device=DEV)
    for r, G in enumerate(Gs):
        nz = gumbel_planes(9, 2, 5, r, W.size, 4)
        _, p, c = ogsq.soft_weight(st.logits, nz, None, st.scales, W.shape, 64, tau, kappa)
        ogsq.backward_accumulate(acc, G.astype(np.float64), p, None, c, st.scales, 64, tau, kappa)
        lin.soft(tau, kappa, 5, r, 9, probs=P[r])
    ogsq.lion_step(st, acc[0] / np.float32(2), acc[1] / np.float32(2))
    Wt = torch.as_tensor(W, device=DEV)
    terms = torch.zeros(2, 3, *W.shape, device=DEV, dtype=torch.bfloat16)
    lin.step(P, torch.as_tensor(np.stack(Gs), device=DEV), tau, kappa,
             nxt={"step": 6, "tau": tau1, "kappa": kappa1, "seed": 9, "w_ref": Wt,
                  "terms": terms})
    lg, mm = lin.logits.cpu().numpy(), lin.mom.cpu().numpy()
    diff = np.abs(lg - st.logits)   # a sign decided by rounding moves a logit by 2 lr
    assert (diff > 1e-7).mean() < 1e-3 and diff.max() <= 2.5e-4
    np.testing.assert_allclose(mm, st.mom_logits, rtol=1e-4, atol=1e-9)
    np.testing.assert_allclose(lin.scales.cpu().numpy(), st.scales, rtol=0, atol=2.5e-4)
    np.testing.assert_allclose(lin.mom_s.cpu().numpy(), st.mom_scales, rtol=1e-4, atol=1e-12)
    for r in range(2):
        Pf = torch.empty(2, W.size, device=DEV)
        Tf = torch.zeros(3, *W.shape, device=DEV, dtype=torch.bfloat16)
        lin.soft(tau1, kappa1, 6, r, 9, w_ref=Wt, terms=Tf, probs=Pf)
        assert torch.equal(Pf, P[r]) and torch.equal(Tf, terms[r])


def test_ternary_harden():
    W, lin, st = make_ternary()
    lg = np.random.default_rng(5).standard_normal(st.logits.shape).astype(np.float32)
    lg[:, :4] = 0.0     # zero logits decode as kept / positive (>= 0)
    lg[0, 4:8] = -0.0
    st.logits = lg
    lin.logits.copy_(torch.as_tensor(lg, device=DEV))
    got = lin.hard_codes()
    assert np.array_equal(got, st.hard_codes())
    assert set(np.unique(got)) <= {0, 1, 2}


def test_ternary_qk_stage_200_steps():
    """200 qk-stage Lion steps of a ternary linear (host Gumbel planes) against the oracle,
    held to the oracle's own float32-level spread: GPU-vs-oracle at most 1.5x the distance of
    an oracle run whose weight gradients carry 1e-7 relative jitter (or 1e-3)."""
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, SoftLinear, train_linears
    rng = np.random.default_rng(0)
    out_f, in_f, n_seq, T = 128, 512, 32, 257
    W = (0.02 * rng.standard_normal((out_f, in_f))).astype(np.float32)
    sch = np.exp(rng.standard_normal(in_f)).astype(np.float32)
    X = rng.standard_normal((n_seq * T, in_f)).astype(np.float32) * sch
    H, _ = og.hessian_from_inputs(X)
    g = og.quantize_gptq(W, H, 1, 64)
    codes, s16 = g["codes"], g["scales"].astype(np.float16)
    Xs = X.reshape(n_seq, T, in_f)[:, 1:]
    rows = lambda idx: Xs[idx].reshape(-1, in_f)
    st = ogsq.LinearState(1, codes, s16, 64, seed=0, linear_id=1)
    hist_o = ogsq.train_linear(st, rows, W, n_seq, 200, seed=1, noise_seed=77)
    jit = np.random.default_rng(9)
    st_j = ogsq.LinearState(1, codes, s16, 64, seed=0, linear_id=1)
    hist_j = ogsq.train_linear(st_j, rows, W, n_seq, 200, seed=1, noise_seed=77,
                               perturb=lambda G: G * (1 + 1e-7 * jit.standard_normal(G.shape)))
    lin = SoftLinear("q_proj", 1, codes, s16, 64, seed=0, linear_id=1)
    noise_of = lambda t, r, l: torch.as_tensor(gumbel_planes(77, 1, t, r, W.size, 4), device=DEV)
    hist, _ = train_linears([lin], torch.as_tensor(X.reshape(n_seq, T, in_f), device=DEV),
                            {"q_proj": torch.as_tensor(W, device=DEV)}, n_seq,
                            BlockOpts(steps=200), seed=1, noise_of=noise_of, noise_seed=77)
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))
    g_ = (rel(lin.logits.cpu().numpy(), st.logits), rel(lin.scales.cpu().numpy(), st.scales),
          abs(hist[-1] - hist_o[-1]) / hist_o[-1], 1 - (lin.hard_codes() == st.hard_codes()).mean())
    j_ = (rel(st_j.logits, st.logits), rel(st_j.scales, st.scales),
          abs(hist_j[-1] - hist_o[-1]) / hist_o[-1], 1 - (st_j.hard_codes() == st.hard_codes()).mean())
    print(f"ternary qk: GPU logits {g_[0]:.2e} scales {g_[1]:.2e} loss {g_[2]:.2e} codes "
          f"{1 - g_[3]:.6f} | jittered oracle {j_[0]:.2e} {j_[1]:.2e} {j_[2]:.2e} {1 - j_[3]:.6f}")
    for a, b in zip(g_, j_):
        assert a <= max(1e-3, 1.5 * b), (g_, j_)
