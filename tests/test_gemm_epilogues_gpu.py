"""Batched / causal / fused-epilogue forms of the tensor-core GEMM (gsq_gemm) against float64
torch references of the same float32 operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def terms_of(x, n=3):
    from gsq_rco_mlx_b200.gemm import Terms, split_into
    return split_into(x.contiguous(), Terms(x.shape[0], x.shape[1], n))


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


def check():
    from gsq_rco_mlx_b200.gemm import check_err
    torch.cuda.synchronize()
    check_err(torch.device(DEV))


def test_batched_affine_offsets_bn64():
    """28 (head, sequence) products P_h V_kv(h) with 7 heads per kv head, N = 64 tiles."""
    from gsq_rco_mlx_b200.gemm import Terms, gemm
    torch.manual_seed(0)
    S, Hq, Hkv, T, D = 2, 14, 2, 256, 64
    P = torch.randn(S * Hq * T, T, device=DEV).bfloat16().float()  # one exact term
    V = torch.randn(S * Hkv * D, T, device=DEV)          # V^T per (seq, kv head): [64, T]
    Pt, Vt = terms_of(P, 1), terms_of(V)
    out = torch.zeros(S * Hq * T, D, device=DEV)
    # batch z = s * 14 + h: A rows z * T; B rows (z // 7) * 64; C offset z * T * D
    gemm(Pt, Vt, M=T, N=D, K=T, batch=S * Hq, bn=64, C=out, ldc=D,
         a_off=(1, T, 0), b_off=(7, D, 0), c_off=(1, T * D, 0))
    check()
    ref = torch.empty_like(out, dtype=torch.float64)
    for z in range(S * Hq):
        ref[z * T:(z + 1) * T] = P[z * T:(z + 1) * T].double() @ V[(z // 7) * D:(z // 7 + 1) * D].double().T
    assert rel(out, ref) < 2e-6


def test_causal_skips_upper_blocks():
    from gsq_rco_mlx_b200.gemm import gemm
    torch.manual_seed(1)
    T, N = 1024, 192
    P = torch.tril(torch.rand(T, T, device=DEV)).bfloat16().float()
    B = torch.randn(N, T, device=DEV)
    out = torch.zeros(T, N, device=DEV)
    gemm(terms_of(P, 1), terms_of(B), C=out, causal=True)
    check()
    assert rel(out, P.double() @ B.double().T) < 2e-6


def test_residual_loss_epilogue():
    """r = acc + bias + resid - target, per-tile sum r^2, out_scale r as C, row and
    transposed terms."""
    from gsq_rco_mlx_b200.gemm import Terms, gemm
    torch.manual_seed(2)
    M, N, K = 300, 256, 192
    A, B = torch.randn(M, K, device=DEV), torch.randn(N, K, device=DEV)
    bias = torch.randn(N, device=DEV)
    resid = torch.randn(M, N, device=DEV).bfloat16()
    target = torch.randn(M, N, device=DEV).bfloat16()
    tiles = 3 * 2
    sq = torch.zeros(tiles, device=DEV, dtype=torch.float64)
    C = torch.empty(M, N, device=DEV)
    cs, ct = Terms(M, N), Terms(N, M)
    gemm(terms_of(A), terms_of(B), C=C, bias=bias, resid=resid, target=target, epi=1,
         out_scale=0.25, sq_partial=sq, c_terms=cs, ct_terms=ct)
    check()
    r = A.double() @ B.double().T + bias.double() + resid.double() - target.double()
    assert abs(sq.sum().item() - (r ** 2).sum().item()) <= 2e-6 * (r ** 2).sum().item()
    assert rel(C, 0.25 * r) < 2e-6
    assert torch.equal(cs.value(), C) and torch.equal(ct.value(), C.T)


def _silu(g):
    return g * torch.sigmoid(g)


def test_swiglu_forward_and_backward_epilogues():
    from gsq_rco_mlx_b200.gemm import Terms, gemm
    torch.manual_seed(3)
    M, W, K = 260, 384, 256      # W = intermediate width (gate/up rows each)
    X = torch.randn(M, K, device=DEV).bfloat16().float()   # exactly bf16 rows (normed input)
    Wg, Wu = 0.05 * torch.randn(W, K, device=DEV), 0.05 * torch.randn(W, K, device=DEV)
    g_out = torch.empty(M, W, device=DEV)
    u_out = torch.empty(M, W, device=DEV)
    d_row, d_t = Terms(M, W), Terms(W, M)
    gemm(terms_of(X, 1), terms_of(Wg), B2=terms_of(Wu), epi=2, aux0=g_out, aux1=u_out,
         c_terms=d_row, ct_terms=d_t)
    check()
    g_ref = X.double() @ Wg.double().T
    u_ref = X.double() @ Wu.double().T
    assert rel(g_out, g_ref) < 2e-6 and rel(u_out, u_ref) < 2e-6
    d_ref = _silu(g_out.double()) * u_out.double()
    assert rel(d_row.value(), d_ref) < 1e-6
    assert torch.equal(d_t.value(), d_row.value().T)
    # backward: dd = dR w_down, with the gate/up stored above
    Nout = 128
    dR = torch.randn(M, Nout, device=DEV)
    Wd = 0.05 * torch.randn(Nout, W, device=DEV)
    grads_t = Terms(2 * W, M)
    gemm(terms_of(dR), terms_of(Wd.T.contiguous()), epi=3, aux0=g_out, aux1=u_out,
         ct_terms=grads_t, ct_up_rows=W)
    check()
    dd = dR.double() @ Wd.double()
    g, u = g_out.double().requires_grad_(), u_out.double().requires_grad_()
    (_silu(g) * u * dd).sum().backward()
    got = grads_t.value()
    assert rel(got[:W].T, g.grad) < 2e-6
    assert rel(got[W:].T, u.grad) < 2e-6


@pytest.mark.parametrize("M,N,K,splits,bn", [(896, 896, 4094, 6, 128), (128, 896, 4094, 21, 128),
                                             (200, 130, 1000, 3, 64)])
def test_split_k_matches_single_pass(M, N, K, splits, bn):
    """Weight-gradient shapes (few output tiles, long k): split-K partials summed in part order,
    alpha / beta applied once, within the float32-faithful bound of the single-pass GEMM."""
    from gsq_rco_mlx_b200.gemm import gemm
    torch.manual_seed(7)
    A, B = torch.randn(M, K, device=DEV), torch.randn(N, K, device=DEV)
    C0 = torch.randn(M, N, device=DEV)
    one, many = C0.clone(), C0.clone()
    gemm(terms_of(A), terms_of(B), C=one, alpha=0.5, beta=2.0, bn=bn, split_k=1)
    gemm(terms_of(A), terms_of(B), C=many, alpha=0.5, beta=2.0, bn=bn, split_k=splits)
    check()
    ref = 0.5 * (A.double() @ B.double().T) + 2.0 * C0.double()
    assert rel(one, ref) < 2e-6 and rel(many, ref) < 2e-6
    # deterministic: a second run gives the same bits
    again = C0.clone()
    gemm(terms_of(A), terms_of(B), C=again, alpha=0.5, beta=2.0, bn=bn, split_k=splits)
    check()
    assert torch.equal(again, many)


def test_auto_split_policy():
    from gsq_rco_mlx_b200.gemm import auto_split
    assert auto_split(896, 896, 4094) > 1        # 49 tiles
    assert auto_split(128, 896, 4094) > 1        # 7 tiles
    assert auto_split(4096, 4864, 896) == 1      # 1216 tiles


def test_swiglu_backward_bn64_equals_bn128():
    """The SwiGLU-backward epilogue on 128 x 64 tiles (more TMEM chunk slots ahead of the
    epilogue) writes the same [dg | du] row terms as on 128 x 128 tiles, bit for bit: each
    output element is folded from the same k-block chunks in the same order."""
    from gsq_rco_mlx_b200.gemm import Terms, gemm
    torch.manual_seed(3)
    M, W, Nout = 700, 384, 256
    g_in = torch.randn(M, W, device=DEV)
    u_in = torch.randn(M, W, device=DEV)
    dR = torch.randn(M, Nout, device=DEV)
    Wd = 0.05 * torch.randn(Nout, W, device=DEV)
    outs = []
    for bn in (128, 64):
        rows = Terms(M, 2 * W)
        gemm(terms_of(dR), terms_of(Wd.T.contiguous()), epi=3, aux0=g_in, aux1=u_in,
             c_terms=rows, ct_up_rows=W, bn=bn)
        check()
        outs.append([t.clone() for t in rows.t])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_plan_runs_equal_single_calls():
    """A GemmPlan (checks and tensor maps built once) run twice gives the bits of gemm() on the
    same operands, also when the operands' contents change between runs."""
    from gsq_rco_mlx_b200.gemm import GemmPlan, gemm
    torch.manual_seed(5)
    M, N, K = 300, 260, 1000
    A, B = torch.randn(M, K, device=DEV), torch.randn(N, K, device=DEV)
    At, Bt = terms_of(A), terms_of(B)
    ref, got = torch.zeros(M, N, device=DEV), torch.zeros(M, N, device=DEV)
    plan = GemmPlan(At, Bt, C=got, alpha=0.5)
    for _ in range(2):
        gemm(At, Bt, C=ref, alpha=0.5)
        plan.run()
        check()
        assert torch.equal(ref, got)
        A2 = torch.randn(M, K, device=DEV)
        for dst, src in zip(At.t, terms_of(A2).t):
            dst.copy_(src)


@pytest.mark.parametrize("bn", [64, 128])
def test_one_small_accumulator_equals_two(bn):
    """One TMEM accumulator for the cross products (and one more hi x hi chunk slot) gives the
    bits of two: the same products are folded in the same order. 256+ tiles, so every CTA
    reuses the single accumulator."""
    from gsq_rco_mlx_b200.gemm import Terms, gemm
    torch.manual_seed(9)
    M, N, K = 4096, 1024, 896
    A, B = torch.randn(M, K, device=DEV), torch.randn(N, K, device=DEV)
    R = torch.randn(M, N, device=DEV).bfloat16()
    Tg = (R.float() + 1e-3 * torch.randn(M, N, device=DEV)).bfloat16()
    outs = []
    for sb in (2, 1):
        C = torch.zeros(M, N, device=DEV)
        rows = Terms(M, N)
        sq = torch.zeros((M // 128) * (N // 128), device=DEV, dtype=torch.float64)
        gemm(terms_of(A), terms_of(B), C=C, bn=bn, small_bufs=sb)
        gemm(terms_of(A), terms_of(B), epi=1, resid=R, target=Tg, out_scale=0.5, sq_partial=sq,
             c_terms=rows, bn=bn, small_bufs=sb)
        check()
        outs.append((C, [t.clone() for t in rows.t], sq.clone()))
    (c2, r2, s2), (c1, r1, s1) = outs
    assert torch.equal(c1, c2) and torch.equal(s1, s2)
    for a, b in zip(r1, r2):
        assert torch.equal(a, b)
