"""Tensor-core split-bf16 GEMM (tcgen05) vs float64 matmul: float32-level accuracy with
three terms per side, bf16 accuracy with one; epilogue outputs (C, C terms, C^T terms,
per-tile sum of squares); ragged and padded shapes."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def run(M, N, K, na, nb, seed=0, alpha=1.0, scale_b=1.0):
    from gsq_rco_mlx_b200.gemm import Terms, check_err, gemm_tc, split_into
    g = torch.Generator(device="cpu").manual_seed(seed)
    A = torch.randn(M, K, generator=g, dtype=torch.float64)
    B = torch.randn(N, K, generator=g, dtype=torch.float64) * scale_b
    Ad, Bd = A.float().to(DEV), B.float().to(DEV)
    At, Bt = Terms(M, K, 3), Terms(N, K, 3)
    split_into(Ad, At)
    split_into(Bd, Bt)
    C = torch.empty(M, N, device=DEV)
    gemm_tc(At, Bt, na=na, nb=nb, alpha=alpha, C=C)
    torch.cuda.synchronize()
    check_err(torch.device(DEV))
    # reference on the same float32-rounded operands, each cut to the terms used
    Ar = sum(t[:, :K].double() for t in At.t[:na]).cpu()
    Br = sum(t[:, :K].double() for t in Bt.t[:nb]).cpu()
    ref = alpha * (Ar @ Br.T)
    return C.double().cpu(), ref, Ad.double().cpu() @ Bd.double().cpu().T * alpha


def test_gemm_tc_single_tile_exact_bf16():
    """1 term per side, one 128 x 128 x 64 tile: exact bf16 products, fp32 accumulation."""
    C, ref, _ = run(128, 128, 64, 1, 1)
    err = (C - ref).abs().max() / ref.abs().max()
    assert err < 1e-6, err


@pytest.mark.parametrize("shape", [(128, 128, 256), (300, 200, 100), (1022, 640, 896),
                                   (96, 4864, 1022)])
def test_gemm_tc_fp32_faithful(shape):
    """Three terms per side: the error against the float64 product of the float32 operands
    stays at the level of a float32 GEMM (cuBLAS SGEMM, TF32 off, on the same operands)."""
    M, N, K = shape
    C, ref, full = run(M, N, K, 3, 3, seed=M)
    g = torch.Generator(device="cpu").manual_seed(M)
    A = torch.randn(M, K, generator=g, dtype=torch.float64).float().to(DEV)
    B = torch.randn(N, K, generator=g, dtype=torch.float64).float().to(DEV)
    torch.backends.cuda.matmul.allow_tf32 = False
    sg = (A @ B.T).double().cpu()
    err_ours = ((C - full).norm() / full.norm()).item()
    err_sgemm = ((sg - full).norm() / full.norm()).item()
    assert err_ours <= 4 * err_sgemm + 1e-9, (err_ours, err_sgemm)
    assert err_ours < 2e-6, err_ours


def test_gemm_tc_epilogue_outputs():
    from gsq_rco_mlx_b200.gemm import Terms, check_err, gemm_tc, split_into
    M, N, K = 515, 260, 200
    torch.manual_seed(0)
    A = torch.randn(M, K, device=DEV)
    B = torch.randn(N, K, device=DEV)
    At, Bt = split_into(A, Terms(M, K)), split_into(B, Terms(N, K))
    C = torch.empty(M, N, device=DEV)
    cs, ct = Terms(M, N), Terms(N, M)
    tiles = ((M + 127) // 128) * ((N + 127) // 128)
    sq = torch.zeros(tiles, device=DEV, dtype=torch.float64)
    gemm_tc(At, Bt, alpha=0.5, C=C, c_terms=cs, ct_terms=ct, sq_partial=sq)
    torch.cuda.synchronize()
    check_err(torch.device(DEV))
    ref = 0.5 * (A.double() @ B.double().T)
    assert ((C.double() - ref).norm() / ref.norm()).item() < 2e-6
    assert torch.equal(cs.value(), C)
    assert torch.equal(ct.value(), C.T)
    assert abs(sq.sum().item() - (C.double() ** 2).sum().item()) <= 1e-9 * (C.double() ** 2).sum().item()
    # beta accumulation into C
    C2 = C.clone()
    gemm_tc(At, Bt, alpha=0.5, C=C2, beta=1.0)
    torch.cuda.synchronize()
    assert ((C2.double() - 2 * ref).norm() / ref.norm()).item() < 2e-6


def test_gemm_tc_exact_operand_three_products():
    """An exactly-bf16 A (one term) against a three-term B: float32-level result."""
    from gsq_rco_mlx_b200.gemm import Terms, gemm_tc, split_into
    M, N, K = 1022, 384, 896
    torch.manual_seed(1)
    A = torch.randn(M, K, device=DEV).bfloat16().float()
    B = torch.randn(N, K, device=DEV)
    At, Bt = split_into(A, Terms(M, K, 1)), split_into(B, Terms(N, K))
    C = torch.empty(M, N, device=DEV)
    gemm_tc(At, Bt, C=C)
    ref = A.double() @ B.double().T
    assert ((C.double() - ref).norm() / ref.norm()).item() < 2e-6


@pytest.mark.parametrize("terms", [(1, 1), (3, 3), (1, 3)])
@pytest.mark.parametrize("majors", [(1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("shape,bn", [((300, 200, 100), 128), ((256, 320, 640), 128),
                                      ((200, 96, 1000), 64)])
def test_mn_major_operands_equal_k_major(terms, majors, shape, bn):
    """An MN-major operand (a row-major [K][M] / [K][N] matrix read as its own transpose) gives
    bit-for-bit the product of the K-major copy: same products, same accumulation order."""
    from gsq_rco_mlx_b200.gemm import Terms, gemm, check_err
    M, N, K = shape
    na, nb = terms
    g = torch.Generator(device="cuda").manual_seed(M + N + K + 7 * na + nb)

    def pair(rows, cols, n):
        km = Terms(rows, cols, n, "cuda")
        mn = Terms(cols, rows, n, "cuda")
        for i in range(n):
            x = (torch.randn(rows, cols, device="cuda", generator=g) * 2.0 ** (-8 * i)).bfloat16()
            km.t[i][:, :cols] = x
            mn.t[i][:, :rows] = x.T
        return km, mn
    A, Amn = pair(M, K, na)
    B, Bmn = pair(N, K, nb)
    ref = torch.empty(M, N, device="cuda")
    out = torch.empty(M, N, device="cuda")
    gemm(A, B, C=ref, bn=bn, split_k=1)
    am, bm = majors
    gemm(Amn if am else A, Bmn if bm else B, M=M, N=N, K=K, C=out, bn=bn, split_k=1,
         a_major=am, b_major=bm)
    torch.cuda.synchronize()
    check_err(torch.device("cuda"))
    assert torch.equal(out, ref)


@pytest.mark.parametrize("causal", [0, 2])
def test_mn_major_batched_a_equals_k_major(causal):
    """A batched MN-major A (each batch's rows at a_off along K), with and without the causal
    k-range, gives bit-for-bit the product of its K-major transposed copy: the vo stage's
    dV = P^T dO reading P directly. K not a multiple of 64 is refused for a batched MN-major A."""
    from gsq_rco_mlx_b200.gemm import Terms, gemm, check_err
    B, T, hd = 3, 256, 64
    g = torch.Generator(device="cuda").manual_seed(11 + causal)
    P, PT = Terms(B * T, T, 1, "cuda"), Terms(B * T, T, 1, "cuda")
    x = torch.randn(B, T, T, device="cuda", generator=g).bfloat16()
    P.t[0][:, :T] = x.reshape(B * T, T)
    PT.t[0][:, :T] = x.transpose(1, 2).reshape(B * T, T)
    D = Terms(B * hd, T, 3, "cuda")
    for i in range(3):
        D.t[i][:, :T] = (torch.randn(B * hd, T, device="cuda", generator=g)
                         * 2.0 ** (-8 * i)).bfloat16()
    ref = torch.empty(B, T, hd, device="cuda")
    out = torch.empty(B, T, hd, device="cuda")
    kw = dict(M=T, N=hd, K=T, batch=B, bn=64, causal=causal, a_off=(1, T, 0),
              b_off=(1, hd, 0), ldc=hd, c_off=(1, T * hd, 0))
    gemm(PT, D, C=ref, **kw)
    gemm(P, D, C=out, a_major=1, **kw)
    torch.cuda.synchronize()
    check_err(torch.device("cuda"))
    assert torch.equal(out, ref)
    kw["K"] = T - 32
    with pytest.raises(ValueError):
        gemm(P, D, C=out, a_major=1, **kw)
