"""The qk-stage step through the micro-batch Gram matrix: G = 2 D (X^T X) / (M out) and the
loss sum D * (D X^T X) equal the residual form 2 (X D^T)^T X / (M out) and sum (X D^T)^2 of
src/gsq_rco/gsq/staged.py:327-328 (float64 on the CPU), at the q / k shapes of the block."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("x_terms", [1, 3])
def test_gram_step_matches_residual_form(x_terms):
    from gsq_rco_mlx_b200.gsq.staged import LinearStep, SoftLinear
    rng = np.random.default_rng(x_terms)
    M, in_f = 2 * 2047, 896
    lins = []
    for i, out_f in enumerate((896, 128)):
        codes = rng.integers(0, 8, size=(out_f, in_f)).astype(np.uint8)
        s16 = (0.01 + 0.002 * rng.random((out_f, in_f // 64))).astype(np.float16)
        lins.append(SoftLinear(("q_proj", "k_proj")[i], 3, codes, s16, 64, seed=i, linear_id=i))
    X = torch.randn(1, M + 1, in_f, generator=torch.Generator().manual_seed(5))
    if x_terms == 1:
        X = X.bfloat16().float()
    W = {l.name: (0.02 * torch.randn(l.out_f, in_f, generator=torch.Generator().manual_seed(
        7 + i))) for i, l in enumerate(lins)}
    step = LinearStep(lins, M, in_f, 2, x_terms=x_terms)
    Xd = X.to(DEV)
    step.stage(Xd.view(-1, in_f), [0], M, M + 1, 1)
    step.first_forward({k: v.to(DEV) for k, v in W.items()}, 0, 2.0, 100.0, 3)
    step.contract()
    torch.cuda.synchronize()
    Xr = X[0, 1:].double()
    for li, lin in enumerate(lins):
        for r in range(2):
            D = sum(t.double() for t in step.Dbuf[lin.name][r].cpu())   # w_bar - W as terms
            R = Xr @ D.T
            G_ref = 2.0 / (M * lin.out_f) * (R.T @ Xr)
            G = step.grads[lin.name][r].double().cpu()
            rel = float((G - G_ref).norm() / G_ref.norm())
            loss = float(step.loss[li * 2 + r].item())
            loss_ref = float((R * R).sum())
            assert rel < 1e-5, (lin.name, r, rel)
            assert abs(loss - loss_ref) <= 1e-6 * loss_ref, (lin.name, r, loss, loss_ref)


@pytest.mark.parametrize("rows,cols,ld", [(300, 200, 208), (37, 203, 211), (2000, 896, 896)])
def test_dot_terms_matches_float64(rows, cols, ld):
    from gsq_rco_mlx_b200 import _lib
    g = torch.Generator().manual_seed(1)
    x = torch.randn(rows, cols, generator=g)
    t0 = x.bfloat16()
    t1 = (x - t0.float()).bfloat16()
    t2 = (x - t0.float() - t1.float()).bfloat16()
    terms = torch.zeros(3, rows, ld, dtype=torch.bfloat16)
    for i, t in enumerate((t0, t1, t2)):
        terms[i, :, :cols] = t
    G = torch.randn(rows, cols, generator=g)
    td, Gd = terms.to(DEV), G.to(DEV)
    part = torch.zeros(1024, device=DEV, dtype=torch.float64)
    out = torch.zeros(1, device=DEV, dtype=torch.float64)
    _lib.call("gsq_dot_terms", _lib.ptr(td[0]), _lib.ptr(td[1]), _lib.ptr(td[2]), ld,
              _lib.ptr(Gd), cols, rows, cols, 0.5, _lib.ptr(part), _lib.ptr(out),
              _lib.stream_ptr())
    d = (t0.float() + t1.float() + t2.float()).double()
    ref = 0.5 * float((d * G.double()).sum())
    assert abs(float(out.item()) - ref) <= 1e-12 * float((d * G.double()).abs().sum())
