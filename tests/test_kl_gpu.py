"""The RCO KL head (tied-embedding logits, KL(p_ref || p_q) and its gradient) and the
straight-through dots on the GPU against the CPU restatement (oracle/kl.py)."""
import numpy as np
import pytest
import torch

from oracle import kl as okl

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(V, n, H=896, seed=0):
    g = torch.Generator().manual_seed(seed)
    E = (0.02 * torch.randn(V, H, generator=g)).bfloat16()
    hr = torch.randn(n, H, generator=g).bfloat16()
    hq = (hr.float() + 0.1 * torch.randn(n, H, generator=g)).bfloat16()
    return E, hq, hr


@pytest.mark.parametrize("V,n,chunk", [(4096, 300, 128), (151936, 40, 32)])
def test_kl_head_matches_oracle(V, n, chunk):
    from gsq_rco_mlx_b200.rco.kl import KLHead, kl_value_and_grad_hidden
    E, hq, hr = _case(V, n)
    head = KLHead(E.to(DEV), chunk=chunk)
    kl, grad = kl_value_and_grad_hidden(head, hq.to(DEV), hr.to(DEV))
    kl_o, grad_o = okl.kl_value_and_grad_hidden(hq.double(), hr.double(), E.double())
    assert abs(kl - kl_o) <= 1e-4 * abs(kl_o), (kl, kl_o)
    gg = grad.double().cpu()
    rel = float((gg - grad_o).norm() / grad_o.norm())
    assert rel < 1e-2, rel
    # bf16(D E) after bf16(q - p): float32 vs float64 accumulation flips the last bit of a few
    # percent of the elements
    assert float((gg == grad_o).double().mean()) >= 0.90


def test_kl_head_c_entry_equals_python_head():
    """kl_head_fwd_bwd (the KL head as one C-ABI call) against the Python KL head on the same
    inputs: the same launches in the same order, so the same bits."""
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.gemm import err_flag
    from gsq_rco_mlx_b200.rco.kl import KLHead
    V, n, chunk, H = 4096, 300, 128, 896
    E, hq, hr = _case(V, n, H, seed=4)
    head = KLHead(E.to(DEV), chunk=chunk)
    hq, hr = hq.to(DEV), hr.to(DEV)
    total, grad = head.kl_sum_and_grad(hq, hr)
    zq = torch.empty(chunk, V, device=DEV, dtype=torch.bfloat16)
    zr, D = torch.empty_like(zq), torch.empty_like(zq)
    rows = torch.empty(n, device=DEV, dtype=torch.float64)
    total_c = torch.empty(1, device=DEV, dtype=torch.float64)
    grad_c = torch.empty(n, H, device=DEV, dtype=torch.bfloat16)
    err = err_flag(torch.device(DEV))
    _lib.call("kl_head_fwd_bwd", _lib.ptr(hq), _lib.ptr(hr), n, H, _lib.ptr(head.E),
              _lib.ptr(head.ET.t[0]), head.ET.ld, V, chunk, _lib.ptr(zq), _lib.ptr(zr),
              _lib.ptr(D), _lib.ptr(rows), _lib.ptr(total_c), _lib.ptr(grad_c), _lib.ptr(err),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(total_c, total) and torch.equal(grad_c, grad)


def test_ste_dots_matches_oracle():
    from gsq_rco_mlx_b200.rco.kl import ste_dots
    rng = np.random.default_rng(3)
    out_f, in_f = 896, 4864
    G = rng.standard_normal((out_f, in_f)).astype(np.float32) * 1e-3
    W = torch.as_tensor(0.02 * rng.standard_normal((out_f, in_f)), dtype=torch.float32).bfloat16()
    cands = []
    for bits in (2, 3, 4):
        codes = rng.integers(0, 2 ** bits, size=(out_f, in_f)).astype(np.uint8)
        scales = (0.01 * rng.random((out_f, in_f // 64))).astype(np.float32)
        cands.append((codes, scales, bits))
    got = ste_dots(torch.as_tensor(G, device=DEV), W.to(DEV),
                   [(torch.as_tensor(c, device=DEV), torch.as_tensor(s, device=DEV), b)
                    for c, s, b in cands]).cpu().numpy()
    want = okl.ste_dots(G, W.float().numpy(), cands)
    assert np.allclose(got, want, rtol=1e-9, atol=0), (got, want)
