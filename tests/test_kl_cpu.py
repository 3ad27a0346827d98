"""The KL-head oracle (evaluate.py:111-151 restated): its logit gradient q - p is the gradient
of the row KL (float64 autograd without the bf16 roundings), and the dots oracle on a
hand-checked case."""
import numpy as np
import torch

from oracle import kl as okl


def test_kl_gradient_is_q_minus_p_times_E():
    g = torch.Generator().manual_seed(0)
    E = torch.randn(40, 8, generator=g, dtype=torch.float64)
    hq = torch.randn(5, 8, generator=g, dtype=torch.float64, requires_grad=True)
    hr = torch.randn(5, 8, generator=g, dtype=torch.float64)
    lq = torch.log_softmax(hq @ E.T, -1)
    lr = torch.log_softmax(hr @ E.T, -1)
    kl = (lr.exp() * (lr - lq)).sum()
    kl.backward()
    q, p = lq.exp(), lr.exp()
    assert torch.allclose(hq.grad, (q - p).detach() @ E, atol=1e-12)


def test_ste_dots_small_case():
    G = np.array([[1.0, 2.0, -1.0, 0.5]], dtype=np.float32)
    W = np.array([[0.0, 0.25, -0.5, 1.0]], dtype=np.float32)
    codes = np.array([[2, 3, 0, 1]], dtype=np.uint8)       # 2-bit grid [-2, -1, 0, 1]
    scales = np.array([[0.5]], dtype=np.float32)
    # wq = [0, 0.5, -1, -0.5]; wq - W = [0, 0.25, -0.5, -1.5]
    want = 1.0 * 0 + 2.0 * 0.25 + (-1.0) * (-0.5) + 0.5 * (-1.5)
    got = okl.ste_dots(G, W, [(codes, scales, 2)], group_size=4)
    assert abs(got[0] - want) < 1e-12
