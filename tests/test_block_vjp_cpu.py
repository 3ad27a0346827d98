"""The block-vjp oracle (oracle/block_vjp.py): its forward is oracle.block.block_hard bit for bit,
and without the bf16 roundings its explicit backward equals float64 autograd of the same smooth
function (the check of the formulas: RMSNorm, SwiGLU, causal softmax, RoPE, GQA sums)."""
import torch

from oracle import block as ob
from oracle import block_vjp as ov

F64 = torch.float64


def small(seed=0, H=128, nh=2, nkv=1, inter=256):
    g = torch.Generator().manual_seed(seed)
    hd = 64
    def w(*s):
        return (0.05 * torch.randn(*s, generator=g)).bfloat16()
    return {"q_proj": w(nh * hd, H), "k_proj": w(nkv * hd, H), "v_proj": w(nkv * hd, H),
            "o_proj": w(H, nh * hd), "gate_proj": w(inter, H), "up_proj": w(inter, H),
            "down_proj": w(H, inter), "q_bias": w(nh * hd), "k_bias": w(nkv * hd),
            "v_bias": w(nkv * hd), "in_norm": (1 + 0.1 * torch.randn(H, generator=g)).bfloat16(),
            "post_norm": (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()}


def test_forward_keep_is_block_hard():
    W = small(1)
    h = torch.randn(24, 128, generator=torch.Generator().manual_seed(2)).bfloat16().float()
    out, _ = ob.block_hard(h, W, 2, 1)
    out2, _ = ov.forward_keep(h, W, 2, 1)
    assert torch.equal(out, out2)


def _smooth(h, Wt, nh, nkv, eps=1e-6):
    """The block without roundings, float64, differentiable in h and the weights."""
    T, H = h.shape
    hd = Wt["q_proj"].shape[0] // nh
    def rms(x, w):
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w
    hn = rms(h, Wt["in_norm"])
    q = hn @ Wt["q_proj"].T + Wt["q_bias"]
    k = hn @ Wt["k_proj"].T + Wt["k_bias"]
    v = hn @ Wt["v_proj"].T + Wt["v_bias"]
    cos, sin = ob.rope_tables(T, hd)
    c, s = torch.as_tensor(cos, dtype=F64), torch.as_tensor(sin, dtype=F64)
    def rope(x):
        x1, x2 = x[..., :hd // 2], x[..., hd // 2:]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], -1)
    qr = rope(q.view(T, nh, hd).transpose(0, 1))
    kr = rope(k.view(T, nkv, hd).transpose(0, 1)).repeat_interleave(nh // nkv, 0)
    vv = v.view(T, nkv, hd).transpose(0, 1).repeat_interleave(nh // nkv, 0)
    S = (qr @ kr.transpose(1, 2)) * 0.125
    S = S.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), -torch.inf)
    o = (torch.softmax(S, -1) @ vv).transpose(0, 1).reshape(T, nh * hd)
    h1 = h + o @ Wt["o_proj"].T
    mn = rms(h1, Wt["post_norm"])
    g, u = mn @ Wt["gate_proj"].T, mn @ Wt["up_proj"].T
    return h1 + (g * torch.sigmoid(g) * u) @ Wt["down_proj"].T


def test_explicit_backward_equals_autograd_without_rounding():
    nh, nkv = 2, 1
    W = small(3, nh=nh, nkv=nkv)
    gen = torch.Generator().manual_seed(4)
    h = torch.randn(20, 128, generator=gen, dtype=F64)
    cot = torch.randn(20, 128, generator=gen, dtype=F64)
    Wt = {k: v.to(F64).clone().requires_grad_(True) for k, v in W.items()}
    hh = h.clone().requires_grad_(True)
    (_smooth(hh, Wt, nh, nkv) * cot).sum().backward()
    dh, grads = ov.block_vjp(h.float(), {k: v.float() for k, v in W.items()}, cot.float(),
                             nh, nkv, rounding=False)
    # float32 forward values in the oracle: agreement to float32 accuracy
    assert float((dh.double() - hh.grad).norm() / hh.grad.norm()) < 1e-5
    for name, G in grads.items():
        ref = Wt[name].grad
        assert float((G.double() - ref).norm() / ref.norm()) < 1e-5, name
