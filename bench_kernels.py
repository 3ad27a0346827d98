"""Representative launches of the hot kernels at Qwen2.5-0.5B block shapes, for profilers and
micro-timing (one process, one GPU, a few GB of device memory).

  python bench.py --workload kernels --cases mlp_gemms,attn,... [--once]
  (cases: mlp_gemms, attn, attn1, soft_step, cublas, packed, eval_batch)

--once runs every case a single time (an ncu capture: `-k regex:<kernel> -c <n>`); otherwise
each case is timed with CUDA events over 10 launches after 3 warm-up launches and printed with
its executed bf16 TFLOP/s (GEMMs) or algorithmic GB/s (streams).

mlp_gemms: the six GEMMs of one mlp-stage resample (micro-batch 2 x 2047 rows) and the hard
  SwiGLU GEMM of the block forward (8 x 2048 rows):
    F1 gate|up = mn [Wg|Wu]^T (1 x 3 terms, SwiGLU epilogue)   F3 residual loss (3 x 3)
    B1 dL/dWd (3 x 3, MN-major operands)   B2 SwiGLU backward (3 x 3, MN-major weight)
    B3 dL/dWg, dL/dWu (3 x 1, two MN-major launches)
attn: the causal scores GEMM and softmax of 8 sequences x 14 heads x 2048 positions (attn1: one
  sequence, 235 MB of scores: the profiler-sized case).
soft_step: the fused backward + Lion + next forward of one up_proj-shaped soft linear (R = 2).
cublas: library bf16 GEMMs of the mlp shapes, for context only (not on any product path).
packed: the packed-weight dequant of one layer and the fused dequant-GEMV (HBM streams).
eval_batch: one 8-window batch of the packed 24-layer eval (forward, head, NLL rows).
"""
from __future__ import annotations

import sys

import torch

from gsq_rco_mlx_b200 import _lib
from gsq_rco_mlx_b200.gemm import Terms, check_err, gemm
from gsq_rco_mlx_b200.gsq.staged import _col_terms

H, I, HEADS, KV, HD, T = 896, 4864, 14, 2, 64, 2048


class Bytes(int):
    """A case's algorithmic byte count (printed as GB/s), where other cases give FLOPs."""


def _terms(rows, cols, n, dev, g):
    t = Terms(rows, cols, n, dev)
    for i, x in enumerate(t.t):
        x.copy_((torch.randn(x.shape, device=dev, generator=g) * (0.05 * 2.0 ** (-8 * i)))
                .bfloat16())
    return t


def mlp_gemms(dev, g):
    """The six GEMMs of one resample of the mlp stage step (one micro-batch of 2 x 2047
    positions) as the stage runs them, plus the hard (bf16) SwiGLU forward of 8 sequences: F1
    SwiGLU forward, F3 residual loss, B1 dWd, B2 SwiGLU backward, B3 dWg / dWu (the weight
    gradients read row-major activations as MN-major operands)."""
    M = 2 * (T - 1)
    MN, H1, Y = _terms(M, H, 1, dev, g), _terms(M, H, 1, dev, g), _terms(M, H, 1, dev, g)
    Dg, Du, Dd = _terms(I, H, 3, dev, g), _terms(I, H, 3, dev, g), _terms(H, I, 3, dev, g)
    gg, uu = torch.empty(M, I, device=dev), torch.empty(M, I, device=dev)
    DIN, DR = Terms(M, I, 3, dev), Terms(M, H, 3, dev)
    DGU = Terms(M, 2 * I, 3, dev)
    DG, DU = _col_terms(DGU, 0, I), _col_terms(DGU, I, I)
    grad_gu, grad_d = torch.empty(2, I, H, device=dev), torch.empty(H, I, device=dev)
    sq = torch.zeros(((M + 127) // 128) * 7, device=dev, dtype=torch.float64)
    R = 8 * T
    MNt = _terms(R, H, 1, dev, g)
    Wg1, Wu1 = _terms(I, H, 1, dev, g), _terms(I, H, 1, dev, g)
    d_in = torch.empty(R, I, device=dev, dtype=torch.bfloat16)

    def b3():
        gemm(DG, MN, C=grad_gu[0], ldc=H, a_major=1, b_major=1)
        gemm(DU, MN, C=grad_gu[1], ldc=H, a_major=1, b_major=1)
    return {
        "F1 swiglu fwd (1x3)": (3 * 2 * M * 2 * I * H, lambda: gemm(
            MN, Dg, B2=Du, epi=2, aux0=gg, aux1=uu, c_terms=DIN)),
        "F3 resid (3x3)": (6 * 2 * M * H * I, lambda: gemm(
            DIN, Dd, epi=1, resid=H1.t[0], target=Y.t[0], ld_rt=H1.ld, out_scale=1e-3,
            sq_partial=sq, c_terms=DR)),
        "B1 gradWd (3x3, MN-major)": (6 * 2 * H * I * M, lambda: gemm(
            DR, DIN, C=grad_d, a_major=1, b_major=1)),
        "B2 swiglu bwd (3x3)": (6 * 2 * M * I * H, lambda: gemm(
            DR, Dd, b_major=1, epi=3, aux0=gg, aux1=uu, c_terms=DGU, ct_up_rows=I)),
        "B2 swiglu bwd (3x3) bn 64": (6 * 2 * M * I * H, lambda: gemm(
            DR, Dd, b_major=1, epi=3, aux0=gg, aux1=uu, c_terms=DGU, ct_up_rows=I, bn=64)),
        "B2 bn 64, 1 small acc": (6 * 2 * M * I * H, lambda: gemm(
            DR, Dd, b_major=1, epi=3, aux0=gg, aux1=uu, c_terms=DGU, ct_up_rows=I, bn=64,
            small_bufs=1)),
        "B2 bn 128, 1 small acc": (6 * 2 * M * I * H, lambda: gemm(
            DR, Dd, b_major=1, epi=3, aux0=gg, aux1=uu, c_terms=DGU, ct_up_rows=I,
            small_bufs=1)),
        "F1 1 small acc": (3 * 2 * M * 2 * I * H, lambda: gemm(
            MN, Dg, B2=Du, epi=2, aux0=gg, aux1=uu, c_terms=DIN, small_bufs=1)),
        "F3 1 small acc": (6 * 2 * M * H * I, lambda: gemm(
            DIN, Dd, epi=1, resid=H1.t[0], target=Y.t[0], ld_rt=H1.ld, out_scale=1e-3,
            sq_partial=sq, c_terms=DR, small_bufs=1)),
        "B1 1 small acc": (6 * 2 * H * I * M, lambda: gemm(
            DR, DIN, C=grad_d, a_major=1, b_major=1, small_bufs=1)),
        "B3 gradWgu (3x1, MN-major)": (3 * 2 * 2 * I * H * M, b3),
        "hard swiglu bf16 (1x1)": (2 * R * 2 * I * H, lambda: gemm(
            MNt, Wg1, B2=Wu1, epi=5, c_terms=Terms(R, I, 1, ld=I, tensors=[d_in]))),
    }


def attn(dev, g, seqs=8):
    B = seqs * HEADS
    q, k = _terms(B * T, HD, 3, dev, g), _terms(seqs * KV * T, HD, 3, dev, g)  # f32 after RoPE
    scores = torch.empty(B, T, T, device=dev)
    P = torch.empty(B * T, T, device=dev, dtype=torch.bfloat16)
    st = _lib.stream_ptr()
    return {
        "scores (3x3) causal": (6 * 2 * B * T * T * HD // 2, lambda: gemm(
            q, k, M=T, N=T, K=HD, batch=B, alpha=0.125, C=scores, ldc=T, a_off=(1, T, 0),
            b_off=(HEADS // KV, T, 0), c_off=(1, T * T, 0), skip_upper=True)),
        "softmax causal": (None, lambda: _lib.call(
            "gsq_softmax_causal", _lib.ptr(scores), B, T, _lib.ptr(P), None, st)),
    }


def soft_step(dev, g):
    from gsq_rco_mlx_b200.gsq.staged import SoftLinear
    import numpy as np
    out_f, in_f, R = I, H, 2
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 8, size=(out_f, in_f)).astype(np.uint8)
    s16 = (0.01 + 0.001 * rng.random((out_f, in_f // 64))).astype(np.float16)
    lin = SoftLinear("up_proj", 3, codes, s16, 64, seed=0)
    probs = torch.rand(R, lin.K, lin.d, device=dev)
    grad = torch.randn(R, out_f, in_f, device=dev) * 1e-3
    terms = torch.empty(R, 3, out_f, in_f, device=dev, dtype=torch.bfloat16)
    nxt = {"step": 1, "tau": 1.9, "kappa": 102.0, "seed": 5, "terms": terms}
    return {"soft_step up_proj (R=2)": (None, lambda: lin.step(probs, grad, 2.0, 100.0, nxt=nxt))}


def cublas(dev, g):
    """Library bf16 GEMMs of the same shapes (context for the tile-level figures above)."""
    M, R = 2 * (T - 1), 8 * T
    a1, b1 = torch.randn(R, H, device=dev).bfloat16(), torch.randn(2 * I, H, device=dev).bfloat16()
    a2, b2 = torch.randn(M, I, device=dev).bfloat16(), torch.randn(H, I, device=dev).bfloat16()
    a3, b3 = torch.randn(H, M, device=dev).bfloat16(), torch.randn(I, M, device=dev).bfloat16()
    return {
        "cublas bf16 16384x9728x896": (2 * R * 2 * I * H, lambda: a1 @ b1.T),
        "cublas bf16 4094x896x4864": (2 * M * H * I, lambda: a2 @ b2.T),
        "cublas bf16 896x4864x4094": (2 * H * I * M, lambda: a3 @ b3.T),
    }


def _packed_linear(N, K, bits, dev, g):
    """A packed linear with random words (every bit pattern is a valid code stream) and fp16
    g64 scales, generated on the device."""
    from gsq_rco_mlx_b200.common.evaluate import PackedLinear
    words = torch.randint(-2 ** 31, 2 ** 31, (N, K * bits // 32), device=dev, dtype=torch.int64,
                          generator=g).to(torch.int32)
    s = (0.01 * torch.randn(N, K // 64, device=dev, generator=g)).half()
    return PackedLinear(words, s, (-(1 << (bits - 1)) * s.float()).half(), bits, 64, K)


def packed(dev, g):
    """Packed 3-bit weights (fp16 g64 scales): the dequant stream of one decoder layer's seven
    linears into bf16, and the fused dequant-GEMV of a 65536 x 8192 weight (201 MB packed, more
    than L2) at 1 and 8 rows. Figures are algorithmic bytes: packed words + scales + biases read,
    bf16 weights written (dequant) or X read / Y written (GEMV)."""
    shapes = [(1024, H), (128, H), (H, H), (I, H), (I, H), (H, I)]
    lins = [_packed_linear(n, k, 3, dev, g) for n, k in shapes]
    outs = [torch.empty(n, k, device=dev, dtype=torch.bfloat16) for n, k in shapes]
    dq_bytes = sum(n * k * 3 // 8 + 2 * 2 * n * k // 64 + 2 * n * k for n, k in shapes)
    big = _packed_linear(65536, 8192, 3, dev, g)
    gv_bytes = 65536 * 8192 * 3 // 8 + 2 * 2 * 65536 * 8192 // 64
    x1 = torch.randn(1, 8192, device=dev, generator=g).bfloat16()
    x8 = torch.randn(8, 8192, device=dev, generator=g).bfloat16()
    y1 = torch.empty(1, 65536, device=dev, dtype=torch.bfloat16)
    y8 = torch.empty(8, 65536, device=dev, dtype=torch.bfloat16)

    def dq():
        for lin, o in zip(lins, outs):
            lin.dequant(o)
    return {
        "qdequant layer (3-bit)": (Bytes(dq_bytes), dq),
        "qgemv 65536x8192 M=1": (Bytes(gv_bytes), lambda: big(x1, out=y1)),
        "qgemv 65536x8192 M=8": (Bytes(gv_bytes), lambda: big(x8, out=y8)),
    }


def eval_batch(dev, g):
    """One 8-window x 2048 batch of the packed eval through 24 random 3-bit layers and the
    tied head (next-token NLL): the launch mix of bench.py's eval step."""
    import numpy as np
    from gsq_rco_mlx_b200.common.evaluate import Evaluator, PackedModel
    from gsq_rco_mlx_b200.gsq.e2e import LIN_ORDER, BlockConfig
    from gsq_rco_mlx_b200.rco.database import random_model
    cfg = BlockConfig()
    model = random_model(n_layers=24, seed=0, device=dev)
    layers = []
    for L, W in enumerate(model.layers):
        d = {k: W[k] for k in ("q_bias", "k_bias", "v_bias", "in_norm", "post_norm")}
        for name in LIN_ORDER:
            n, k = W[name].shape
            d[name] = _packed_linear(n, k, 3, dev, g)
        layers.append(d)
    del model.layers
    pm = PackedModel(cfg, model.embed, model.norm, layers)
    ev = Evaluator(pm, T, 8)
    rng = np.random.default_rng(2)
    win = rng.integers(0, model.embed.shape[0], size=(8, T))
    tok = torch.as_tensor(win.reshape(-1).astype(np.int32)).to(dev)
    tg = np.full(win.shape, -1, dtype=np.int32)
    tg[:, :-1] = win[:, 1:]
    tgt = torch.as_tensor(tg.reshape(-1)).to(dev)
    out = torch.zeros(1, device=dev, dtype=torch.float64)
    return {"eval batch 8 x 2048": (None, lambda: ev.forward_nll(tok, tgt, 8, out))}


def vjp_gemms(dev, g):
    """Two GEMMs of the block vector-Jacobian product at one sequence (14 heads x 2048): the
    probability cotangent dP = dO V^T per head (bf16 chain, causal tiles) and the MLP's
    dd = cot Wd with the bf16 SwiGLU backward epilogue ([dg | du] rows)."""
    B, R = HEADS, T
    do = _terms(B * T, HD, 1, dev, g)
    vr = _terms(KV * T, HD, 1, dev, g)
    dP = Terms(B * T, T, 1, dev, ld=T)
    cot = _terms(R, H, 1, dev, g)
    WdT = _terms(I, H, 1, dev, g)
    gg = torch.randn(R, I, device=dev, generator=g)
    uu = torch.randn(R, I, device=dev, generator=g)
    dGU = Terms(R, 2 * I, 1, dev, ld=2 * I)
    return {
        "dP = dO V^T (1x1, causal)": (2 * B * T * T * HD // 2, lambda: gemm(
            do, vr, M=T, N=T, K=HD, batch=B, epi=4, a_off=(1, T, 0), b_off=(HEADS // KV, T, 0),
            c_terms=dP, c_off=(1, T * T, 0), skip_upper=True)),
        "dd SwiGLU bwd bf16 (1x1)": (2 * R * I * H, lambda: gemm(
            cot, WdT, epi=6, aux0=gg, aux1=uu, ld_aux=I, c_terms=dGU, ct_up_rows=I)),
    }


def vo_step(dev, g):
    """The vo stage step at the block's widths on one micro-batch of 2 sequences x 2048 (R = 2):
    stage() gathers the rows, RoPEs q / k, runs the causal scores GEMM and the windowed softmax;
    contract() runs both resamples' GEMMs (V, P V, Y, dWo, dO, P^T dO, dWv) with the
    transposes and head sums between them. Times only (the products mix 1, 3 and 6 bf16
    products per float32 product)."""
    import numpy as np
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig
    from gsq_rco_mlx_b200.gsq.staged import SoftLinear, VOStep
    cfg = BlockConfig()
    rng = np.random.default_rng(0)

    def lin(name, out_f, in_f, i):
        codes = rng.integers(0, 8, size=(out_f, in_f)).astype(np.uint8)
        s16 = (0.01 + 0.001 * rng.random((out_f, in_f // 64))).astype(np.float16)
        return SoftLinear(name, 3, codes, s16, 64, seed=i, linear_id=i)
    v, o = lin("v_proj", KV * HD, H, 2), lin("o_proj", H, HEADS * HD, 3)
    bv = (0.02 * torch.randn(KV * HD, device=dev, generator=g)).bfloat16()
    step = VOStep([v, o], cfg, 2, T, 2, bv)
    hn = torch.randn(4 * T, H, device=dev, generator=g).bfloat16()
    a = (0.02 * torch.randn(4 * T, H, device=dev, generator=g)).bfloat16()
    qk = torch.randn(4 * T, (HEADS + KV) * HD, device=dev, generator=g).bfloat16()
    step.first_forward(0, 2.0, 100.0, 5)
    return {"vo stage(): gathers, RoPE, scores, softmax": (None, lambda: step.stage(hn, a, qk,
                                                                                    [1, 3])),
            "vo contract(): 2 resamples": (None, step.contract)}


CASES = {"mlp_gemms": mlp_gemms, "vo_step": vo_step, "vjp_gemms": vjp_gemms, "attn": attn, "attn1": lambda dev, g: attn(dev, g, seqs=1),
         "soft_step": soft_step, "cublas": cublas, "packed": packed, "eval_batch": eval_batch}


def main(argv):
    names = [a for a in argv if not a.startswith("--")] or list(CASES)
    once = "--once" in argv
    _lib.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    for name in names:
        for label, (flops, fn) in CASES[name](dev, g).items():
            if once:
                fn()
                torch.cuda.synchronize()
                continue
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                fn()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / 10 * 1000
            extra = ""
            if isinstance(flops, Bytes):
                extra = f"  {flops / us / 1e3:8.1f} GB/s algorithmic"
            elif flops:
                extra = f"  {flops / us / 1e6:8.1f} TFLOP/s executed bf16"
            print(f"{label:28s} {us:9.1f} us{extra}", flush=True)
    check_err(dev)


if __name__ == "__main__":
    main(sys.argv[1:])
