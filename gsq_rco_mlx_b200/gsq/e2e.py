"""Qwen2 decoder block on the GPU (reference src/gsq_rco/gsq/e2e.py), for the GSQ stages.

The reference runs one sequence at a time through MLX (``Qwen2Stream``). Here a chunk of S
sequences x T positions runs at once, bf16 storage exactly where the reference's arrays are
bf16, as seven tensor-core GEMMs with fused epilogues plus four elementwise kernels:

  hn  = rmsnorm(h)                                     gsq_rmsnorm
  q|k = bf16(bf16(hn [Wq|Wk]^T) + [bq|bk])             gemm, bf16-chain epilogue (one GEMM)
  v^T = bf16(bf16(hn Wv^T) + bv), transposed per seq   gemm, batched over sequences
  rope(q), rope(k) as float32 operand terms            gsq_rope_split
  S   = rope(q) rope(k)^T / 8 (float32-faithful)       gemm, batched (seq, head), causal tiles
  P   = bf16(softmax(S)) (causal)                      gsq_softmax_causal
  o   = bf16(P v)                                      gemm, batched (seq, head), causal k-range
  h1  = bf16(h + bf16(o Wo^T))                         gemm, bf16 chain with residual
  mn  = rmsnorm(h1)                                    gsq_rmsnorm
  d   = bf16(bf16(g bf16(sigmoid g)) u), g|u = mn [Wg|Wu]^T    gemm, dual-B bf16 SwiGLU epilogue
  out = bf16(h1 + bf16(d Wd^T))                        gemm, bf16 chain with residual

Optional transposed taps (the K-major operands of the Hessian GEMMs) of the four linear inputs
(hn, o, mn, d), with the columns of position 0 zeroed because every Hessian skips position 0
(staged.py:14-15). ``hessian_add`` folds X^T X of a tap into a float64 Hessian.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .. import _lib
from ..gemm import Terms, err_flag, gemm, pad8

LIN_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
TAPS = ("hn", "o", "mn", "d_in")  # inputs of q/k/v, o, gate/up, down


@dataclass(frozen=True)
class BlockConfig:
    hidden: int = 896
    n_heads: int = 14
    n_kv: int = 2
    head_dim: int = 64
    inter: int = 4864
    eps: float = 1e-6
    theta: float = 1e6

    @property
    def rep(self):
        return self.n_heads // self.n_kv


def rope_tables(T, head_dim=64, theta=1e6):
    """cos / sin [T, head_dim / 2] float32 (e2e.py:96-100)."""
    ex = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    freq = (np.float32(1.0) / (np.float32(theta) ** ex)).astype(np.float32)
    ang = np.arange(T, dtype=np.float32)[:, None] * freq[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def wterms(W):
    """A bf16 [out, in] weight as a one-term GEMM operand."""
    return Terms(W.shape[0], W.shape[1], 1, ld=W.shape[1], tensors=[W])


class BlockWeights:
    """bf16 CUDA weights of one block plus the stacked forms the fused GEMMs read."""

    def __init__(self, W: dict, qk=None):
        """qk: an existing [Wq; Wk] buffer whose row blocks are W["q_proj"] and W["k_proj"]
        (weights dequantized in place); otherwise the stacked copy is made here."""
        self.W = {k: v.contiguous() for k, v in W.items()}
        w = self.W
        self.qk = torch.cat([w["q_proj"], w["k_proj"]]).contiguous() if qk is None else qk
        self.qk_bias = torch.cat([w["q_bias"], w["k_bias"]]).float().contiguous()
        self.v_bias = w["v_bias"].float().contiguous()

    def replace(self, **kw):
        W = dict(self.W)
        W.update(kw)
        return BlockWeights(W)

    def transposed(self, key):
        """K-major transposed copies for the backward GEMMs (made once, cached): "down" Wd^T
        [I, H], "gate_up" [Wg; Wu]^T [H, 2I], "o" Wo^T [nh hd, H], "qkv" [Wq; Wk; Wv]^T
        [H, (nh + 2 nkv) hd]."""
        cache = self.__dict__.setdefault("_T", {})
        if key not in cache:
            w = self.W
            src = {"down": w["down_proj"], "o": w["o_proj"],
                   "gate_up": torch.cat([w["gate_proj"], w["up_proj"]]),
                   "qkv": torch.cat([w["q_proj"], w["k_proj"], w["v_proj"]])}[key].contiguous()
            r, c = src.shape
            t = Terms(c, r, 1, src.device)
            _lib.call("gsq_transpose_bf16", _lib.ptr(src), r, c, c, 0, _lib.ptr(t.t[0]), t.ld, 0,
                      1, 0, _lib.stream_ptr())
            cache[key] = t
        return cache[key]


class Qwen2Block:
    """Buffers and launches of the block forward for chunks of up to S sequences of T."""

    def __init__(self, cfg: BlockConfig, S: int, T: int, device=None):
        self.cfg, self.S, self.T = cfg, int(S), int(T)
        dev = device or _lib.device()
        self.dev = dev
        c = cfg
        R = S * T
        bf = torch.bfloat16
        self.hn = torch.empty(R, c.hidden, device=dev, dtype=bf)
        self.qk = torch.empty(R, (c.n_heads + c.n_kv) * c.head_dim, device=dev, dtype=bf)
        self.vT = Terms(S * c.n_kv * c.head_dim, T, 1, dev)
        self.q_rot = Terms(S * c.n_heads * T, c.head_dim, 3, dev)
        self.k_rot = Terms(S * c.n_kv * T, c.head_dim, 3, dev)
        self.scores = torch.empty(S * c.n_heads, T, T, device=dev, dtype=torch.float32)
        self.P = Terms(S * c.n_heads * T, T, 1, dev, ld=T)
        self.o = torch.empty(R, c.hidden, device=dev, dtype=bf)
        self.h1 = torch.empty(R, c.hidden, device=dev, dtype=bf)
        self.mn = torch.empty(R, c.hidden, device=dev, dtype=bf)
        self.d_in = torch.empty(R, c.inter, device=dev, dtype=bf)
        self.taps_t = {}
        cos, sin = rope_tables(T, c.head_dim, c.theta)
        self.cos = torch.as_tensor(cos, device=dev)
        self.sin = torch.as_tensor(sin, device=dev)

    def tap(self, name):
        """Transposed tap buffer [width, S*T] (bf16), allocated on first use."""
        if name not in self.taps_t:
            width = self.cfg.inter if name == "d_in" else self.cfg.hidden
            self.taps_t[name] = Terms(width, self.S * self.T, 1, self.dev)
        return self.taps_t[name]

    # ------------------------------------------------------------------------ forward ---
    def attention(self, hn, W: BlockWeights, S, o_out, o_tap=None, probs_t=None):
        """Causal GQA self-attention before o_proj of S sequences: o_out bf16 [S*T, H]."""
        c, T = self.cfg, self.T
        R = S * T
        st = _lib.stream_ptr()
        hnT = Terms(R, c.hidden, 1, ld=c.hidden, tensors=[hn])
        # q | k in one GEMM, bf16 chain with bias
        gemm(hnT, wterms(W.qk), M=R, epi=4, bias=W.qk_bias,
             c_terms=Terms(R, self.qk.shape[1], 1, ld=self.qk.shape[1], tensors=[self.qk[:R]]))
        # v^T per sequence: [s][kv * 64 + d][t]
        nkvd = c.n_kv * c.head_dim
        gemm(hnT, wterms(W.W["v_proj"]), M=T, batch=S, epi=4, bias=W.v_bias,
             a_off=(1, T, 0), ct_terms=self.vT, t_off=(1, nkvd, 0, 0, 0))
        qd = c.n_heads * c.head_dim
        t = self.q_rot.t
        _lib.call("gsq_rope_split", _lib.ptr(self.qk), self.qk.shape[1], S, T, c.n_heads,
                  _lib.ptr(self.cos), _lib.ptr(self.sin), _lib.ptr(t[0]), _lib.ptr(t[1]),
                  _lib.ptr(t[2]), st)
        t = self.k_rot.t
        kview = self.qk[:, qd:]
        _lib.call("gsq_rope_split", C_ptr(kview), self.qk.shape[1], S, T, c.n_kv,
                  _lib.ptr(self.cos), _lib.ptr(self.sin), _lib.ptr(t[0]), _lib.ptr(t[1]),
                  _lib.ptr(t[2]), st)
        # scores (seq, head) = q_rot k_rot^T / sqrt(64), causal tiles only
        B = S * c.n_heads
        gemm(self.q_rot, self.k_rot, M=T, N=T, K=c.head_dim, batch=B, alpha=1.0 / 8.0,
             C=self.scores, ldc=T, a_off=(1, T, 0), b_off=(c.rep, T, 0), c_off=(1, T * T, 0),
             skip_upper=True)
        _lib.call("gsq_softmax_causal", _lib.ptr(self.scores), B, T, _lib.ptr(self.P.t[0]),
                  _lib.ptr(probs_t), st)
        # o (seq, head) = P v, written at columns h * 64 of row s * T + t
        Ot = Terms(R, c.hidden, 1, ld=c.hidden, tensors=[o_out])
        gemm(self.P, self.vT, M=T, N=c.head_dim, K=T, batch=B, bn=64, causal=1, epi=4,
             a_off=(1, T, 0), b_off=(c.rep, c.head_dim, 0),
             c_off=(c.n_heads, T * c.hidden, c.head_dim), c_terms=Ot,
             ct_terms=o_tap, t_off=(c.n_heads, 0, c.head_dim, T, 0))

    def forward(self, h, W: BlockWeights, S=None, out=None, taps=(), attn_out=None, upto=None,
                mn=None, gu=None):
        """Block forward of S sequences h bf16 [S*T, H] -> out bf16 [S*T, H]. taps: names of
        TAPS to write transposed (self.tap(name)), position-0 columns zeroed.
        attn_out: also the attention output after o_proj (no residual; the vo-stage target);
        without `out` the forward ends there. upto: end after the named site ("hn", "o", "mn",
        "d_in") when only its tap is wanted. mn: bf16 [S*T, H] post-attention-norm rows of an
        earlier pass; the forward then starts at the MLP, with h the attention block output h1
        (unused for upto="d_in")."""
        c, T = self.cfg, self.T
        S = self.S if S is None else S
        R = S * T
        st = _lib.stream_ptr()
        if mn is not None:
            return self._mlp(h, mn, W, R, T, st, out, taps, upto)
        hn_tap = self.tap("hn") if "hn" in taps else None
        _lib.call("gsq_rmsnorm", _lib.ptr(h), c.hidden, _lib.ptr(W.W["in_norm"]), R, c.hidden,
                  float(c.eps), _lib.ptr(self.hn), c.hidden,
                  _lib.ptr(hn_tap.t[0] if hn_tap else None), hn_tap.ld if hn_tap else 0, T, 1, st)
        if upto == "hn":
            return None
        o_tap = self.tap("o") if "o" in taps else None
        self.attention(self.hn[:R], W, S, self.o[:R], o_tap=o_tap)
        if o_tap is not None:
            _lib.call("gsq_zero_cols", _lib.ptr(o_tap.t[0]), c.hidden, o_tap.ld, R, T, st)
        if upto == "o":
            return None
        Ot = Terms(R, c.hidden, 1, ld=c.hidden, tensors=[self.o[:R]])
        if attn_out is not None:
            gemm(Ot, wterms(W.W["o_proj"]), epi=4,
                 c_terms=Terms(R, c.hidden, 1, ld=c.hidden, tensors=[attn_out]))
            if out is None:
                return attn_out
        gemm(Ot, wterms(W.W["o_proj"]), epi=4, resid=h, ld_rt=c.hidden,
             c_terms=Terms(R, c.hidden, 1, ld=c.hidden, tensors=[self.h1[:R]]))
        mn_tap = self.tap("mn") if "mn" in taps else None
        _lib.call("gsq_rmsnorm", _lib.ptr(self.h1), c.hidden, _lib.ptr(W.W["post_norm"]), R,
                  c.hidden, float(c.eps), _lib.ptr(self.mn), c.hidden,
                  _lib.ptr(mn_tap.t[0] if mn_tap else None), mn_tap.ld if mn_tap else 0, T, 1, st)
        if upto == "mn":
            return None
        return self._mlp(self.h1[:R], self.mn[:R], W, R, T, st, out, taps, upto, gu)

    def _mlp(self, h1, mn, W: BlockWeights, R, T, st, out, taps, upto, gu=None):
        """out = h1 + down(SwiGLU(mn)) (bf16 chain); the d_in tap if asked; gu = (g, u) float32
        buffers receive the bf16 gate / up values (for the backward)."""
        c = self.cfg
        d_tap = self.tap("d_in") if "d_in" in taps else None
        MNt = Terms(R, c.hidden, 1, ld=c.hidden, tensors=[mn])
        gemm(MNt, wterms(W.W["gate_proj"]), B2=wterms(W.W["up_proj"]), epi=5,
             c_terms=Terms(R, c.inter, 1, ld=c.inter, tensors=[self.d_in[:R]]), ct_terms=d_tap,
             aux0=None if gu is None else gu[0], aux1=None if gu is None else gu[1],
             ld_aux=c.inter)
        if d_tap is not None:
            _lib.call("gsq_zero_cols", _lib.ptr(d_tap.t[0]), c.inter, d_tap.ld, R, T, st)
        if upto == "d_in":
            return None
        out = torch.empty(R, c.hidden, device=self.dev, dtype=torch.bfloat16) if out is None else out
        Dt = Terms(R, c.inter, 1, ld=c.inter, tensors=[self.d_in[:R]])
        gemm(Dt, wterms(W.W["down_proj"]), epi=4, resid=h1, ld_rt=c.hidden,
             c_terms=Terms(R, c.hidden, 1, ld=c.hidden, tensors=[out]))
        return out

    # ------------------------------------------------------------------------ backward ---
    def _bwd_buffers(self, S):
        """Work buffers of vjp for S sequences (allocated on first use, reused)."""
        key = ("bwd", S)
        if getattr(self, "_bwd_key", None) == key:
            return self._bwd
        c, T, dev = self.cfg, self.T, self.dev
        R, H, I, hd = S * T, c.hidden, c.inter, c.head_dim
        QD, KD = c.n_heads * hd, c.n_kv * hd
        B = S * c.n_heads
        bf = torch.bfloat16
        b = {
            "g": torch.empty(R, I, device=dev), "u": torch.empty(R, I, device=dev),
            "out": torch.empty(R, H, device=dev, dtype=bf),
            "dGU": torch.empty(R, 2 * I, device=dev, dtype=bf),
            "dmn": torch.empty(R, H, device=dev, dtype=bf),
            "dh1": torch.empty(R, H, device=dev, dtype=bf),
            "doh": torch.empty(B * T, hd, device=dev, dtype=bf), "doT": Terms(B * hd, T, 1, dev),
            "vrows": torch.empty(S * c.n_kv * T, hd, device=dev, dtype=bf),
            "dP": torch.empty(B * T, T, device=dev, dtype=bf),
            "dS": Terms(B * T, T, 3, dev), "dST": Terms(B * T, T, 3, dev),
            "PT": Terms(B * T, T, 1, dev),
            "qT": Terms(B * hd, T, 3, dev), "kT": Terms(S * c.n_kv * hd, T, 3, dev),
            "dqr": torch.empty(B * T, hd, device=dev), "dkr": torch.empty(B * T, hd, device=dev),
            "dvh": torch.empty(B * T, hd, device=dev),
            "dk": torch.empty(S * c.n_kv * T, hd, device=dev),
            "dQKV": torch.empty(R, QD + 2 * KD, device=dev, dtype=bf),
            "dhn": torch.empty(R, H, device=dev, dtype=bf),
        }
        self._bwd_key, self._bwd = key, b
        return b

    def _T(self, x, rows, cols, ld, out, ld_out=None, batch=1, bs_in=0, bs_out=0,
           skip_upper=False):
        """out[z] = x[z]^T (bf16): out a Terms (term 0, its ld) or a tensor with ld_out;
        skip_upper leaves the transposes of a causal block's zero tiles unwritten."""
        if isinstance(out, Terms):
            out, ld_out = out.t[0], out.ld
        _lib.call("gsq_transpose_bf16", _lib.ptr(x), rows, cols, ld, bs_in, _lib.ptr(out),
                  ld_out, bs_out, batch, int(skip_upper), _lib.stream_ptr())

    def new_grads(self, W: BlockWeights):
        """Zeroed float32 weight gradients of the seven linears; gate / up and q / k / v are views
        of one stacked buffer each (the layouts the weight-gradient GEMMs write)."""
        c, dev = self.cfg, self.dev
        H, I = c.hidden, c.inter
        QD, KD = c.n_heads * c.head_dim, c.n_kv * c.head_dim
        gu = torch.zeros(2 * I, H, device=dev)
        qkv = torch.zeros(QD + 2 * KD, H, device=dev)
        return {"_gu": gu, "_qkv": qkv, "gate_proj": gu[:I], "up_proj": gu[I:],
                "q_proj": qkv[:QD], "k_proj": qkv[QD:QD + KD], "v_proj": qkv[QD + KD:],
                "o_proj": torch.zeros(H, QD, device=dev),
                "down_proj": torch.zeros(H, I, device=dev)}

    def vjp(self, h, W: BlockWeights, cot, S=None, dh=None, grads=None, accumulate=False):
        """Vector-Jacobian product of the block (the RCO objective's _layer_vjp,
        src/gsq_rco/rco/allocate.py:156-167, of the block of e2e.py:160-174): h, cot bf16
        [S*T, H] (block input, cotangent of the block output) -> dh bf16 [S*T, H] (cotangent of
        the input) and the float32 weight gradients grads[name] [out, in] (added to when
        accumulate, e.g. over chunks). Cotangents of bf16 forward tensors are rounded to bf16,
        those of the float32 scores and RoPE'd q / k stay float32."""
        c, T = self.cfg, self.T
        S = self.S if S is None else S
        R, H, I, hd = S * T, c.hidden, c.inter, c.head_dim
        nh, nkv, rep = c.n_heads, c.n_kv, c.rep
        QD, KD = nh * hd, nkv * hd
        B = S * nh
        st = _lib.stream_ptr()
        b = self._bwd_buffers(S)
        dev = self.dev
        if grads is None:
            grads = self.new_grads(W)
        beta = 1.0 if accumulate else 0.0
        dh = torch.empty(R, H, device=dev, dtype=torch.bfloat16) if dh is None else dh
        # forward recompute, keeping the intermediates (and bf16 g, u)
        self.forward(h, W, S=S, out=b["out"][:R], gu=(b["g"][:R], b["u"][:R]))
        rows = lambda x, n=None: Terms(x.shape[0] if n is None else n, x.shape[1], 1,
                                       ld=x.shape[1], tensors=[x if n is None else x[:n]])
        # weight gradients dW = dY^T X: both row-major [R, .] activations read as MN-major
        # operands (the same products as their transposes)
        wgrad = lambda dy, x, out: gemm(rows(dy, R), rows(x, R), M=dy.shape[1], N=x.shape[1],
                                        K=R, C=out, beta=beta, a_major=1, b_major=1)
        # MLP: dd = bf16(cot Wd) with the SwiGLU backward in the epilogue ([dg | du] rows)
        gemm(rows(cot), W.transposed("down"), epi=6, aux0=b["g"], aux1=b["u"], ld_aux=I,
             c_terms=Terms(R, 2 * I, 1, ld=2 * I, tensors=[b["dGU"][:R]]), ct_up_rows=I)
        gemm(rows(b["dGU"], R), W.transposed("gate_up"), epi=4, c_terms=rows(b["dmn"], R))
        wgrad(b["dGU"], self.mn, grads["_gu"])
        wgrad(cot, self.d_in, grads["down_proj"])
        _lib.call("gsq_rmsnorm_bwd", _lib.ptr(self.h1), H, _lib.ptr(W.W["post_norm"]),
                  _lib.ptr(b["dmn"]), H, _lib.ptr(cot), H, _lib.ptr(b["dh1"]), H, R, H,
                  float(c.eps), st)
        # o_proj: do per (sequence, head) = bf16(dh1 Wo[:, h]) and its transpose
        wgrad(b["dh1"], self.o, grads["o_proj"])
        gemm(rows(b["dh1"], R), W.transposed("o"), M=T, N=hd, K=H, batch=B, bn=64, epi=4,
             a_off=(nh, T, 0), b_off=(nh, 0, hd),
             c_terms=Terms(B * T, hd, 1, ld=hd, tensors=[b["doh"]]), c_off=(1, T * hd, 0),
             ct_terms=b["doT"], t_off=(1, hd, 0, 0, 0))
        # attention: dP = bf16(do v^T); dS; dq, dk (float32); dv
        self._T(self.vT.t[0], hd, T, self.vT.ld, b["vrows"], hd, batch=S * nkv,
                bs_in=hd * self.vT.ld, bs_out=T * hd)
        gemm(Terms(B * T, hd, 1, ld=hd, tensors=[b["doh"]]),
             Terms(S * nkv * T, hd, 1, ld=hd, tensors=[b["vrows"]]), M=T, N=T, K=hd, batch=B,
             epi=4, a_off=(1, T, 0), b_off=(rep, T, 0),
             c_terms=Terms(B * T, T, 1, ld=T, tensors=[b["dP"]]), c_off=(1, T * T, 0),
             skip_upper=True)
        dS, dST = b["dS"], b["dST"]
        _lib.call("gsq_softmax_bwd", _lib.ptr(self.scores), _lib.ptr(b["dP"]), B, T, T,
                  _lib.ptr(dS.t[0]), _lib.ptr(dS.t[1]), _lib.ptr(dS.t[2]), dS.ld, 0.125, st)
        for i in range(3):
            self._T(dS.t[i], T, T, dS.ld, dST.t[i], dST.ld, batch=B, bs_in=T * dS.ld,
                    bs_out=T * dST.ld, skip_upper=True)
            self._T(self.q_rot.t[i], T, hd, self.q_rot.ld, b["qT"].t[i], b["qT"].ld, batch=B,
                    bs_in=T * self.q_rot.ld, bs_out=hd * b["qT"].ld)
            self._T(self.k_rot.t[i], T, hd, self.k_rot.ld, b["kT"].t[i], b["kT"].ld,
                    batch=S * nkv, bs_in=T * self.k_rot.ld, bs_out=hd * b["kT"].ld)
        self._T(self.P.t[0], T, T, self.P.ld, b["PT"], batch=B, bs_in=T * self.P.ld,
                bs_out=T * b["PT"].ld, skip_upper=True)
        gemm(dS, b["kT"], M=T, N=hd, K=T, batch=B, bn=64, causal=1, a_off=(1, T, 0),
             b_off=(rep, hd, 0), C=b["dqr"], ldc=hd, c_off=(1, T * hd, 0))
        gemm(dST, b["qT"], M=T, N=hd, K=T, batch=B, bn=64, causal=2, a_off=(1, T, 0),
             b_off=(1, hd, 0), C=b["dkr"], ldc=hd, c_off=(1, T * hd, 0))
        gemm(b["PT"], b["doT"], M=T, N=hd, K=T, batch=B, bn=64, causal=2, a_off=(1, T, 0),
             b_off=(1, hd, 0), C=b["dvh"], ldc=hd, c_off=(1, T * hd, 0))
        QKV = QD + 2 * KD
        dQKV = b["dQKV"]
        _lib.call("gsq_rope_bwd", _lib.ptr(b["dqr"]), hd, S, T, nh, _lib.ptr(self.cos),
                  _lib.ptr(self.sin), _lib.ptr(dQKV), QKV, 0, st)
        _lib.call("gsq_group_sum", _lib.ptr(b["dkr"]), hd, S, nh, rep, T, _lib.ptr(b["dk"]),
                  None, 0, 0, st)
        _lib.call("gsq_rope_bwd", _lib.ptr(b["dk"]), hd, S, T, nkv, _lib.ptr(self.cos),
                  _lib.ptr(self.sin), _lib.ptr(dQKV), QKV, QD, st)
        _lib.call("gsq_group_sum", _lib.ptr(b["dvh"]), hd, S, nh, rep, T, None,
                  _lib.ptr(dQKV), QKV, QD + KD, st)
        # q / k / v projections and the input norm
        gemm(rows(dQKV, R), W.transposed("qkv"), epi=4, c_terms=rows(b["dhn"], R))
        wgrad(dQKV, self.hn, grads["_qkv"])
        _lib.call("gsq_rmsnorm_bwd", _lib.ptr(h), H, _lib.ptr(W.W["in_norm"]), _lib.ptr(b["dhn"]),
                  H, _lib.ptr(b["dh1"]), H, _lib.ptr(dh), H, R, H, float(c.eps), st)
        return dh, grads

    def hessian_add(self, name, H, n, S=None):
        """Fold X^T X of tap `name` (positions 1.. of S sequences) into the float64 Hessian
        H (reference gptq.py:89-101 / staged.py:143-155): H <- H n/(n+m) + 2/(n+m) X^T X.
        Returns the new count n + m."""
        S = self.S if S is None else S
        tp = self.tap(name)
        m = S * (self.T - 1)
        width = tp.rows
        G = torch.empty(width, width, device=self.dev, dtype=torch.float32)
        gemm(tp, tp, K=S * self.T, C=G)
        total = n + m
        _lib.call("gsq_hess_accum", _lib.ptr(H), _lib.ptr(G), width * width, float(n / total),
                  float(2.0 / total), _lib.stream_ptr())
        return total


def C_ptr(t):
    """Device pointer of a (possibly strided) tensor view, for kernels that take a leading
    dimension argument."""
    import ctypes
    return ctypes.c_void_p(t.data_ptr())
