"""Quantized-model eval on the GPU: packed MLX-affine linears, the chunked next-token NLL through
the tied head, and perplexity over token windows.

Reference: src/gsq_rco/common/evaluate.py:35-78 (nll_from_hidden, perplexity), run by the
reference on an mlx-lm checkpoint written by src/gsq_rco/gsq/export.py (QuantizedLinear layers
holding affine packed weights). Here the checkpoint's packed words stay packed in HBM:

  PackedLinear   words / scales / biases of one linear; __call__ is qgemm_packed (M <= 8: one
                 fused dequant-GEMV HBM stream; larger M: dequant + tensor-core GEMM)
  PackedModel    the decoder with packed linears; block(L) dequantizes layer L's seven linears
                 into one bf16 scratch set (14.9M weights, 30 MB: it stays in L2 for the block's
                 GEMMs) and returns the block weights the forward engine reads
  LogitHead      bf16(h E^T) chunks of the tied embedding and the NLL row pass
  perplexity     windows -> embedding -> blocks -> final norm -> head -> NLL sum, windows
                 sharded over data-parallel ranks with one all-reduce of the NLL sum
"""
from __future__ import annotations

import json
import math
import os

import numpy as np
import torch

from .. import _lib
from ..gemm import Terms, gemm
from ..gsq.e2e import LIN_ORDER, BlockConfig, BlockWeights, Qwen2Block
from ..gsq.export import BKEY, NKEY, SafetensorsFile, mlx_bits, module_path, to_mlx_affine

QGEMV_MAX_ROWS = 8


class PackedLinear:
    """One linear W [N][K] in the MLX affine packed form, resident on the GPU."""

    def __init__(self, words, scales, biases, bits: int, group_size: int, in_features: int):
        if words.dtype != torch.int32 or not words.is_cuda:
            raise ValueError("words must be a CUDA int32 tensor (uint32 bit patterns)")
        if scales.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError(f"unsupported scale dtype {scales.dtype}")
        if biases.dtype != scales.dtype or biases.shape != scales.shape:
            raise ValueError("scales and biases must share dtype and shape")
        self.words = words.contiguous()
        self.scales, self.biases = scales.contiguous(), biases.contiguous()
        self.bits, self.group_size = int(bits), int(group_size)
        self.N, self.K = int(words.shape[0]), int(in_features)
        if self.words.shape[1] * 32 != self.K * self.bits:
            raise ValueError(f"{self.words.shape[1]} words per row do not hold {self.K} x "
                             f"{self.bits}-bit values")
        if self.scales.shape != (self.N, self.K // self.group_size):
            raise ValueError(f"scales shape {tuple(self.scales.shape)} != "
                             f"{(self.N, self.K // self.group_size)}")
        self.sdtype = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}[self.scales.dtype]
        self._ws = None
        self._err = None

    @classmethod
    def from_native(cls, codes, scales, bits, group_size=64, scale_dtype="bfloat16",
                    device=None):
        """Pack native (codes, scales) on the host (to_mlx_affine) and upload."""
        dev = device or _lib.device()
        packed, sc, bi = to_mlx_affine(np.asarray(codes), np.asarray(scales, np.float32), bits,
                                       group_size, scale_dtype)
        words = torch.from_numpy(packed.view(np.int32).copy()).to(dev)
        return cls(words, sc.to(dev), bi.to(dev), mlx_bits(bits), group_size,
                   np.asarray(codes).shape[1])

    def dequant(self, out):
        """out bf16 [N][ld] (a row-major view with 16-byte aligned rows) = the dense weight."""
        if out.dtype != torch.bfloat16 or out.shape[0] != self.N or out.shape[1] != self.K:
            raise ValueError(f"out must be bf16 [{self.N}, {self.K}]")
        if out.stride(1) != 1:
            raise ValueError("out rows must be contiguous")
        _lib.call("qdequant_packed", _lib.ptr(self.words), _lib.ptr(self.scales),
                  _lib.ptr(self.biases), self.sdtype, self.N, self.K, self.bits,
                  self.group_size, C_view_ptr(out), out.stride(0), _lib.stream_ptr())
        return out

    def __call__(self, x, out=None, y_f32=False):
        """y = x W^T for x bf16 [M, K] (QuantizedLinear's matmul): bf16 [M, N] (or float32).
        M <= 8: the fused matrix-vector kernel on the unrounded weight s q + bias; larger M: the
        bf16-dequantized weight on the tensor cores (MLX's two forms)."""
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != self.K:
            raise ValueError(f"x must be bf16 [M, {self.K}]")
        x = x.contiguous()
        M = x.shape[0]
        dt = torch.float32 if y_f32 else torch.bfloat16
        if out is None:
            out = torch.empty(M, self.N, device=x.device, dtype=dt)
        if out.dtype != dt or out.shape != (M, self.N) or not out.is_contiguous():
            raise ValueError(f"out must be contiguous {dt} [{M}, {self.N}]")
        ws, nbytes = None, 0
        if M > QGEMV_MAX_ROWS:
            if self._ws is None:
                self._ws = torch.empty(self.N * self.K, device=x.device, dtype=torch.bfloat16)
            if self._err is None:
                self._err = torch.zeros(1, device=x.device, dtype=torch.int32)
            ws, nbytes = self._ws, self._ws.numel() * 2
        _lib.call("qgemm_packed", _lib.ptr(x), M, self.K, self.K, _lib.ptr(self.words),
                  _lib.ptr(self.scales), _lib.ptr(self.biases), self.sdtype, self.N, self.bits,
                  self.group_size, _lib.ptr(out), self.N, int(y_f32), _lib.ptr(ws), nbytes,
                  _lib.ptr(self._err), _lib.stream_ptr())
        return out


def C_view_ptr(t):
    """Device pointer of a CUDA tensor view whose rows may be strided (no contiguity check)."""
    import ctypes
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return ctypes.c_void_p(t.data_ptr())


class PackedModel:
    """A Qwen2-architecture decoder whose block linears are PackedLinear (dense tensors are
    accepted for linears the checkpoint left unquantized), with the tied bf16 embedding, the
    bf16 norms and biases."""

    def __init__(self, cfg: BlockConfig, embed, norm, layers: list):
        self.cfg, self.embed, self.norm, self.layers = cfg, embed, norm, layers
        self.dev = embed.device
        c, H = cfg, cfg.hidden
        QD, KD = c.n_heads * c.head_dim, c.n_kv * c.head_dim
        bf, dev = torch.bfloat16, self.dev
        # one dequant scratch set shared by every layer (stream order serialises them)
        self._qk = torch.empty(QD + KD, H, device=dev, dtype=bf)
        self._scratch = {"q_proj": self._qk[:QD], "k_proj": self._qk[QD:],
                         "v_proj": torch.empty(KD, H, device=dev, dtype=bf),
                         "o_proj": torch.empty(H, QD, device=dev, dtype=bf),
                         "gate_proj": torch.empty(c.inter, H, device=dev, dtype=bf),
                         "up_proj": torch.empty(c.inter, H, device=dev, dtype=bf),
                         "down_proj": torch.empty(H, c.inter, device=dev, dtype=bf)}
        self._bw = []
        for W in layers:
            d = {k: W[k] for k in ("q_bias", "k_bias", "v_bias", "in_norm", "post_norm")}
            d.update(self._scratch)
            self._bw.append(BlockWeights(d, qk=self._qk))

    @property
    def n_layers(self):
        return len(self.layers)

    def block(self, L: int) -> BlockWeights:
        """Dequantize layer L's linears into the scratch set; its block weights."""
        for name in LIN_ORDER:
            lin, dst = self.layers[L][name], self._scratch[name]
            if isinstance(lin, PackedLinear):
                lin.dequant(dst)
            else:
                dst.copy_(lin)
        return self._bw[L]

    def packed_bytes(self) -> int:
        """Bytes of the packed words, scales and biases of every linear."""
        n = 0
        for W in self.layers:
            for name in LIN_ORDER:
                lin = W[name]
                if isinstance(lin, PackedLinear):
                    n += lin.words.numel() * 4 + 2 * lin.scales.numel() * lin.scales.element_size()
        return n

    @classmethod
    def from_quantized(cls, model, quantized: dict, scale_dtype="bfloat16"):
        """A QwenModel (bf16 on the GPU) with the linears of `quantized` ({module path:
        dict(codes, scales, bits, group_size)}) packed; the others stay dense."""
        layers = []
        for L, W in enumerate(model.layers):
            d = {k: W[k] for k in ("q_bias", "k_bias", "v_bias", "in_norm", "post_norm")}
            for name in LIN_ORDER:
                q = quantized.get(module_path(L, name))
                d[name] = W[name] if q is None else PackedLinear.from_native(
                    q["codes"], q["scales"], q["bits"], q["group_size"], scale_dtype,
                    device=model.embed.device)
            layers.append(d)
        return cls(model.cfg, model.embed, model.norm, layers)

    @classmethod
    def load(cls, model_dir, device=None):
        """An exported checkpoint (export_mlx_lm) onto the GPU: packed linears stay packed."""
        dev = device or _lib.device()
        with open(os.path.join(model_dir, "config.json")) as f:
            conf = json.load(f)
        H, nh = conf["hidden_size"], conf["num_attention_heads"]
        cfg = BlockConfig(hidden=H, n_heads=nh, n_kv=conf["num_key_value_heads"],
                          head_dim=H // nh, inter=conf["intermediate_size"],
                          eps=float(conf["rms_norm_eps"]), theta=float(conf["rope_theta"]))
        quant = conf.get("quantization", {})
        st = SafetensorsFile(os.path.join(model_dir, "model.safetensors"))

        def dense(name):
            if st.dtype(name) != "BF16":
                raise TypeError(f"{name} is {st.dtype(name)}, expected BF16")
            return st.tensor(name).to(dev)

        layers = []
        for L in range(conf["num_hidden_layers"]):
            p = f"model.layers.{L}."
            d = {k: dense(p + n) for k, n in {**BKEY, **NKEY}.items()}
            for name in LIN_ORDER:
                path = module_path(L, name)
                if st.dtype(path + ".weight") == "U32":
                    qc = quant.get(path, quant)
                    bits, gs = int(qc["bits"]), int(qc["group_size"])
                    words = st.tensor(path + ".weight").to(dev)
                    in_f = words.shape[1] * 32 // bits
                    d[name] = PackedLinear(words, st.tensor(path + ".scales").to(dev),
                                           st.tensor(path + ".biases").to(dev), bits, gs, in_f)
                else:
                    d[name] = dense(path + ".weight")
            layers.append(d)
        return cls(cfg, dense("model.embed_tokens.weight"), dense("model.norm.weight"), layers)


class LogitHead:
    """Chunks of bf16(h E^T) (the tied head in the model dtype, evaluate.py:28-33) and the NLL
    row pass; one [chunk, V] bf16 logit buffer."""

    def __init__(self, E, chunk: int = 1024):
        if E.dtype != torch.bfloat16 or E.dim() != 2:
            raise ValueError("E must be a bf16 [V, H] tensor")
        self.E = E.contiguous()
        self.V, self.H = self.E.shape
        if self.V % 8:
            raise ValueError(f"vocabulary {self.V} must be a multiple of 8")
        self.chunk = int(chunk)
        self.Et = Terms(self.V, self.H, 1, ld=self.H, tensors=[self.E])
        self.z = torch.empty(self.chunk, self.V, device=E.device, dtype=torch.bfloat16)

    def nll_rows(self, h, targets, out):
        """out f64 [n]: next-token NLL of each row of h bf16 [n, H] (targets int32 [n], < 0 for
        unscored rows)."""
        n = h.shape[0]
        st = _lib.stream_ptr()
        for a in range(0, n, self.chunk):
            b = min(n, a + self.chunk)
            m = b - a
            zt = Terms(m, self.V, 1, ld=self.V, tensors=[self.z[:m]])
            gemm(Terms(m, self.H, 1, ld=self.H, tensors=[h[a:b]]), self.Et, epi=4, c_terms=zt)
            _lib.call("gsq_nll_rows", _lib.ptr(self.z), m, self.V, self.V,
                      _lib.ptr(targets[a:b]), _lib.ptr(out[a:b]), st)
        return out


def nll_from_hidden(head: LogitHead, h, targets):
    """Summed next-token NLL over rows (evaluate.py:35-52): (float64 CUDA [1], n rows scored).
    h bf16 [B*T, H] normed hidden states, targets int [B*T] (the token each row predicts)."""
    tg = torch.as_tensor(np.asarray(targets, dtype=np.int32)).to(h.device) \
        if not torch.is_tensor(targets) else targets.to(h.device, torch.int32)
    rows = torch.empty(h.shape[0], device=h.device, dtype=torch.float64)
    head.nll_rows(h, tg, rows)
    total = torch.empty(1, device=h.device, dtype=torch.float64)
    _lib.call("gsq_sum_f64", _lib.ptr(rows), rows.numel(), _lib.ptr(total), _lib.stream_ptr())
    return total, int((tg >= 0).sum().item())


class Evaluator:
    """Buffers of the windowed eval: forward engine, head and per-batch token / target rows.
    Reused across perplexity() calls on windows of one length."""

    def __init__(self, model: PackedModel, seq_len: int, chunk_seqs: int = 4,
                 head_chunk: int = 1024):
        self.model, self.S, self.cs = model, int(seq_len), int(chunk_seqs)
        dev, H = model.dev, model.cfg.hidden
        self.eng = Qwen2Block(model.cfg, self.cs, self.S, dev)
        self.head = LogitHead(model.embed, head_chunk)
        n = self.cs * self.S
        self.h = [torch.empty(n, H, device=dev, dtype=torch.bfloat16) for _ in range(2)]
        self.hn = torch.empty(n, H, device=dev, dtype=torch.bfloat16)
        self.tok = torch.empty(n, device=dev, dtype=torch.int32)
        self.tgt = torch.empty(n, device=dev, dtype=torch.int32)
        self.rows = torch.empty(n, device=dev, dtype=torch.float64)
        self.pin_tok = torch.empty(n, dtype=torch.int32).pin_memory()
        self.pin_tgt = torch.empty(n, dtype=torch.int32).pin_memory()
        self._copied = torch.cuda.Event()
        self._copied.record()

    def batch_nll(self, win: np.ndarray, out_sum):
        """out_sum f64 CUDA [1] = summed NLL of windows win [s, S] (s <= chunk_seqs): each window
        is fed whole and position t scored against token t + 1 (t < S - 1); the last position's
        output is not scored (causality: positions < S - 1 equal a forward of tokens[:-1])."""
        s, S = win.shape
        n = s * S
        self._copied.synchronize()  # the previous batch's copies have read the pinned rows
        tok = self.pin_tok[:n].numpy().reshape(s, S)
        tgt = self.pin_tgt[:n].numpy().reshape(s, S)
        tok[:] = win
        tgt[:, :-1] = win[:, 1:]
        tgt[:, -1] = -1
        self.tok[:n].copy_(self.pin_tok[:n], non_blocking=True)
        self.tgt[:n].copy_(self.pin_tgt[:n], non_blocking=True)
        self._copied.record()
        return self.forward_nll(self.tok[:n], self.tgt[:n], s, out_sum)

    def forward_nll(self, tok, tgt, s: int, out_sum):
        """out_sum f64 CUDA [1] = summed NLL of s windows already on the device: tok, tgt int32
        [s * S] (ids and the targets of each position, -1 where not scored)."""
        S, n = self.S, s * self.S
        if s > self.cs or tok.numel() != n or tgt.numel() != n:
            raise ValueError(f"expected {s} <= {self.cs} windows of {S} ids and targets")
        model, c = self.model, self.model.cfg
        st = _lib.stream_ptr()
        h, nxt = self.h
        _lib.call("gsq_embed", _lib.ptr(tok), n, _lib.ptr(model.embed), c.hidden,
                  _lib.ptr(h), st)
        for L in range(model.n_layers):
            W = model.block(L)
            self.eng.forward(h[:n], W, S=s, out=nxt[:n])
            h, nxt = nxt, h
        _lib.call("gsq_rmsnorm", _lib.ptr(h), c.hidden, _lib.ptr(model.norm), n, c.hidden,
                  float(c.eps), _lib.ptr(self.hn), c.hidden, None, 0, 1, 0, st)
        self.head.nll_rows(self.hn[:n], tgt, self.rows[:n])
        _lib.call("gsq_sum_f64", _lib.ptr(self.rows), n, _lib.ptr(out_sum), st)
        return out_sum


def perplexity(model: PackedModel, windows, chunk_seqs: int = 4, progress: bool = False,
               dp=None, evaluator: Evaluator = None) -> dict:
    """Perplexity of token windows [N, S] (evaluate.py:55-78): each window contributes S - 1
    predictions. Windows are split contiguously over the data-parallel ranks (dp: a
    gsq.staged.DataParallel; one all-reduce of the float64 NLL sum). Returns dict(ppl,
    nll_per_token, n_tokens, n_windows, seq_len)."""
    from ..gsq.staged import DataParallel
    windows = np.asarray(windows)
    if windows.ndim != 2 or windows.shape[1] < 2:
        raise ValueError(f"windows must be [N, S] with S >= 2, got {windows.shape}")
    if windows.min(initial=0) < 0 or windows.max(initial=0) >= model.embed.shape[0]:
        raise ValueError("token ids outside the vocabulary")
    dp = dp or DataParallel()
    n_windows, seq_len = windows.shape
    ev = evaluator or Evaluator(model, seq_len, chunk_seqs)
    if ev.S != seq_len:
        raise ValueError(f"evaluator built for windows of {ev.S}, got {seq_len}")
    a, b = dp.share(0, n_windows)
    dev = model.dev
    n_batches = max(1, -(-(b - a) // ev.cs))
    sums = torch.zeros(n_batches, device=dev, dtype=torch.float64)
    for j, w0 in enumerate(range(a, b, ev.cs)):
        w1 = min(b, w0 + ev.cs)
        ev.batch_nll(windows[w0:w1].astype(np.int32), sums[j:j + 1])
        if progress and (j + 1) % 10 == 0:
            print(f"  ppl: {w1 - a}/{b - a} windows (rank {dp.rank})", flush=True)
    total = torch.zeros(1, device=dev, dtype=torch.float64)
    _lib.call("gsq_sum_f64", _lib.ptr(sums), n_batches, _lib.ptr(total), _lib.stream_ptr())
    dp.allreduce(total)
    n_tokens = n_windows * (seq_len - 1)
    nll = float(total.item()) / n_tokens
    return {"ppl": math.exp(nll), "nll_per_token": nll, "n_tokens": n_tokens,
            "n_windows": n_windows, "seq_len": seq_len}
