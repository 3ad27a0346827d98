"""App-H: end-to-end fine-tune of the group scales of a quantized stack (codes fixed).

Reference: src/gsq_rco/gsq/staged.py:555-634 (scale_finetune), off by default in the reference
pipeline (pipeline.py:176-206). Per step, one calibration sequence: the quantized forward with
W = bf16(s[r][c / g] grid[code]) for every quantized linear, the mean token KL(p_fp || p_q)
against the final-normed FP hidden states through the tied head (evaluate.py:128-151), its
gradient chained back through the final norm and every block (the same vector-Jacobian products
as the RCO objective: gsq.e2e.Qwen2Block.vjp), reduced per group to dL/ds = sum_c G grid[code]
(gsq_scale_grad), and one Lion step on every scale (lr for all of them, lion.py:44-56).

The block vjp gives float32 weight gradients (the reference's MLX autodiff carries bf16 ones);
everything else follows the reference's order: KL before the update of its step, returned per
step.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _lib
from ..rco.kl import KLHead
from .e2e import LIN_ORDER, BlockWeights, Qwen2Block
from .lion import BETAS, LR_SCALES, WEIGHT_DECAY


def _rmsnorm_rows(x, w, eps, out):
    _lib.call("gsq_rmsnorm", _lib.ptr(x), x.shape[1], _lib.ptr(w), x.shape[0], x.shape[1],
              float(eps), _lib.ptr(out), x.shape[1], None, 0, 1, 0, _lib.stream_ptr())
    return out


class ScaleFinetune:
    """The training state of App-H on the GPU: fixed codes, float32 scales and their Lion
    momentum per quantized linear; the FP blocks of unquantized layers."""

    def __init__(self, model, qblocks: dict, tokens, group_size: int = 64, lr: float = LR_SCALES):
        self.model, self.gs, self.lr = model, int(group_size), float(lr)
        self.cfg = model.cfg
        self.dev = model.embed.device
        self.tokens = np.asarray(tokens, dtype=np.int32)
        if self.tokens.ndim != 2:
            raise ValueError("tokens must be [N, T]")
        self.T = self.tokens.shape[1]
        self.q = {}
        for L, lins in qblocks.items():
            for name in LIN_ORDER:
                qq = lins[name]
                codes = torch.as_tensor(np.ascontiguousarray(qq["codes"])).to(self.dev)
                s = torch.as_tensor(np.asarray(qq["scales"], dtype=np.float32)).to(self.dev)
                self.q[(L, name)] = {"codes": codes, "bits": int(qq["bits"]), "scales": s,
                                     "mom": torch.zeros_like(s), "grad": torch.empty_like(s)}
        self.eng = Qwen2Block(self.cfg, 1, self.T, self.dev)
        self.head = KLHead(model.embed, chunk=min(8192, self.T))
        self.h_ref = self._reference_states()

    def _weights(self, L):
        W = dict(self.model.layers[L])
        for name in LIN_ORDER:
            qq = self.q.get((L, name))
            if qq is None:
                continue
            out = torch.empty_like(self.model.layers[L][name])
            out_f, in_f = out.shape
            _lib.call("gsq_dequant_bf16", _lib.ptr(qq["codes"]), _lib.ptr(qq["scales"]), out_f,
                      in_f, qq["bits"], self.gs, _lib.ptr(out), _lib.stream_ptr())
            W[name] = out
        return BlockWeights(W)

    def _embed(self, n):
        tok = torch.as_tensor(self.tokens[n]).to(self.dev)
        h = torch.empty(self.T, self.cfg.hidden, device=self.dev, dtype=torch.bfloat16)
        _lib.call("gsq_embed", _lib.ptr(tok), self.T, _lib.ptr(self.model.embed),
                  self.cfg.hidden, _lib.ptr(h), _lib.stream_ptr())
        return h

    def _reference_states(self):
        """Final-normed FP hidden states of every calibration sequence (pipeline.py:180-186)."""
        out = torch.empty(len(self.tokens) * self.T, self.cfg.hidden, device=self.dev,
                          dtype=torch.bfloat16)
        Wfp = [BlockWeights(W) for W in self.model.layers]
        for n in range(len(self.tokens)):
            h = self._embed(n)
            for W in Wfp:
                nxt = torch.empty_like(h)
                self.eng.forward(h, W, S=1, out=nxt)
                h = nxt
            _rmsnorm_rows(h, self.model.norm, self.cfg.eps, out[n * self.T:(n + 1) * self.T])
        return out

    def step(self, t: int) -> float:
        """One fine-tune step on sequence t % N: the KL before the update (float)."""
        n = t % len(self.tokens)
        cfg, T, H = self.cfg, self.T, self.cfg.hidden
        st = _lib.stream_ptr()
        Ws = [self._weights(L) for L in range(len(self.model.layers))]
        states = [self._embed(n)]
        for W in Ws:
            nxt = torch.empty_like(states[-1])
            self.eng.forward(states[-1], W, S=1, out=nxt)
            states.append(nxt)
        hq = torch.empty(T, H, device=self.dev, dtype=torch.bfloat16)
        _rmsnorm_rows(states[-1], self.model.norm, cfg.eps, hq)
        kl_sum, g = self.head.kl_sum_and_grad(hq, self.h_ref[n * T:(n + 1) * T])
        # mean over the sequence's positions (evaluate.py:150), then through the final norm
        _lib.call("gsq_div_bf16", _lib.ptr(g), g.numel(), float(T), st)
        cot = torch.empty(T, H, device=self.dev, dtype=torch.bfloat16)
        _lib.call("gsq_rmsnorm_bwd", _lib.ptr(states[-1]), H, _lib.ptr(self.model.norm),
                  _lib.ptr(g), H, None, 0, _lib.ptr(cot), H, T, H, float(cfg.eps), st)
        for L in reversed(range(len(self.model.layers))):
            grads = self.eng.new_grads(Ws[L])
            g_in = torch.empty_like(cot)
            self.eng.vjp(states[L], Ws[L], cot, S=1, dh=g_in, grads=grads)
            for name in LIN_ORDER:
                qq = self.q.get((L, name))
                if qq is None:
                    continue
                out_f, in_f = grads[name].shape
                _lib.call("gsq_scale_grad", _lib.ptr(grads[name]),
                          _lib.ptr(qq["codes"]), out_f, in_f, qq["bits"], self.gs,
                          _lib.ptr(qq["grad"]), st)
            cot = g_in
        b1, b2 = BETAS
        for qq in self.q.values():
            _lib.call("gsq_lion_f32", _lib.ptr(qq["scales"]), _lib.ptr(qq["mom"]),
                      _lib.ptr(qq["grad"]), qq["scales"].numel(), self.lr, float(WEIGHT_DECAY),
                      float(b1), float(b2), st)
        return float(kl_sum.item()) / T

    def scales(self) -> dict:
        """{layer: {linear: fp16 scales}} (the stored form)."""
        out = {}
        for (L, name), qq in self.q.items():
            out.setdefault(L, {})[name] = qq["scales"].cpu().numpy().astype(np.float16)
        return out


def scale_finetune(model, qblocks: dict, tokens, steps: int, lr: float = LR_SCALES,
                   group_size: int = 64, log=print):
    """(scales, kl) as the reference's scale_finetune (staged.py:555-634): scales[layer][name]
    the fine-tuned fp16 scales, kl the KL of each step before its update. qblocks[layer][name] =
    {"codes" uint8, "scales" float16, "bits"}; tokens [N, T] calibration ids; model a QwenModel
    with the FP weights (biases, norms, unquantized layers, the tied embedding)."""
    ft = ScaleFinetune(model, qblocks, tokens, group_size, lr)
    kls = []
    for t in range(steps):
        kls.append(ft.step(t))
        if (t + 1) % max(1, steps // 4) == 0:
            log(f"    scale fine-tune step {t + 1}/{steps}: KL "
                f"{np.mean(kls[-max(1, steps // 4):]):.5f}")
    return ft.scales(), kls
