"""RCO bit allocation with the KL objective on the GPU (reference src/gsq_rco/rco/allocate.py).

KLObjective is the grad_fn of rco.loop.rco_loop: for a DP assignment z (one option per linear)
it assembles every linear from the database (dequant in the model dtype), runs the windows of
the sample through the stack, measures the mean token KL of the final hidden states against the
full-precision model's (tied-embedding head, rco.kl), and chains the gradient back block by
block (Qwen2Block.vjp) to the weight gradients dL/dW_i, whose inner products with every
candidate's residual Delta_ik = dequant(db[i, k]) - W_i are the straight-through upstream
(allocate.py:100-174). On the GPU:
  * the 25 decoder states of the sample's windows stay resident (bf16);
  * each layer's chosen weights are assembled once per sample (gsq_dequant_bf16);
  * the block backward runs in chunks of sequences, accumulating the weight gradients;
  * ste_dots streams each linear's gradient against its K candidates.
Across ranks the sample's windows are shared out; one all-reduce sums the upstream [n, K] and
the loss (the DP, manifold and Adam stay on the host, identical on every rank).
"""
from __future__ import annotations

from fractions import Fraction

import numpy as np
import torch

from .. import _lib
from ..gsq.e2e import BlockWeights, LIN_ORDER, Qwen2Block
from .database import QwenModel, SITE_OF
from .kl import DotsWorkspace, KLHead, kl_value_and_grad_hidden, ste_dots
from .loop import TAU0, TAU_MIN, integer_weights, rco_loop
from .manifold import dp_knapsack, expected_cost

MAX_TICKS = 256
MAX_TABLE_ENTRIES = 100_000_000
LINEARS = LIN_ORDER
N_PER_LAYER = len(LINEARS)


def budget_grid(avg_bits, total_units: int, n_groups: int):
    """The budget avg_bits * total_units held exactly on the DP's integer grid
    (allocate.py:33-51 semantics): avg_bits is taken as the decimal it prints as (2.976 is
    2976/1000, not its binary neighbour), ticks = the smallest grid scale that makes the budget
    a whole number. Returns (budget float, ticks, budget_int). Raises ValueError when the grid
    would need more than MAX_TICKS ticks per unit or the DP table would exceed
    MAX_TABLE_ENTRIES bytes."""
    exact = Fraction(str(float(avg_bits))) * int(total_units)
    ticks, budget_int = exact.denominator, exact.numerator
    if ticks > MAX_TICKS:
        raise ValueError(f"budget_grid: {avg_bits} bits on average needs a grid of {ticks} "
                         f"ticks per unit, above {MAX_TICKS}; shorten its decimal expansion")
    if n_groups * (budget_int + 1) > MAX_TABLE_ENTRIES:
        raise ValueError(f"budget_grid: a DP table of {n_groups} groups x {budget_int + 1} "
                         f"budgets is above {MAX_TABLE_ENTRIES} entries")
    return float(exact), int(ticks), int(budget_int)


def _grid(bank, avg_bits):
    """(w_int [n_groups], total units, budget, ticks, budget_int) of a bank and an average."""
    w_int, _ = integer_weights(bank.counts)
    total = int(np.sum(w_int))
    return (w_int, total) + budget_grid(avg_bits, total, len(bank.groups))


class Bank:
    """The quantized database on the GPU (rco.database.build_database results, keep="device"):
    groups i = (layer, name) in layer-major LINEARS order, options k = bit widths."""

    def __init__(self, manifest: dict, results: dict, group_size: int = 64):
        self.options = tuple(int(b) for b in manifest["options"])
        self.group_size = int(group_size)
        self.n_layers = int(manifest["n_layers"])
        self.groups = [(L, name) for L in range(self.n_layers) for name in LINEARS]
        self.counts = np.asarray(manifest["counts"], dtype=np.int64)
        self.sensitivity = np.asarray(manifest["sensitivity"], dtype=np.float64)
        self._r = results

    def cands(self, i):
        L, name = self.groups[i]
        return [(*self._r[(L, name, b)], b) for b in self.options]

    def dequant_bf16(self, i, k, out):
        codes, scales, bits = self.cands(i)[k]
        out_f, in_f = codes.shape
        _lib.call("gsq_dequant_bf16", _lib.ptr(codes), _lib.ptr(scales), out_f, in_f, int(bits),
                  self.group_size, _lib.ptr(out), _lib.stream_ptr())
        return out


def _rmsnorm_rows(x, w, eps, out):
    _lib.call("gsq_rmsnorm", _lib.ptr(x), x.shape[1], _lib.ptr(w), x.shape[0], x.shape[1],
              float(eps), _lib.ptr(out), x.shape[1], None, 0, 1, 0, _lib.stream_ptr())
    return out


class KLObjective:
    """Mean token KL(p_fp || p_z) over calibration windows (Eq. 6) as the RCO grad_fn
    (allocate.py:54-174)."""

    def __init__(self, model: QwenModel, bank: Bank, windows, *, windows_per_sample: int = 1,
                 chunk_seqs: int = 2, dp=None):
        windows = np.asarray(windows, dtype=np.int32)
        if windows.ndim != 2 or windows.shape[1] < 2:
            raise ValueError(f"windows must be [N, T] with T >= 2, got {windows.shape}")
        if not 1 <= windows_per_sample <= len(windows):
            raise ValueError(f"windows_per_sample must be in 1..{len(windows)}")
        if len(model.layers) != bank.n_layers:
            raise ValueError(f"model has {len(model.layers)} layers, database {bank.n_layers}")
        from ..gsq.staged import DataParallel
        self.model, self.bank, self.windows = model, bank, windows
        self.m = int(windows_per_sample)
        self.n_layers = bank.n_layers
        self.K = len(bank.options)
        self.dp = dp or DataParallel()
        cfg = model.cfg
        self.cfg, self.T = cfg, windows.shape[1]
        self.dev = model.embed.device
        self.cs = int(chunk_seqs)
        self.eng = Qwen2Block(cfg, self.cs, self.T, self.dev)
        self.head = KLHead(model.embed, chunk=8192)
        self.dots_ws = DotsWorkspace(self.dev)
        self.W_fp = [BlockWeights(W) for W in model.layers]
        # the reference hidden states (after the final norm) of every window, computed once
        self.h_ref = torch.empty(len(windows) * self.T, cfg.hidden, device=self.dev,
                                 dtype=torch.bfloat16)
        for a in range(0, len(windows), self.cs):
            ids = list(range(a, min(len(windows), a + self.cs)))
            st = self._states(ids, lambda L: self.W_fp[L])
            _rmsnorm_rows(st[-1], model.norm, cfg.eps,
                          self.h_ref[ids[0] * self.T:(ids[-1] + 1) * self.T])

    def _my_ids(self, ids):
        """This rank's share of a sample's windows (contiguous)."""
        a, b = self.dp.share(0, len(ids))
        return ids[a:b]

    def _states(self, ids, weights_of):
        """Decoder states [embedding, after block 0, ..., after block L-1] of windows ids
        (allocate.py:135-149), bf16 [len(ids) * T, H] each."""
        T, H = self.T, self.cfg.hidden
        n = len(ids) * T
        tok = torch.as_tensor(self.windows[ids].reshape(-1), device=self.dev)
        h = torch.empty(n, H, device=self.dev, dtype=torch.bfloat16)
        _lib.call("gsq_embed", _lib.ptr(tok), n, _lib.ptr(self.model.embed), H, _lib.ptr(h),
                  _lib.stream_ptr())
        states = [h]
        for L in range(self.n_layers):
            W = weights_of(L)
            nxt = torch.empty_like(h)
            for a in range(0, len(ids), self.cs):
                s = min(self.cs, len(ids) - a)
                rows = slice(a * T, (a + s) * T)
                self.eng.forward(states[-1][rows], W, S=s, out=nxt[rows])
            states.append(nxt)
        return states

    def _installed(self, L, choice):
        W = dict(self.model.layers[L])
        for j, name in enumerate(LINEARS):
            i = L * N_PER_LAYER + j
            out = torch.empty_like(self.model.layers[L][name])
            W[name] = self.bank.dequant_bf16(i, int(choice[i]), out)
        return BlockWeights(W)

    def __call__(self, z, p, step, sample, rng):
        """rco_loop grad_fn: (upstream [n_groups, K], loss) for one Gumbel sample."""
        choice = np.asarray(z).argmax(axis=1)
        ids = sorted(int(w) for w in rng.choice(len(self.windows), size=self.m, replace=False))
        loss, upstream = self.loss_and_upstream(choice, ids)
        return upstream, loss

    def mean_kl(self, choice, window_ids) -> float:
        return self.loss_and_upstream(choice, window_ids, upstream=False)[0]

    def loss_and_upstream(self, choice, window_ids, upstream: bool = True):
        """allocate.py:100-123 over this rank's share of the windows, summed over the ranks."""
        choice = np.asarray(choice).astype(int)
        all_ids = [int(w) for w in window_ids]
        ids = self._my_ids(all_ids)
        cfg, T, H = self.cfg, self.T, self.cfg.hidden
        n_all = len(all_ids) * T
        Ws = [self._installed(L, choice) for L in range(self.n_layers)]
        st = _lib.stream_ptr()
        up = torch.zeros(len(self.bank.groups), self.K, device=self.dev, dtype=torch.float64)
        tot = torch.zeros(1, device=self.dev, dtype=torch.float64)
        if ids:
            states = self._states(ids, lambda L: Ws[L])
            n = len(ids) * T
            hq = torch.empty(n, H, device=self.dev, dtype=torch.bfloat16)
            _rmsnorm_rows(states[-1], self.model.norm, cfg.eps, hq)
            href = torch.cat([self.h_ref[w * T:(w + 1) * T] for w in ids])
            kl_sum, g = self.head.kl_sum_and_grad(hq, href)
            tot += kl_sum
            if upstream:
                # mean over all the sample's positions (evaluate.py:150): bf16(g / n)
                _lib.call("gsq_div_bf16", _lib.ptr(g), g.numel(), float(n_all), st)
                # through the final norm, then block by block
                cot = torch.empty(n, H, device=self.dev, dtype=torch.bfloat16)
                _lib.call("gsq_rmsnorm_bwd", _lib.ptr(states[-1]), H, _lib.ptr(self.model.norm),
                          _lib.ptr(g), H, None, 0, _lib.ptr(cot), H, n, H, float(cfg.eps), st)
                for L in reversed(range(self.n_layers)):
                    grads = self.eng.new_grads(Ws[L])
                    g_in = torch.empty_like(cot)
                    for a in range(0, len(ids), self.cs):
                        s = min(self.cs, len(ids) - a)
                        rows = slice(a * T, (a + s) * T)
                        self.eng.vjp(states[L][rows], Ws[L], cot[rows], S=s, dh=g_in[rows],
                                     grads=grads, accumulate=a > 0)
                    for j, name in enumerate(LINEARS):
                        i = L * N_PER_LAYER + j
                        ste_dots(grads[name], self.model.layers[L][name], self.bank.cands(i),
                                 self.bank.group_size, ws=self.dots_ws, out=up[i])
                    cot = g_in
        self.dp.allreduce(up, tot)
        loss = float(tot.item()) / n_all
        return loss, (up.cpu().numpy() if upstream else None)


def initial_logits(bank: Bank, init: str) -> np.ndarray:
    """alpha0 = 0 or -S / mean(S) (allocate.py:177-192)."""
    n, K = len(bank.groups), len(bank.options)
    if init == "zero":
        return np.zeros((n, K))
    if init == "sensitivity":
        s = np.asarray(bank.sensitivity, dtype=np.float64)
        return -s / float(s.mean())
    raise ValueError(f"init must be 'zero' or 'sensitivity', got {init!r}")


def rco_allocate(objective: KLObjective, bank: Bank, avg_bits, *, steps: int, g: int,
                 lr: float, seed: int, tau0: float = TAU0, tau_min: float = TAU_MIN,
                 init: str = "zero", callback=None) -> dict:
    """RCO (Alg. 1) with the exact budget (allocate.py:195-224): the decoded choice per group,
    the per-step history, the budget grid and the decoded / expected average bits."""
    w_int, total, budget, ticks, budget_int = _grid(bank, avg_bits)
    bits = np.asarray(bank.options, dtype=np.float64)
    run = rco_loop(initial_logits(bank, init), bits, w_int, budget, steps=steps, g=g, lr=lr,
                   seed=seed, tau0=tau0, tau_min=tau_min, grad_fn=objective, ticks=ticks,
                   callback=callback)
    if run["budget_int"] != budget_int:
        raise RuntimeError(f"rco_allocate: the loop enforced budget {run['budget_int']}, the "
                           f"grid says {budget_int}")
    choice = np.argmax(run["z_final"], axis=1)
    cost_int, avg = decoded_cost(bank, choice)
    expected = float(expected_cost(run["logits"], bits, w_int)) / total
    return dict(choice=choice, history=run["history"], budget=budget, budget_int=budget_int,
                ticks=ticks, total_units=total, decoded_int_cost=cost_int,
                decoded_avg_bits=avg, expected_avg_bits=expected)


def decoded_cost(bank: Bank, choice):
    """(sum_i w_i b_{k_i}, that sum / sum_i w_i): the integer cost and average bits of a
    choice (allocate.py:243-247)."""
    w_int, _ = integer_weights(bank.counts)
    chosen_bits = np.asarray(bank.options, dtype=np.int64)[np.asarray(choice)]
    cost = int(np.dot(w_int, chosen_bits))
    return cost, cost / int(np.sum(w_int))


def proxy_dp_choice(bank: Bank, avg_bits):
    """Baseline allocation: the exact knapsack on minus the per-linear output-MSE
    sensitivities under the same budget (allocate.py:250-256)."""
    w_int, _, _, ticks, budget_int = _grid(bank, avg_bits)
    option_cost = ticks * np.asarray(bank.options, dtype=np.int64)
    z = dp_knapsack(-np.asarray(bank.sensitivity, dtype=np.float64), option_cost, w_int,
                    budget_int)
    return np.argmax(np.asarray(z), axis=1)


def uniform_choice(bank: Bank, bits: int):
    """Baseline allocation: every linear at ``bits`` (one of the bank's options)."""
    try:
        k = bank.options.index(int(bits))
    except ValueError:
        raise ValueError(f"uniform_choice: {bits} bits is not an option of the bank "
                         f"{bank.options}") from None
    return np.full(len(bank.groups), k, dtype=np.int64)
