"""The RCO quantized-weight database on the GPU (reference src/gsq_rco/rco/database.py).

For every linear i of the first n_layers blocks and every option k (bit width b_k) the
database holds the GPTQ quantizer of that linear (signed scales, group size 64) and its
sensitivity, the output MSE 1/2 tr(dW H dW^T) on the calibration Hessian
(database.py:158-241). Hessians are the Gram matrices 2 X^T X / M of the full-precision
model's inputs to each linear, position 0 of every window excluded, computed layer by layer on
the full-precision stream (database.py:184-214).

B200 layout of the work, per layer:
  * one block forward per chunk of 8 windows writes all four taps at once (transposed bf16
    operands, position-0 columns zero): q/k/v input, o input, gate/up input, down input;
  * each tap's Gram X^T X runs on the tensor cores (one bf16 term: exact products, float32
    accumulation folded in float32 registers) and folds into the float64 Hessian with the
    reference's running-mean update H <- H n/(n+m) + 2/(n+m) X^T X;
  * one factorisation (upper factor of the damped inverse Hessian) per site serves every
    linear and bit width that reads the site (q/k/v share one, gate/up share one);
  * the GPTQ sweeps of the 7 linears x K options.

Across ranks (torch.distributed initialised, world > 1): the calibration windows are split
into contiguous shards, each rank runs the forward of its shard and its running-mean
Hessians, one all-reduce per site combines them (weights n_rank / n), and the (linear,
option) solves are shared out by longest-processing-time on their float64 cost. Codes,
scales and sensitivities are all-gathered so that every rank returns the full database.

On-disk layout when db_dir is given (database.py:10-18): manifest.json, sensitivity.npy,
L{layer:02d}.{name}.b{bits}.{codes,scales}.npy.
"""
from __future__ import annotations

import hashlib
import json
import os
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .. import _lib
from ..gsq.e2e import BlockConfig, BlockWeights, LIN_ORDER, Qwen2Block
from ..gsq.gptq import gptq_factor, quantize_gptq

FORMAT = "rco_mlx.database/1"
MAX_OPTIONS = 255
LINEARS = LIN_ORDER
SITE_OF = {"q_proj": "qkv", "k_proj": "qkv", "v_proj": "qkv", "o_proj": "o",
           "gate_proj": "gate_up", "up_proj": "gate_up", "down_proj": "down"}
TAP_OF_SITE = {"qkv": "hn", "o": "o", "gate_up": "mn", "down": "d_in"}
SITES = ("qkv", "o", "gate_up", "down")


@dataclass(frozen=True)
class DBSpec:
    """database.py:52-60 (calibration source fields kept for the manifest identity)."""
    options: tuple = (2, 3, 4, 5, 6, 8)
    group_size: int = 64
    quantizer: str = "gptq"
    damp: float = 0.01
    n_layers: int = 24
    calib_split: str = "train"
    calib_seed: int = 0


@dataclass
class QwenModel:
    """A Qwen2-architecture decoder stack on the GPU: the tied token embedding (bf16 [V, H]),
    one weight dict per block (the keys of gsq.e2e.BlockWeights) and the final RMSNorm weight
    (bf16 [H])."""
    cfg: BlockConfig
    embed: torch.Tensor
    layers: list
    norm: torch.Tensor = None


def _check_spec(spec: DBSpec, n_model_layers: int):
    """database.py:117-127."""
    opts = tuple(int(b) for b in spec.options)
    if not opts or len(opts) > MAX_OPTIONS:
        raise ValueError(f"need 1..{MAX_OPTIONS} options, got {opts}")
    if any(not 2 <= b <= 8 for b in opts) or list(opts) != sorted(set(opts)):
        raise ValueError(f"options must be strictly increasing bit-widths in 2..8, got {opts}")
    if spec.quantizer != "gptq":
        raise ValueError(f"quantizer {spec.quantizer!r}: this build implements 'gptq'")
    if not 1 <= spec.n_layers <= n_model_layers:
        raise ValueError(f"n_layers must be in 1..{n_model_layers}, got {spec.n_layers}")
    return opts


def _name(layer: int, name: str, bits: int, kind: str) -> str:
    return f"L{layer:02d}.{name}.b{bits}.{kind}.npy"


def sha256_array(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def identity(spec: DBSpec, model_sha: str, tokens) -> dict:
    """The fields that decide whether a stored database is valid (database.py:79-103)."""
    tokens = np.asarray(tokens)
    return {
        "format": FORMAT,
        "model_weights_sha256": model_sha,
        "options": [int(b) for b in spec.options],
        "group_size": int(spec.group_size),
        "quantizer": spec.quantizer,
        "damp": float(spec.damp),
        "signed_scale": True,
        "n_layers": int(spec.n_layers),
        "calibration": {
            "split": spec.calib_split, "seed": int(spec.calib_seed),
            "n_windows": int(tokens.shape[0]), "window_len": int(tokens.shape[1]),
            "excluded_positions": [0], "tokens_sha256": sha256_array(tokens),
            "hessian_rows": int(tokens.shape[0] * (tokens.shape[1] - 1)),
        },
        "hessian": "2/M X^T X in float64 (running mean per chunk), FP-model inputs",
    }


# ------------------------------------------------------------------------ sharding ---

def solve_cost(out_f: int, in_f: int) -> float:
    """Relative cost of one GPTQ solve: the float64 sweep, out * in^2."""
    return float(out_f) * float(in_f) * float(in_f)


def assign_lpt(costs, world: int):
    """Longest-processing-time assignment of jobs to ranks: jobs in decreasing cost (ties by
    index) each go to the least-loaded rank (ties by rank). Returns owner[job]."""
    order = sorted(range(len(costs)), key=lambda j: (-costs[j], j))
    load = [0.0] * world
    owner = [0] * len(costs)
    for j in order:
        r = min(range(world), key=lambda q: (load[q], q))
        owner[j] = r
        load[r] += costs[j]
    return owner


def shard_windows(n: int, world: int, rank: int):
    """Contiguous window range [a, b) of this rank (sizes differ by at most one)."""
    base, extra = divmod(n, world)
    a = rank * base + min(rank, extra)
    return a, a + base + (1 if rank < extra else 0)


def _dist():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        return dist
    return None


def combine_hessian(H, n_local: int, n_total: int, dist=None):
    """Running-mean Hessians of the shards -> the Hessian of all rows (in place)."""
    if dist is None:
        return H
    H.mul_(n_local / n_total)
    dist.all_reduce(H)
    return H


# ------------------------------------------------------------------------- builder ---

def build_database(model: QwenModel, tokens, spec: DBSpec, db_dir=None, model_sha: str = "",
                   log=print, chunk_windows: int = 8, keep: str = "host", timings=None,
                   n_streams: int = 8, hessians_out=None):
    """Quantize every linear of the first spec.n_layers layers at every option
    (database.py:158-241). tokens: int32 [N, T] calibration windows.

    Returns (manifest, results): results[(layer, name, bits)] = (codes uint8 [out, in],
    scales float32 [out, groups]) as numpy arrays (keep="host") or CUDA tensors
    (keep="device"); manifest["sensitivity"] is the [n_groups, K] float64 array. With db_dir
    the reference's files are written (manifest last, atomically). timings: optional dict
    that receives per-phase seconds. hessians_out: optional dict that receives each layer's
    site Hessians (float64 CUDA) as hessians_out[(layer, site)]."""
    tokens = np.asarray(tokens, dtype=np.int32)
    if tokens.ndim != 2 or tokens.shape[1] < 2:
        raise ValueError(f"tokens must be [N, T] with T >= 2, got {tokens.shape}")
    opts = _check_spec(spec, len(model.layers))
    dist = _dist()
    world = dist.get_world_size() if dist else 1
    rank = dist.get_rank() if dist else 0
    cfg = model.cfg
    dev = model.embed.device
    N, T = tokens.shape
    a, b = shard_windows(N, world, rank)
    n_loc = b - a
    if n_loc == 0:
        raise ValueError(f"{N} windows cannot be shared by {world} ranks")
    cs = min(chunk_windows, n_loc)
    tm = timings if timings is not None else {}
    for k in ("forward", "hessian", "factor", "sweep", "gather"):
        tm.setdefault(k, 0.0)

    def tick():
        torch.cuda.synchronize(dev)
        return time.perf_counter()

    eng = Qwen2Block(cfg, cs, T, dev)
    streams = [torch.cuda.Stream(dev) for _ in range(n_streams)]
    ids = torch.as_tensor(tokens[a:b].reshape(-1), device=dev)
    H_ = cfg.hidden
    h = torch.empty(n_loc * T, H_, device=dev, dtype=torch.bfloat16)
    h_next = torch.empty_like(h)
    _lib.call("gsq_embed", _lib.ptr(ids), ids.numel(), _lib.ptr(model.embed), H_, _lib.ptr(h),
              _lib.stream_ptr())
    m_total = N * (T - 1)

    groups = [(L, name) for L in range(spec.n_layers) for name in LINEARS]
    sens = np.zeros((len(groups), len(opts)), dtype=np.float64)
    counts = []
    results = {}
    db = None
    if db_dir is not None and rank == 0:
        db = Path(db_dir)
        db.mkdir(parents=True, exist_ok=True)
        (db / ".gitignore").write_text("*\n")

    for L in range(spec.n_layers):
        t0 = tick()
        W = BlockWeights(model.layers[L])
        Hs = {s: torch.zeros(cfg.inter if s == "down" else H_, cfg.inter if s == "down" else H_,
                             device=dev, dtype=torch.float64) for s in SITES}
        n = {s: 0 for s in SITES}
        th = 0.0
        for c0 in range(0, n_loc, cs):
            s_ = min(cs, n_loc - c0)
            rows = slice(c0 * T, (c0 + s_) * T)
            eng.forward(h[rows], W, S=s_, out=h_next[rows], taps=tuple(TAP_OF_SITE.values()))
            t1 = time.perf_counter()
            for site in SITES:
                n[site] = eng.hessian_add(TAP_OF_SITE[site], Hs[site], n[site], S=s_)
            th += time.perf_counter() - t1
        for site in SITES:
            combine_hessian(Hs[site], n[site], m_total, dist)
            if hessians_out is not None:
                hessians_out[(L, site)] = Hs[site].clone()
        t2 = tick()
        tm["forward"] += t2 - t0 - th
        tm["hessian"] += th
        h, h_next = h_next, h

        # solves: (linear, option) jobs by LPT over the ranks
        jobs = [(name, bits) for name in LINEARS for bits in opts]
        shapes = {name: tuple(model.layers[L][name].shape) for name in LINEARS}
        owner = assign_lpt([solve_cost(*shapes[nm]) for nm, _ in jobs], world)
        mine = [j for j, r in enumerate(owner) if r == rank]
        factors = {}
        local = {}
        t3 = tick()
        for site in sorted({SITE_OF[jobs[j][0]] for j in mine}, key=SITES.index):
            factors[site] = gptq_factor(Hs[site], spec.damp)
        t4 = tick()
        tm["factor"] += t4 - t3
        # the solves of the layer are independent once their factor exists: round-robin over a
        # pool of streams so that the small ones (k / v: 128 rows) run beside the large ones
        main = torch.cuda.current_stream(dev)
        for q in streams:
            q.wait_stream(main)
        for n_j, j in enumerate(mine):
            name, bits = jobs[j]
            site = SITE_OF[name]
            with torch.cuda.stream(streams[n_j % len(streams)]):
                Wf = model.layers[L][name].float()
                local[j] = quantize_gptq(Wf, Hs[site], bits, spec.group_size, spec.damp,
                                         device=True, factor=factors[site])
        for q in streams:
            main.wait_stream(q)
        tm["sweep"] += tick() - t4
        for name in LINEARS:
            counts.append(int(model.layers[L][name].numel()))
        t4 = tick()
        for j, (name, bits) in enumerate(jobs):
            i = L * len(LINEARS) + LINEARS.index(name)
            k = opts.index(bits)
            out_f, in_f = shapes[name]
            G = -(-in_f // spec.group_size)
            if owner[j] == rank:
                codes, scales, err = local[j]["codes"], local[j]["scales"], local[j]["err"]
            else:
                codes = torch.empty(out_f, in_f, device=dev, dtype=torch.uint8)
                scales = torch.empty(out_f, G, device=dev, dtype=torch.float32)
                err = torch.zeros((), device=dev, dtype=torch.float64)
            if dist is not None:
                dist.broadcast(codes, owner[j])
                dist.broadcast(scales, owner[j])
                err = err.reshape(1)
                dist.broadcast(err, owner[j])
            sens[i, k] = float(err.reshape(-1)[0].item())
            if keep == "host" or db is not None:
                c_h, s_h = codes.cpu().numpy(), scales.cpu().numpy()
                if db is not None:
                    np.save(db / _name(L, name, bits, "codes"), c_h)
                    np.save(db / _name(L, name, bits, "scales"), s_h)
                results[(L, name, bits)] = (c_h, s_h) if keep == "host" else (codes, scales)
            else:
                results[(L, name, bits)] = (codes, scales)
        tm["gather"] += tick() - t4
        del Hs, factors, local
        log(f"[build-db] layer {L:2d}: {len(jobs)} solves ({len(mine)} on rank {rank})")

    manifest = identity(spec, model_sha, tokens)
    manifest.update({"counts": counts,
                     "groups": [f"{L}.{name}" for L, name in groups],
                     "sensitivity_file": "sensitivity.npy"})
    if db is not None:
        np.save(db / "sensitivity.npy", sens)
        tmp = db / "manifest.json.tmp"
        tmp.write_text(json.dumps(manifest, indent=1))
        os.replace(tmp, db / "manifest.json")
    manifest["sensitivity"] = sens
    return manifest, results


def random_model(n_layers=24, seed=0, device=None, cfg: BlockConfig = None, vocab=151936):
    """A random-init Qwen2.5-0.5B-architecture stack: bf16 weights N(0, 0.02^2) drawn layer by
    layer in a fixed order (torch CPU generator), unit norms, a tied embedding."""
    cfg = cfg or BlockConfig()
    dev = device or _lib.device()
    g = torch.Generator(device="cpu").manual_seed(seed)
    H, I, nh, nkv, hd = cfg.hidden, cfg.inter, cfg.n_heads, cfg.n_kv, cfg.head_dim
    embed = (0.02 * torch.randn(vocab, H, generator=g)).bfloat16().to(dev)
    shapes = {"q_proj": (nh * hd, H), "k_proj": (nkv * hd, H), "v_proj": (nkv * hd, H),
              "o_proj": (H, nh * hd), "gate_proj": (I, H), "up_proj": (I, H),
              "down_proj": (H, I), "q_bias": (nh * hd,), "k_bias": (nkv * hd,),
              "v_bias": (nkv * hd,)}
    layers = []
    for _ in range(n_layers):
        W = {k: (0.02 * torch.randn(*s, generator=g)).bfloat16().to(dev) for k, s in shapes.items()}
        W["in_norm"] = torch.ones(H, dtype=torch.bfloat16, device=dev)
        W["post_norm"] = torch.ones(H, dtype=torch.bfloat16, device=dev)
        layers.append(W)
    return QwenModel(cfg, embed, layers, torch.ones(H, dtype=torch.bfloat16, device=dev))
