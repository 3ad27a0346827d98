"""Block-by-block GSQ quantization of a whole decoder stack on the GPU.

Reference: src/gsq_rco/gsq/pipeline.py:32-174 (run_quantize without its CLI): every block is
trained on the quantized prefix x_q against the FP block applied to x_q (gsq.staged
quantize_block), then x_q <- Q_block(x_q), so each block runs once per stream. One shard per
block, layer_XX.npz, in the reference's format (pipeline.py:88-108): per linear
`<name>.codes` uint8, `<name>.scales` float16, `<name>.bits`, and the JSON `meta` (layer,
fingerprint, bits) and `stats`. resume=True replays finished blocks from their shards (checked
against the fingerprint), so no block is skipped in the stream.

The calibration stream stays in HBM ([N*T, H] bf16: 470 MB for 128 x 2048 tokens); the block
loop is sequential by construction (block i+1 trains on block i's quantized output). Under a
DataParallel each rank computes its position windows of every stage step (quantize_block), and
the stream advance is sharded by sequences with one all-gather per block.
"""
from __future__ import annotations

import json
import os
import time

import numpy as np
import torch

from .. import _lib
from .e2e import LIN_ORDER, BlockConfig, BlockWeights, Qwen2Block
from .export import export_mlx_lm, module_path
from .staged import BlockOpts, DataParallel, _hard_bf16, quantize_block


def fingerprint(opts: BlockOpts, n_cal: int, seq_len: int, cal_seed: int = 0,
                model: str = "Qwen2.5-0.5B") -> dict:
    """Settings that must match for shards to be reused on resume (pipeline.py:64-71)."""
    from .lion import LR_SCALES, SCALE_LR_RULE
    return {"model": model, "group_size": opts.group_size, "damp": opts.damp,
            "block_size": opts.block_size, "steps": opts.steps,
            "micro_batch": opts.micro_batch, "resamples": opts.resamples,
            "lr_logits": opts.lr_logits, "lr_scales": LR_SCALES,
            "scale_lr_rule": SCALE_LR_RULE, "seed": opts.seed, "n_cal": n_cal,
            "seq_len": seq_len, "cal_seed": cal_seed}


def load_bits(layers, alloc=None, uniform_bits=None) -> dict:
    """{layer: {linear: bits}} from an allocation ({"per_linear_bits": {"<layer>.<linear>": b}}
    or {"per_layer_bits": {"<layer>": b}}) or one uniform width (pipeline.py:32-61)."""
    layers = list(layers)
    if (alloc is None) == (uniform_bits is None):
        raise ValueError("give exactly one of alloc and uniform_bits")
    if uniform_bits is not None:
        per = {(i, n): int(uniform_bits) for i in layers for n in LIN_ORDER}
    elif "per_linear_bits" in alloc:
        per = {}
        for key, b in alloc["per_linear_bits"].items():
            i, name = key.split(".", 1)
            per[(int(i), name)] = int(b)
    elif "per_layer_bits" in alloc:
        per = {(i, n): int(alloc["per_layer_bits"][str(i)]) for i in layers for n in LIN_ORDER}
    else:
        raise ValueError("allocation needs per_linear_bits or per_layer_bits")
    out = {}
    for i in layers:
        missing = [n for n in LIN_ORDER if (i, n) not in per]
        if missing:
            raise ValueError(f"layer {i} has no bits for {missing}")
        out[i] = {n: per[(i, n)] for n in LIN_ORDER}
        for n, b in out[i].items():
            if not 1 <= b <= 8:
                raise ValueError(f"layer {i} {n}: bits {b} outside 1..8")
    return out


def save_shard(path: str, layer: int, lins: dict, bits: dict, fp: dict, stats: dict) -> None:
    """One block's stored form (pipeline.py:88-99), written atomically."""
    arrays = {"meta": np.array(json.dumps({"layer": layer, "fingerprint": fp, "bits": bits})),
              "stats": np.array(json.dumps(stats))}
    for name, q in lins.items():
        arrays[f"{name}.codes"] = np.asarray(q["codes"], dtype=np.uint8)
        arrays[f"{name}.scales"] = np.asarray(q["scales"], dtype=np.float16)
        arrays[f"{name}.bits"] = np.array(int(q["bits"]))
    tmp = path + ".tmp.npz"
    np.savez_compressed(tmp, **arrays)
    os.replace(tmp, path)


def load_shard(path: str):
    """-> (meta dict, stats dict, {linear: {codes, scales, bits}}) (pipeline.py:102-110)."""
    with np.load(path) as z:
        meta = json.loads(str(z["meta"]))
        stats = json.loads(str(z["stats"]))
        lins = {n: {"codes": z[f"{n}.codes"], "scales": z[f"{n}.scales"],
                    "bits": int(z[f"{n}.bits"])} for n in LIN_ORDER}
    return meta, stats, lins


def hard_block(lins: dict, base: dict, group_size: int = 64) -> dict:
    """bf16 CUDA weights of a quantized block from its stored form (staged.py:525-532): the
    linears dequantized with their fp16 scales; base holds the FP biases and norms."""
    W = dict(base)
    for name in LIN_ORDER:
        q = lins[name]
        codes = torch.as_tensor(np.ascontiguousarray(q["codes"])).to(_lib.device())
        W[name] = _hard_bf16(codes, q["scales"], int(q["bits"]), group_size)
    return W


def advance(eng: Qwen2Block, h, W: dict, T: int, dp: DataParallel = None):
    """h <- block(h) over every calibration sequence (staged.py:535-537): sequences sharded
    over the ranks, gathered with one all-gather. h: bf16 CUDA [N*T, H], updated in place."""
    dp = dp or DataParallel()
    N = h.shape[0] // T
    Wb = BlockWeights(W)
    per = -(-N // dp.world)
    a, b = min(N, dp.rank * per), min(N, (dp.rank + 1) * per)
    out = torch.empty(per * T, h.shape[1], device=h.device, dtype=h.dtype)
    for s0 in range(a, b, eng.S):
        s = min(eng.S, b - s0)
        eng.forward(h[s0 * T:(s0 + s) * T], Wb, S=s, out=out[(s0 - a) * T:(s0 - a + s) * T])
    if dp.dist is None:
        h.copy_(out[:N * T])
        return h
    full = torch.empty(dp.world * per * T, h.shape[1], device=h.device, dtype=h.dtype)
    dp.dist.all_gather_into_tensor(full, out, group=dp.group)
    h.copy_(full[:N * T])
    return h


def quantize_model(model, cal_tokens, bits_by_layer: dict, opts: BlockOpts, out_dir: str,
                   resume: bool = False, dp: DataParallel = None, cal_seed: int = 0,
                   log=print) -> dict:
    """Quantize the blocks listed in bits_by_layer along the calibration stream of cal_tokens
    int [N, T] (pipeline.py:120-174); blocks not listed stay FP in the stream. Writes
    out_dir/layer_XX.npz (rank 0) and returns {"layers": {i: stats}, "seconds": total}."""
    dp = dp or DataParallel()
    cal = np.asarray(cal_tokens, dtype=np.int32)
    N, T = cal.shape
    cfg = model.cfg
    os.makedirs(out_dir, exist_ok=True)
    fp = fingerprint(opts, N, T, cal_seed)
    shard_path = lambda i: os.path.join(out_dir, f"layer_{i:02d}.npz")
    layers = sorted(bits_by_layer)
    done = {i for i in layers if os.path.exists(shard_path(i))}
    if done and not resume:
        raise FileExistsError(f"{len(done)} shard(s) already in {out_dir}: pass resume=True")
    for i in sorted(done):
        meta = load_shard(shard_path(i))[0]
        if meta["fingerprint"] != fp or {k: int(v) for k, v in meta["bits"].items()} != \
                bits_by_layer[i]:
            raise ValueError(f"{shard_path(i)} was made with other settings")
    t_all = time.perf_counter()
    dev = model.embed.device
    ids = torch.as_tensor(cal.reshape(-1)).to(dev)
    h = torch.empty(N * T, cfg.hidden, device=dev, dtype=torch.bfloat16)
    _lib.call("gsq_embed", _lib.ptr(ids), N * T, _lib.ptr(model.embed), cfg.hidden, _lib.ptr(h),
              _lib.stream_ptr())
    eng = Qwen2Block(cfg, min(8, N), T, dev)
    stats_all = {}
    for i, Wfp in enumerate(model.layers):
        t0 = time.perf_counter()
        if i not in bits_by_layer:
            Wq = Wfp
        elif i in done:
            _, stats, lins = load_shard(shard_path(i))
            Wq = hard_block(lins, {k: Wfp[k] for k in Wfp if k not in LIN_ORDER},
                            opts.group_size)
            stats_all[i] = stats
            log(f"layer {i}: replayed from {shard_path(i)}")
        else:
            shard, stats, Wq = quantize_block(h, Wfp, bits_by_layer[i], opts, i, cfg=cfg, T=T,
                                              log=lambda *a: None, dp=dp)
            torch.cuda.synchronize()
            stats["seconds"] = round(time.perf_counter() - t0, 3)
            if dp.rank == 0:
                save_shard(shard_path(i), i, shard, bits_by_layer[i], fp, stats)
            stats_all[i] = stats
            log(f"layer {i}: quantized in {stats['seconds']:.2f}s")
        advance(eng, h, Wq, T, dp)
    torch.cuda.synchronize()
    if dp.dist is not None:
        dp.dist.barrier(group=dp.group)
    return {"layers": stats_all, "seconds": round(time.perf_counter() - t_all, 3)}


def finetune_shards(model, out_dir: str, layers, cal_tokens, steps: int, group_size: int = 64,
                    log=print) -> dict:
    """App-H on the written shards (pipeline.py:176-206): the group scales of every quantized
    block fine-tuned end to end (gsq.finetune.scale_finetune, one calibration sequence per step)
    and written back into the shards with the KL of the first and last steps in their stats."""
    from .finetune import scale_finetune
    from .lion import LR_SCALES
    t0 = time.perf_counter()
    shard_path = lambda i: os.path.join(out_dir, f"layer_{i:02d}.npz")
    shards = {i: load_shard(shard_path(i)) for i in layers}
    qblocks = {i: lins for i, (_, _, lins) in shards.items()}
    new, kls = scale_finetune(model, qblocks, cal_tokens, steps, LR_SCALES, group_size, log)
    w = max(1, min(10, len(kls) // 2))  # averaging window: at most half the steps
    summary = {"steps": steps, "window": w, "kl_first": float(np.mean(kls[:w])),
               "kl_last": float(np.mean(kls[-w:]))}
    for i, (meta, stats, lins) in shards.items():
        for name in LIN_ORDER:
            lins[name]["scales"] = new[i][name]
        stats["scale_finetune"] = dict(summary)
        save_shard(shard_path(i), i, lins, {k: int(v) for k, v in meta["bits"].items()},
                   meta["fingerprint"], stats)
    summary["seconds"] = round(time.perf_counter() - t0, 1)
    return summary


def export_quantized(out_dir: str, base_dir: str, layers, group_size: int = 64,
                     scale_dtype: str = "bfloat16") -> str:
    """The mlx-lm checkpoint of the quantized blocks' shards (pipeline.py:256-266 with
    export.py:137-215): out_dir/mlx next to the shards."""
    quantized = {}
    for i in layers:
        _, _, lins = load_shard(os.path.join(out_dir, f"layer_{i:02d}.npz"))
        for name in LIN_ORDER:
            q = lins[name]
            quantized[module_path(i, name)] = dict(
                codes=q["codes"], scales=q["scales"].astype(np.float32), bits=q["bits"],
                group_size=group_size)
    return export_mlx_lm(os.path.join(out_dir, "mlx"), quantized, base_dir, scale_dtype)
