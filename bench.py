"""Benchmark of the GSQ hot path on B200 (one JSON line on rank 0).

Workload "block" (default; the metric's "GSQ steps/s per block"): one random-init
Qwen2.5-0.5B-architecture decoder block (hidden 896, 14 q / 2 kv heads of 64, SwiGLU 4864,
RMSNorm eps 1e-6, RoPE theta 1e6, bf16 weights ~ N(0, 0.02^2), unit norms), calibration 128
sequences x 2048 uniform-random token ids over vocab 151936 through a random-init bf16
embedding. GPTQ 3-bit group-64 warm start, then the GSQ stages qk / vo / mlp, micro-batch 2,
2 Gumbel resamples, Lion, tau 2 -> 0.05, kappa 100 -> 500. A step = one Lion step of each of the
three stages (qk + vo + mlp), so value = block steps/s. Inputs are synthetic (seeded), with the
configuration's shapes and distributions; every stage step's working set (the block's soft
weights, probabilities, momenta: > 1 GB) exceeds the 126 MB L2.

Workload "linear": one up_proj-shaped linear (W 4864 x 896, X 16384 x 896 as 32 x 512), the
qk-stage step of one linear.

Workload "gptq": GPTQ of the 168 linears of a random-init 24-layer stack at 2, 3 and 4 bits from
Hessians over 128 x 2048 tokens; value = seconds per model (lower is
better); under torchrun the windows and solves are sharded (strong scaling, NCCL all-reduce of
the Hessians).

Workload "rco": RCO allocation on the same stack and a GPTQ database at
2 / 3 / 4 bits: seconds per RCO step of 8 Gumbel samples x 32 windows x 2048 tokens (forward,
KL head, backward through 24 blocks, straight-through dots); at most 2 timed steps after 3
warm-up steps (a step takes seconds); windows sharded over ranks under torchrun.

Workload "eval": the quantized-model eval on the same stack: packed
mixed 2 / 3 / 4-bit MLX-affine linears (a 3.0-bit allocation from the GPTQ database, fp16 g64
scales), 146 windows x 2048 ids, next-token NLL; value = scored tokens per second of one pass
over all windows (each window's 8-window batch dequantizes every layer into L2-resident bf16
scratch, then runs the bf16 tensor-core forward and the head + NLL row pass).

Workload "pipeline": the full 3-bit pipeline on the stack (build-db, RCO allocate, quantize the
24 blocks on the quantized stream, export, eval), each phase timed; value = wall-clock seconds
with the allocate phase at 100 RCO steps (those of the 100 not among the --rco-steps measured
ones counted at the measured mean).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload block|linear|gptq|rco|eval|pipeline] [--rco-steps S]

N > 1 runs under torchrun, one rank per GPU. Block: the ranks quantize one block together,
data-parallel over the positions of each micro-batch sequence with one NCCL all-reduce of the
weight gradients per stage step (strong scaling). GPTQ: windows and solves sharded. --impl
reference times the CPU restatement of the same work on this host's cores (the reference's GSQ
path is MLX-only and cannot run here).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

VOCAB, HID, NH, NKV, HD, INTER = 151936, 896, 14, 2, 64, 4864
N_SEQ, T_SEQ = 128, 2048
LIN = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="block",
                    choices=["block", "linear", "gptq", "rco", "eval", "pipeline", "kernels"])
    ap.add_argument("--cases", default="",
                    help="kernels: comma-separated cases of bench_kernels.py (default all)")
    ap.add_argument("--once", action="store_true",
                    help="kernels: run each case once (for a profiler capture)")
    ap.add_argument("--rco-steps", type=int, default=2,
                    help="pipeline: RCO steps run (the rest of the 100 extrapolated)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--split", default="sequences", choices=["sequences", "positions"],
                    help="block, N > 1: each rank its own micro-batch of 2 sequences (weak "
                         "scaling; global micro-batch 2N) or the positions of one shared "
                         "micro-batch (strong scaling)")
    ap.add_argument("--no-secondary", action="store_true",
                    help="block: skip the GPTQ s/model and RCO s/step fields")
    ap.add_argument("--e2e-steps", type=int, default=200)
    return ap.parse_args()


def dist_setup():
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return rank, world, local


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = f"/tmp/.gsq_clocks_{os.getpid()}.csv"

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        try:
            os.remove(self.path)
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    return json.load(open(p)) if os.path.exists(p) else {}


# ----------------------------------------------------------------------------- block ---

def make_block(seed, dev):
    """Random-init block (bf16 N(0, 0.02^2), fixed draw order), embedding and calibration ids."""
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    shapes = {"q_proj": (NH * HD, HID), "k_proj": (NKV * HD, HID), "v_proj": (NKV * HD, HID),
              "o_proj": (HID, NH * HD), "gate_proj": (INTER, HID), "up_proj": (INTER, HID),
              "down_proj": (HID, INTER), "q_bias": (NH * HD,), "k_bias": (NKV * HD,),
              "v_bias": (NKV * HD,)}
    W = {k: (0.02 * torch.randn(*s, generator=g)).bfloat16().to(dev) for k, s in shapes.items()}
    W["in_norm"] = torch.ones(HID, dtype=torch.bfloat16, device=dev)
    W["post_norm"] = torch.ones(HID, dtype=torch.bfloat16, device=dev)
    return W


def make_calibration(dev, seed=0):
    import torch
    gen = torch.Generator(device="cpu").manual_seed(seed)
    E = (0.02 * torch.randn(VOCAB, HID, generator=gen)).bfloat16()
    ids = np.random.default_rng(seed).integers(0, VOCAB, size=(N_SEQ, T_SEQ)).astype(np.int32)
    return E, ids


def embed(E_dev, ids, dev):
    import torch
    from gsq_rco_mlx_b200 import _lib
    ids_t = torch.as_tensor(ids.reshape(-1), device=dev)
    h = torch.empty(ids.size, HID, device=dev, dtype=torch.bfloat16)
    _lib.call("gsq_embed", _lib.ptr(ids_t), ids.size, _lib.ptr(E_dev), HID, _lib.ptr(h),
              _lib.stream_ptr())
    return h


# DRAM bytes (read + write) per gemm_tc_kernel launch, mean over the four GEMMs of one mlp-stage
# resample in the ncu capture summarised in profiles/gemm_tc_mlp_stage.md (F1, F3, B1, B2 as the
# stage issues them)
GEMM_TRAFFIC_PER_LAUNCH = int(round((60 + 227 + 200 + 16 + 162 + 10 + 342 + 217) / 4 * 1e6))
GEMM_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum, mean per launch over "
                       "F1, F3, B1, B2 of one mlp-stage resample (profiles/gemm_tc_mlp_stage.md)")


def gemm_flops_of_mlp_stage(M):
    """Algorithmic (float32-equivalent) FLOPs of one mlp-stage resample: 5 GEMMs."""
    return 2 * M * (2 * INTER) * HID + 2 * M * HID * INTER * 4


def run_block(args):
    import torch
    import torch.distributed as dist
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.gemm import LaunchLog
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, DataParallel, StageTimer, quantize_block

    rank, world, local = dist_setup()
    _lib.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = BlockConfig()
    W = make_block(1000, dev)
    dp = DataParallel(split=args.split)
    E, ids = make_calibration(dev)
    E_dev = E.to(dev)
    h = embed(E_dev, ids, dev)
    del E_dev
    bits = {n: 3 for n in LIN}
    quiet = lambda *a: None

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up: a short full run (allocations, first launches)
    quantize_block(h, W, bits, BlockOpts(steps=args.warmup + 1), layer=0, cfg=cfg, T=T_SEQ,
                   log=quiet, dp=dp)
    barrier()
    clocks = Clocks(local)
    clocks.start()
    timer = StageTimer(args.warmup, nvtx=True)
    opts = BlockOpts(steps=args.warmup + args.steps)
    _, stats, _ = quantize_block(h, W, bits, opts, layer=0, cfg=cfg, T=T_SEQ, log=quiet,
                                 timer=timer, dp=dp)
    barrier()
    clk = clocks.stop()
    ms = {s: max_over_ranks(timer.ms[s]) for s in ("qk", "vo", "mlp")}
    ms_step = ms["qk"] + ms["vo"] + ms["mlp"]

    # roofline of the dominant kernel (the tensor-core GEMM): CUDA events around every GEMM
    # launch of 3 timed steps per stage (the log is active only inside the timed window), with
    # the algorithmic float32-equivalent FLOPs 2 M N K of each launch
    rl_log = LaunchLog()
    rl_steps = 3
    quantize_block(h, W, bits, BlockOpts(steps=args.warmup + rl_steps), layer=0, cfg=cfg,
                   T=T_SEQ, log=quiet, dp=dp, timer=StageTimer(args.warmup, launch_log=rl_log))
    by_stage = rl_log.by_tag()
    stage_gemm = {}
    fl = fl_exec = t_ms = 0.0
    for stage in ("qk", "vo", "mlp"):
        rows = by_stage.get(stage, [])
        f = sum(2.0 * M * N * K * b for (M, N, K, p, b, t) in rows)
        fe = sum(2.0 * M * N * K * b * p for (M, N, K, p, b, t) in rows)
        tt = max_over_ranks(sum(t for (*_, t) in rows))
        fl, fl_exec, t_ms = fl + f, fl_exec + fe, t_ms + tt
        stage_gemm[stage] = {
            "gemm_launches_per_step": len(rows) // rl_steps,
            "gemm_ms_per_step": round(tt / rl_steps, 4),
            "gemm_share_of_stage": round(tt / rl_steps / ms[stage], 3),
            "f32eq_gflop_per_step": round(f / rl_steps / 1e9, 2),
            "f32eq_tflops": round(f / (tt * 1e-3) / 1e12, 1) if tt else None,
            "executed_bf16_tflops": round(fe / (tt * 1e-3) / 1e12, 1) if tt else None}
    achieved = fl / (t_ms * 1e-3) / 1e12
    pk = peaks()
    peak = float(pk.get("bf16_tflops", 1590.0))

    if args.e2e_steps == 0:  # profiling runs: no end-to-end pass
        res = {"ms_step": ms_step, "stage_ms": ms}
        if rank == 0:
            print(json.dumps(res), flush=True)
        return
    # end to end through the public API: host calibration stream in, stored shards out
    h_host = h.cpu().pin_memory()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    h_dev = h_host.to(dev, non_blocking=True)
    shard, st2, _ = quantize_block(h_dev, W, bits, BlockOpts(steps=args.e2e_steps), layer=0,
                                   cfg=cfg, T=T_SEQ, log=quiet, dp=dp)
    e1.record()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    d2h = sum(v["codes"].nbytes + v["scales"].nbytes for v in shard.values())

    # weak scaling: a step of the N ranks trains on N micro-batches of 2 sequences, so the
    # whole job's throughput is N micro-batch steps per step time
    per_step = dp.total(1)
    value = 1000.0 / ms_step * per_step
    res = {
        "metric": "GSQ steps/s per block (Qwen2.5-0.5B block, 3-bit g64: one qk + vo + mlp Lion step)",
        "value": round(value, 3), "unit": "block steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak" if args.split == "sequences" else "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: random-init bf16 block and embedding, uniform-random token ids",
        "config": {"workload": "one Qwen2.5-0.5B block, calib 128 x 2048, micro-batch 2, R=2",
                   "stage_ms_per_step": {k: round(v, 4) for k, v in ms.items()},
                   "block_seconds_200_steps": round(e2e_ms / 1000, 3),
                   "parallelism": (f"one block, data-parallel over {world} GPU(s): each rank "
                                   "its own micro-batch of 2 sequences of one global sorted "
                                   f"draw of {2 * per_step} (value = {per_step} micro-batch "
                                   "steps per step), NCCL all-reduce of dL/dw per step")
                   if args.split == "sequences" else
                   (f"one block, data-parallel over {world} GPU(s): position windows of each "
                    "micro-batch sequence, NCCL all-reduce of dL/dw per step"),
                   "l2": "per-step working set > L2 (126 MB)"},
        "e2e": {"value": round(args.e2e_steps * per_step / (e2e_ms / 1000), 3),
                "unit": "block steps/s",
                "h2d_bytes_per_step": int(h_host.numel() * 2 / args.e2e_steps),
                "d2h_bytes_per_step": int(d2h / args.e2e_steps),
                "what": "quantize_block(200 steps per stage) from pinned host activations to "
                        "host shards, GPTQ init and hardening included"},
        "gpu_launches": None,
        "roofline": {"kernel": "gemm_tc_kernel: every launch of 3 timed block steps",
                     "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": GEMM_TRAFFIC_PER_LAUNCH,
                     "traffic_source": GEMM_TRAFFIC_SOURCE,
                     "gemm_ms_per_step": round(t_ms / rl_steps, 4),
                     "gemm_share_of_step": round(t_ms / rl_steps / ms_step, 3),
                     "executed_bf16_tflops": round(fl_exec / (t_ms * 1e-3) / 1e12, 1),
                     "executed_frac": round(fl_exec / (t_ms * 1e-3) / 1e12 / peak, 4),
                     "per_stage": stage_gemm,
                     "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
                     if "bf16_tflops" in pk else "fallback 1590 TFLOP/s",
                     "note": "achieved = float32-equivalent GEMM FLOPs 2MNK of the timed steps / "
                             "their GEMM time; the float32-faithful split engine executes 3-6 "
                             "bf16 products per float32 product (executed_bf16_tflops)"},
        "clocks": clk,
    }
    res["gpu_launches"] = int(sum(timer.launches.values()))
    if not args.no_secondary:
        del h, h_dev, h_host
        torch.cuda.empty_cache()
        res["config"].update(measure_gptq_rco(dev, world, barrier, max_over_ranks))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_block()
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measure_gptq_rco(dev, world, barrier, max_over_ranks, rco_steps=2):
    """The other two parts of the metric, measured in the same run at the same N: GPTQ seconds
    per model (the 24-layer stack at 2 / 3 / 4 bits from Hessians over 128 x 2048 tokens, after
    a one-layer warm-up) and RCO seconds per step (g = 8 samples x 32 windows x 2048 tokens on
    that database, ``rco_steps`` timed after one warm-up step). Windows, solves and samples'
    windows are sharded over the ranks as in the gptq / rco workloads; CUDA events, max over
    ranks."""
    import torch
    from gsq_rco_mlx_b200.rco.allocate import Bank, KLObjective, rco_allocate
    from gsq_rco_mlx_b200.rco.database import DBSpec, build_database, random_model
    quiet = lambda *a: None
    model = random_model(n_layers=24, seed=0, device=dev)
    tokens = np.random.default_rng(0).integers(0, VOCAB, size=(N_SEQ, T_SEQ)).astype(np.int32)
    build_database(model, tokens, DBSpec(options=GPTQ_OPTIONS, n_layers=1), log=quiet,
                   keep="device")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tm = {}
    barrier()
    e0.record()
    man, res = build_database(model, tokens, DBSpec(options=GPTQ_OPTIONS, n_layers=24),
                              log=quiet, keep="device", timings=tm)
    e1.record()
    barrier()
    gptq_s = max_over_ranks(e0.elapsed_time(e1) / 1000)
    bank = Bank(man, res)
    windows = np.random.default_rng(1).integers(0, VOCAB, size=(RCO_WINDOWS, T_SEQ)).astype(
        np.int32)
    obj = KLObjective(model, bank, windows, windows_per_sample=RCO_WIN_PER_SAMPLE, chunk_seqs=8)
    rco_allocate(obj, bank, 3.0, steps=1, g=RCO_G, lr=0.1, seed=0)
    barrier()
    e0.record()
    rco_allocate(obj, bank, 3.0, steps=rco_steps, g=RCO_G, lr=0.1, seed=1)
    e1.record()
    barrier()
    rco_s = max_over_ranks(e0.elapsed_time(e1) / 1000 / rco_steps)
    del obj, bank, man, res, model
    torch.cuda.empty_cache()
    return {"gptq_s_per_model": round(gptq_s, 3),
            "gptq_phase_seconds": {k: round(v, 3) for k, v in tm.items()},
            "rco_s_per_step": round(rco_s, 3),
            "secondary_what": "gptq_s_per_model: 24-layer GPTQ database (168 linears x {2,3,4} "
                              "bits, Hessians over 128 x 2048 tokens); rco_s_per_step: one RCO "
                              f"step of g=8 samples x 32 windows x 2048 tokens ({rco_steps} "
                              "timed after 1 warm-up); same N, CUDA events, max over ranks"}


def cpu_baseline_block(steps=1, warmup=0):
    """The CPU restatement (oracle port) of the block step in the reference's float32
    arithmetic — one Lion step each of the qk stage (q_proj, k_proj on the normed rows), the vo
    stage (v_proj, o_proj through the hard attention probabilities) and the mlp stage (gate,
    up, down) — at the configuration's micro-batch (2 sequences x 2048 positions, R = 2), on
    all of this host's cores: float32 GEMMs (torch / numpy BLAS) and the elementwise Gumbel /
    softmax / backward / Lion passes in the oracle's C backend over every core. Returns the
    block steps/s of ``steps`` timed steps after ``warmup`` untimed ones."""
    import torch
    from oracle import block as ob
    from oracle import gptq as og
    from oracle import gsq as ogsq
    torch.set_num_threads(os.cpu_count())
    prev = ogsq.set_backend("c")
    rng = np.random.default_rng(0)
    T, M = T_SEQ, 2 * (T_SEQ - 1)
    F32 = torch.float32

    def rows(shape, scale=1.0):  # exactly-bf16 float32 activations
        x = scale * rng.standard_normal(shape).astype(np.float32)
        return torch.as_tensor(x).bfloat16().float()

    def linear(out_f, in_f, i):
        W = (0.02 * rng.standard_normal((out_f, in_f))).astype(np.float32)
        r = og.quantize_rtn(W, 3, 64)
        return W, ogsq.LinearState(3, r["codes"], r["scales"].astype(np.float16), 64, seed=i,
                                   linear_id=i)

    qk = [linear(NH * HD, HID, 0), linear(NKV * HD, HID, 1)]
    hn_rows = rows((M, HID)).numpy()
    vo = [linear(NKV * HD, HID, 2)[1], linear(HID, NH * HD, 3)[1]]
    hn_seqs = [rows((T, HID)) for _ in range(2)]
    A_seqs = [rows((T, HID), 0.02) for _ in range(2)]
    bv = rows((NKV * HD,), 0.02)
    scores = 4.0 * torch.randn(NH, T, T, generator=torch.Generator().manual_seed(0))
    scores = scores.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), -torch.inf)
    P = torch.softmax(scores, dim=-1).bfloat16().float()
    del scores
    mlp = [linear(INTER, HID, 4)[1], linear(INTER, HID, 5)[1], linear(HID, INTER, 6)[1]]
    mn, h1, Y = rows((T, HID)), rows((T, HID), 0.02), rows((T, HID), 0.02)

    def block_step(t):
        tau, kappa = ogsq.gs_schedules(t, 200)
        for W, st in qk:
            noises = [st.noise(0, t, r) for r in range(2)]
            _, glog, gs, _ = ogsq.linear_loss_and_grads(hn_rows, W, st.logits, st.Ckd,
                                                        st.scales, noises, 64, tau, kappa,
                                                        gemm_dtype=np.float32)
            ogsq.lion_step(st, glog, gs)
        ob.train_vo(vo, hn_seqs, A_seqs, lambda t_, idx: [P, P], bv, 1, NH, NKV, micro_batch=2,
                    dtype=F32)
        ob.train_mlp(mlp, [mn, mn], [h1, h1], [Y, Y], 1, micro_batch=2, dtype=F32)

    try:
        for t in range(warmup):
            block_step(t)
        t0 = time.perf_counter()
        for t in range(steps):
            block_step(warmup + t)
        dt = (time.perf_counter() - t0) / steps
    finally:
        ogsq.set_backend(prev)
    return {"value": round(1.0 / dt, 5), "unit": "block steps/s",
            "cores": os.cpu_count(), "kind": "port",
            "sample": f"{steps} block step(s) (qk + vo + mlp Lion steps) at micro-batch 2 x 2048, "
                      f"R=2, after {warmup} warm-up: float32 restatement (the reference's "
                      "arithmetic; its MLX path is unavailable), all host cores"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    steps, warmup = max(3, min(args.steps, 5)), 1
    cb = cpu_baseline_block(steps=steps, warmup=warmup)
    v = cb["value"]
    res = {"impl": "reference",
           "metric": "GSQ steps/s per block (Qwen2.5-0.5B block, 3-bit g64: one qk + vo + mlp Lion step)",
           "value": round(v, 5), "unit": "block steps/s", "n_gpus": world, "steps": steps,
           "warmup": warmup, "ms_per_step": round(1000 / v, 1), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "one Qwen2.5-0.5B block, calib 128 x 2048, micro-batch 2, R=2"},
           "cpu_baseline": cb,
           "e2e": {"value": round(v, 5), "unit": "block steps/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


# ------------------------------------------------------------------------------ gptq ---

GPTQ_OPTIONS = (2, 3, 4)


def run_gptq(args):
    """Config 3: GPTQ of every linear of a random-init 24-layer Qwen2.5-0.5B stack at 2, 3 and 4
    bits (504 solves) from Hessians over 128 x 2048 uniform-random tokens. A step is one full
    build (Hessian forward of 24 layers + 504 solves); the metric is seconds per model. Under
    torchrun the windows and the solves are shared over the ranks (strong scaling)."""
    import torch
    import torch.distributed as dist
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.rco.database import DBSpec, build_database, random_model

    rank, world, local = dist_setup()
    _lib.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n_layers = 24
    model = random_model(n_layers=n_layers, seed=0, device=dev)
    tokens = np.random.default_rng(0).integers(0, VOCAB, size=(N_SEQ, T_SEQ)).astype(np.int32)
    quiet = lambda *a: None

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up: one layer (allocations, first launches)
    for _ in range(max(1, args.warmup)):
        build_database(model, tokens, DBSpec(options=GPTQ_OPTIONS, n_layers=1), log=quiet,
                       keep="device")
    barrier()
    clocks = Clocks(local)
    clocks.start()
    tm = {}
    n0 = _lib.Launches.n
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(max(1, args.steps)):
        barrier()
        e0.record()
        man, res = build_database(model, tokens, DBSpec(options=GPTQ_OPTIONS, n_layers=n_layers),
                                  log=quiet, keep="device", timings=tm)
        e1.record()
        barrier()
        times.append(max_over_ranks(e0.elapsed_time(e1) / 1000))
    clk = clocks.stop()
    launches = (_lib.Launches.n - n0) // max(1, args.steps)
    sec = statistics.median(times)
    # end to end: host tokens in, host codes / scales / sensitivities out
    barrier()
    t0 = time.perf_counter()
    man, res = build_database(model, tokens, DBSpec(options=GPTQ_OPTIONS, n_layers=n_layers),
                              log=quiet, keep="host")
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    d2h = sum(c.nbytes + sc.nbytes for c, sc in res.values())
    steps = max(1, args.steps)
    phase = {k: round(v / steps, 3) for k, v in tm.items()}
    out = {
        "metric": "GPTQ s/model (24-layer Qwen2.5-0.5B architecture, 168 linears x {2,3,4} bits, "
                  "Hessians over 128 x 2048 tokens)",
        "value": round(sec, 3), "unit": "s/model", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(sec * 1000, 1), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64 solves, bf16/f32 Hessians",
        "data": "synthetic: random-init bf16 24-layer stack, uniform-random token ids",
        "config": {"workload": "24-layer GPTQ, options (2, 3, 4), g64, damp 0.01",
                   "phase_seconds_per_model": phase,
                   "parallelism": f"windows and solves sharded over {world} rank(s)",
                   "l2": "per-layer working set (470 MB of hidden states) > L2"},
        "e2e": {"value": round(e2e_s, 3), "unit": "s/model",
                "h2d_bytes_per_step": int(tokens.nbytes), "d2h_bytes_per_step": int(d2h),
                "what": "build_database from host token ids to host codes, scales, sensitivities"},
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline_gptq()
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline_gptq():
    """The numpy restatement of the reference GPTQ (float64, the reference's own CPU path) on a
    bounded sample: one solve of each distinct shape at 3 bits on this host's cores, scaled to
    the 504 solves of the model (the Hessian forward is not included: a lower bound)."""
    from oracle import gptq as og
    rng = np.random.default_rng(0)
    per_shape = {}
    for (o, i) in ((HID, HID), (NKV * HD, HID), (INTER, HID), (HID, INTER)):
        X = rng.standard_normal((4096, i)).astype(np.float32)
        H = 2.0 * (X.astype(np.float64).T @ X.astype(np.float64)) / X.shape[0]
        W = (0.02 * rng.standard_normal((o, i))).astype(np.float32)
        t0 = time.perf_counter()
        og.quantize_gptq(W, H, 3, 64, 0.01)
        per_shape[(o, i)] = time.perf_counter() - t0
    per_layer = (2 * per_shape[(HID, HID)] + 2 * per_shape[(NKV * HD, HID)] +
                 2 * per_shape[(INTER, HID)] + per_shape[(HID, INTER)])
    total = per_layer * len(GPTQ_OPTIONS) * 24
    return {"value": round(total, 1), "unit": "s/model (solves only, lower bound)",
            "cores": os.cpu_count(), "kind": "port",
            "sample": "one 3-bit solve per distinct linear shape (q/o, k/v, gate/up, down) with "
                      "H from 4096 rows, scaled to 24 layers x 7 linears x 3 options"}


def run_reference_gptq(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cb = cpu_baseline_gptq()
    res = {"impl": "reference",
           "metric": "GPTQ s/model (24-layer Qwen2.5-0.5B architecture, 168 linears x {2,3,4} bits, "
                     "Hessians over 128 x 2048 tokens)",
           "value": cb["value"], "unit": "s/model", "n_gpus": world, "steps": 1, "warmup": 0,
           "ms_per_step": round(cb["value"] * 1000, 1), "higher_is_better": False,
           "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
           "config": {"workload": "24-layer GPTQ, options (2, 3, 4), g64, damp 0.01"},
           "cpu_baseline": cb,
           "e2e": {"value": cb["value"], "unit": "s/model", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


# ------------------------------------------------------------------------------- rco ---

RCO_G, RCO_WINDOWS, RCO_WIN_PER_SAMPLE = 8, 32, 32


def rco_setup(dev):
    from gsq_rco_mlx_b200.rco.allocate import Bank, KLObjective
    from gsq_rco_mlx_b200.rco.database import DBSpec, build_database, random_model
    model = random_model(n_layers=24, seed=0, device=dev)
    calib = np.random.default_rng(0).integers(0, VOCAB, size=(N_SEQ, T_SEQ)).astype(np.int32)
    man, res = build_database(model, calib, DBSpec(options=GPTQ_OPTIONS, n_layers=24),
                              log=lambda *a: None, keep="device")
    windows = np.random.default_rng(1).integers(0, VOCAB, size=(RCO_WINDOWS, T_SEQ)).astype(
        np.int32)
    return model, Bank(man, res), windows, KLObjective


def run_rco(args):
    """Config 4: RCO allocation on the 24-layer stack (options 2 / 3 / 4, 3.0 bits exactly),
    g = 8 Gumbel samples per step, each the mean token KL over 32 windows x 2048 with its
    straight-through upstream (forward and backward through the 24 blocks). A step is one RCO
    step (8 samples + DP + manifold Adam); the metric is seconds per step. Under torchrun each
    sample's windows are shared over the ranks (one all-reduce of the upstream per sample)."""
    import torch
    import torch.distributed as dist
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.rco.allocate import rco_allocate

    rank, world, local = dist_setup()
    _lib.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    steps, warmup = max(1, min(args.steps, 2)), max(3, min(args.warmup, 3))
    model, bank, windows, KLObjective = rco_setup(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    t_init = time.perf_counter()
    obj = KLObjective(model, bank, windows, windows_per_sample=RCO_WIN_PER_SAMPLE, chunk_seqs=8)
    barrier()
    t_init = time.perf_counter() - t_init
    rco_allocate(obj, bank, 3.0, steps=warmup, g=RCO_G, lr=0.1, seed=0)
    barrier()
    clocks = Clocks(local)
    clocks.start()
    n0 = _lib.Launches.n
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    t0 = time.perf_counter()
    e0.record()
    res = rco_allocate(obj, bank, 3.0, steps=steps, g=RCO_G, lr=0.1, seed=1)
    e1.record()
    barrier()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    sec = max_over_ranks(e0.elapsed_time(e1) / 1000 / steps)
    launches = (_lib.Launches.n - n0) // steps
    e2e = max_over_ranks((t_init + wall) / steps)
    out = {
        "metric": "RCO s per step (24-layer Qwen2.5-0.5B architecture, options {2,3,4}, 3.0 bits, "
                  "g=8 samples x 32 windows x 2048 tokens)",
        "value": round(sec, 3), "unit": "s/step", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(sec * 1000, 1), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 model, f32/f64 objective",
        "data": "synthetic: random-init 24-layer stack, uniform-random token windows",
        "config": {"workload": "RCO allocation, windows_per_sample 32, g 8, Adam lr 0.1",
                   "decoded_avg_bits": res["decoded_avg_bits"],
                   "parallelism": f"windows of each sample sharded over {world} rank(s)",
                   "l2": "25 decoder states of 32 x 2048 tokens (3 GB) > L2"},
        "e2e": {"value": round(e2e, 3), "unit": "s/step",
                "h2d_bytes_per_step": int(RCO_G * RCO_WIN_PER_SAMPLE * T_SEQ * 4),
                "d2h_bytes_per_step": int(RCO_G * 168 * len(GPTQ_OPTIONS) * 8),
                "what": "KLObjective construction (reference states) amortised over the steps, "
                        "plus rco_allocate steps from host token windows to the host allocation"},
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline_rco()
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline_rco():
    """The CPU restatement of the objective (oracle.block / oracle.block_vjp / oracle.kl) on a
    bounded sample: one window of 2048 tokens forward + backward through 2 blocks plus its KL
    head, scaled to 24 blocks x 32 windows x 8 samples per step."""
    import torch
    from oracle import block as ob
    from oracle import block_vjp as ov
    from oracle import kl as okl
    torch.set_num_threads(os.cpu_count())
    g = torch.Generator().manual_seed(0)
    W = {"q_proj": (NH * HD, HID), "k_proj": (NKV * HD, HID), "v_proj": (NKV * HD, HID),
         "o_proj": (HID, NH * HD), "gate_proj": (INTER, HID), "up_proj": (INTER, HID),
         "down_proj": (HID, INTER), "q_bias": (NH * HD,), "k_bias": (NKV * HD,),
         "v_bias": (NKV * HD,)}
    W = {k: (0.02 * torch.randn(*s, generator=g)).bfloat16().float() for k, s in W.items()}
    W["in_norm"] = torch.ones(HID)
    W["post_norm"] = torch.ones(HID)
    h = (0.02 * torch.randn(T_SEQ, HID, generator=g)).bfloat16().float()
    t0 = time.perf_counter()
    x = h
    for _ in range(2):
        x = ob.block_hard(x, W)[0]
    cot = (1e-3 * torch.randn(T_SEQ, HID, generator=g)).bfloat16().float()
    for _ in range(2):
        cot = ov.block_vjp(h, W, cot)[0]
    t_blocks = time.perf_counter() - t0
    E = (0.02 * torch.randn(VOCAB // 16, HID, generator=g)).bfloat16().double()
    t0 = time.perf_counter()
    okl.kl_chunk_value_grad(x[:512].double(), h[:512].double(), E)
    t_head = (time.perf_counter() - t0) * 16 * (T_SEQ / 512)
    per_window = t_blocks * 12 + t_head
    total = per_window * RCO_WIN_PER_SAMPLE * RCO_G
    return {"value": round(total, 1), "unit": "s/step (extrapolated)", "cores": os.cpu_count(),
            "kind": "port",
            "sample": "one 2048-token window forward + backward through 2 blocks (x12 for 24) "
                      "and 512 rows of the KL head over 1/16 of the vocabulary (scaled), "
                      "x 32 windows x 8 samples"}


def run_reference_rco(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cb = cpu_baseline_rco()
    res = {"impl": "reference",
           "metric": "RCO s per step (24-layer Qwen2.5-0.5B architecture, options {2,3,4}, 3.0 "
                     "bits, g=8 samples x 32 windows x 2048 tokens)",
           "value": cb["value"], "unit": "s/step", "n_gpus": world, "steps": 1, "warmup": 0,
           "ms_per_step": round(cb["value"] * 1000, 1), "higher_is_better": False,
           "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
           "config": {"workload": "RCO allocation, windows_per_sample 32, g 8"},
           "cpu_baseline": cb,
           "e2e": {"value": cb["value"], "unit": "s/step", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


# ------------------------------------------------------------------------------ eval ---

EVAL_WINDOWS, EVAL_CHUNK = 146, 8


def eval_setup(dev):
    """The 24-layer stack, its GPTQ database at 2 / 3 / 4 bits (fp16-rounded scales as the
    shards store them), a mixed allocation at exactly 3.0 bits (the DP on the database's
    sensitivities) packed into MLX affine words, and 146 windows of 2048 ids (seed 2)."""
    import torch
    from gsq_rco_mlx_b200.common.evaluate import PackedModel
    from gsq_rco_mlx_b200.gsq.export import module_path
    from gsq_rco_mlx_b200.rco.allocate import Bank, decoded_cost, proxy_dp_choice
    from gsq_rco_mlx_b200.rco.database import DBSpec, build_database, random_model
    model = random_model(n_layers=24, seed=0, device=dev)
    calib = np.random.default_rng(0).integers(0, VOCAB, size=(N_SEQ, T_SEQ)).astype(np.int32)
    man, res = build_database(model, calib, DBSpec(options=GPTQ_OPTIONS, n_layers=24),
                              log=lambda *a: None, keep="device")
    bank = Bank(man, res)
    choice = proxy_dp_choice(bank, 3.0)
    quantized = {}
    for i, (L, name) in enumerate(bank.groups):
        codes, scales, bits = bank.cands(i)[int(choice[i])]
        quantized[module_path(L, name)] = dict(
            codes=codes.cpu().numpy(),
            scales=scales.cpu().numpy().astype(np.float16).astype(np.float32),
            bits=int(bits), group_size=64)
    pm = PackedModel.from_quantized(model, quantized, scale_dtype="float16")
    windows = np.random.default_rng(2).integers(0, VOCAB, size=(EVAL_WINDOWS, T_SEQ)).astype(
        np.int32)
    hist = {b: int(sum(1 for q in quantized.values() if q["bits"] == b)) for b in GPTQ_OPTIONS}
    info = {"bits_histogram": hist, "avg_bits": round(decoded_cost(bank, choice)[1], 4),
            "packed_mb": round(pm.packed_bytes() / 1e6, 1)}
    return pm, windows, info


def eval_flops_per_token(T):
    """Algorithmic FLOPs per scored token: the 168 linears, the causal attention (q k^T and
    P v over the average T / 2 keys), the tied head."""
    lin = 2 * 24 * (HID * (NH + 2 * NKV) * HD + HID * NH * HD + 3 * HID * INTER)
    attn = 24 * 2 * 2 * (T / 2) * HD * NH
    head = 2 * HID * VOCAB
    return lin + attn + head


def run_eval(args):
    """Config 5: the quantized-model eval: packed mixed 2 / 3 / 4-bit linears (fp16 group-64
    scales), 146 windows x 2048 ids, next-token NLL. A step is one pass over all 146 windows;
    the metric is scored tokens per second. Under torchrun the windows are sharded over the
    ranks with one all-reduce of the NLL sum."""
    import torch
    import torch.distributed as dist
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.common.evaluate import Evaluator, perplexity
    from gsq_rco_mlx_b200.gemm import LaunchLog
    from gsq_rco_mlx_b200.gsq.staged import DataParallel

    rank, world, local = dist_setup()
    _lib.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    steps, warmup = max(1, min(args.steps, 5)), max(3, min(args.warmup, 5))
    pm, windows, info = eval_setup(dev)
    dp = DataParallel()
    ev = Evaluator(pm, T_SEQ, EVAL_CHUNK)
    a, b = dp.share(0, EVAL_WINDOWS)
    # device-resident windows of this rank (the timed step reads no host memory)
    mine = windows[a:b]
    tok = torch.as_tensor(mine.reshape(-1)).to(dev)
    tgt_h = np.full(mine.shape, -1, dtype=np.int32)
    tgt_h[:, :-1] = mine[:, 1:]
    tgt = torch.as_tensor(tgt_h.reshape(-1)).to(dev)
    n_b = -(-(b - a) // EVAL_CHUNK)
    sums = torch.zeros(max(1, n_b), device=dev, dtype=torch.float64)
    total = torch.zeros(1, device=dev, dtype=torch.float64)

    def step():
        for j in range(n_b):
            w0, w1 = j * EVAL_CHUNK, min(b - a, (j + 1) * EVAL_CHUNK)
            ev.forward_nll(tok[w0 * T_SEQ:w1 * T_SEQ], tgt[w0 * T_SEQ:w1 * T_SEQ], w1 - w0,
                           sums[j:j + 1])
        _lib.call("gsq_sum_f64", _lib.ptr(sums), n_b, _lib.ptr(total), _lib.stream_ptr())
        dp.allreduce(total)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(warmup):
        step()
    barrier()
    clocks = Clocks(local)
    clocks.start()
    n0 = _lib.Launches.n
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    barrier()
    clk = clocks.stop()
    sec = max_over_ranks(e0.elapsed_time(e1) / 1000 / steps)
    launches = (_lib.Launches.n - n0) // steps
    nll = float(total.item()) / (EVAL_WINDOWS * (T_SEQ - 1))
    n_tok = EVAL_WINDOWS * (T_SEQ - 1)

    # roofline of the dominant kernel (the tensor-core GEMM) over one batch's launches
    with LaunchLog() as log:
        ev.forward_nll(tok[:EVAL_CHUNK * T_SEQ], tgt[:EVAL_CHUNK * T_SEQ],
                       min(EVAL_CHUNK, b - a), sums[:1])
    rows = log.summary()
    fl = sum(2.0 * M * N * K * bt for (M, N, K, p, bt, t) in rows)
    t_ms = sum(t for (*_, t) in rows)
    pk = peaks()
    peak = float(pk.get("bf16_tflops", 1590.0))
    achieved = fl / (t_ms * 1e-3) / 1e12

    # end to end through the public API: host windows in, the perplexity dict out
    barrier()
    t0 = time.perf_counter()
    r = perplexity(pm, windows, chunk_seqs=EVAL_CHUNK, dp=dp, evaluator=ev)
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    out = {
        "metric": "eval tokens/s (24-layer Qwen2.5-0.5B architecture, packed mixed 2/3/4-bit "
                  "g64 fp16 scales, 146 x 2048 windows, next-token NLL)",
        "value": round(n_tok / sec, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(sec * 1000, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init 24-layer stack, GPTQ database, uniform-random windows",
        "config": {"workload": "packed-model eval, 146 windows x 2048",
                   **info, "nll_per_token": round(nll, 6), "windows_per_batch": EVAL_CHUNK,
                   "parallelism": f"windows sharded over {world} rank(s), NCCL all-reduce of "
                                  "the NLL sum",
                   "l2": "per-batch activations (8 x 2048 x 896 bf16 per state, logits "
                         "1024 x 151936) > L2",
                   "algorithmic_tflops": round(eval_flops_per_token(T_SEQ) * n_tok / sec / 1e12,
                                               1)},
        "e2e": {"value": round(n_tok / e2e_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(windows.nbytes * 2),
                "d2h_bytes_per_step": 8,
                "what": "perplexity(): host windows copied per batch (ids and targets), "
                        "NLL sum read back; ppl " + f"{r['ppl']:.3f}"},
        "gpu_launches": int(launches),
        "roofline": {"kernel": "gemm_tc_kernel (all launches of one 8-window batch)",
                     "bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops)"
                     if "bf16_tflops" in pk else "fallback 1590 TFLOP/s",
                     "note": "2MNK per launch (the attention scores' three bf16 terms counted "
                             "once)"},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline_eval()
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline_eval(T=512):
    """The CPU restatement of the dense bf16-dequantized eval (oracle.block / oracle.evaluate)
    on a bounded sample: one window of T tokens through 2 blocks and the tied head over the
    full vocabulary for its rows, scaled to 24 blocks; tokens per second."""
    import torch
    from oracle import block as ob
    from oracle import evaluate as oe
    torch.set_num_threads(os.cpu_count())
    g = torch.Generator().manual_seed(0)
    W = {"q_proj": (NH * HD, HID), "k_proj": (NKV * HD, HID), "v_proj": (NKV * HD, HID),
         "o_proj": (HID, NH * HD), "gate_proj": (INTER, HID), "up_proj": (INTER, HID),
         "down_proj": (HID, INTER), "q_bias": (NH * HD,), "k_bias": (NKV * HD,),
         "v_bias": (NKV * HD,)}
    W = {k: (0.02 * torch.randn(*s, generator=g)).bfloat16().float() for k, s in W.items()}
    W["in_norm"] = torch.ones(HID)
    W["post_norm"] = torch.ones(HID)
    E = (0.02 * torch.randn(VOCAB, HID, generator=g)).bfloat16().float()
    ids = torch.randint(0, VOCAB, (T + 1,), generator=g)
    t0 = time.perf_counter()
    h = E[ids[:-1]]
    for _ in range(2):
        h = ob.block_hard(h, W)[0]
    t_blocks = time.perf_counter() - t0
    t0 = time.perf_counter()
    hn = ob.rmsnorm(h, torch.ones(HID))
    z = ob.bf(hn.double() @ E.double().T)
    oe.nll_rows(z, ids[1:].numpy())
    t_head = time.perf_counter() - t0
    per_window = t_blocks * 12 + t_head
    return {"value": round(T / per_window, 2), "unit": "tokens/s (extrapolated)",
            "cores": os.cpu_count(), "kind": "port",
            "sample": f"one {T}-token window through 2 blocks (x12 for 24) and the tied head over "
                      "the full vocabulary (torch-CPU float64 restatement; the MLX path is "
                      "unavailable)"}


def run_reference_eval(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cb = cpu_baseline_eval()
    res = {"impl": "reference",
           "metric": "eval tokens/s (24-layer Qwen2.5-0.5B architecture, packed mixed 2/3/4-bit "
                     "g64 fp16 scales, 146 x 2048 windows, next-token NLL)",
           "value": cb["value"], "unit": "tokens/s", "n_gpus": world, "steps": 1, "warmup": 0,
           "ms_per_step": round(EVAL_WINDOWS * (T_SEQ - 1) / cb["value"] * 1000, 1),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
           "data": "synthetic",
           "config": {"workload": "packed-model eval, 146 windows x 2048"},
           "cpu_baseline": cb,
           "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


# -------------------------------------------------------------------------- pipeline ---

def run_pipeline(args):
    """The full 3-bit pipeline on the 24-layer stack, each phase timed on the host clock:
    build-db (Hessians + GPTQ at 2 / 3 / 4 bits over 128 x 2048 calibration ids), allocate (RCO,
    3.0 bits, 8 samples x 32 windows x 2048; --rco-steps of the 100, the rest extrapolated
    from their mean), quantize (24 blocks x qk / vo / mlp x 200 Lion steps on the quantized
    stream, shards), export (MLX affine checkpoint), eval (packed model, 146 x 2048 windows).
    value = the pipeline wall-clock in seconds with the allocate phase at 100 steps."""
    import shutil
    import tempfile
    import torch
    import torch.distributed as dist
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.common.evaluate import PackedModel, perplexity
    from gsq_rco_mlx_b200.gsq import pipeline as pl
    from gsq_rco_mlx_b200.gsq.export import save_base_checkpoint
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, DataParallel
    from gsq_rco_mlx_b200.rco.allocate import Bank, KLObjective, rco_allocate
    from gsq_rco_mlx_b200.rco.database import DBSpec, build_database, random_model

    rank, world, local = dist_setup()
    _lib.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dp = DataParallel()
    rco_steps = max(1, min(args.rco_steps, 100))

    def sync():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    model = random_model(n_layers=24, seed=0, device=dev)
    calib = np.random.default_rng(0).integers(0, VOCAB, size=(N_SEQ, T_SEQ)).astype(np.int32)
    rco_win = np.random.default_rng(1).integers(0, VOCAB, size=(RCO_WINDOWS, T_SEQ)).astype(
        np.int32)
    ev_win = np.random.default_rng(2).integers(0, VOCAB, size=(EVAL_WINDOWS, T_SEQ)).astype(
        np.int32)
    # one work directory for every rank (rank 0 writes the shards and the export, every rank
    # loads the export for the eval)
    work = [tempfile.mkdtemp(prefix="gsq_pipeline_") if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(work, src=0)
    work = work[0]
    quiet = lambda *a: None
    t = {}
    clocks = Clocks(local)
    clocks.start()
    sync()
    t0 = time.perf_counter()
    man, res = build_database(model, calib, DBSpec(options=GPTQ_OPTIONS, n_layers=24), log=quiet,
                              keep="device")
    bank = Bank(man, res)
    sync()
    t["build_db"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    obj = KLObjective(model, bank, rco_win, windows_per_sample=RCO_WIN_PER_SAMPLE, chunk_seqs=8,
                      dp=dp)
    sync()
    t["allocate_setup"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    alloc = rco_allocate(obj, bank, 3.0, steps=rco_steps, g=RCO_G, lr=0.1, seed=0)
    sync()
    t_rco = time.perf_counter() - t0
    t["allocate_steps_measured"] = t_rco
    t["allocate"] = t["allocate_setup"] + t_rco / rco_steps * 100
    per_linear = {f"{L}.{n}": int(bank.options[int(k)])
                  for (L, n), k in zip(bank.groups, alloc["choice"])}
    del obj
    torch.cuda.empty_cache()
    bits = pl.load_bits(range(24), alloc={"per_linear_bits": per_linear})
    t0 = time.perf_counter()
    qres = pl.quantize_model(model, calib, bits, BlockOpts(steps=200), os.path.join(work, "q"),
                             dp=dp, log=quiet)
    sync()
    t["quantize"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    if rank == 0:
        save_base_checkpoint(model, os.path.join(work, "base"))
        pl.export_quantized(os.path.join(work, "q"), os.path.join(work, "base"), range(24))
    sync()
    t["export"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    pm = PackedModel.load(os.path.join(work, "q", "mlx"), device=dev)
    r = perplexity(pm, ev_win, chunk_seqs=EVAL_CHUNK, dp=dp)
    sync()
    t["eval"] = time.perf_counter() - t0
    clk = clocks.stop()
    total = t["build_db"] + t["allocate"] + t["quantize"] + t["export"] + t["eval"]
    measured = total - t["allocate"] + t["allocate_setup"] + t_rco
    out = {
        "metric": "full 3-bit pipeline wall-clock (24-layer Qwen2.5-0.5B architecture: build-db, "
                  "allocate, quantize, export, eval)",
        "value": round(total, 2), "unit": "s", "n_gpus": world, "steps": 1, "warmup": 0,
        "ms_per_step": round(total * 1000, 1), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16 model, f32/f64 optimisation",
        "data": "synthetic: random-init 24-layer stack, uniform-random calibration, RCO and "
                "eval windows",
        "config": {"workload": "full pipeline: 128 x 2048 calibration, RCO 100 steps (g 8, 32 "
                               "windows), 24 blocks x 200 steps per stage, 146 eval windows",
                   "phase_seconds": {k: round(v, 2) for k, v in t.items()},
                   "rco_steps_measured": rco_steps,
                   "measured_seconds": round(measured, 2),
                   "decoded_avg_bits": round(alloc["decoded_avg_bits"], 4),
                   "quantize_seconds_per_block": round(t["quantize"] / 24, 3),
                   "eval_ppl": round(r["ppl"], 3),
                   "parallelism": f"every phase data-parallel over {world} rank(s)"},
        "e2e": {"value": round(total, 2), "unit": "s",
                "h2d_bytes_per_step": int(calib.nbytes + rco_win.nbytes + ev_win.nbytes),
                "d2h_bytes_per_step": int(sum(os.path.getsize(os.path.join(work, "q", f))
                                              for f in os.listdir(os.path.join(work, "q"))
                                              if f.endswith(".npz")) if rank == 0 else 0),
                "what": "host ids in, shards and the checkpoint on disk, the eval dict out"},
        "gpu_launches": None,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
        shutil.rmtree(work, ignore_errors=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- linear ---

OUT_F, IN_F, N_SEQ_L, T_SEQ_L = 4864, 896, 32, 512
STAGE_STEPS = 200
RESAMPLES = 2
MICRO = 2


def make_inputs(seed=0):
    rng = np.random.default_rng(seed)
    W = (0.02 * rng.standard_normal((OUT_F, IN_F))).astype(np.float32)
    sch = np.exp(rng.standard_normal(IN_F)).astype(np.float32)
    X = (rng.standard_normal((N_SEQ_L * T_SEQ_L, IN_F)).astype(np.float32) * sch)
    return W, X


def run_linear(args):
    """The qk-stage step of one up_proj-shaped linear (W 4864 x 896, X 16384 x 896)."""
    import torch
    import torch.distributed as dist
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.gsq import gptq
    from gsq_rco_mlx_b200.gsq.quant import gs_schedules
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, LinearStep, SoftLinear

    rank, world, local = dist_setup()
    _lib.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    W, X = make_inputs(seed=rank)
    Wd = torch.as_tensor(W, device=dev)
    Xd = torch.as_tensor(X, device=dev)
    H, _ = gptq.hessian_from_inputs(Xd, device=True)
    g = gptq.quantize_gptq(Wd, H, 3, 64, device=True)
    lin = SoftLinear("up_proj", 3, g["codes"].cpu().numpy(), g["scales"].cpu().numpy().astype(np.float16),
                     64, seed=rank, linear_id=5)
    rng = np.random.default_rng(1)
    M = MICRO * (T_SEQ_L - 1)
    opts = BlockOpts(resamples=RESAMPLES, micro_batch=MICRO)
    lstep = LinearStep([lin], M, IN_F, RESAMPLES, x_terms=3)
    targets = {"up_proj": Wd}
    Xmb = torch.empty(M, IN_F, device=dev)
    Xpin = torch.from_numpy(np.ascontiguousarray(X.reshape(N_SEQ_L, T_SEQ_L, IN_F)[:, 1:])).pin_memory()
    loss_host = torch.empty(RESAMPLES, dtype=torch.float64).pin_memory()
    stream = torch.cuda.current_stream()
    bwd_events = []

    lstep.first_forward(targets, 0, *gs_schedules(0, STAGE_STEPS), 77)

    def step(t, host_inputs=False, time_bwd=False):
        tau, kappa = gs_schedules(t % STAGE_STEPS, STAGE_STEPS)
        idx = np.sort(rng.choice(N_SEQ_L, size=MICRO, replace=False))
        if host_inputs:
            for j, s in enumerate(idx):
                Xmb[j * (T_SEQ_L - 1):(j + 1) * (T_SEQ_L - 1)].copy_(Xpin[s], non_blocking=True)
            lstep.stage(Xmb, [0, 1], T_SEQ_L - 1, T_SEQ_L - 1, 0)
        else:
            lstep.stage(Xd, idx, T_SEQ_L - 1, T_SEQ_L, 1)
        lstep.contract()
        if time_bwd:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        t1 = t + 1
        lstep.update(targets, t, tau, kappa, opts, 77,
                     nxt=(t1, *gs_schedules(t1 % STAGE_STEPS, STAGE_STEPS)))
        if time_bwd:
            e1.record(stream)
            bwd_events.append((e0, e1))
        if host_inputs:
            loss_host.copy_(lstep.loss, non_blocking=True)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for t in range(args.warmup):
        step(t)
    barrier()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for t in range(args.steps):
        step(args.warmup + t, time_bwd=True)
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    clk = clocks.stop()
    bwd_ms = statistics.mean(a.elapsed_time(b) for a, b in bwd_events)
    # end to end through the public API: host rows in, loss out, every step
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for t in range(args.steps):
        step(args.warmup + args.steps + t, host_inputs=True)
    e3.record(stream)
    barrier()
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))

    d = OUT_F * IN_F
    # algorithmic bytes of the fused step pass per weight: read logits + momentum (40 B), code
    # (1), FP weight (4), per resample the stored probabilities (20) and the weight gradient
    # (4); write logits + momentum (40), per resample the next probabilities (20) and the next
    # soft weight as three bf16 terms (6); plus the group scales and their momentum
    bwd_bytes = d * (40 + 1 + 4 + 40 + RESAMPLES * (20 + 4 + 20 + 6)) + \
        4 * 4 * OUT_F * (IN_F // 64)
    achieved = bwd_bytes / (bwd_ms * 1e-3) / 1e9
    peaks = globals()["peaks"]()
    peak = float(peaks.get("hbm_gbs", 6650.0))
    value = world * args.steps / (ms * 1e-3)
    res = {
        "metric": "GSQ steps/s (single linear up_proj 4864x896, 3-bit, micro-batch 2x511, R=2)",
        "value": round(value, 3), "unit": "steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) x lognormal channels, random-init weights)",
        "config": {"workload": "single linear GSQ (W 4864x896, X 16384x896 as 32x512)",
                   "rows_per_step": M, "resamples": RESAMPLES, "bits": 3, "group_size": 64,
                   "parallelism": f"replicas x{world}", "l2": "per-step working set > L2 (126 MB)"},
        "e2e": {"value": round(world * args.steps / (ms_e2e * 1e-3), 3), "unit": "steps/s",
                "h2d_bytes_per_step": M * IN_F * 4, "d2h_bytes_per_step": RESAMPLES * 8},
        "gpu_launches": args.steps * (RESAMPLES * 4 + 2),
        "roofline": {"kernel": "soft_step_kernel", "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": None, "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)"
                     if "hbm_gbs" in peaks else "fallback 6650 GB/s"},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_linear(W, X, lin_codes=g["codes"].cpu().numpy(),
                                                  s16=g["scales"].cpu().numpy().astype(np.float16),
                                                  n_steps=2)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline_linear(W, X, lin_codes, s16, n_steps=2):
    """The CPU restatement of the same step (oracle port), on this host's cores."""
    from oracle import gsq as ogsq
    st = ogsq.LinearState(3, lin_codes, s16, 64, seed=0, linear_id=5)
    Xs = X.reshape(N_SEQ_L, T_SEQ_L, IN_F)[:, 1:]
    t0 = time.perf_counter()
    ogsq.train_linear(st, lambda idx: Xs[idx].reshape(-1, IN_F), W, N_SEQ_L, n_steps, seed=1,
                      noise_seed=77)
    dt = time.perf_counter() - t0
    return {"value": round(n_steps / dt, 4), "unit": "steps/s", "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"{n_steps} steps of the same workload (numpy float32 elementwise, float64 GEMMs)"}



def main():
    args = parse()
    if args.workload == "kernels":
        import bench_kernels
        return bench_kernels.main([c for c in args.cases.split(",") if c] +
                                  (["--once"] if args.once else []))
    if args.workload == "linear":
        return run_linear(args)
    if args.workload == "gptq":
        return run_reference_gptq(args) if args.impl == "reference" else run_gptq(args)
    if args.workload == "rco":
        return run_reference_rco(args) if args.impl == "reference" else run_rco(args)
    if args.workload == "eval":
        return run_reference_eval(args) if args.impl == "reference" else run_eval(args)
    if args.workload == "pipeline":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the full pipeline's GSQ, RCO "
                              "and eval phases are MLX-only in the reference (MLX absent)"}))
            return None
        return run_pipeline(args)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_block(args)


if __name__ == "__main__":
    main()
