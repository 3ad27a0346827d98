"""Benchmark of the GSQ hot path on B200 (one JSON line on rank 0).

Workload "linear": one Qwen2.5-0.5B up_proj-shaped linear W [4864 x 896] (0.02 N(0,1), seed
0), calibration X [16384 x 896] = N(0,1) x per-channel lognormal scales viewed as 32
sequences x 512 positions (position 0 dropped), GPTQ 3-bit group-64 init with fp16 scales,
then GSQ Lion steps at micro-batch 2 (1022 rows), 2 Gumbel resamples, tau 2 -> 0.05,
kappa 100 -> 500 over 200 steps. A step = one Lion step (soft weights, residual and
weight-gradient contractions, loss, fused backward + Lion). Inputs are synthetic (seeded)
with the shapes and distributions of the configuration; the per-step working set (~300 MB)
exceeds the 126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU, each rank quantizing its own linear (weak
scaling: per-GPU work fixed). --impl reference times the CPU restatement of the same step
(the reference's GSQ path is MLX-only and cannot run here).
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

OUT_F, IN_F, N_SEQ, T_SEQ = 4864, 896, 32, 512
STAGE_STEPS = 200
RESAMPLES = 2
MICRO = 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def make_inputs(seed=0):
    rng = np.random.default_rng(seed)
    W = (0.02 * rng.standard_normal((OUT_F, IN_F))).astype(np.float32)
    sch = np.exp(rng.standard_normal(IN_F)).astype(np.float32)
    X = (rng.standard_normal((N_SEQ * T_SEQ, IN_F)).astype(np.float32) * sch)
    return W, X


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out" if os.path.isdir(os.path.join(ROOT, "gpurun_out"))
                                 else "", f".clocks_{os.getpid()}.csv")

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
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
                "reasons": sorted(reasons)}


def run_ours(args):
    import torch
    import torch.distributed as dist
    from gsq_rco_mlx_b200 import _lib
    from gsq_rco_mlx_b200.gsq import gptq
    from gsq_rco_mlx_b200.gsq.quant import gs_schedules
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, LinearStep, SoftLinear

    rank, world, local = dist_setup(args.gpus)
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
    M = MICRO * (T_SEQ - 1)
    opts = BlockOpts(resamples=RESAMPLES, micro_batch=MICRO)
    lstep = LinearStep([lin], M, IN_F, RESAMPLES, x_terms=3)
    targets = {"up_proj": Wd}
    Xmb = torch.empty(M, IN_F, device=dev)
    Xpin = torch.from_numpy(np.ascontiguousarray(X.reshape(N_SEQ, T_SEQ, IN_F)[:, 1:])).pin_memory()
    loss_host = torch.empty(RESAMPLES, dtype=torch.float64).pin_memory()
    stream = torch.cuda.current_stream()
    bwd_events = []

    lstep.first_forward(targets, 0, *gs_schedules(0, STAGE_STEPS), 77)

    def step(t, host_inputs=False, time_bwd=False):
        tau, kappa = gs_schedules(t % STAGE_STEPS, STAGE_STEPS)
        idx = np.sort(rng.choice(N_SEQ, size=MICRO, replace=False))
        if host_inputs:
            for j, s in enumerate(idx):
                Xmb[j * (T_SEQ - 1):(j + 1) * (T_SEQ - 1)].copy_(Xpin[s], non_blocking=True)
            lstep.stage(Xmb, [0, 1], T_SEQ - 1, T_SEQ - 1, 0)
        else:
            lstep.stage(Xd, idx, T_SEQ - 1, T_SEQ, 1)
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
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) \
        if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = float(peaks.get("hbm_gbs", 6650.0))
    value = world * args.steps / (ms * 1e-3)
    res = {
        "metric": "GSQ steps/s (single linear up_proj 4864x896, 3-bit, micro-batch 2x511, R=2)",
        "value": round(value, 3), "unit": "steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) x lognormal channels, random-init weights)",
        "config": {"workload": "config 1: single linear GSQ (W 4864x896, X 16384x896 as 32x512)",
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
    if rank == 0 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(W, X, lin_codes=g["codes"].cpu().numpy(),
                                           s16=g["scales"].cpu().numpy().astype(np.float16),
                                           n_steps=2)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline(W, X, lin_codes, s16, n_steps=2):
    """The CPU restatement of the same step (oracle port), on this host's cores."""
    from oracle import gsq as ogsq
    st = ogsq.LinearState(3, lin_codes, s16, 64, seed=0, linear_id=5)
    Xs = X.reshape(N_SEQ, T_SEQ, IN_F)[:, 1:]
    t0 = time.perf_counter()
    ogsq.train_linear(st, lambda idx: Xs[idx].reshape(-1, IN_F), W, N_SEQ, n_steps, seed=1,
                      noise_seed=77)
    dt = time.perf_counter() - t0
    return {"value": round(n_steps / dt, 4), "unit": "steps/s", "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"{n_steps} steps of the same workload (numpy float32 elementwise, float64 GEMMs)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import gptq as og
    W, X = make_inputs(seed=0)
    H, _ = og.hessian_from_inputs(X)
    g = og.quantize_gptq(W[:64], H, 3, 64)  # init codes for the sample rows only (bounded)
    rng = np.random.default_rng(0)
    codes = np.concatenate([g["codes"]] * (OUT_F // 64))
    scales = np.concatenate([g["scales"]] * (OUT_F // 64)).astype(np.float16)
    per = []
    for _ in range(max(1, min(args.steps, 3))):
        r = cpu_baseline(W, X, codes, scales, n_steps=1)
        per.append(r["value"])
    v = statistics.median(per)
    res = {"impl": "reference",
           "metric": "GSQ steps/s (single linear up_proj 4864x896, 3-bit, micro-batch 2x511, R=2)",
           "value": round(v, 4), "unit": "steps/s", "n_gpus": world, "steps": len(per),
           "warmup": 0, "ms_per_step": round(1000 / v, 2), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "config 1: single linear GSQ (W 4864x896, X 16384x896 as 32x512)"},
           "cpu_baseline": {"value": round(v, 4), "unit": "steps/s", "cores": os.cpu_count(),
                            "kind": "port",
                            "sample": "1-step samples of the same workload; the reference's MLX "
                                      "path is unavailable, this is the numpy restatement"},
           "e2e": {"value": round(v, 4), "unit": "steps/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
