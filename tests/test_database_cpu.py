"""Sharding of the database build across ranks (host logic; world size 2 over gloo on CPU)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def test_lpt_assignment_balances_and_is_deterministic():
    from gsq_rco_mlx_b200.rco.database import assign_lpt, solve_cost
    shapes = [(896, 896), (128, 896), (128, 896), (896, 896), (4864, 896), (4864, 896),
              (896, 4864)]
    costs = [solve_cost(*s) for s in shapes for _ in (2, 3, 4)]
    for world in (1, 2, 4, 8):
        owner = assign_lpt(costs, world)
        assert owner == assign_lpt(costs, world)
        load = np.zeros(world)
        for c, r in zip(costs, owner):
            load[r] += c
        # LPT bound: max load <= mean + largest job
        assert load.max() <= load.sum() / world + max(costs) + 1e-6
        assert set(owner) == set(range(min(world, len(costs))))


def test_shard_windows_cover_all():
    from gsq_rco_mlx_b200.rco.database import shard_windows
    for n in (1, 7, 128):
        for world in (1, 2, 3, 8):
            if n < world:
                continue
            spans = [shard_windows(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _combine_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from gsq_rco_mlx_b200.rco.database import combine_hessian, shard_windows
        from oracle.gptq import hessian_from_inputs
        rng = np.random.default_rng(0)
        X = rng.standard_normal((23, 6))            # all rows, same on every rank
        a, b = shard_windows(23, world, rank)
        H_loc, n = None, 0
        for r0 in range(a, b, 4):                   # running mean over this rank's rows
            H_loc, n = hessian_from_inputs(X[r0:min(b, r0 + 4)], H_loc, n)
        H = torch.as_tensor(H_loc)
        combine_hessian(H, n, 23, dist)
        if rank == 0:
            ref, _ = hessian_from_inputs(X)
            out.put(float(np.abs(H.numpy() - ref).max() / np.abs(ref).max()))
    finally:
        dist.destroy_process_group()


def test_combine_hessian_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_combine_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) < 1e-12
