"""Host logic of the GSQ stage data parallelism (gsq.staged.DataParallel), world size 2 over gloo."""
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def test_windows_single_process():
    from gsq_rco_mlx_b200.gsq.staged import DataParallel
    dp = DataParallel()
    assert dp.world == 1 and dp.window(1, 2048) == (1, 2048)
    dp.allreduce(torch.ones(3))  # no-op


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from gsq_rco_mlx_b200.gsq.staged import DataParallel
        dp = DataParallel()
        w = dp.window(1, 2048)
        g = torch.full((4,), float(rank + 1))
        dp.allreduce(g)
        q.put((rank, w, g.tolist()))
    finally:
        dist.destroy_process_group()


def test_windows_and_allreduce_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=60) for _ in range(2))
    for p in procs:
        p.join(60)
    assert all(p.exitcode == 0 for p in procs)
    (r0, w0, g0), (r1, w1, g1) = res
    assert w0 == (1, 1025) and w1 == (1025, 2048)
    assert g0 == g1 == [3.0] * 4
