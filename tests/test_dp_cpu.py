"""Host logic of the GSQ stage data parallelism (gsq.staged.DataParallel), world size 2 over gloo."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def test_windows_single_process():
    from gsq_rco_mlx_b200.gsq.staged import DataParallel
    for split in ("sequences", "positions"):
        dp = DataParallel(split=split)
        assert dp.world == 1 and dp.window(1, 2048) == (1, 2048)
        assert dp.total(2) == 2
        # one process draws the reference's micro-batch: sorted, without replacement
        a = dp.draw(np.random.default_rng(3), 128, 2)
        b = np.sort(np.random.default_rng(3).choice(128, size=2, replace=False))
        assert np.array_equal(a, b)
        dp.allreduce(torch.ones(3))  # no-op
    with pytest.raises(ValueError):
        DataParallel(split="tokens")


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from gsq_rco_mlx_b200.gsq.staged import DataParallel
        pos = DataParallel(split="positions")
        seq = DataParallel(split="sequences")
        w = pos.window(1, 2048)
        rng = np.random.default_rng(7)
        draws = [seq.draw(rng, 128, 2).tolist() for _ in range(3)]
        g = torch.full((4,), float(rank + 1))
        seq.allreduce(g)
        q.put((rank, w, seq.window(1, 2048), seq.total(2), pos.total(2), pos.share(0, 5),
               draws, g.tolist()))
    finally:
        dist.destroy_process_group()


def test_windows_draws_and_allreduce_two_ranks():
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
    (r0, w0, sw0, st0, pt0, sh0, d0, g0), (r1, w1, sw1, st1, pt1, sh1, d1, g1) = res
    assert w0 == (1, 1025) and w1 == (1025, 2048)          # positions: halves of 1..2047
    assert sw0 == sw1 == (1, 2048)                          # sequences: every position
    assert st0 == st1 == 4 and pt0 == pt1 == 2
    assert sh0 == (0, 3) and sh1 == (3, 5)
    # sequences: the ranks' draws are the two halves of one sorted global draw of 4
    rng = np.random.default_rng(7)
    for t in range(3):
        glob = np.sort(rng.choice(128, size=4, replace=False)).tolist()
        assert d0[t] == glob[:2] and d1[t] == glob[2:]
    assert g0 == g1 == [3.0] * 4
