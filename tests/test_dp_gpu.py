"""Data parallelism of the GSQ stages (the rank windows of gsq.staged.DataParallel): the
gradients and loss partials of position windows, summed, equal those of the whole micro-batch
(float32-faithful sums in another order). The windows run one after the other on one GPU, which
is what the ranks compute before their all-reduce; the 2-GPU run covers the all-reduce itself."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def _setup(seed):
    from tests.test_stages_gpu import _pair, _weights
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig, BlockWeights, Qwen2Block
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    W = _weights(seed)
    N, T = 4, 64
    h = (0.5 * torch.randn(N * T, cfg.hidden, generator=torch.Generator().manual_seed(seed))
         ).bfloat16()
    blk = Qwen2Block(cfg, N, T)
    Wd = BlockWeights({k: v.to(DEV) for k, v in W.items()})
    return cfg, W, Wd, blk, h.to(DEV), N, T, _pair


def test_mlp_windows_sum_to_full_step():
    from gsq_rco_mlx_b200.gsq.staged import MLPStep
    cfg, W, Wd, blk, h, N, T, _pair = _setup(1)
    Y = blk.forward(h, Wd).clone()
    mn, h1 = blk.mn.clone(), blk.h1.clone()
    lins = [_pair(n, W[n].float().numpy(), 3, i + 4)[0] for i, n in
            enumerate(("gate_proj", "up_proj", "down_proj"))]
    full = MLPStep(lins, cfg, 2, T, 2)
    parts = [MLPStep(lins, cfg, 2, T, 2, window=w) for w in ((1, 30), (30, 64))]
    for st in [full] + parts:
        st.first_forward(0, 2.0, 100.0, 9)
        st.stage(mn, h1, Y, [0, 2])
        st.contract()
    torch.cuda.synchronize()
    assert _rel(parts[0].gflat + parts[1].gflat, full.gflat) < 2e-6
    assert _rel(parts[0].loss + parts[1].loss, full.loss) < 1e-9


def test_vo_windows_sum_to_full_step():
    from gsq_rco_mlx_b200.gsq.e2e import wterms
    from gsq_rco_mlx_b200.gsq.staged import VOStep, _bf16_rows
    from gsq_rco_mlx_b200.gemm import gemm
    cfg, W, Wd, blk, h, N, T, _pair = _setup(2)
    A = torch.empty(N * T, cfg.hidden, device=DEV, dtype=torch.bfloat16)
    blk.forward(h, Wd, attn_out=A)
    hn = blk.hn.clone()
    qk = torch.empty(N * T, 3 * 64, device=DEV, dtype=torch.bfloat16)
    gemm(_bf16_rows(hn), wterms(Wd.qk), epi=4, bias=Wd.qk_bias, c_terms=_bf16_rows(qk))
    lins = [_pair(n, W[n].float().numpy(), 3, i + 2)[0] for i, n in
            enumerate(("v_proj", "o_proj"))]
    full = VOStep(lins, cfg, 2, T, 2, Wd.W["v_bias"])
    parts = [VOStep(lins, cfg, 2, T, 2, Wd.W["v_bias"], window=w) for w in ((0, 24), (24, 64))]
    for st in [full] + parts:
        st.first_forward(0, 2.0, 100.0, 11)
        st.stage(hn, A, qk, [1, 3])
        st.contract()
    torch.cuda.synchronize()
    # probabilities of the query rows: the window rows of the full P, bit for bit
    Pf = full.P.t[0].view(2 * cfg.n_heads, T, -1)[:, 24:64, :64]
    P1 = parts[1].P.t[0].view(2 * cfg.n_heads, 40, -1)[:, :, :64]
    assert torch.equal(Pf, P1)
    assert _rel(parts[0].gflat + parts[1].gflat, full.gflat) < 2e-6
    assert _rel(parts[0].loss + parts[1].loss, full.loss) < 1e-9


def test_linear_windows_sum_to_full_step():
    from gsq_rco_mlx_b200.gsq.staged import LinearStep
    from tests.test_stages_gpu import _pair
    rng = np.random.default_rng(0)
    out_f, in_f, T, m = 256, 128, 64, 2
    W = (0.02 * rng.standard_normal((out_f, in_f))).astype(np.float32)
    lin = _pair("q_proj", W, 3, 0)[0]
    x = torch.as_tensor(rng.standard_normal((4 * T, in_f)).astype(np.float32), device=DEV)
    targets = {"q_proj": torch.as_tensor(W, device=DEV)}
    full = LinearStep([lin], m * (T - 1), in_f, 2)
    parts = [LinearStep([lin], m * (b - a), in_f, 2, M_total=m * (T - 1)) for a, b in
             ((1, 40), (40, 64))]
    for st, (a, b) in zip([full] + parts, ((1, 64), (1, 40), (40, 64))):
        st.first_forward(targets, 0, 2.0, 100.0, 5)
        st.stage(x, [0, 3], b - a, T, a)
        st.contract()
    torch.cuda.synchronize()
    assert _rel(parts[0].gflat + parts[1].gflat, full.gflat) < 2e-6
    # the qk loss is sum D * G of the float32 gradients: float32 accuracy
    assert _rel(parts[0].loss + parts[1].loss, full.loss) < 1e-6


def _dp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from gsq_rco_mlx_b200.gsq.staged import BlockOpts, DataParallel, MLPStep, train_stage
        cfg, W, Wd, blk, h, N, T, _pair = _setup(1)
        Y = blk.forward(h, Wd).clone()
        mn, h1 = blk.mn.clone(), blk.h1.clone()
        lins = [_pair(n, W[n].float().numpy(), 3, i + 4)[0] for i, n in
                enumerate(("gate_proj", "up_proj", "down_proj"))]
        dp = DataParallel(split="positions")
        step = MLPStep(lins, cfg, 2, T, 2, window=dp.window(1, T))
        hist = train_stage(step, lambda idx: (mn, h1, Y, idx), N, BlockOpts(steps=6), seed=5,
                           noise_seed=9, dp=dp)[0]
        out = torch.cat([l.logits.flatten() for l in lins])
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        if rank == 0:
            q.put((hist, [g.cpu() for g in gathered]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_mlp_stage_two_ranks_matches_one():
    import torch.multiprocessing as mp
    from gsq_rco_mlx_b200.gsq.staged import BlockOpts, MLPStep, train_stage
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    hist2, logits = q.get(timeout=300)
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert torch.equal(logits[0], logits[1])          # ranks stay identical
    cfg, W, Wd, blk, h, N, T, _pair = _setup(1)
    Y = blk.forward(h, Wd).clone()
    mn, h1 = blk.mn.clone(), blk.h1.clone()
    lins = [_pair(n, W[n].float().numpy(), 3, i + 4)[0] for i, n in
            enumerate(("gate_proj", "up_proj", "down_proj"))]
    step = MLPStep(lins, cfg, 2, T, 2)
    hist1 = train_stage(step, lambda idx: (mn, h1, Y, idx), N, BlockOpts(steps=6), seed=5,
                        noise_seed=9)[0]
    one = torch.cat([l.logits.flatten() for l in lins]).cpu()
    assert _rel(logits[0], one) < 1e-5
    assert abs(hist2[-1] - hist1[-1]) <= 1e-5 * abs(hist1[-1])


def test_mlp_sequence_shares_sum_to_global_step():
    """The "sequences" split: two ranks' steps over their halves of a global micro-batch of 4
    sequences (loss normalised by the global count) sum to one step over all 4."""
    from gsq_rco_mlx_b200.gsq.staged import MLPStep
    cfg, W, Wd, blk, h, N, T, _pair = _setup(3)
    Y = blk.forward(h, Wd).clone()
    mn, h1 = blk.mn.clone(), blk.h1.clone()
    lins = [_pair(n, W[n].float().numpy(), 3, i + 4)[0] for i, n in
            enumerate(("gate_proj", "up_proj", "down_proj"))]
    full = MLPStep(lins, cfg, 4, T, 2)
    parts = [MLPStep(lins, cfg, 2, T, 2, m_total=4) for _ in range(2)]
    ids = [0, 1, 2, 3]
    for st, idx in ((full, ids), (parts[0], ids[:2]), (parts[1], ids[2:])):
        st.first_forward(0, 2.0, 100.0, 9)
        st.stage(mn, h1, Y, idx)
        st.contract()
    torch.cuda.synchronize()
    assert _rel(parts[0].gflat + parts[1].gflat, full.gflat) < 2e-6
    assert _rel(parts[0].loss + parts[1].loss, full.loss) < 1e-9
