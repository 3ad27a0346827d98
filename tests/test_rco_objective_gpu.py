"""The RCO KL objective on the GPU (reference src/gsq_rco/rco/allocate.py:54-174) against the
oracle chain: assembled-weight forwards (oracle.block), the KL head (oracle.kl), the final-norm
and per-block backward (oracle.block_vjp) and the straight-through dots, summed over windows."""
import numpy as np
import pytest
import torch

from oracle import block as ob
from oracle import block_vjp as ov
from oracle import gptq as og
from oracle import kl as okl

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


@pytest.fixture(scope="module")
def setup():
    from gsq_rco_mlx_b200.gsq.e2e import BlockConfig
    from gsq_rco_mlx_b200.rco.allocate import Bank, KLObjective
    from gsq_rco_mlx_b200.rco.database import DBSpec, build_database, random_model
    cfg = BlockConfig(hidden=128, n_heads=2, n_kv=1, inter=256)
    model = random_model(n_layers=2, seed=11, device=torch.device(DEV), cfg=cfg, vocab=1024)
    model.norm = (1 + 0.1 * torch.randn(128, generator=torch.Generator().manual_seed(1))
                  ).bfloat16().to(DEV)
    windows = np.random.default_rng(5).integers(0, 1024, size=(4, 64)).astype(np.int32)
    man, res = build_database(model, windows, DBSpec(options=(2, 3, 4), n_layers=2),
                              log=lambda *a: None, keep="device", chunk_windows=2)
    bank = Bank(man, res)
    obj = KLObjective(model, bank, windows, windows_per_sample=2, chunk_seqs=1)
    return cfg, model, bank, obj, windows


def _assembled(bank, model, L, choice):
    W = {k: v.cpu() for k, v in model.layers[L].items()}
    for j, name in enumerate(NAMES):
        codes, scales, bits = bank.cands(L * 7 + j)[int(choice[L * 7 + j])]
        wq = og.dequantize(codes.cpu().numpy(), scales.cpu().numpy(), bits, 64)
        W[name] = torch.as_tensor(wq).bfloat16()
    return W


def oracle_objective(cfg, model, bank, windows, choice, ids):
    E = model.embed.cpu()
    wn = model.norm.cpu()
    Wq = [_assembled(bank, model, L, choice) for L in range(2)]
    Wfp = [{k: v.cpu() for k, v in model.layers[L].items()} for L in range(2)]
    T = windows.shape[1]
    n_all = len(ids) * T
    total, up = 0.0, np.zeros((14, 3))
    for w in ids:
        h0 = E[torch.as_tensor(windows[w], dtype=torch.long)].float()
        states = [h0]
        for L in range(2):
            states.append(ob.block_hard(states[-1], Wq[L], 2, 1)[0])
        href = h0
        for L in range(2):
            href = ob.block_hard(href, Wfp[L], 2, 1)[0]
        hq = ob.rmsnorm(states[-1], wn)
        hr = ob.rmsnorm(href, wn)
        v, g = okl.kl_chunk_value_grad(hq.double(), hr.double(), E.double())
        total += v
        g = ob.bf((g / n_all).float())
        cot = ob.bf(ov.rmsnorm_bwd(states[-1], wn, g).float())
        for L in reversed(range(2)):
            dh, grads = ov.block_vjp(states[L], {k: v.float() for k, v in Wq[L].items()}, cot,
                                     2, 1)
            for j, name in enumerate(NAMES):
                up[L * 7 + j] += okl.ste_dots(
                    grads[name].numpy(), Wfp[L][name].float().numpy(),
                    [(c.cpu().numpy(), s.cpu().numpy(), b) for c, s, b in bank.cands(L * 7 + j)])
            cot = dh
    return total / n_all, up


def test_objective_matches_oracle(setup):
    cfg, model, bank, obj, windows = setup
    choice = np.array([1, 0, 2, 1, 1, 0, 2] * 2)
    ids = [0, 2]
    loss, up = obj.loss_and_upstream(choice, ids)
    loss_o, up_o = oracle_objective(cfg, model, bank, windows, choice, ids)
    assert abs(loss - loss_o) <= 1e-3 * abs(loss_o) + 1e-9, (loss, loss_o)
    rel = float(np.linalg.norm(up - up_o) / np.linalg.norm(up_o))
    assert rel < 5e-2, rel
    # the objective's own consistency: forward-only loss equals the loss of the full call
    assert abs(obj.mean_kl(choice, ids) - loss) <= 1e-9 * abs(loss) + 1e-12


def test_rco_allocate_runs(setup):
    from gsq_rco_mlx_b200.rco.allocate import rco_allocate
    cfg, model, bank, obj, windows = setup
    res = rco_allocate(obj, bank, 3.0, steps=2, g=2, lr=0.1, seed=0)
    assert res["decoded_int_cost"] <= res["budget_int"]
    assert len(res["history"]) == 2 and res["choice"].shape == (14,)
