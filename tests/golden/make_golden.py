"""Generate the golden vectors of the hot path by running the reference's own numpy code.

Run where a checkout of the reference (egesabanci/gsq-rco-mlx) is readable:
    python tests/golden/make_golden.py --reference PATH_TO_CHECKOUT
It imports the reference package from PATH/src and its test oracles from PATH/tests, and
writes small .npz fixtures next to this script. The fixtures are
committed; nothing at test time reads the reference.

The reference's GSQ, Lion and KL code is MLX-only and MLX cannot run here. Its numpy test
oracle (tests/oracles.py) only needs two Lion constants from gsq_rco.gsq.lion, whose module
imports mlx.core at the top; a throwaway empty module object stands in for ``mlx.core`` while
this script imports them (no MLX function is called).
"""
from __future__ import annotations

import sys
import types
from pathlib import Path

import numpy as np

REF = None  # the reference checkout, set by main() from --reference
OUT = Path(__file__).resolve().parent


def _import_reference():
    sys.path.insert(0, str(REF / "src"))
    sys.path.insert(0, str(REF / "tests"))
    # the numpy modules first, so their optional-MLX probes see no MLX
    import gsq_rco.gsq.gptq as gptq
    import gsq_rco.gsq.quant as quant
    import gsq_rco.rco.manifold as manifold
    import gsq_rco.rco.loop as loop
    if "mlx" not in sys.modules:
        mlx = types.ModuleType("mlx")
        core = types.ModuleType("mlx.core")
        core.array = type("array", (), {})  # isinstance(x, mx.array) is False for numpy
        mlx.core = core
        sys.modules["mlx"] = mlx
        sys.modules["mlx.core"] = core
    import oracles
    return gptq, quant, manifold, loop, oracles


def gen_gptq(gptq):
    """GPTQ / RTN / Hessian cases (gsq/gptq.py) incl. the edge cases of tests/test_gptq.py:155-233."""
    out = {}
    rng = np.random.default_rng(100)
    cases = []
    # the single-linear workload's statistics at a reduced shape: W ~ 0.02 N(0,1),
    # X = N(0,1) * lognormal channel scales
    for ci, (o, i, bits, gs, bsz) in enumerate([(96, 256, 3, 64, 128), (64, 256, 2, 64, 128),
                                                 (64, 256, 4, 64, 128), (48, 320, 3, 64, 128),
                                                 (40, 100, 3, 64, 128), (32, 192, 3, 64, 64)]):
        W = (0.02 * rng.standard_normal((o, i))).astype(np.float32)
        sch = np.exp(rng.standard_normal(i))
        X = rng.standard_normal((1024, i)) * sch
        if ci == 3:
            X[:, 7] = 0.0  # a dead input column
        H, n = None, 0
        for a in range(0, X.shape[0], 256):
            H, n = gptq.hessian_from_inputs(X[a:a + 256], H, n)
        r = gptq.quantize_gptq(W, H, bits, gs, 0.01, bsz)
        cases.append(dict(W=W, H=H, bits=bits, gs=gs, block=bsz, codes=r["codes"],
                          scales=r["scales"], w_q=r["w_q"], err=r["err"]))
    for ci, c in enumerate(cases):
        for k, v in c.items():
            out[f"gptq{ci}_{k}"] = np.asarray(v)
    out["gptq_n"] = np.array(len(cases))
    # H = I equals RTN (tests/test_gptq.py:187-190) and RTN at every width incl. ragged groups
    Wd = rng.standard_normal((6, 100)) * 0.05
    out["rtn_W"] = Wd
    for bits in (1, 2, 3, 4, 8):
        r = gptq.quantize_rtn(Wd, bits, 64)
        out[f"rtn{bits}_codes"], out[f"rtn{bits}_scales"], out[f"rtn{bits}_wq"] = \
            r["codes"], r["scales"], r["w_q"]
    out["gptq_eye_codes"] = gptq.quantize_gptq(Wd, np.eye(100), 3, 64)["codes"]
    # block-size invariance (tests/test_gptq.py:211-224)
    Xb = rng.standard_normal((512, 96)) @ rng.standard_normal((96, 96)) * 0.1
    Hb, _ = gptq.hessian_from_inputs(Xb)
    Wbk = rng.standard_normal((12, 96)) * 0.05
    out["blk_W"], out["blk_H"] = Wbk, Hb
    out["blk_codes96"] = gptq.quantize_gptq(Wbk, Hb, 2, 24, block_size=96)["codes"]
    out["blk_codes16"] = gptq.quantize_gptq(Wbk, Hb, 2, 24, block_size=16)["codes"]
    # streaming Hessian (tests/test_gptq.py:226-233)
    Ha, na = gptq.hessian_from_inputs(Xb[:200])
    Hab, nab = gptq.hessian_from_inputs(Xb[200:], Ha, na)
    out["hess_X"], out["hess_H"], out["hess_n"] = Xb, Hab, np.array(nab)  # 512 x 96
    np.savez_compressed(OUT / "gptq.npz", **out)


def gen_dp(manifold, loop):
    """DP decode cases (rco/manifold.py:304-380) incl. tests/test_rco_phase1.py:202-307."""
    out = {}
    rb = np.random.default_rng(11)
    n = 0
    for _ in range(60):
        N, K = int(rb.integers(3, 8)), int(rb.integers(2, 5))
        s = rb.standard_normal((N, K))
        c = rb.integers(1, 8, size=K)
        w = rb.integers(1, 4, size=N)
        lo, hi = int((w * c.min()).sum()), int((w * c.max()).sum())
        B = int(rb.integers(lo, hi + 1))
        z = manifold.dp_knapsack(s, c, w, B, use_topk=False)
        out.update({f"dp{n}_s": s, f"dp{n}_c": c, f"dp{n}_w": w, f"dp{n}_B": np.array(B),
                    f"dp{n}_z": z})
        n += 1
    # ties: zero scores pick the cheapest optimum (tests/test_rco_phase1.py:216-221)
    s = np.zeros((6, 3)); c = np.array([2, 3, 5]); w = np.ones(6, dtype=np.int64)
    out.update({f"dp{n}_s": s, f"dp{n}_c": c, f"dp{n}_w": w, f"dp{n}_B": np.array(20),
                f"dp{n}_z": manifold.dp_knapsack(s, c, w, 20)})
    n += 1
    # quantized scores: many exact ties inside the table
    s = rb.integers(-3, 4, size=(40, 4)).astype(np.float64)
    c = np.array([2, 3, 4, 8]); w = rb.integers(1, 6, size=40)
    B = int(0.6 * (w * c.max()).sum())
    out.update({f"dp{n}_s": s, f"dp{n}_c": c, f"dp{n}_w": w, f"dp{n}_B": np.array(B),
                f"dp{n}_z": manifold.dp_knapsack(s, c, w, B)})
    n += 1
    # the RCO decode at the Qwen2.5-0.5B budget: N = 168, options {2,3,4}, 3.0 bits -> B' = 9360
    w_int, unit = loop.integer_weights(np.array([802816, 114688, 114688, 802816,
                                                 4358144, 4358144, 4358144] * 24))
    out["qwen_w_int"], out["qwen_unit"] = w_int, np.array(unit)
    for r in range(3):
        s = rb.standard_normal((168, 3)) * (10.0 ** r)
        c = np.array([2, 3, 4])
        B = 3 * int(w_int.sum())
        out.update({f"dp{n}_s": s, f"dp{n}_c": c, f"dp{n}_w": w_int, f"dp{n}_B": np.array(B),
                    f"dp{n}_z": manifold.dp_knapsack(s, c, w_int, B)})
        n += 1
    # K = 6 at B' = 20000 (tests/test_rco_phase1.py:276-292)
    rl = np.random.default_rng(21)
    s = rl.standard_normal((168, 6)); c = np.array([1, 2, 3, 4, 6, 8])
    w = rl.integers(1, 40, size=168)
    out.update({f"dp{n}_s": s, f"dp{n}_c": c, f"dp{n}_w": w, f"dp{n}_B": np.array(20000),
                f"dp{n}_z": manifold.dp_knapsack(s, c, w, 20000)})
    n += 1
    # K = 2 uniform weights: the top-k shortcut (manifold.py:378-379)
    for _ in range(20):
        N = int(rb.integers(4, 12))
        s = rb.standard_normal((N, 2)); c = rb.integers(0, 6, size=2)
        w = np.full(N, int(rb.integers(1, 4)))
        base = int(N * w[0] * c.min())
        B = int(rb.integers(base, int(N * w[0] * c.max()) + 1))
        out.update({f"dp{n}_s": s, f"dp{n}_c": c, f"dp{n}_w": w, f"dp{n}_B": np.array(B),
                    f"dp{n}_z": manifold.dp_knapsack(s, c, w, B)})
        n += 1
    out["dp_n"] = np.array(n)
    np.savez_compressed(OUT / "dp.npz", **out)


def gen_rco_host(manifold, loop):
    """Host-side RCO math (rco/manifold.py:61-207, rco/loop.py:57-307) on small cases."""
    out = {}
    rng = np.random.default_rng(0)
    costs = np.array([2.0, 3.0, 4.0, 8.0])
    w = np.ones(20)
    a = rng.standard_normal((20, 4))
    out["a"], out["costs"], out["w"] = a, costs, w
    out["softmax"] = manifold.softmax(a)
    out["expected_cost"] = np.array(manifold.expected_cost(a, costs, w))
    out["normal"] = manifold.normal_vector(a, costs, w)
    g = rng.standard_normal((20, 4))
    out["g"] = g
    out["proj"] = manifold.project_tangent(g, out["normal"])
    out["retract_B52"] = manifold.retract(a, costs, w, budget=52.0)
    close = np.array([2.0, 2.1, 2.2, 2.3])
    abig = np.random.default_rng(0).standard_normal((20, 4)) * 30.0
    out["abig"], out["close"] = abig, close
    out["retract_big"] = manifold.retract(abig, close, w, budget=2.15 * 20)
    out["tau"] = np.array([loop.tau_schedule(t, 10) for t in range(10)])
    up = rng.standard_normal((20, 4)); p = manifold.softmax(a)
    out["up"], out["ste"] = up, loop.ste_grad(up, p, 0.3)
    ci, wi, Bi = loop.to_int_grid(costs, np.arange(1, 21), 2.5 * 210, ticks=2)
    out["tig_c"], out["tig_w"], out["tig_B"] = ci, wi, np.array(Bi)
    # rco_loop on a linear objective with the numpy Generator stream (loop.py:180-307)
    target = rng.standard_normal((12, 3))
    out["lin_target"] = target
    wl = np.array([7, 1, 1, 7, 38, 38, 38, 7, 1, 1, 7, 38])

    def grad_fn(z, p, t, j, rng_):
        return -target, float(-(z * target).sum())
    res = loop.rco_loop(np.zeros((12, 3)), np.array([2.0, 3.0, 4.0]), wl, 3.0 * wl.sum(),
                        steps=15, g=4, lr=0.1, seed=3, grad_fn=grad_fn)
    out["lin_w"] = wl
    out["lin_logits"], out["lin_m"], out["lin_v"] = res["logits"], res["momentum"], res["velocity"]
    out["lin_z"] = res["z_final"]
    out["lin_cost"] = np.array([h["cost"] for h in res["history"]])
    out["lin_loss"] = np.array([h["loss"] for h in res["history"]])
    np.savez_compressed(OUT / "rco_host.npz", **out)


def gen_gsq(gptq, quant, oracles):
    """Grid, schedules, local shift, inits (gsq/quant.py, gsq/gptq.py:192-232), and the
    reference test oracle's analytic 2-bit GSQ loss/gradients and Lion (tests/oracles.py)."""
    out = {}
    for b in range(1, 9):
        out[f"grid{b}"] = quant.get_grid(b)
    out["sched"] = np.array([quant.gs_schedules(t, 200) for t in range(200)])
    r = np.random.default_rng(11)
    j0 = r.integers(0, 8, size=512)
    out["ls_j0"] = j0
    out["ls_C"] = quant.local_shift_values(j0, quant.get_grid(3))
    lg = r.standard_normal((512, 5)).astype(np.float32)
    out["ls_logits"] = lg
    out["ls_idx"] = np.asarray(quant.local_shift_indices(j0, lg, 8))
    out["ls_edge"] = np.asarray(quant.local_shift_indices(
        np.array([0, 7]), np.array([[-99., -99., -99., -99., 99.], [99., -99., -99., -99., -99.]],
                                    dtype=np.float32), 8))
    out["init_shift"] = gptq.init_shift_logits(300, alpha=6.0, std=0.01, seed=5)
    codes = r.integers(0, 4, size=(8, 16)).astype(np.uint8)
    out["init2_codes"] = codes
    out["init2"] = gptq.init_logits_2bit_from_codes(codes, 4, alpha=6.0, std=0.01, seed=6)
    # tests/oracles.py:311-347, 2-bit full grid; the Gumbel draws are reproduced from the same
    # numpy stream (oracles.py:43-56) and stored so the restatement can be fed the same noise.
    X = oracles.synthetic_calibration(8, 16, 32, seed=2).astype(np.float64)
    W = oracles.synthetic_weights((16, 32), seed=1)
    rtn = gptq.quantize_rtn(W, 2, 16)
    logits = gptq.init_logits_2bit_from_codes(rtn["codes"], 4, seed=3).astype(np.float64)
    scales = rtn["scales"].astype(np.float64)
    tau, kappa = quant.gs_schedules(37, 200)
    loss, glog, gsc = oracles.linear_loss_and_grads_np(X, W, logits, quant.get_grid(2), scales,
                                                       16, tau, kappa, n_resamples=3, seed=9)
    rng = np.random.default_rng(9)
    noises = [oracles.sample_gumbel((W.size, 4), rng=rng) for _ in range(3)]
    out.update(lg_X=X, lg_W=W, lg_codes=rtn["codes"], lg_logits=logits, lg_scales=scales,
               lg_tau=np.array(tau), lg_kappa=np.array(kappa), lg_noise=np.stack(noises),
               lg_loss=np.array(loss), lg_glog=glog, lg_gscale=gsc)
    # oracles.Lion, three steps
    P = r.standard_normal((50,)).astype(np.float32)
    opt = oracles.Lion({"p": P}, lr=1e-2)
    Gs = r.standard_normal((3, 50)).astype(np.float32)
    traj = [P]
    for t in range(3):
        P = opt.step({"p": P}, {"p": Gs[t]})["p"]
        traj.append(P)
    out["lion_G"], out["lion_traj"] = Gs, np.stack(traj)
    np.savez_compressed(OUT / "gsq.npz", **out)


def gen_ternary(gptq, oracles):
    """Ternary (1-bit) soft weights: the mask / sign logit init (gsq/gptq.py:222-232) and the
    reference test oracle's soft and hard ternary weights (tests/oracles.py:92-103, 126-160)
    from fixed Gumbel draws, at a moderate and a saturating (tau, kappa)."""
    out = {}
    r = np.random.default_rng(21)
    q = r.integers(-1, 2, size=600).astype(np.float32)
    lm, lb = gptq.init_ternary_logits(q, alpha=3.0, std=0.01, seed=4)
    out.update(init_q=q, init_lm=lm, init_lb=lb)
    lm = r.standard_normal(600).astype(np.float32) * 0.05
    lb = r.standard_normal(600).astype(np.float32) * 0.05
    noise = np.stack([oracles.sample_gumbel((600,), rng=r) for _ in range(4)]).astype(np.float32)
    out.update(lm=lm, lb=lb, noise=noise, scale=np.float32(0.037))
    for j, (tau, kappa) in enumerate(((1.7, 6.0), (0.5, 200.0))):
        out[f"tau{j}"], out[f"kappa{j}"] = np.float64(tau), np.float64(kappa)
        out[f"soft{j}"] = np.asarray(oracles.ternary_soft(lm, lb, 0.037, tau, kappa,
                                                          noise=tuple(noise)))
    w, (m, b) = oracles.ternary_hard(lm, lb, 0.037)
    out.update(hard=np.asarray(w), hard_m=np.asarray(m), hard_b=np.asarray(b))
    np.savez_compressed(OUT / "ternary.npz", **out)


def gen_export():
    """Packed words of the MLX affine export (gsq/export.py:61-73, pack_codes; mlx_bits :52-58;
    bits_report :218-250 on the hand-made case of tests/test_export.py:139-150). export.py
    imports mlx.core for its scale casts only; the stand-in module gains the dtype names its
    module-level table reads (never called)."""
    core = sys.modules["mlx.core"]
    for name in ("bfloat16", "float16", "float32", "uint16", "uint32"):
        if not hasattr(core, name):
            setattr(core, name, object())
    import gsq_rco.gsq.export as ex
    out = {}
    rng = np.random.default_rng(7)
    for bits in (2, 3, 4, 5, 6, 8):
        codes = rng.integers(0, 1 << bits, size=(5, 256), dtype=np.uint8)
        codes[0] = 0
        codes[1] = (1 << bits) - 1
        codes[2, ::2] = (1 << bits) - 1
        out[f"codes{bits}"] = codes
        out[f"words{bits}"] = ex.pack_codes(codes, bits)
    ternary = rng.integers(0, 3, size=(3, 128), dtype=np.uint8)
    out["codes_t"], out["words_t"] = ternary, ex.pack_codes(ternary + np.uint8(1), ex.mlx_bits(1))
    out["mlx_bits"] = np.array([ex.mlx_bits(b) for b in (1, 2, 3, 4, 5, 6, 8)])
    hand = {"a": dict(codes=np.zeros((4, 128), np.uint8), scales=np.ones((4, 2), np.float16),
                      bits=2, group_size=64),
            "b": dict(codes=np.zeros((2, 64), np.uint8), scales=np.ones((2, 1), np.float16),
                      bits=1, group_size=64)}
    rep = ex.bits_report(hand, 640)
    for k in ("code_bpp", "native_bpp", "mlx_bpp", "shard_bpp"):
        out[f"report_{k}"] = np.float64(rep[k])
    np.savez_compressed(OUT / "export.npz", **out)


def main():
    import argparse
    global REF
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True,
                    help="path of a checkout of the reference repository")
    ap.add_argument("--only", default="gptq,dp,rco_host,gsq,ternary,export",
                    help="comma-separated fixture names to (re)generate")
    args = ap.parse_args()
    REF = Path(args.reference).resolve()
    only = set(args.only.split(","))
    gptq, quant, manifold, loop, oracles = _import_reference()
    gens = {"gptq": lambda: gen_gptq(gptq), "dp": lambda: gen_dp(manifold, loop),
            "rco_host": lambda: gen_rco_host(manifold, loop),
            "gsq": lambda: gen_gsq(gptq, quant, oracles),
            "ternary": lambda: gen_ternary(gptq, oracles), "export": gen_export}
    for name, gen in gens.items():
        if name in only:
            gen()
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
