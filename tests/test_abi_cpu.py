"""CPU checks: the C-ABI library loads and exports every declared symbol; the host-side
RCO math and validation follow the reference (golden vectors); no GPU needed."""
import os
import re

import numpy as np
import pytest

from gsq_rco_mlx_b200 import _lib
from gsq_rco_mlx_b200.gsq import quant
from gsq_rco_mlx_b200.rco import loop, manifold

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")


def declared_symbols():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"^(?:int|const char \*)\s*(\w+)\(", text, flags=re.M)
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
    assert set(_lib.SIGNATURES) | {"gsq_status_string"} >= set(names)
    assert lib.gsq_abi_version() == 2
    assert lib.gsq_status_string(1) == b"invalid argument"


def declared_arities():
    """{name: parameter count} of every function the headers declare (void lists count 0)."""
    out = {}
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if not fn.endswith(".h"):
            continue
        text = re.sub(r"/\*.*?\*/", " ", open(os.path.join(ROOT, "include", fn)).read(),
                      flags=re.S)
        for m in re.finditer(r"^(?:int|const char \*)\s*(\w+)\(([^)]*)\);", text, flags=re.M):
            params = m.group(2).strip()
            out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_signatures_match_the_header():
    """Every ctypes argument list in the package has as many entries as the declaration in
    include/ has parameters (an ABI drift would pass wrong values silently)."""
    arity = declared_arities()
    assert len(arity) == len(declared_symbols())
    for name, argtypes in _lib.SIGNATURES.items():
        assert name in arity, name
        assert len(argtypes) == arity[name], (name, len(argtypes), arity[name])


def test_bad_arguments_are_rejected_without_launch():
    """Argument validation happens before any CUDA call (no device needed)."""
    lib = _lib.load()
    assert lib.gsq_soft_fwd(None, None, None, None, 0, 0, 0, 0, 4, 4, 64, 3, 1.0, 100.0,
                            None, None, None, None, None) == _lib.GSQ_EINVAL
    assert lib.gsq_soft_fwd(None, None, None, None, 0, 0, 0, 0, 4, 4, 64, 8, 1.0, 100.0,
                            None, None, None, None, None) == _lib.GSQ_ENOTSUP
    assert lib.mckp_dp_f64(None, None, 1, 3, 2, 10, None, None, None, None) == _lib.GSQ_EINVAL
    # the allocation-free DP refuses null pointers and sizes beyond its fixed array before
    # touching the device
    import ctypes as C
    fake = C.c_void_p(256)  # never dereferenced: every call below is refused first
    assert lib.mckp_dp_f64_noalloc(None, fake, 1, 168, 3, 9360, fake, None) == _lib.GSQ_EINVAL
    assert lib.mckp_dp_f64_noalloc(fake, None, 1, 168, 3, 9360, fake, None) == _lib.GSQ_EINVAL
    assert lib.mckp_dp_f64_noalloc(fake, fake, 1, 168, 3, 9360, None, None) == _lib.GSQ_EINVAL
    assert lib.mckp_dp_f64_noalloc(fake, fake, 1, 168, 3, 20000, fake, None) == _lib.GSQ_EINVAL
    assert lib.mckp_dp_f64_noalloc(fake, fake, 20, 168, 3, 9360, fake, None) == _lib.GSQ_EINVAL
    assert lib.mckp_dp_f64_noalloc(fake, fake, 1, 168, 300, 100, fake, None) == _lib.GSQ_EINVAL
    assert lib.gptq_sweep(None, None, None, 4, 4, 3, 64, 128, 1, None, None, None,
                          None) == _lib.GSQ_EINVAL
    # the KL head entry: null pointers, widths that are not multiples of 8, a short ET stride
    kl = lambda *a: lib.kl_head_fwd_bwd(*a)
    ok = [fake, fake, 40, 896, fake, fake, 151936, 151936, 32, fake, fake, fake, fake, fake,
          fake, fake, None]
    for i, bad in [(0, None), (4, None), (15, None), (3, 900), (7, 151930), (6, 151928),
                   (8, 0), (2, 0)]:
        args = list(ok)
        args[i] = bad
        assert kl(*args) == _lib.GSQ_EINVAL, (i, bad)
    assert lib.gsq_soft_bwd_lion(None, None, None, None, None, None, None, 2, 4, 4, 64, 3, 1.0,
                                 100.0, 1e-4, 5e-5, 1.0, 0.9, 0.95, 0, None, 0, 0, 0, 1.0, 1.0,
                                 None, None, None, None) == _lib.GSQ_EINVAL


def test_product_path_refuses_to_run_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError):
        _lib.lib()


def test_host_grid_and_schedules():
    z = np.load(os.path.join(GOLD, "gsq.npz"))
    for b in range(1, 9):
        assert np.array_equal(quant.get_grid(b), z[f"grid{b}"])
    assert np.array_equal(np.array([quant.gs_schedules(t, 200) for t in range(200)]), z["sched"])
    assert np.array_equal(quant.local_shift_values(z["ls_j0"], quant.get_grid(3)), z["ls_C"])
    assert np.array_equal(quant.local_shift_indices(z["ls_j0"], z["ls_logits"], 8), z["ls_idx"])


def _retract_ok(out, a, c, w, budget, gold, tol=1e-8):
    """out is a + t c for one scalar t, meets the budget to tol, and its shift is within the
    tolerance's reach of the reference's shift (both are valid retractions: any t with
    |C - B| <= tol is one; the slope of C along c bounds how far two such t can be apart)."""
    t = (out - a) / c[None, :]
    assert np.allclose(t, t.flat[0], rtol=0, atol=1e-9 * max(1.0, abs(t.flat[0])))
    assert abs(manifold.expected_cost(out, c, w) - budget) <= tol
    t_gold = float(((gold - a) / c[None, :]).mean())
    _, slope = manifold.Budget(c, w).cost_and_slope(out)
    assert abs(t.flat[0] - t_gold) <= 2 * tol / slope + 1e-12


def test_host_manifold_matches_reference():
    z = np.load(os.path.join(GOLD, "rco_host.npz"))
    a, c, w = z["a"], z["costs"], z["w"]
    np.testing.assert_allclose(manifold.softmax(a), z["softmax"], rtol=1e-15)
    assert manifold.expected_cost(a, c, w) == pytest.approx(float(z["expected_cost"]), rel=1e-15)
    np.testing.assert_allclose(manifold.normal_vector(a, c, w), z["normal"], rtol=1e-14,
                               atol=1e-15)
    np.testing.assert_allclose(manifold.project_tangent(z["g"], z["normal"]), z["proj"],
                               rtol=1e-13, atol=1e-15)
    _retract_ok(manifold.retract(a, c, w, budget=52.0), a, c, w, 52.0, z["retract_B52"])
    _retract_ok(manifold.retract(z["abig"], z["close"], w, budget=2.15 * 20), z["abig"],
                z["close"], w, 2.15 * 20, z["retract_big"])
    assert np.array_equal(np.array([loop.tau_schedule(t, 10) for t in range(10)]), z["tau"])
    np.testing.assert_allclose(loop.ste_grad(z["up"], manifold.softmax(a), 0.3), z["ste"],
                               rtol=1e-14, atol=1e-15)
    ci, wi, Bi = loop.to_int_grid(c, np.arange(1, 21), 2.5 * 210, ticks=2)
    assert np.array_equal(ci, z["tig_c"]) and np.array_equal(wi, z["tig_w"]) and Bi == int(z["tig_B"])
    with pytest.raises(ValueError):
        manifold.retract(a, c, w, budget=160.5)        # above every reachable cost
    with pytest.raises(ValueError):
        manifold.retract(a, c, w, budget=52.0, max_shift=1e-3)   # no bracket within reach
    with pytest.raises(RuntimeError):
        manifold.retract(a, c, w, budget=52.0, iters=1, tol=1e-300)
    with pytest.raises(ValueError):
        loop.to_int_grid(c, np.full(20, 1.5), 10.0)


def test_rco_loop_matches_reference_trajectory():
    """rco_loop on the reference's linear objective (15 steps, g = 4, seed 3): the random
    stream, Adam, retraction and transport follow the reference's run, and the decoded
    allocation is identical. The knapsack decode is the oracle's (no GPU here)."""
    from oracle import dp as odp
    z = np.load(os.path.join(GOLD, "rco_host.npz"))
    target, wl = z["lin_target"], z["lin_w"]

    def grad_fn(zz, p, t, j, rng_):
        return -target, float(-(zz * target).sum())
    res = loop.rco_loop(np.zeros((12, 3)), np.array([2.0, 3.0, 4.0]), wl, 3.0 * wl.sum(),
                        steps=15, g=4, lr=0.1, seed=3, grad_fn=grad_fn,
                        decode=odp.dp_knapsack)
    np.testing.assert_allclose(res["logits"], z["lin_logits"], rtol=1e-6, atol=1e-8)
    np.testing.assert_allclose(res["momentum"], z["lin_m"], rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(res["velocity"], z["lin_v"], rtol=1e-5, atol=1e-12)
    assert np.array_equal(res["z_final"], z["lin_z"])
    np.testing.assert_allclose([h["cost"] for h in res["history"]], z["lin_cost"], atol=2e-8)
    np.testing.assert_array_equal([h["loss"] for h in res["history"]], z["lin_loss"])
    with pytest.raises(ValueError):
        loop.rco_loop(np.zeros((12, 3)), np.array([2.0, 3.0, 4.0]), wl, 3.0 * wl.sum())


def test_integer_weights_and_dp_validation():
    w, unit = loop.integer_weights(np.array([802816, 114688, 114688, 802816,
                                             4358144, 4358144, 4358144] * 24))
    z = np.load(os.path.join(GOLD, "dp.npz"))
    assert unit == int(z["qwen_unit"]) == 114688
    assert np.array_equal(w, z["qwen_w_int"])
    with pytest.raises(ValueError):
        manifold.dp_knapsack(np.zeros((3, 2)), np.array([2, 3]), np.ones(3, dtype=int), 5)
    with pytest.raises(ValueError):
        manifold.dp_knapsack(np.zeros((3, 2)), np.array([2.5, 3.0]), np.ones(3, dtype=int), 9)
    # K = 2 uniform weights decodes on the host (no GPU needed), as in the reference
    for n in range(int(z["dp_n"])):
        s, c, wv, B = z[f"dp{n}_s"], z[f"dp{n}_c"], z[f"dp{n}_w"], int(z[f"dp{n}_B"])
        if s.shape[1] == 2 and np.all(wv == wv[0]):
            assert np.array_equal(manifold.dp_knapsack(s, c, wv, B), z[f"dp{n}_z"])


def test_gemm_descriptor_layout_matches_header(tmp_path):
    """The ctypes mirror of gsq_gemm_desc has the C struct's size and field offsets."""
    import ctypes
    import shutil
    import subprocess
    from gsq_rco_mlx_b200.gemm import GemmDesc
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    names = [f[0] for f in GemmDesc._fields_]
    src = tmp_path / "off.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "gsq_rco_b200.h"\n'
                   'int main(void){printf("%zu", sizeof(gsq_gemm_desc));\n' +
                   "".join(f'printf(" %zu", offsetof(gsq_gemm_desc, {n}));\n' for n in names) +
                   'return 0;}\n')
    exe = tmp_path / "off"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(GemmDesc)
    assert vals[1:] == [getattr(GemmDesc, n).offset for n in names]


def declared_arities():
    """{name: number of parameters} of every prototype in include/*.h."""
    out = {}
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^(?:int|const char \*)\s*(\w+)\(([^;]*?)\)\s*;", text,
                             flags=re.M | re.S):
            params = " ".join(m.group(2).split())
            out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_signatures_match_header_arity():
    """Every ctypes binding in _lib.SIGNATURES has as many arguments as the header's
    prototype, so the Python side cannot drift from the C ABI silently."""
    arity = declared_arities()
    assert len(arity) >= 14
    for name, argtypes in _lib.SIGNATURES.items():
        assert name in arity, name
        assert len(argtypes) == arity[name], (name, len(argtypes), arity[name])
