"""C backend of the GSQ oracle's elementwise passes (TEST INFRASTRUCTURE ONLY).

Same arithmetic as oracle/gsq.py and oracle/philox.py (numpy), in oracle/gsq_c.c split over the
host's cores. It makes parity runs at full layer sizes (up_proj: 4.36M weights x 5 candidates,
200 steps) finish in minutes; tests/test_oracle_golden.py checks it against the numpy
restatement. ``oracle.gsq.set_backend("c")`` switches the oracle's training loops to it.
"""
from __future__ import annotations

import ctypes as C
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build", "libgsq_oracle.so")
_lib = None
_pool = None
_THREADS = max(1, min(32, os.cpu_count() or 1))


def lib():
    global _lib, _pool
    if _lib is None:
        if not os.path.exists(_PATH):
            raise RuntimeError(f"{_PATH} is missing: run `make -C oracle`")
        L = C.CDLL(_PATH)
        vp, i32, i64, u32, u64, f32, f64 = (C.c_void_p, C.c_int, C.c_int64, C.c_uint32,
                                            C.c_uint64, C.c_float, C.c_double)
        L.og_gumbel_planes.argtypes = [u64, u32, u32, u32, i64, i32, vp, i64, i64]
        L.og_soft_weight.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, f32, f32, vp, vp, vp,
                                     i64, i64]
        L.og_soft_backward_acc.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, f64, f64,
                                           vp, vp, i64, i64]
        L.og_scale_grad_acc.argtypes = [vp, vp, i32, i32, i32, vp, i64, i64]
        L.og_lion.argtypes = [vp, vp, vp, f32, f32, f32, f32, f32, f32, i64, i64]
        for fn in (L.og_gumbel_planes, L.og_soft_weight, L.og_soft_backward_acc,
                   L.og_scale_grad_acc, L.og_lion):
            fn.restype = None
        _lib = L
        _pool = ThreadPoolExecutor(max_workers=_THREADS)
    return _lib


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def _over(n, fn):
    """fn(i0, i1) over [0, n) in one chunk per host thread."""
    lib()
    step = -(-n // _THREADS)
    list(_pool.map(lambda i0: fn(i0, min(n, i0 + step)), range(0, n, step)))


def gumbel_planes(seed, linear_id, step, resample, d, n_planes):
    out = np.empty((n_planes, d), dtype=np.float32)
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    _over(d, lambda a, b: _lib.og_gumbel_planes(seed, int(linear_id) & 0xFFFFFFFF, int(step),
                                                 int(resample), d, n_planes, _ptr(out), a, b))
    return out


def soft_weight(logits_kd, noise_kd, Ckd, scales, shape, group_size, tau, kappa):
    """(w_bar [out, in], p [K, d], c [out, in]) float32, as oracle.gsq.soft_weight."""
    out_f, in_f = shape
    K, d = logits_kd.shape
    lg = np.ascontiguousarray(logits_kd, dtype=np.float32)
    nz = np.ascontiguousarray(noise_kd, dtype=np.float32)
    ck = np.ascontiguousarray(Ckd, dtype=np.float32)
    sc = np.ascontiguousarray(scales, dtype=np.float32)
    w = np.empty(d, dtype=np.float32)
    c = np.empty(d, dtype=np.float32)
    p = np.empty((K, d), dtype=np.float32)
    _over(d, lambda a, b: _lib.og_soft_weight(_ptr(lg), _ptr(nz), _ptr(ck), _ptr(sc), out_f,
                                               in_f, int(group_size), K, float(np.float32(tau)),
                                               float(np.float32(kappa)), _ptr(w), _ptr(p),
                                               _ptr(c), a, b))
    return w.reshape(shape), p, c.reshape(shape)


def soft_backward_acc(G, p, Ckd, c, scales, group_size, tau, kappa, glog_acc, gs_acc):
    """glog_acc [K, d] += float32(dL/dlogits), gs_acc [out, G] += float32(dL/dscales) of one
    draw with G = dL/dw_bar [out, in] (float64), as oracle.gsq.soft_backward."""
    out_f, in_f = G.shape
    K, d = p.shape
    Gd = np.ascontiguousarray(G, dtype=np.float64)
    pp = np.ascontiguousarray(p, dtype=np.float32)
    ck = np.ascontiguousarray(Ckd, dtype=np.float32)
    cc = np.ascontiguousarray(c, dtype=np.float32)
    sc = np.ascontiguousarray(scales, dtype=np.float32)
    assert glog_acc.flags.c_contiguous and gs_acc.flags.c_contiguous
    _over(d, lambda a, b: _lib.og_soft_backward_acc(_ptr(Gd), _ptr(pp), _ptr(ck), _ptr(cc),
                                                     _ptr(sc), out_f, in_f, int(group_size), K,
                                                     float(tau), float(kappa), _ptr(glog_acc),
                                                     None, a, b))
    _over(gs_acc.size, lambda a, b: _lib.og_scale_grad_acc(_ptr(Gd), _ptr(cc), out_f, in_f,
                                                            int(group_size), _ptr(gs_acc), a, b))


def lion_(P, M, G, lr, wd, betas):
    """In-place float32 Lion on contiguous P, M with gradient G, as oracle.gsq.lion."""
    b1, b2 = betas
    f = np.float32
    Gf = np.ascontiguousarray(G, dtype=np.float32)
    assert P.dtype == np.float32 and M.dtype == np.float32
    assert P.flags.c_contiguous and M.flags.c_contiguous
    args = (float(f(lr)), float(f(wd)), float(f(b1)), float(f(1 - b1)), float(f(b2)),
            float(f(1 - b2)))
    _over(P.size, lambda a, b: _lib.og_lion(_ptr(P), _ptr(M), _ptr(Gf), *args, a, b))
