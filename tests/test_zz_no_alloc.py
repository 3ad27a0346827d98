"""The allocation-free DP entry point (mckp_dp_f64_noalloc) against the allocating one.

Some callers of this library cannot allocate device memory: a serving runtime that owns every
device byte through its own pool, or a host-language binding with no CUDA allocator. The
allocation-free entry point keeps its scratch (the DP choice table) in a fixed array inside the
library. This file is collected last on purpose; the test passes alone in a fresh process and
after the other tests, and runs two calls in a row, because the array is shared by every call
and keeps the previous call's contents."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _decode(lib, name, S, step, B, choice=None):
    dev = torch.device("cuda", 0)
    n_inst, N, K = S.shape
    s_t = torch.as_tensor(np.ascontiguousarray(S), device=dev)
    st_t = torch.as_tensor(np.ascontiguousarray(step), device=dev)
    z = torch.full((n_inst, N), -1, device=dev, dtype=torch.int32)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if name == "mckp_dp_f64":
        ch = torch.empty(n_inst * N * (B + 1), device=dev, dtype=torch.uint8)
        rc = lib.mckp_dp_f64(C.c_void_p(s_t.data_ptr()), C.c_void_p(st_t.data_ptr()), n_inst, N,
                             K, B, C.c_void_p(ch.data_ptr()), None, C.c_void_p(z.data_ptr()),
                             stream)
    else:
        rc = lib.mckp_dp_f64_noalloc(C.c_void_p(s_t.data_ptr()), C.c_void_p(st_t.data_ptr()),
                                     n_inst, N, K, B, C.c_void_p(z.data_ptr()), stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return z.cpu().numpy()


def test_noalloc_dp_matches_allocating_dp_twice():
    from gsq_rco_mlx_b200 import _lib
    lib = _lib.lib()
    w = np.array([7, 1, 1, 7, 38, 38, 38] * 24, dtype=np.int64)
    costs = np.array([2, 3, 4], dtype=np.int64)
    step = w[:, None] * costs[None, :]
    B = 3 * int(w.sum())
    rng = np.random.default_rng(12)
    # two calls in a row, different scores and instance counts: the second call must not see
    # anything of the first in the shared array
    for n_inst, scale in ((8, 1.0), (3, 100.0)):
        S = rng.standard_normal((n_inst, 168, 3)) * scale
        z_ref = _decode(lib, "mckp_dp_f64", S, step, B)
        z_new = _decode(lib, "mckp_dp_f64_noalloc", S, step, B)
        assert np.array_equal(z_new, z_ref)
        assert np.all((z_new >= 0) & (z_new < 3))
    # sizes beyond the fixed array or the shared-memory rows are refused with GSQ_EINVAL
    dev = torch.device("cuda", 0)
    s_t = torch.zeros(1, 168, 3, device=dev, dtype=torch.float64)
    st_t = torch.as_tensor(step, device=dev)
    z = torch.zeros(1, 168, device=dev, dtype=torch.int32)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.mckp_dp_f64_noalloc(C.c_void_p(s_t.data_ptr()), C.c_void_p(st_t.data_ptr()), 1,
                                   168, 3, 20000, C.c_void_p(z.data_ptr()), stream) == _lib.GSQ_EINVAL
    assert lib.mckp_dp_f64_noalloc(C.c_void_p(s_t.data_ptr()), C.c_void_p(st_t.data_ptr()), 20,
                                   168, 3, 9360, C.c_void_p(z.data_ptr()), stream) == _lib.GSQ_EINVAL
