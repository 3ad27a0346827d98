"""ctypes binding of libgsqrco_b200.so (the C ABI in include/gsq_rco_b200.h).

The library is the only compute path of this package: if it is missing, or no CUDA device is
present, every call raises. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libgsqrco_b200.so"

GSQ_OK, GSQ_EINVAL, GSQ_ECUDA, GSQ_ETIMEOUT, GSQ_ENOTSUP = range(5)

_vp, _i32, _i64, _u32, _u64, _f32, _f64 = (C.c_void_p, C.c_int, C.c_int64, C.c_uint32,
                                             C.c_uint64, C.c_float, C.c_double)

# name -> argument types (restype is int for every entry point except the status string)
SIGNATURES = {
    "gsq_abi_version": [],
    "gsq_soft_fwd": [_vp, _vp, _vp, _vp, _u64, _u32, _u32, _u32, _i32, _i32, _i32, _i32, _f32,
                     _f32, _vp, _vp, _vp, _vp, _vp],
    "gsq_soft_step": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32,
                      _f32, _f32, _f32, _f64, _f64, _f64, _i32, _vp, _u64, _u32, _u32, _f32,
                      _f32, _vp, _vp, _vp, _vp],
    "gsq_soft_bwd_lion": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                          _f32, _f32, _f32, _f32, _f64, _f64, _f64, _i32, _vp, _u64, _u32, _u32,
                          _f32, _f32, _vp, _vp, _vp, _vp],
    "gsq_harden": [_vp, _vp, _i32, _i32, _i32, _vp, _vp],
    "gsq_lion_f32": [_vp, _vp, _vp, _i64, _f32, _f64, _f64, _f64, _vp],
    "gsq_gemm_f32": [_i32, _i32, _i32, _f32, _vp, _i64, _i64, _vp, _i64, _i64, _f32, _vp, _i64,
                     _vp],
    "gsq_gemm_f64": [_i32, _i32, _i32, _f64, _vp, _i64, _i64, _vp, _i64, _i64, _f64, _vp, _i64,
                     _i32, _vp],
    "gsq_sumsq_f32": [_vp, _i64, _vp, _vp, _vp],
    "gsq_gemm_tc": [_i32, _i32, _i32, _vp, _i32, _i64, _vp, _i32, _i64, _i32, _f32, _vp, _i64,
                    _f32, _vp, _i32, _i64, _vp, _i32, _i64, _vp, _vp, _vp],
    "gsq_split_bf16": [_vp, _i32, _i32, _i64, _i32, _vp, _vp, _vp, _i64, _vp],
    "gsq_gemm": [_vp, _vp],
    "gsq_gemm_plan_create": [_vp, _vp],
    "gsq_gemm_plan_run": [_vp, _vp],
    "gsq_gemm_plan_destroy": [_vp],
    "gsq_rmsnorm": [_vp, _i64, _vp, _i32, _i32, _f32, _vp, _i64, _vp, _i64, _i32, _i32, _vp],
    "gsq_rope_split": [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp],
    "gsq_softmax_causal": [_vp, _i32, _i32, _vp, _vp, _vp],
    "gsq_softmax_causal_rows": [_vp, _i32, _i32, _i32, _i64, _i32, _vp, _i64, _vp],
    "gsq_kl_rows": [_vp, _vp, _i32, _i32, _i64, _vp, _i64, _vp, _vp, _vp],
    "kl_head_fwd_bwd": [_vp, _vp, _i32, _i32, _vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp,
                        _vp, _vp, _vp, _vp],
    "gsq_div_bf16": [_vp, _i64, _f32, _vp],
    "gsq_dequant_bf16": [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp],
    "gsq_rmsnorm_bwd": [_vp, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _f64, _vp],
    "gsq_softmax_bwd": [_vp, _vp, _i32, _i32, _i64, _vp, _vp, _vp, _i64, _f32, _vp],
    "gsq_rope_bwd": [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _i64, _i32, _vp],
    "gsq_group_sum": [_vp, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _i64, _i32, _vp],
    "ste_dots": [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _vp],
    "gsq_embed": [_vp, _i64, _vp, _i32, _vp, _vp],
    "gsq_hess_accum": [_vp, _vp, _i64, _f64, _f64, _vp],
    "gsq_zero_cols": [_vp, _i32, _i64, _i32, _i32, _vp],
    "gsq_gather_split": [_vp, _i32, _i64, _vp, _i32, _i64, _i32, _i32, _i32, _i32, _vp, _i64,
                         _vp, _i64, _vp],
    "gsq_transpose_bf16": [_vp, _i32, _i32, _i64, _i64, _vp, _i64, _i64, _i32, _i32, _vp],
    "gsq_head_group_sum_t": [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _i64, _vp],
    "gsq_sum_f64": [_vp, _i32, _vp, _vp],
    "gsq_dot_terms": [_vp, _vp, _vp, _i64, _vp, _i64, _i32, _i32, _f64, _vp, _vp, _vp],
    "hessian_accum": [_vp, _i64, _i32, _vp, _i64, _vp],
    "gptq_factor": [_vp, _i32, _f64, _vp, _vp, _vp, _vp, _vp],
    "gptq_sweep": [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp],
    "gptq_dequant": [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp],
    "gptq_err": [_vp, _vp, _vp, _i32, _i32, _vp, _vp, _vp],
    "mckp_dp_f64": [_vp, _vp, _i32, _i32, _i32, _i64, _vp, _vp, _vp, _vp],
    "mckp_dp_f64_noalloc": [_vp, _vp, _i32, _i32, _i32, _i64, _vp, _vp],
    "qdequant_packed": [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp],
    "qgemm_packed": [_vp, _i32, _i32, _i64, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _i64,
                     _i32, _vp, _i64, _vp, _vp],
    "gsq_nll_rows": [_vp, _i32, _i32, _i64, _vp, _vp, _vp],
    "gsq_scale_grad": [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp],
}

_lib = None


class GsqError(RuntimeError):
    """A nonzero status from the CUDA library."""


def load():
    """Load the shared library (no GPU needed); raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with python -m gsq_rco_mlx_b200.build")
    lib = C.CDLL(str(LIB_PATH))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = C.c_int
    lib.gsq_status_string.argtypes = [C.c_int]
    lib.gsq_status_string.restype = C.c_char_p
    _lib = lib
    return lib


def lib():
    """The library, on a machine with a CUDA device (the product path requires one)."""
    if not torch.cuda.is_available():
        raise RuntimeError("gsq_rco_mlx_b200 needs a CUDA GPU (sm_100a); none is available")
    return load()


def check(status: int, what: str):
    if status != GSQ_OK:
        msg = load().gsq_status_string(status).decode()
        if status in (GSQ_EINVAL,):
            raise ValueError(f"{what}: {msg}")
        if status == GSQ_ENOTSUP:
            raise NotImplementedError(f"{what}: {msg}")
        raise GsqError(f"{what}: {msg} (status {status})")


def ptr(t):
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


def stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


class Launches:
    """Count of entry-point calls (each launches one kernel; gemm() adds the split-K reduce):
    the bench's `gpu_launches`. Increment is a Python add per call."""
    n = 0


def call(name: str, *args):
    """Call an entry point and raise on a nonzero status."""
    Launches.n += 1
    check(getattr(lib(), name)(*args), name)


def device():
    return torch.device("cuda", torch.cuda.current_device())


_SMS = {}


def num_sms(dev=None):
    """Streaming multiprocessors of the device (148 on B200)."""
    import torch
    d = torch.device(dev) if dev is not None else device()
    key = str(d)
    if key not in _SMS:
        _SMS[key] = torch.cuda.get_device_properties(d).multi_processor_count
    return _SMS[key]
