"""Float32-faithful contractions of the GSQ step on CUDA tensors.

  mm_nt(A, B)  = alpha * A @ B.T     A [M, K], B [N, K]   (the forward residual X (W_bar - W)^T)
  mm_tn(A, B)  = alpha * A.T @ B     A [K, M], B [K, N]   (the weight gradient R^T X)
  sumsq(x)     = sum(x^2) in float64 (deterministic)
"""
from __future__ import annotations

import torch

from . import _lib


def _f32(t):
    if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
        raise ValueError("expected a contiguous CUDA float32 tensor")
    return t


def mm_nt(A, B, alpha=1.0, out=None):
    _f32(A), _f32(B)
    M, K = A.shape
    N, K2 = B.shape
    if K != K2:
        raise ValueError(f"inner dims differ: {K} vs {K2}")
    out = torch.empty(M, N, device=A.device, dtype=torch.float32) if out is None else _f32(out)
    _lib.call("gsq_gemm_f32", M, N, K, float(alpha), _lib.ptr(A), K, 1, _lib.ptr(B), 1, K, 0.0,
              _lib.ptr(out), N, _lib.stream_ptr())
    return out


def mm_tn(A, B, alpha=1.0, out=None):
    _f32(A), _f32(B)
    K, M = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"inner dims differ: {K} vs {K2}")
    out = torch.empty(M, N, device=A.device, dtype=torch.float32) if out is None else _f32(out)
    _lib.call("gsq_gemm_f32", M, N, K, float(alpha), _lib.ptr(A), 1, M, _lib.ptr(B), N, 1, 0.0,
              _lib.ptr(out), N, _lib.stream_ptr())
    return out


class SumSq:
    """Reusable float64 sum-of-squares accumulator (keeps its partials buffer)."""

    def __init__(self, device):
        self.partials = torch.empty(1024, device=device, dtype=torch.float64)

    def __call__(self, x, out):
        _f32(x)
        _lib.call("gsq_sumsq_f32", _lib.ptr(x), x.numel(), _lib.ptr(self.partials), _lib.ptr(out),
                  _lib.stream_ptr())
        return out


# ------------------------------------------------------------ tensor-core engine ---

import ctypes as _C


def pad8(n: int) -> int:
    """Leading dimension for TMA: rows of a multiple of 16 bytes (8 bf16)."""
    return (int(n) + 7) // 8 * 8


class Terms:
    """An fp32 matrix held as up to three bf16 terms [rows, ld] (K-major GEMM operand)."""

    def __init__(self, rows, cols, n_terms=3, device=None, ld=None, tensors=None):
        self.rows, self.cols, self.n = int(rows), int(cols), int(n_terms)
        self.ld = pad8(cols) if ld is None else int(ld)
        if tensors is not None:
            # views of existing storage, e.g. one slice of a [R][3][rows][ld] buffer
            self.t = list(tensors)[:self.n]
            for t in self.t:
                assert t.dtype == torch.bfloat16 and t.shape == (self.rows, self.ld)
            return
        dev = device or _lib.device()
        self.t = [torch.zeros(self.rows, self.ld, device=dev, dtype=torch.bfloat16)
                  for _ in range(self.n)]

    def ptrs(self, n=None):
        n = self.n if n is None else n
        arr = (_C.c_void_p * 3)()
        for i in range(n):
            arr[i] = self.t[i].data_ptr()
        return arr

    def value(self):
        """fp32 reconstruction (tests)."""
        v = self.t[0][:, :self.cols].float()
        for t in self.t[1:]:
            v = v + t[:, :self.cols].float()
        return v


def split_into(x, terms: Terms, transpose=False):
    """Write fp32 x [r, c] (or x^T) into ``terms``."""
    _f32(x)
    r, c = x.shape
    if transpose:
        assert (terms.rows, terms.cols) == (c, r)
    else:
        assert (terms.rows, terms.cols) == (r, c)
    p = [terms.t[i] if i < terms.n else None for i in range(3)]
    _lib.call("gsq_split_bf16", _lib.ptr(x), r, c, c, int(transpose), _lib.ptr(p[0]),
              _lib.ptr(p[1]), _lib.ptr(p[2]), terms.ld, _lib.stream_ptr())
    return terms


_ERR = {}


def err_flag(dev):
    if dev not in _ERR:
        _ERR[dev] = torch.zeros(1, device=dev, dtype=torch.int32)
    return _ERR[dev]


def check_err(dev):
    e = int(err_flag(dev).item())
    if e:
        raise _lib.GsqError(f"tensor-core GEMM: bounded wait timed out (code {e})")


class GemmDesc(_C.Structure):
    """ctypes mirror of gsq_gemm_desc (include/gsq_rco_b200.h)."""
    _fields_ = [
        ("M", _C.c_int), ("N", _C.c_int), ("K", _C.c_int), ("batch", _C.c_int),
        ("a", _C.c_void_p * 3), ("na", _C.c_int), ("lda", _C.c_int64), ("a_rows", _C.c_int64),
        ("b", _C.c_void_p * 3), ("b2", _C.c_void_p * 3), ("nb", _C.c_int), ("ldb", _C.c_int64),
        ("b_rows", _C.c_int64),
        ("order", _C.c_int), ("causal", _C.c_int), ("epi", _C.c_int), ("bn", _C.c_int),
        ("alpha", _C.c_float), ("beta", _C.c_float),
        ("C", _C.c_void_p), ("ldc", _C.c_int64),
        ("cs", _C.c_void_p * 3), ("ncs", _C.c_int), ("ldcs", _C.c_int64),
        ("ct", _C.c_void_p * 3), ("nct", _C.c_int), ("ldct", _C.c_int64), ("ct_up_rows", _C.c_int64),
        ("sq_partial", _C.c_void_p), ("bias", _C.c_void_p), ("resid", _C.c_void_p),
        ("target", _C.c_void_p), ("ld_rt", _C.c_int64), ("out_scale", _C.c_float),
        ("aux0", _C.c_void_p), ("aux1", _C.c_void_p), ("ld_aux", _C.c_int64),
        ("a_div", _C.c_int), ("a_s1", _C.c_int64), ("a_s2", _C.c_int64),
        ("b_div", _C.c_int), ("b_s1", _C.c_int64), ("b_s2", _C.c_int64),
        ("c_div", _C.c_int), ("c_s1", _C.c_int64), ("c_s2", _C.c_int64),
        ("t_div", _C.c_int), ("t_r1", _C.c_int64), ("t_r2", _C.c_int64), ("t_c1", _C.c_int64),
        ("t_c2", _C.c_int64),
        ("err", _C.c_void_p),
        ("skip_upper", _C.c_int),
        ("row_period", _C.c_int),
        ("split_k", _C.c_int),
        ("workspace", _C.c_void_p),
        ("a_major", _C.c_int),
        ("b_major", _C.c_int),
        ("small_bufs", _C.c_int),
    ]


_WS = {}


def _workspace(dev, n_floats):
    """A per-device float32 split-K workspace of at least n_floats (grown on demand)."""
    key = str(dev)
    ws = _WS.get(key)
    if ws is None or ws.numel() < n_floats:
        ws = torch.empty(int(n_floats), device=dev, dtype=torch.float32)
        _WS[key] = ws
    return ws


def auto_split(M, N, K, bn=128):
    """Number of k-parts for an output of fewer tiles than SMs: the split s <= k-blocks / 3
    that minimises ceil(tiles * s / SMs) / s (waves times the per-part k-length)."""
    tiles = -(-M // 128) * -(-N // bn)
    kb = -(-K // 64)
    sms = _lib.num_sms()
    if tiles >= sms:
        return 1
    best, best_cost = 1, None
    for s in range(1, max(1, kb // 3) + 1):
        cost = -(-tiles * s // sms) / s
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = s, cost
    return best


def _tp(t):
    return None if t is None else t.data_ptr()


class LaunchLog:
    """Optional per-launch CUDA events of gemm() calls (for roofline measurements): while
    active, every call records (M, N, K, products, batch, start, end, tag); ``tag`` is the
    log's current tag (a stage name) at the call. ``batch`` is the work in M x N x K boxes:
    the batch count, halved for causal and skip-upper (triangular) products."""
    active = None

    def __init__(self):
        self.rows = []
        self.tag = None

    def __enter__(self):
        LaunchLog.active = self
        return self

    def __exit__(self, *a):
        LaunchLog.active = None

    def summary(self):
        torch.cuda.synchronize()
        out = []
        for (M, N, K, prods, batch, e0, e1, tag) in self.rows:
            out.append((M, N, K, prods, batch, e0.elapsed_time(e1)))
        return out

    def by_tag(self):
        """{tag: [(M, N, K, products, batch, ms), ...]}."""
        torch.cuda.synchronize()
        out = {}
        for (M, N, K, prods, batch, e0, e1, tag) in self.rows:
            out.setdefault(tag, []).append((M, N, K, prods, batch, e0.elapsed_time(e1)))
        return out


def _describe(A: Terms, B: Terms, M=None, N=None, K=None, na=None, nb=None, order=2, alpha=1.0,
         beta=0.0, C=None, ldc=None, c_terms: Terms = None, ct_terms: Terms = None,
         sq_partial=None, bias=None, resid=None, target=None, ld_rt=None, out_scale=1.0,
         aux0=None, aux1=None, ld_aux=None, B2: Terms = None, epi=0, bn=128, causal=False,
         batch=1, a_off=(1, 0, 0), b_off=(1, 0, 0), c_off=(1, 0, 0), t_off=(1, 0, 0, 0, 0),
         ct_up_rows=0, skip_upper=False, row_period=0, split_k="auto", a_major=0, b_major=0,
         small_bufs=0, own_workspace=False):
    """The descriptor of one gemm() call: (GemmDesc, (M, N, K, products, work boxes, launches),
    the split-K workspace tensor or None). own_workspace: a workspace of its own (a plan keeps
    its pointer) instead of the shared, growing one."""
    d = GemmDesc()
    d.M = (A.cols if a_major else A.rows) if M is None else M
    d.N = ((B.cols if b_major else B.rows) if epi not in (2, 5) else 2 * B.rows) if N is None \
        else N
    d.K = (A.rows if a_major else A.cols) if K is None else K
    d.a_major, d.b_major = int(a_major), int(b_major)
    d.batch = batch
    na = A.n if na is None else na
    nb = B.n if nb is None else nb
    for i in range(na):
        d.a[i] = A.t[i].data_ptr()
    d.na, d.lda, d.a_rows = na, A.ld, A.rows
    for j in range(nb):
        d.b[j] = B.t[j].data_ptr()
        if B2 is not None:
            d.b2[j] = B2.t[j].data_ptr()
    d.nb, d.ldb, d.b_rows = nb, B.ld, B.rows
    d.order, d.causal, d.epi, d.bn = order, int(causal), epi, bn
    d.alpha, d.beta = alpha, beta
    d.C = _tp(C)
    d.ldc = (C.stride(0) if C is not None and C.dim() == 2 else d.N) if ldc is None else ldc
    if c_terms is not None:
        for i in range(c_terms.n):
            d.cs[i] = c_terms.t[i].data_ptr()
        d.ncs, d.ldcs = c_terms.n, c_terms.ld
    if ct_terms is not None:
        for i in range(ct_terms.n):
            d.ct[i] = ct_terms.t[i].data_ptr()
        d.nct, d.ldct = ct_terms.n, ct_terms.ld
    d.ct_up_rows = ct_up_rows
    d.sq_partial = _tp(sq_partial)
    d.bias, d.resid, d.target = _tp(bias), _tp(resid), _tp(target)
    d.ld_rt = (d.N if ld_rt is None else ld_rt)
    d.out_scale = out_scale
    d.aux0, d.aux1 = _tp(aux0), _tp(aux1)
    d.ld_aux = (d.N // 2 if epi in (2, 5) else d.N) if ld_aux is None else ld_aux
    d.skip_upper = int(skip_upper)
    d.row_period = int(row_period)
    d.small_bufs = int(small_bufs)
    splittable = (epi == 0 and batch == 1 and not causal and C is not None and bias is None
                  and c_terms is None and ct_terms is None and sq_partial is None)
    if split_k == "auto":
        split_k = auto_split(d.M, d.N, d.K, bn) if splittable else 1
    ws = None
    if split_k > 1:
        d.split_k = int(split_k)
        if own_workspace:
            ws = torch.empty(int(split_k) * d.M * d.N, device=A.t[0].device,
                             dtype=torch.float32)
        else:
            ws = _workspace(A.t[0].device, split_k * d.M * d.N)
        d.workspace = ws.data_ptr()
    d.a_div, d.a_s1, d.a_s2 = a_off
    d.b_div, d.b_s1, d.b_s2 = b_off
    d.c_div, d.c_s1, d.c_s2 = c_off
    d.t_div, d.t_r1, d.t_r2, d.t_c1, d.t_c2 = t_off
    dev = A.t[0].device
    d.err = err_flag(dev).data_ptr()
    extra = 0
    if d.split_k > 1:
        kb = -(-d.K // 64)
        per = -(-kb // d.split_k)
        extra = 1 if -(-kb // per) > 1 else 0  # the split-K reduction
    prods = sum(1 for i in range(na) for j in range(nb) if i + j <= order)
    # a causal product (or a square one whose upper tiles are skipped) does half the work of
    # its M x N x K box: count batch x 1/2
    eff = batch * (0.5 if (causal or skip_upper) else 1.0)
    return d, (d.M, d.N, d.K, prods, eff, 1 + extra), ws


def _launch(entry, arg, info):
    """Call a GEMM entry point (with the launch log's events around it when active)."""
    log = LaunchLog.active
    if log is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    _lib.call(entry, arg, _lib.stream_ptr())
    _lib.Launches.n += info[5] - 1
    if log is not None:
        e1.record()
        log.rows.append((*info[:5], e0, e1, log.tag))


def gemm(A: Terms, B: Terms, **kw):
    """One (batched) tensor-core GEMM with a fused epilogue; see gsq_gemm in the C header.
    Keywords: M, N, K (default: the operand shapes), na, nb, order, alpha, beta, C, ldc,
    c_terms, ct_terms, sq_partial, bias, resid, target, ld_rt, out_scale, aux0, aux1, ld_aux,
    B2, epi, bn, causal, batch, a_off / b_off / c_off = (div, s1, s2), t_off = (div, row_s1,
    row_s2, col_s1, col_s2), ct_up_rows, skip_upper, row_period, split_k, a_major / b_major
    (1: the operand's Terms hold [K][M] / [K][N], a row-major activation read as its own
    transpose). Returns C."""
    d, info, _ = _describe(A, B, **kw)
    _launch("gsq_gemm", _C.byref(d), info)
    return kw.get("C")


class GemmPlan:
    """A gemm() call prepared once (gsq_gemm_plan_create: checks and tensor maps) and run
    many times on the same buffers: the steps of a stage repeat the same products every step.
    Keeps references to its operand tensors so that their storage outlives the plan."""

    def __init__(self, A: Terms, B: Terms, **kw):
        self.d, self.info, self.ws = _describe(A, B, own_workspace=True, **kw)
        self._keep = (A, B, kw)
        h = _C.c_void_p()
        _lib.check(_lib.lib().gsq_gemm_plan_create(_C.byref(self.d), _C.byref(h)),
                   "gsq_gemm_plan_create")
        self.h = h

    def run(self):
        _launch("gsq_gemm_plan_run", self.h, self.info)

    def __del__(self):
        h = getattr(self, "h", None)
        if h is not None and h.value and _lib._lib is not None:
            _lib._lib.gsq_gemm_plan_destroy(h)


class PlanCache:
    """Plans keyed by call site: run(key, A, B, **kw) creates the plan on the first call and
    only launches it afterwards (the operands of a key must not change between calls)."""

    def __init__(self):
        self.plans = {}

    def run(self, key, A: Terms, B: Terms, **kw):
        p = self.plans.get(key)
        if p is None:
            p = self.plans[key] = GemmPlan(A, B, **kw)
        p.run()




def gemm_tc(A: Terms, B: Terms, na=None, nb=None, order=2, alpha=1.0, C=None, beta=0.0,
            c_terms: Terms = None, ct_terms: Terms = None, sq_partial=None):
    """C = alpha A B^T on tcgen05 with split-bf16 operands (see include/gsq_rco_b200.h)."""
    na = A.n if na is None else na
    nb = B.n if nb is None else nb
    if A.cols != B.cols:
        raise ValueError(f"inner dims differ: {A.cols} vs {B.cols}")
    M, N, K = A.rows, B.rows, A.cols
    dev = A.t[0].device
    _lib.call("gsq_gemm_tc", M, N, K, A.ptrs(na), na, A.ld, B.ptrs(nb), nb, B.ld, int(order),
              float(alpha), _lib.ptr(C), N if C is None else C.stride(0), float(beta),
              None if c_terms is None else c_terms.ptrs(), 0 if c_terms is None else c_terms.n,
              0 if c_terms is None else c_terms.ld,
              None if ct_terms is None else ct_terms.ptrs(), 0 if ct_terms is None else ct_terms.n,
              0 if ct_terms is None else ct_terms.ld, _lib.ptr(sq_partial),
              _lib.ptr(err_flag(dev)), _lib.stream_ptr())
    return C
