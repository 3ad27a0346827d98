// Elementwise and row kernels of the decoder block's vector-Jacobian product (the RCO objective's
// per-layer vjp, reference src/gsq_rco/rco/allocate.py:156-167 through mx.vjp of
// src/gsq_rco/gsq/e2e.py:160-174). The contractions run on the tensor-core GEMM; these kernels
// are the RMSNorm, causal-softmax and RoPE backward passes. Cotangents of bf16 forward tensors
// are rounded to bf16; float32 forward tensors (scores, RoPE'd q / k) keep float32 cotangents.
#include <math.h>

#include "common.cuh"

namespace gsq {

__device__ __forceinline__ float ldbf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// out = bf16(resid + bf16(dx)), dx the cotangent of x for y = (x inv) w,
// inv = 1 / sqrt(mean x^2 + eps) (float64), one warp per row.
__global__ void __launch_bounds__(256)
rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x,
                   const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ dy,
                   int64_t ld_dy, const __nv_bfloat16* __restrict__ resid, int64_t ld_r,
                   __nv_bfloat16* __restrict__ out, int64_t ld_o, int rows, int H, double eps) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const __nv_bfloat16* xr = x + r * ld_x;
    const __nv_bfloat16* gr = dy + r * ld_dy;
    double ss = 0.0, dot = 0.0;
    for (int c = lane; c < H; c += 32) {
      const double xv = ldbf(xr + c), wv = ldbf(w + c), gv = ldbf(gr + c);
      ss += xv * xv;
      dot += xv * wv * gv;
    }
    ss = warp_sum_d(ss);
    dot = warp_sum_d(dot);
    const double inv = 1.0 / sqrt(ss / (double)H + eps);
    const double k3 = inv * inv * inv / (double)H * dot;
    for (int c = lane; c < H; c += 32) {
      const double xv = ldbf(xr + c), wv = ldbf(w + c), gv = ldbf(gr + c);
      const float dx = bf16r_dev((float)(inv * wv * gv - k3 * xv));
      const float rv = resid ? ldbf(resid + r * ld_r + c) : 0.f;
      out[r * ld_o + c] = __float2bfloat16_rn(__fadd_rn(rv, dx));
    }
  }
}

// dS = 0.125 Pf (dP - sum_k dP Pf) of the causal softmax Pf = softmax(S) recomputed from the
// float32 scores exactly as the forward (max, float64 sum of exp, float32 reciprocal), written
// as three bf16 terms [B*T][ld_o] (zeros for keys > query up to T). One warp per row.
__global__ void __launch_bounds__(256)
softmax_bwd_kernel(const float* __restrict__ S, const __nv_bfloat16* __restrict__ dP, int B,
                   int T, int64_t ld_p, __nv_bfloat16* __restrict__ o0,
                   __nv_bfloat16* __restrict__ o1, __nv_bfloat16* __restrict__ o2, int64_t ld_o,
                   float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t n_rows = (int64_t)B * T;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int t = (int)(row % T);
    const float* s = S + row * T;
    const __nv_bfloat16* g = dP + row * ld_p;
    float m = -INFINITY;
    for (int k = lane; k <= t; k += 32) m = fmaxf(m, s[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double sum = 0.0;
    for (int k = lane; k <= t; k += 32) sum += (double)expf(__fsub_rn(s[k], m));
    sum = warp_sum_d(sum);
    const float inv = __frcp_rn((float)sum);
    double dot = 0.0;
    for (int k = lane; k <= t; k += 32) {
      const float pf = __fmul_rn(expf(__fsub_rn(s[k], m)), inv);
      dot += (double)ldbf(g + k) * (double)pf;
    }
    dot = warp_sum_d(dot);
    for (int k = lane; k < T; k += 32) {
      float v = 0.f;
      if (k <= t) {
        const float pf = __fmul_rn(expf(__fsub_rn(s[k], m)), inv);
        v = (float)((double)pf * ((double)ldbf(g + k) - dot) * (double)scale);
      }
      __nv_bfloat16 h, mi, l;
      split3_bf16(v, h, mi, l);
      const int64_t o = row * ld_o + k;
      o0[o] = h;
      o1[o] = mi;
      o2[o] = l;
    }
  }
}

// dx = rope_bwd(dy) rounded to bf16: dy float32 [(s * nh + h) * T + t][64] (ld_i) ->
// out bf16 [s * T + t][col0 + h * 64 + d] (ld_o). The half-split rotation's transpose:
// dx1 = dy1 c + dy2 s, dx2 = -dy1 s + dy2 c.
__global__ void rope_bwd_kernel(const float* __restrict__ dy, int64_t ld_i, int S, int T, int nh,
                                const float* __restrict__ cosv, const float* __restrict__ sinv,
                                __nv_bfloat16* __restrict__ out, int64_t ld_o, int col0) {
  const int64_t n = (int64_t)S * nh * T * 32;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(e % 32);
    const int64_t zt = e / 32;             // (s * nh + h) * T + t
    const int t = (int)(zt % T);
    const int64_t z = zt / T;
    const int h = (int)(z % nh), s = (int)(z / nh);
    const float d1 = dy[zt * ld_i + j], d2 = dy[zt * ld_i + 32 + j];
    const float c = cosv[t * 32 + j], sn = sinv[t * 32 + j];
    const float a = __fadd_rn(__fmul_rn(d1, c), __fmul_rn(d2, sn));
    const float b = __fsub_rn(__fmul_rn(d2, c), __fmul_rn(d1, sn));
    __nv_bfloat16* o = out + ((int64_t)s * T + t) * ld_o + col0 + h * 64;
    o[j] = __float2bfloat16_rn(a);
    o[32 + j] = __float2bfloat16_rn(b);
  }
}

// GQA sum over the rep query heads of each kv head: in float32 [(s nh + h) T + t][ld_i] (64 per
// head) -> out_f float32 [(s nkv + kv) T + t][64] and / or out_b bf16 at
// [s T + t][col0 + kv 64 + d] (ld_o).
__global__ void group_sum_kernel(const float* __restrict__ in, int64_t ld_i, int S, int nh,
                                 int rep, int T, float* __restrict__ out_f,
                                 __nv_bfloat16* __restrict__ out_b, int64_t ld_o, int col0) {
  const int nkv = nh / rep;
  const int64_t n = (int64_t)S * nkv * T * 64;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(e % 64);
    const int64_t zt = e / 64;             // (s * nkv + kv) * T + t
    const int t = (int)(zt % T);
    const int64_t zk = zt / T;
    const int kv = (int)(zk % nkv), s = (int)(zk / nkv);
    float acc = 0.f;
    for (int r = 0; r < rep; ++r)
      acc = __fadd_rn(acc, in[(((int64_t)s * nh + kv * rep + r) * T + t) * ld_i + d]);
    if (out_f) out_f[zt * 64 + d] = acc;
    if (out_b) out_b[((int64_t)s * T + t) * ld_o + col0 + kv * 64 + d] = __float2bfloat16_rn(acc);
  }
}

inline unsigned grid_for(int64_t n, int t) {
  int64_t b = (n + t - 1) / t;
  const int64_t cap = (int64_t)num_sms() * 32;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace gsq

using namespace gsq;

extern "C" int gsq_rmsnorm_bwd(const void* x, int64_t ld_x, const void* w, const void* dy,
                               int64_t ld_dy, const void* resid, int64_t ld_r, void* out,
                               int64_t ld_o, int rows, int H, double eps, void* stream) {
  if (!x || !w || !dy || !out || rows <= 0 || H <= 0 || ld_x < H || ld_dy < H || ld_o < H ||
      (resid && ld_r < H))
    return GSQ_EINVAL;
  rmsnorm_bwd_kernel<<<grid_for((int64_t)rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, ld_x, (const __nv_bfloat16*)w, (const __nv_bfloat16*)dy, ld_dy,
      (const __nv_bfloat16*)resid, ld_r, (__nv_bfloat16*)out, ld_o, rows, H, eps);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_softmax_bwd(const float* S, const void* dP, int B, int T, int64_t ld_p,
                               void* o0, void* o1, void* o2, int64_t ld_o, float scale,
                               void* stream) {
  if (!S || !dP || !o0 || !o1 || !o2 || B <= 0 || T <= 0 || ld_p < T || ld_o < T)
    return GSQ_EINVAL;
  softmax_bwd_kernel<<<grid_for((int64_t)B * T * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      S, (const __nv_bfloat16*)dP, B, T, ld_p, (__nv_bfloat16*)o0, (__nv_bfloat16*)o1,
      (__nv_bfloat16*)o2, ld_o, scale);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_rope_bwd(const float* dy, int64_t ld_i, int S, int T, int nh,
                            const float* cosv, const float* sinv, void* out, int64_t ld_o,
                            int col0, void* stream) {
  if (!dy || !cosv || !sinv || !out || S <= 0 || T <= 0 || nh <= 0 || ld_i < 64 ||
      ld_o < col0 + nh * 64 || col0 < 0)
    return GSQ_EINVAL;
  rope_bwd_kernel<<<grid_for((int64_t)S * nh * T * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      dy, ld_i, S, T, nh, cosv, sinv, (__nv_bfloat16*)out, ld_o, col0);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_group_sum(const float* in, int64_t ld_i, int S, int nh, int rep, int T,
                             float* out_f, void* out_b, int64_t ld_o, int col0, void* stream) {
  if (!in || (!out_f && !out_b) || S <= 0 || nh <= 0 || rep <= 0 || nh % rep || T <= 0 ||
      ld_i < 64 || (out_b && ld_o < col0 + (nh / rep) * 64) || col0 < 0)
    return GSQ_EINVAL;
  group_sum_kernel<<<grid_for((int64_t)S * (nh / rep) * T * 64, 256), 256, 0,
                     (cudaStream_t)stream>>>(in, ld_i, S, nh, rep, T, out_f,
                                             (__nv_bfloat16*)out_b, ld_o, col0);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
