// Elementwise kernels of the Qwen2 decoder block the GSQ stages run through: RMSNorm, RoPE
// into GEMM operand terms, the causal row softmax of the attention scores, the embedding
// gather, and the float64 finalisation of a Hessian accumulated by the tensor cores.
//
// Rounding follows the reference block (bf16 storage, float32 norm / rotation / softmax math):
//   rmsnorm: bf16((x * (1 / sqrt(mean(x^2) + eps))) * w), mean(x^2) from a float64 sum
//   rope:    [x1 c - x2 s, x1 s + x2 c] in float32 of bf16 x (half-split, theta per pair)
//   softmax: float32 over keys <= query, exp(x - max) / sum, rounded to bf16; keys > query 0
#include <math.h>

#include "common.cuh"

namespace gsq {

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

// One block = 32 rows: warp w computes the inverse RMS of rows 4w..4w+3, then the block walks
// 32-column tiles writing row-major and (optionally) transposed bf16 outputs. Rows whose
// position within their sequence is 0 are written as zeros to the transposed output when
// zero_pos0 is set (Hessian inputs exclude position 0).
__global__ void __launch_bounds__(256)
rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, const __nv_bfloat16* __restrict__ w,
               int rows, int H, float eps, __nv_bfloat16* __restrict__ y, int64_t ld_y,
               __nv_bfloat16* __restrict__ yt, int64_t ld_yt, int seq_len, int zero_pos0) {
  __shared__ float inv[32];
  __shared__ float tile[32][33];
  const int r0 = blockIdx.x * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int rr = warp; rr < 32; rr += 8) {
    const int r = r0 + rr;
    double s = 0.0;
    if (r < rows)
      for (int c = lane; c < H; c += 32) {
        const float v = bf(x[(int64_t)r * ld_x + c]);
        s += (double)__fmul_rn(v, v);
      }
    s = warp_sum_d(s);
    if (lane == 0) {
      const float var = (float)(s / (double)H);
      inv[rr] = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
    }
  }
  __syncthreads();
  for (int c0 = 0; c0 < H; c0 += 32) {
    for (int rr = warp; rr < 32; rr += 8) {
      const int r = r0 + rr, c = c0 + lane;
      float v = 0.f;
      if (r < rows && c < H) {
        v = bf16r_dev(__fmul_rn(__fmul_rn(bf(x[(int64_t)r * ld_x + c]), inv[rr]), bf(w[c])));
        if (y) y[(int64_t)r * ld_y + c] = __float2bfloat16_rn(v);
      }
      tile[rr][lane] = v;
    }
    __syncthreads();
    if (yt) {
      for (int cc = warp; cc < 32; cc += 8) {
        const int c = c0 + cc, r = r0 + lane;
        if (c < H && r < rows) {
          float v = tile[lane][cc];
          if (zero_pos0 && (r % seq_len) == 0) v = 0.f;
          yt[(int64_t)c * ld_yt + r] = __float2bfloat16_rn(v);
        }
      }
    }
    __syncthreads();
  }
}

// q / k rotation into three bf16 terms, head-major: out[(s * nh + head) * T + t][0..63].
// x: bf16 [S*T][ld_x], head h at columns h*64.. ; cos / sin: float32 [T][32].
__global__ void rope_split_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, int S, int T,
                                  int nh, const float* __restrict__ cosv,
                                  const float* __restrict__ sinv, __nv_bfloat16* __restrict__ o0,
                                  __nv_bfloat16* __restrict__ o1, __nv_bfloat16* __restrict__ o2) {
  const int64_t n = (int64_t)S * T * nh * 32;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(e % 32);
    const int64_t rh = e / 32;             // (s * T + t) * nh + head
    const int head = (int)(rh % nh);
    const int64_t st = rh / nh;            // s * T + t
    const int t = (int)(st % T), s = (int)(st / T);
    const float x1 = bf(x[st * ld_x + head * 64 + j]);
    const float x2 = bf(x[st * ld_x + head * 64 + 32 + j]);
    const float c = cosv[t * 32 + j], sn = sinv[t * 32 + j];
    const float a = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    const float b = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, c));
    const int64_t o = (((int64_t)s * nh + head) * T + t) * 64;
    __nv_bfloat16 h, m, l;
    split3_bf16(a, h, m, l);
    o0[o + j] = h; o1[o + j] = m; o2[o + j] = l;
    split3_bf16(b, h, m, l);
    o0[o + 32 + j] = h; o1[o + 32 + j] = m; o2[o + 32 + j] = l;
  }
}

// Causal softmax of score rows: S float32 [B*T][T] (only keys <= query are defined) ->
// P bf16 [B*T][T] (zeros above the diagonal) and optionally P^T per batch [B][T][T].
// One warp per row.
__global__ void __launch_bounds__(256)
softmax_causal_kernel(const float* __restrict__ S, int B, int T, __nv_bfloat16* __restrict__ P,
                      __nv_bfloat16* __restrict__ PT) {
  const int lane = threadIdx.x & 31;
  const int64_t n_rows = (int64_t)B * T;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int t = (int)(row % T);
    const int64_t b = row / T;
    const float* s = S + row * T;
    float m = -INFINITY;
    for (int k = lane; k <= t; k += 32) m = fmaxf(m, s[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double sum = 0.0;
    for (int k = lane; k <= t; k += 32) sum += (double)expf(__fsub_rn(s[k], m));
    sum = warp_sum_d(sum);
    const float inv = __frcp_rn((float)sum);
    for (int k = lane; k < T; k += 32) {
      float p = 0.f;
      if (k <= t) p = __fmul_rn(expf(__fsub_rn(s[k], m)), inv);
      const __nv_bfloat16 pb = __float2bfloat16_rn(p);
      P[row * T + k] = pb;
      if (PT) PT[(b * T + k) * T + t] = pb;
    }
  }
}

// Vectorised form of softmax_causal_kernel for T % 4 == 0: lanes take consecutive 16-byte
// vectors of the row (512 bytes per warp access), over keys <= query only; the same max, float64
// sum of exp and rounded reciprocal (identical probabilities up to the float64 sum's order
// before its float32 rounding). P is written as 8-byte vectors up to the end of the row's
// 128-key block only: the causal P V product reduces over keys below that end and the causal
// transpose of the backward reads no block beyond it.
__global__ void __launch_bounds__(256)
softmax_causal_v2_kernel(const float* __restrict__ S, int B, int T, __nv_bfloat16* __restrict__ P) {
  const int lane = threadIdx.x & 31;
  const int64_t n_rows = (int64_t)B * T;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int t = (int)(row % T);
    const float4* s4 = reinterpret_cast<const float4*>(S + row * T);
    const int nv = t / 4 + 1;  // vectors holding keys 0..t
    float m = -INFINITY;
#pragma unroll 4
    for (int v = lane; v < nv; v += 32) {
      const float4 q = s4[v];
      const int k0 = 4 * v;
      m = fmaxf(m, q.x);
      if (k0 + 1 <= t) m = fmaxf(m, q.y);
      if (k0 + 2 <= t) m = fmaxf(m, q.z);
      if (k0 + 3 <= t) m = fmaxf(m, q.w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double sum = 0.0;
#pragma unroll 2
    for (int v = lane; v < nv; v += 32) {
      const float4 q = s4[v];
      const int k0 = 4 * v;
      sum += (double)expf(__fsub_rn(q.x, m));
      if (k0 + 1 <= t) sum += (double)expf(__fsub_rn(q.y, m));
      if (k0 + 2 <= t) sum += (double)expf(__fsub_rn(q.z, m));
      if (k0 + 3 <= t) sum += (double)expf(__fsub_rn(q.w, m));
    }
    sum = warp_sum_d(sum);
    const float inv = __frcp_rn((float)sum);
    const int end = min(T, (t / 128 + 1) * 128);
    uint2* p2 = reinterpret_cast<uint2*>(P + row * T);
#pragma unroll 2
    for (int v = lane; v < end / 4; v += 32) {
      const int k0 = 4 * v;
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 <= t) q = s4[v];
      const float x[4] = {q.x, q.y, q.z, q.w};
      __align__(8) __nv_bfloat16 o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = __float2bfloat16_rn(k0 + j <= t ? __fmul_rn(expf(__fsub_rn(x[j], m)), inv) : 0.f);
      p2[v] = *reinterpret_cast<const uint2*>(o);
    }
  }
}

// Row-windowed and vectorised: local row i of batch z is query position t = row0 + i and sees
// keys k <= t; the arithmetic of softmax_causal_v2_kernel (float4 reads, float64 sum, four bf16
// per store). With row0 == 0 (a square causal block) the zeros stop at the end of the query's
// 128-key block, the only keys that the causal P V product and the causal transpose read;
// otherwise (a window of query rows over all keys) every masked key k < cols is written.
// Needs cols, ld_s and ld_p multiples of 4, S 16-byte and P 8-byte aligned.
__global__ void __launch_bounds__(256)
softmax_causal_rows_v2_kernel(const float* __restrict__ S, int B, int rows, int cols,
                              int64_t ld_s, int row0, __nv_bfloat16* __restrict__ P,
                              int64_t ld_p) {
  const int lane = threadIdx.x & 31;
  const int64_t n_rows = (int64_t)B * rows;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int t = row0 + (int)(row % rows);
    const float4* s4 = reinterpret_cast<const float4*>(S + row * ld_s);
    const int nv = t / 4 + 1;  // vectors holding keys 0..t (t < cols, cols % 4 == 0)
    float m = -INFINITY;
#pragma unroll 4
    for (int v = lane; v < nv; v += 32) {
      const float4 q = s4[v];
      const int k0 = 4 * v;
      m = fmaxf(m, q.x);
      if (k0 + 1 <= t) m = fmaxf(m, q.y);
      if (k0 + 2 <= t) m = fmaxf(m, q.z);
      if (k0 + 3 <= t) m = fmaxf(m, q.w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double sum = 0.0;
#pragma unroll 2
    for (int v = lane; v < nv; v += 32) {
      const float4 q = s4[v];
      const int k0 = 4 * v;
      sum += (double)expf(__fsub_rn(q.x, m));
      if (k0 + 1 <= t) sum += (double)expf(__fsub_rn(q.y, m));
      if (k0 + 2 <= t) sum += (double)expf(__fsub_rn(q.z, m));
      if (k0 + 3 <= t) sum += (double)expf(__fsub_rn(q.w, m));
    }
    sum = warp_sum_d(sum);
    const float inv = __frcp_rn((float)sum);
    const int end = row0 == 0 ? min(cols, (t / 128 + 1) * 128) : cols;
    uint2* p2 = reinterpret_cast<uint2*>(P + row * ld_p);
#pragma unroll 2
    for (int v = lane; v < end / 4; v += 32) {
      const int k0 = 4 * v;
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 <= t) q = s4[v];
      const float x[4] = {q.x, q.y, q.z, q.w};
      __align__(8) __nv_bfloat16 o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = __float2bfloat16_rn(k0 + j <= t ? __fmul_rn(expf(__fsub_rn(x[j], m)), inv) : 0.f);
      p2[v] = *reinterpret_cast<const uint2*>(o);
    }
  }
}

// Row-windowed form, any layout: local row i of batch z is query position row0 + i; keys
// k <= row0 + i of the cols stored ones are valid. S [B][rows][ld_s] float32 -> P [B][rows][ld_p]
// bf16 (zeros at masked keys k < cols). One warp per row.
__global__ void __launch_bounds__(256)
softmax_causal_rows_kernel(const float* __restrict__ S, int B, int rows, int cols, int64_t ld_s,
                           int row0, __nv_bfloat16* __restrict__ P, int64_t ld_p) {
  const int lane = threadIdx.x & 31;
  const int64_t n_rows = (int64_t)B * rows;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int i = (int)(row % rows);
    const int last = min(row0 + i, cols - 1);  // last valid key
    const float* s = S + row * ld_s;
    __nv_bfloat16* p = P + row * ld_p;
    float m = -INFINITY;
    for (int k = lane; k <= last; k += 32) m = fmaxf(m, s[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double sum = 0.0;
    for (int k = lane; k <= last; k += 32) sum += (double)expf(__fsub_rn(s[k], m));
    sum = warp_sum_d(sum);
    const float inv = __frcp_rn((float)sum);
    for (int k = lane; k < cols; k += 32) {
      float v = 0.f;
      if (k <= last) v = __fmul_rn(expf(__fsub_rn(s[k], m)), inv);
      p[k] = __float2bfloat16_rn(v);
    }
  }
}

__global__ void embed_kernel(const int32_t* __restrict__ ids, int64_t n, const __nv_bfloat16* __restrict__ E,
                             int H, __nv_bfloat16* __restrict__ out) {
  const int64_t total = n * H;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / H;
    const int c = (int)(e - r * H);
    out[e] = E[(int64_t)ids[r] * H + c];
  }
}

// H64 <- beta H64 + alpha H32 (the float32 Gram of one batch of rows into the float64 H)
__global__ void hess_accum_kernel(double* __restrict__ H, const float* __restrict__ G, int64_t n,
                                  double beta, double alpha) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    H[i] = beta * H[i] + alpha * (double)G[i];
}

// x[r][c] = 0 for the columns c with c % period == 0 (position 0 of every sequence in a
// transposed row buffer [rows][ld]).
__global__ void zero_cols_kernel(__nv_bfloat16* __restrict__ x, int rows, int64_t ld, int cols,
                                 int period) {
  const int n_per_row = (cols + period - 1) / period;
  const int64_t n = (int64_t)rows * n_per_row;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / n_per_row;
    const int c = (int)(e - r * n_per_row) * period;
    x[r * ld + c] = __float2bfloat16_rn(0.f);
  }
}

inline unsigned blocks(int64_t n, int t) {
  int64_t b = (n + t - 1) / t;
  const int64_t cap = (int64_t)num_sms() * 32;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace gsq

using namespace gsq;

extern "C" int gsq_rmsnorm(const void* x, int64_t ld_x, const void* w, int rows, int H, float eps,
                           void* y, int64_t ld_y, void* yt, int64_t ld_yt, int seq_len,
                           int zero_pos0, void* stream) {
  if (!x || !w || rows <= 0 || H <= 0 || ld_x < H || (!y && !yt) || (y && ld_y < H) ||
      (yt && ld_yt < rows) || (zero_pos0 && seq_len <= 0))
    return GSQ_EINVAL;
  rmsnorm_kernel<<<(rows + 31) / 32, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, ld_x, (const __nv_bfloat16*)w, rows, H, eps, (__nv_bfloat16*)y,
      ld_y, (__nv_bfloat16*)yt, ld_yt, seq_len, zero_pos0);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_rope_split(const void* x, int64_t ld_x, int S, int T, int nh,
                              const float* cosv, const float* sinv, void* o0, void* o1, void* o2,
                              void* stream) {
  if (!x || !cosv || !sinv || !o0 || !o1 || !o2 || S <= 0 || T <= 0 || nh <= 0 ||
      ld_x < (int64_t)nh * 64)
    return GSQ_EINVAL;
  const int64_t n = (int64_t)S * T * nh * 32;
  rope_split_kernel<<<blocks(n, 256), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, ld_x, S, T, nh, cosv, sinv, (__nv_bfloat16*)o0,
      (__nv_bfloat16*)o1, (__nv_bfloat16*)o2);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_softmax_causal(const float* S, int B, int T, void* P, void* PT, void* stream) {
  if (!S || !P || B <= 0 || T <= 0) return GSQ_EINVAL;
  const unsigned g = blocks((int64_t)B * T * 32, 256);
  cudaStream_t st = (cudaStream_t)stream;
  auto* Pb = (__nv_bfloat16*)P;
  const bool vec = !PT && T % 4 == 0 && ((uintptr_t)S & 15) == 0 && ((uintptr_t)P & 7) == 0;
  if (vec) softmax_causal_v2_kernel<<<g, 256, 0, st>>>(S, B, T, Pb);
  else
    softmax_causal_kernel<<<g, 256, 0, st>>>(S, B, T, Pb, (__nv_bfloat16*)PT);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_softmax_causal_rows(const float* S, int B, int rows, int cols, int64_t ld_s,
                                       int row0, void* P, int64_t ld_p, void* stream) {
  if (!S || !P || B <= 0 || rows <= 0 || cols <= 0 || row0 < 0 || ld_s < cols || ld_p < cols ||
      row0 + rows > cols)
    return GSQ_EINVAL;
  const unsigned g = blocks((int64_t)B * rows * 32, 256);
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = cols % 4 == 0 && ld_s % 4 == 0 && ld_p % 4 == 0 && ((uintptr_t)S & 15) == 0 &&
                   ((uintptr_t)P & 7) == 0;
  if (vec)
    softmax_causal_rows_v2_kernel<<<g, 256, 0, st>>>(S, B, rows, cols, ld_s, row0,
                                                     (__nv_bfloat16*)P, ld_p);
  else
    softmax_causal_rows_kernel<<<g, 256, 0, st>>>(S, B, rows, cols, ld_s, row0,
                                                  (__nv_bfloat16*)P, ld_p);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_embed(const int32_t* ids, int64_t n, const void* E, int H, void* out,
                         void* stream) {
  if (!ids || !E || !out || n <= 0 || H <= 0) return GSQ_EINVAL;
  embed_kernel<<<blocks(n * H, 256), 256, 0, (cudaStream_t)stream>>>(
      ids, n, (const __nv_bfloat16*)E, H, (__nv_bfloat16*)out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_hess_accum(double* H, const float* G, int64_t n, double beta, double alpha,
                              void* stream) {
  if (!H || !G || n <= 0) return GSQ_EINVAL;
  hess_accum_kernel<<<blocks(n, 256), 256, 0, (cudaStream_t)stream>>>(H, G, n, beta, alpha);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_zero_cols(void* x, int rows, int64_t ld, int cols, int period, void* stream) {
  if (!x || rows <= 0 || cols <= 0 || period <= 0 || ld < cols) return GSQ_EINVAL;
  const int64_t n = (int64_t)rows * ((cols + period - 1) / period);
  zero_cols_kernel<<<blocks(n, 256), 256, 0, (cudaStream_t)stream>>>((__nv_bfloat16*)x, rows, ld,
                                                                      cols, period);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
