// RCO objective kernels: the row statistics of the tied-embedding KL head and the
// straight-through dot products of the linear gradients with the database candidates.
//
// KL head (reference src/gsq_rco/common/evaluate.py:111-151): with z = bf16(h E^T) the logits of
// the quantized stream (zq) and of the full-precision stream (zr), per row
//   lse = logsumexp(z), q = exp(zq - lse_q), p = exp(zr - lse_r),
//   KL_row = sum_v p (zr - lse_r - zq + lse_q),   D = bf16(q - p)   (dKL_row / dzq = q - p).
// The two logit GEMMs and the gradient GEMM D E run on the tensor cores (gemm_tc.cu); this file
// holds the row pass between them: one CTA per row, three sweeps over the vocabulary row (the
// later two from L2).
//
// STE dots (reference src/gsq_rco/rco/allocate.py:169-174): for one linear with gradient G and
// reference weight W (bf16), dot_k = sum G (f32(bf16(s_k grid_k[code_k])) - f32(W)) for the K
// database options, accumulated in float64 (deterministic two-level reduction).
#include <math.h>
#include <string.h>

#include "common.cuh"

namespace gsq {

constexpr int kKlThreads = 512;
constexpr int kMaxOptions = 8;

__device__ __forceinline__ float block_max_f(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : -INFINITY;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

__device__ __forceinline__ double block_sum_d(double v, double* sh) {
  v = warp_sum_d(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0.0;
  if (w == 0) {
    v = warp_sum_d(v);
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

// 8 bf16 of a 16-byte aligned vector as floats
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __low2float(b[i]);
    f[2 * i + 1] = __high2float(b[i]);
  }
}

// One CTA per row; V % 8 == 0 and 16-byte aligned rows (checked by the host).
__global__ void __launch_bounds__(kKlThreads)
kl_rows_kernel(const __nv_bfloat16* __restrict__ zq, const __nv_bfloat16* __restrict__ zr,
               int V, int64_t ld, __nv_bfloat16* __restrict__ D, int64_t ld_d,
               double* __restrict__ kl_rows, float* __restrict__ lse_out) {
  __shared__ float shf[32];
  __shared__ double shd[32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* a = zq + row * ld;
  const __nv_bfloat16* b = zr + row * ld;
  const int nv = V / 8;
  float mq = -INFINITY, mr = -INFINITY;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float x[8], y[8];
    load8(a + 8 * i, x);
    load8(b + 8 * i, y);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mq = fmaxf(mq, x[j]);
      mr = fmaxf(mr, y[j]);
    }
  }
  mq = block_max_f(mq, shf);
  mr = block_max_f(mr, shf);
  double sq = 0.0, sr = 0.0;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float x[8], y[8];
    load8(a + 8 * i, x);
    load8(b + 8 * i, y);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sq += (double)expf(__fsub_rn(x[j], mq));
      sr += (double)expf(__fsub_rn(y[j], mr));
    }
  }
  sq = block_sum_d(sq, shd);
  sr = block_sum_d(sr, shd);
  const float lq = __fadd_rn(mq, logf((float)sq));
  const float lr = __fadd_rn(mr, logf((float)sr));
  double kl = 0.0;
  __nv_bfloat16* d = D + row * ld_d;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float x[8], y[8];
    load8(a + 8 * i, x);
    load8(b + 8 * i, y);
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float lpq = __fsub_rn(x[j], lq), lpr = __fsub_rn(y[j], lr);
      const float q = expf(lpq), p = expf(lpr);
      kl += (double)__fmul_rn(p, __fsub_rn(lpr, lpq));
      o[j] = __float2bfloat16_rn(__fsub_rn(q, p));
    }
    *reinterpret_cast<uint4*>(d + 8 * i) = *reinterpret_cast<const uint4*>(o);
  }
  kl = block_sum_d(kl, shd);
  if (threadIdx.x == 0) {
    kl_rows[row] = kl;
    if (lse_out) {
      lse_out[2 * row] = lq;
      lse_out[2 * row + 1] = lr;
    }
  }
}

// Next-token NLL of one logit row (evaluate.py:35-52): nll = logsumexp(z) - z[target] with z
// the float32 value of the bf16 logits, the max and the float64 sum of exp(z - max) as in
// kl_rows_kernel. target < 0 marks a row that is not scored (nll = 0). One CTA per row.
__global__ void __launch_bounds__(kKlThreads)
nll_rows_kernel(const __nv_bfloat16* __restrict__ z, int V, int64_t ld,
                const int32_t* __restrict__ targets, double* __restrict__ nll) {
  __shared__ float shf[32];
  __shared__ double shd[32];
  const int64_t row = blockIdx.x;
  const int t = targets[row];
  if (t < 0 || t >= V) {  // not scored, or an id outside the vocabulary (NaN)
    if (threadIdx.x == 0) nll[row] = t < 0 ? 0.0 : (double)NAN;
    return;
  }
  const __nv_bfloat16* a = z + row * ld;
  const int nv = V / 8;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float x[8];
    load8(a + 8 * i, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, x[j]);
  }
  m = block_max_f(m, shf);
  double s = 0.0;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float x[8];
    load8(a + 8 * i, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += (double)expf(__fsub_rn(x[j], m));
  }
  s = block_sum_d(s, shd);
  if (threadIdx.x == 0) {
    const float lse = __fadd_rn(m, logf((float)s));
    nll[row] = (double)__fsub_rn(lse, __bfloat162float(a[t]));
  }
}

// Group-scale gradient of a stored-form linear W = bf16(s[r][c / gs] grid[code[r][c]]) with its
// codes fixed (App-H scale fine-tune, staged.py:555-634, the mx.take backward): out[r][g] =
// sum over the group's columns of G[r][c] grid[code[r][c]] (float64 sum, float32 out). One warp
// per (row, group), lanes over the group's columns.
__global__ void __launch_bounds__(256)
scale_grad_kernel(const float* __restrict__ G, const uint8_t* __restrict__ codes, int out_f,
                  int in_f, int bits, int gs, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int ng = (in_f + gs - 1) / gs;
  const int64_t units = (int64_t)out_f * ng;
  for (int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < units;
       u += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int r = (int)(u / ng), g = (int)(u - (int64_t)r * ng);
    const int c0 = g * gs, c1 = min(c0 + gs, in_f);
    double acc = 0.0;
    for (int c = c0 + lane; c < c1; c += 32) {
      const int64_t i = (int64_t)r * in_f + c;
      acc += (double)G[i] * (double)grid_value(bits, codes[i]);
    }
    acc = warp_sum_d(acc);
    if (lane == 0) out[u] = (float)acc;
  }
}

struct DotOpts {
  const uint8_t* codes[kMaxOptions];
  const float* scales[kMaxOptions];
  int bits[kMaxOptions];
};

// partials[block][k] = sum over this block's elements of G (f32(bf16(s grid[c])) - f32(W))
__global__ void __launch_bounds__(256)
ste_dots_kernel(const float* __restrict__ G, const __nv_bfloat16* __restrict__ W, int out_f,
                int in_f, int gs, int K, const __grid_constant__ DotOpts opt,
                double* __restrict__ partials) {
  __shared__ double sh[kMaxOptions][8];
  double acc[kMaxOptions];
#pragma unroll
  for (int k = 0; k < kMaxOptions; ++k) acc[k] = 0.0;
  const int64_t d = (int64_t)out_f * in_f;
  const int ng = (in_f + gs - 1) / gs;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < d;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / in_f), c = (int)(e - (int64_t)r * in_f);
    const float g = G[e], w = __bfloat162float(W[e]);
#pragma unroll
    for (int k = 0; k < kMaxOptions; ++k) {
      if (k < K) {
        const float s = opt.scales[k][(int64_t)r * ng + c / gs];
        const float q = bf16r_dev(__fmul_rn(grid_value(opt.bits[k], opt.codes[k][e]), s));
        acc[k] += (double)__fmul_rn(g, __fsub_rn(q, w));
      }
    }
  }
  const int wid = threadIdx.x >> 5, l = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kMaxOptions; ++k) {
    if (k < K) {
      const double v = warp_sum_d(acc[k]);
      if (l == 0) sh[k][wid] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < K) {
    double t = 0.0;
    for (int i = 0; i < 8; ++i) t += sh[threadIdx.x][i];
    partials[(int64_t)blockIdx.x * K + threadIdx.x] = t;
  }
}

__global__ void dots_final_kernel(const double* __restrict__ partials, int n_blocks, int K,
                                  double* __restrict__ out) {
  __shared__ double sh[32];
  for (int k = 0; k < K; ++k) {
    double s = 0.0;
    for (int i = threadIdx.x; i < n_blocks; i += blockDim.x) s += partials[(int64_t)i * K + k];
    s = block_sum_d(s, sh);
    if (threadIdx.x == 0) out[k] = s;
    __syncthreads();
  }
}

// x = bf16(f32(x) / divisor): the mean-over-positions scaling of the bf16 head gradient
// (evaluate.py:150, a bf16 array divided by the position count).
__global__ void div_bf16_kernel(__nv_bfloat16* __restrict__ x, int64_t n, float divisor) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    x[i] = __float2bfloat16_rn(__fdiv_rn(__bfloat162float(x[i]), divisor));
}

// w = bf16(scales[r][c / gs] grid[codes[r, c]]): an assembled database weight in the model dtype
// (database.py:244-256 dequant, then allocate.py:117 astype(bf16)).
__global__ void dequant_bf16_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ sc,
                                    int out_f, int in_f, int bits, int gs,
                                    __nv_bfloat16* __restrict__ w) {
  const int64_t d = (int64_t)out_f * in_f;
  const int ng = (in_f + gs - 1) / gs;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < d;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / in_f), c = (int)(e - (int64_t)r * in_f);
    w[e] = __float2bfloat16_rn(__fmul_rn(grid_value(bits, codes[e]), sc[(int64_t)r * ng + c / gs]));
  }
}

}  // namespace gsq

using namespace gsq;

extern "C" int gsq_dequant_bf16(const uint8_t* codes, const float* scales, int out_f, int in_f,
                                int bits, int group_size, void* w, void* stream) {
  if (!codes || !scales || !w || out_f <= 0 || in_f <= 0 || bits < 1 || bits > 8 ||
      group_size <= 0)
    return GSQ_EINVAL;
  const int64_t d = (int64_t)out_f * in_f;
  int64_t b = (d + 255) / 256;
  if (b > (int64_t)num_sms() * 16) b = (int64_t)num_sms() * 16;
  dequant_bf16_kernel<<<(unsigned)b, 256, 0, (cudaStream_t)stream>>>(
      codes, scales, out_f, in_f, bits, group_size, (__nv_bfloat16*)w);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_div_bf16(void* x, int64_t n, float divisor, void* stream) {
  if (!x || n <= 0 || !(divisor != 0.f)) return GSQ_EINVAL;
  int64_t b = (n + 255) / 256;
  if (b > (int64_t)num_sms() * 16) b = (int64_t)num_sms() * 16;
  div_bf16_kernel<<<(unsigned)b, 256, 0, (cudaStream_t)stream>>>((__nv_bfloat16*)x, n, divisor);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_kl_rows(const void* zq, const void* zr, int n, int V, int64_t ld, void* D,
                           int64_t ld_d, double* kl_rows, float* lse, void* stream) {
  if (!zq || !zr || !D || !kl_rows || n <= 0 || V <= 0 || (V & 7) || ld < V || ld_d < V ||
      (ld & 7) || (ld_d & 7) || ((uintptr_t)zq & 15) || ((uintptr_t)zr & 15) ||
      ((uintptr_t)D & 15))
    return GSQ_EINVAL;
  kl_rows_kernel<<<n, kKlThreads, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)zq, (const __nv_bfloat16*)zr, V, ld, (__nv_bfloat16*)D, ld_d,
      kl_rows, lse);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

// One bf16 product out = bf16(A B^T) of single-term row-major operands (A [M][lda], B [N][ldb],
// the reduction index contiguous) through gsq_gemm's bf16-chain epilogue: the descriptor the
// library's Python gemm() builds for the same call.
static int bf16_product(const void* A, int64_t lda, int M, const void* B, int64_t ldb, int N,
                        int K, void* out, int64_t ldo, int* err, void* stream) {
  gsq_gemm_desc d;
  memset(&d, 0, sizeof(d));
  d.M = M;
  d.N = N;
  d.K = K;
  d.batch = 1;
  d.a[0] = A;
  d.na = 1;
  d.lda = lda;
  d.a_rows = M;
  d.b[0] = B;
  d.nb = 1;
  d.ldb = ldb;
  d.b_rows = N;
  d.order = 2;
  d.epi = 4;
  d.bn = 128;
  d.alpha = 1.f;
  d.ldc = N;
  d.cs[0] = out;
  d.ncs = 1;
  d.ldcs = ldo;
  d.ld_rt = N;
  d.out_scale = 1.f;
  d.ld_aux = N;
  d.a_div = d.b_div = d.c_div = d.t_div = 1;
  d.err = err;
  return gsq_gemm(&d, stream);
}

extern "C" int kl_head_fwd_bwd(const void* h_q, const void* h_ref, int n, int H, const void* E,
                               const void* ET, int64_t ld_et, int V, int chunk, void* zq,
                               void* zr, void* D, double* kl_rows, double* total, void* grad,
                               int* err, void* stream) {
  if (!h_q || !h_ref || !E || !ET || !zq || !zr || !D || !kl_rows || !total || !grad || !err ||
      n <= 0 || H <= 0 || (H & 7) || V <= 0 || (V & 7) || chunk <= 0 || ld_et < V || (ld_et & 7))
    return GSQ_EINVAL;
  const auto* hq = static_cast<const __nv_bfloat16*>(h_q);
  const auto* hr = static_cast<const __nv_bfloat16*>(h_ref);
  auto* g = static_cast<__nv_bfloat16*>(grad);
  for (int a = 0; a < n; a += chunk) {
    const int m = n - a < chunk ? n - a : chunk;
    int rc = bf16_product(hq + (int64_t)a * H, H, m, E, H, V, H, zq, V, err, stream);
    if (rc == GSQ_OK) rc = bf16_product(hr + (int64_t)a * H, H, m, E, H, V, H, zr, V, err, stream);
    if (rc == GSQ_OK) rc = gsq_kl_rows(zq, zr, m, V, V, D, V, kl_rows + a, nullptr, stream);
    if (rc == GSQ_OK) rc = bf16_product(D, V, m, ET, ld_et, H, V, g + (int64_t)a * H, H, err, stream);
    if (rc != GSQ_OK) return rc;
  }
  return gsq_sum_f64(kl_rows, n, total, stream);
}

extern "C" int ste_dots(const float* G, const void* W, int out_f, int in_f, int group_size,
                        int K, const uint8_t* const* codes, const float* const* scales,
                        const int* bits, double* partials, int max_blocks, double* out,
                        void* stream) {
  if (!G || !W || !codes || !scales || !bits || !partials || !out || out_f <= 0 ||
      in_f <= 0 || group_size <= 0 || K < 1 || K > kMaxOptions || max_blocks < 1)
    return GSQ_EINVAL;
  DotOpts opt;
  for (int k = 0; k < kMaxOptions; ++k) {
    opt.codes[k] = k < K ? codes[k] : nullptr;
    opt.scales[k] = k < K ? scales[k] : nullptr;
    opt.bits[k] = k < K ? bits[k] : 0;
    if (k < K && (!codes[k] || !scales[k] || bits[k] < 1 || bits[k] > 8)) return GSQ_EINVAL;
  }
  const int64_t d = (int64_t)out_f * in_f;
  int64_t nb = (d + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (nb > cap) nb = cap;
  if (nb > max_blocks) nb = max_blocks;
  cudaStream_t st = (cudaStream_t)stream;
  ste_dots_kernel<<<(unsigned)nb, 256, 0, st>>>(G, (const __nv_bfloat16*)W, out_f, in_f,
                                                group_size, K, opt, partials);
  GSQ_CHECK_LAUNCH();
  dots_final_kernel<<<1, 256, 0, st>>>(partials, (int)nb, K, out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_nll_rows(const void* z, int n, int V, int64_t ld, const int32_t* targets,
                            double* nll, void* stream) {
  if (!z || !targets || !nll || n <= 0 || V <= 0 || (V & 7) || ld < V || (ld & 7) ||
      ((uintptr_t)z & 15))
    return GSQ_EINVAL;
  nll_rows_kernel<<<n, kKlThreads, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)z, V, ld,
                                                              targets, nll);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_scale_grad(const float* G, const uint8_t* codes, int out_f, int in_f,
                              int bits, int group_size, float* out, void* stream) {
  if (!G || !codes || !out || out_f <= 0 || in_f <= 0 || group_size <= 0 || bits < 1 ||
      bits > 8)
    return GSQ_EINVAL;
  const int ng = (in_f + group_size - 1) / group_size;
  int64_t blocks = ((int64_t)out_f * ng * 32 + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  scale_grad_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, (cudaStream_t)stream>>>(
      G, codes, out_f, in_f, bits, group_size, out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
