// GSQ soft-quantized linear: Gumbel-softmax soft weight (forward), fused soft backward +
// Lion (one HBM pass over the training state), argmax decode, and a flat Lion step.
//
// Elementwise arithmetic uses explicit round-to-nearest intrinsics so that no multiply-add is
// contracted: every product and sum is rounded as in the float32 arrays of the reference.
#include <math.h>

#include "common.cuh"

namespace gsq {

template <int K>
struct SoftMath {
  // p = softmax((kappa * l + g) / tau) and the candidate values C_k of weight i.
  __device__ __forceinline__ static void probs(const float* __restrict__ logits, int64_t d,
                                               int64_t i, const float g[K], float tau,
                                               float kappa, float p[K]) {
    float y[K];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      y[k] = __fdiv_rn(__fadd_rn(__fmul_rn(kappa, logits[k * d + i]), g[k]), tau);
      m = fmaxf(m, y[k]);
    }
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      y[k] = expf(__fsub_rn(y[k], m));
      sum = k == 0 ? y[0] : __fadd_rn(sum, y[k]);
    }
#pragma unroll
    for (int k = 0; k < K; ++k) p[k] = __fdiv_rn(y[k], sum);
  }

  __device__ __forceinline__ static void candidates(int bits, int j0, float C[K]) {
    if (K == 4) {
#pragma unroll
      for (int k = 0; k < K; ++k) C[k] = (float)(k - 2);  // 2-bit grid [-2, -1, 0, 1]
    } else {
      const int top = (1 << bits) - 1;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int j = min(max(j0 + k - 2, 0), top);
        C[k] = grid_value(bits, j);
      }
    }
  }

  __device__ __forceinline__ static void noise(const float* __restrict__ noise_r, int64_t d,
                                               int64_t i, const NoiseKey& nk, float g[K]) {
    if (noise_r) {
#pragma unroll
      for (int k = 0; k < K; ++k) g[k] = noise_r[k * d + i];
    } else {
      gumbel_weight<K>(nk, (uint32_t)i, g);
    }
  }
};

template <int K>
__global__ void __launch_bounds__(256)
soft_fwd_kernel(const float* __restrict__ logits, const uint8_t* __restrict__ j0,
                const float* __restrict__ scales, const float* __restrict__ noise, NoiseKey nk,
                int out_f, int in_f, int G, int gs, int bits, float tau, float kappa,
                const float* __restrict__ w_ref, float* __restrict__ w_out,
                __nv_bfloat16* __restrict__ w_hi, __nv_bfloat16* __restrict__ w_mid,
                __nv_bfloat16* __restrict__ w_lo) {
  const int64_t d = (int64_t)out_f * in_f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d;
       i += (int64_t)gridDim.x * blockDim.x) {
    float g[K], p[K], C[K];
    SoftMath<K>::noise(noise, d, i, nk, g);
    SoftMath<K>::probs(logits, d, i, g, tau, kappa, p);
    SoftMath<K>::candidates(bits, K == 5 ? (int)j0[i] : 0, C);
    float c = __fmul_rn(p[0], C[0]);
#pragma unroll
    for (int k = 1; k < K; ++k) c = __fadd_rn(c, __fmul_rn(p[k], C[k]));
    const int row = (int)(i / in_f), col = (int)(i - (int64_t)row * in_f);
    float w = __fmul_rn(scales[(int64_t)row * G + col / gs], c);
    if (w_ref) w = __fsub_rn(w, w_ref[i]);
    if (w_out) w_out[i] = w;
    if (w_hi) {
      __nv_bfloat16 h, m, l;
      split3_bf16(w, h, m, l);
      w_hi[i] = h;
      if (w_mid) w_mid[i] = m;
      if (w_lo) w_lo[i] = l;
    }
  }
}

__device__ __forceinline__ float sgn(float x) { return (float)((x > 0.f) - (x < 0.f)); }

struct LionConst {
  float b1, omb1, b2, omb2, wd;
};

// theta <- theta - lr (sign(b1 m + (1 - b1) g) + wd theta);  m <- b2 m + (1 - b2) g
__device__ __forceinline__ void lion1(float& p, float& m, float g, float lr, const LionConst& c) {
  const float u = sgn(__fadd_rn(__fmul_rn(c.b1, m), __fmul_rn(c.omb1, g)));
  p = __fsub_rn(p, __fmul_rn(lr, __fadd_rn(u, __fmul_rn(c.wd, p))));
  m = __fadd_rn(__fmul_rn(c.b2, m), __fmul_rn(c.omb2, g));
}

constexpr int kMaxResamples = 8;

// One warp per (row, group): the group's weights are strided over the lanes (MAXW per lane),
// the scale gradient of each resample is a warp reduction, and lane 0 applies the scale's
// Lion step. The resample loop is outermost so that only the per-weight gradient sums stay
// live across resamples.
template <int K, int MAXW>
__global__ void __launch_bounds__(256)
soft_bwd_lion_kernel(float* __restrict__ logits, float* __restrict__ mom,
                     const uint8_t* __restrict__ j0, float* __restrict__ scales,
                     float* __restrict__ mom_s, const float* __restrict__ grad_w,
                     const float* __restrict__ noise, uint64_t seed, uint32_t linear_id,
                     uint32_t step, int R, int out_f, int in_f, int G, int gs, int bits,
                     float tau, float kappa, float lr_l, float lr_s, LionConst lc) {
  const int64_t d = (int64_t)out_f * in_f;
  const int lane = threadIdx.x & 31;
  const int64_t n_units = (int64_t)out_f * G;
  const float kt = __fdiv_rn(kappa, tau);
  const float fR = (float)R;
  for (int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; unit < n_units;
       unit += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int row = (int)(unit / G), grp = (int)(unit - (int64_t)row * G);
    const float s = scales[unit];
    const int c_begin = grp * gs, c_end = min(c_begin + gs, in_f);
    float acc[MAXW][K];
    float gsum = 0.f;
#pragma unroll 1
    for (int r = 0; r < R; ++r) {
      const NoiseKey nk = make_noise_key(seed, linear_id, step, (uint32_t)r);
      const float* noise_r = noise ? noise + (int64_t)r * K * d : nullptr;
      const float* grad_r = grad_w + (int64_t)r * d;
      double part = 0.0;
#pragma unroll
      for (int t = 0; t < MAXW; ++t) {
        const int col = c_begin + lane + 32 * t;
        if (col >= c_end) continue;
        const int64_t i = (int64_t)row * in_f + col;
        float C[K], g[K], p[K];
        SoftMath<K>::candidates(bits, K == 5 ? (int)j0[i] : 0, C);
        SoftMath<K>::noise(noise_r, d, i, nk, g);
        SoftMath<K>::probs(logits, d, i, g, tau, kappa, p);
        float c = __fmul_rn(p[0], C[0]);
#pragma unroll
        for (int k = 1; k < K; ++k) c = __fadd_rn(c, __fmul_rn(p[k], C[k]));
        const float G_r = grad_r[i];
        part += (double)G_r * (double)c;
        const float sG = __fmul_rn(s, G_r);
        float u[K];
        float pu = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          u[k] = __fmul_rn(sG, C[k]);
          pu = k == 0 ? __fmul_rn(p[0], u[0]) : __fadd_rn(pu, __fmul_rn(p[k], u[k]));
        }
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const float gl = __fmul_rn(kt, __fmul_rn(p[k], __fsub_rn(u[k], pu)));
          acc[t][k] = r == 0 ? gl : __fadd_rn(acc[t][k], gl);
        }
      }
      const float gr = (float)warp_sum_d(part);
      gsum = r == 0 ? gr : __fadd_rn(gsum, gr);
    }
#pragma unroll
    for (int t = 0; t < MAXW; ++t) {
      const int col = c_begin + lane + 32 * t;
      if (col >= c_end) continue;
      const int64_t i = (int64_t)row * in_f + col;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        float pv = logits[k * d + i], mv = mom[k * d + i];
        lion1(pv, mv, __fdiv_rn(acc[t][k], fR), lr_l, lc);
        logits[k * d + i] = pv;
        mom[k * d + i] = mv;
      }
    }
    if (lane == 0) {
      float sv = s, mv = mom_s[unit];
      lion1(sv, mv, __fdiv_rn(gsum, fR), lr_s, lc);
      scales[unit] = sv;
      mom_s[unit] = mv;
    }
  }
}

template <int K>
__global__ void harden_kernel(const float* __restrict__ logits, const uint8_t* __restrict__ j0,
                              int64_t d, int bits, uint8_t* __restrict__ codes) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d;
       i += (int64_t)gridDim.x * blockDim.x) {
    int best = 0;
    float bv = logits[i];
#pragma unroll
    for (int k = 1; k < K; ++k) {
      const float v = logits[k * d + i];
      if (v > bv) { bv = v; best = k; }
    }
    if (K == 5) best = min(max((int)j0[i] + best - 2, 0), (1 << bits) - 1);
    codes[i] = (uint8_t)best;
  }
}

__global__ void lion_flat_kernel(float* __restrict__ p, float* __restrict__ m,
                                 const float* __restrict__ g, int64_t n, float lr, LionConst lc) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float pv = p[i], mv = m[i];
    lion1(pv, mv, g[i], lr, lc);
    p[i] = pv;
    m[i] = mv;
  }
}

inline LionConst lion_const(double wd, double b1, double b2) {
  LionConst c;
  c.b1 = (float)b1;
  c.omb1 = (float)(1.0 - b1);
  c.b2 = (float)b2;
  c.omb2 = (float)(1.0 - b2);
  c.wd = (float)wd;
  return c;
}

inline int n_logit_planes(int bits) { return bits == 2 ? 4 : (bits >= 3 && bits <= 7 ? 5 : 0); }

inline unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace gsq

using namespace gsq;

extern "C" int gsq_soft_fwd(const float* logits, const uint8_t* j0, const float* scales,
                            const float* noise, uint64_t seed, uint32_t linear_id, uint32_t step,
                            uint32_t resample, int out_f, int in_f, int group_size, int bits,
                            float tau, float kappa, const float* w_ref, float* w_out, void* w_hi,
                            void* w_mid, void* w_lo, void* stream) {
  const int K = n_logit_planes(bits);
  if (K == 0) return GSQ_ENOTSUP;
  if (out_f <= 0 || in_f <= 0 || group_size <= 0 || !logits || !scales || (K == 5 && !j0) ||
      !(tau > 0.f))
    return GSQ_EINVAL;
  if ((int64_t)out_f * in_f > 0xFFFFFFFFll) return GSQ_EINVAL;  // Philox counter is 32-bit
  if (!w_out && !w_hi) return GSQ_EINVAL;
  const int G = (in_f + group_size - 1) / group_size;
  const NoiseKey nk = make_noise_key(seed, linear_id, step, resample);
  const int64_t d = (int64_t)out_f * in_f;
  cudaStream_t st = (cudaStream_t)stream;
  auto* hi = (__nv_bfloat16*)w_hi;
  auto* mid = (__nv_bfloat16*)w_mid;
  auto* lo = (__nv_bfloat16*)w_lo;
  if (K == 5)
    soft_fwd_kernel<5><<<grid_for(d, 256), 256, 0, st>>>(logits, j0, scales, noise, nk, out_f,
                                                        in_f, G, group_size, bits, tau, kappa,
                                                        w_ref, w_out, hi, mid, lo);
  else
    soft_fwd_kernel<4><<<grid_for(d, 256), 256, 0, st>>>(logits, j0, scales, noise, nk, out_f,
                                                        in_f, G, group_size, bits, tau, kappa,
                                                        w_ref, w_out, hi, mid, lo);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_soft_bwd_lion(float* logits, float* mom_logits, const uint8_t* j0,
                                 float* scales, float* mom_scales, const float* grad_w,
                                 const float* noise, uint64_t seed, uint32_t linear_id,
                                 uint32_t step, int resamples, int out_f, int in_f,
                                 int group_size, int bits, float tau, float kappa,
                                 float lr_logits, float lr_scales, double wd, double beta1,
                                 double beta2, void* stream) {
  const int K = n_logit_planes(bits);
  if (K == 0) return GSQ_ENOTSUP;
  if (out_f <= 0 || in_f <= 0 || group_size <= 0 || resamples < 1 ||
      resamples > kMaxResamples || !logits || !mom_logits || !scales || !mom_scales ||
      !grad_w || (K == 5 && !j0) || !(tau > 0.f))
    return GSQ_EINVAL;
  if ((int64_t)out_f * in_f > 0xFFFFFFFFll) return GSQ_EINVAL;
  const int G = (in_f + group_size - 1) / group_size;
  const int64_t units = (int64_t)out_f * G;
  const LionConst lc = lion_const(wd, beta1, beta2);
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = grid_for(units * 32, 256);
  const int per_lane = (group_size + 31) / 32;
#define GSQ_BWD_LAUNCH(KK, MW)                                                               \
  soft_bwd_lion_kernel<KK, MW><<<grid, 256, 0, st>>>(                                        \
      logits, mom_logits, j0, scales, mom_scales, grad_w, noise, seed, linear_id, step,     \
      resamples, out_f, in_f, G, group_size, bits, tau, kappa, lr_logits, lr_scales, lc)
  if (per_lane > 8) return GSQ_ENOTSUP;
  if (K == 5) {
    if (per_lane == 1) GSQ_BWD_LAUNCH(5, 1);
    else if (per_lane == 2) GSQ_BWD_LAUNCH(5, 2);
    else if (per_lane <= 4) GSQ_BWD_LAUNCH(5, 4);
    else GSQ_BWD_LAUNCH(5, 8);
  } else {
    if (per_lane == 1) GSQ_BWD_LAUNCH(4, 1);
    else if (per_lane == 2) GSQ_BWD_LAUNCH(4, 2);
    else if (per_lane <= 4) GSQ_BWD_LAUNCH(4, 4);
    else GSQ_BWD_LAUNCH(4, 8);
  }
#undef GSQ_BWD_LAUNCH
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_harden(const float* logits, const uint8_t* j0, int out_f, int in_f, int bits,
                          uint8_t* codes, void* stream) {
  const int K = n_logit_planes(bits);
  if (K == 0) return GSQ_ENOTSUP;
  if (out_f <= 0 || in_f <= 0 || !logits || !codes || (K == 5 && !j0)) return GSQ_EINVAL;
  const int64_t d = (int64_t)out_f * in_f;
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 5)
    harden_kernel<5><<<grid_for(d, 256), 256, 0, st>>>(logits, j0, d, bits, codes);
  else
    harden_kernel<4><<<grid_for(d, 256), 256, 0, st>>>(logits, j0, d, bits, codes);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_lion_f32(float* param, float* mom, const float* grad, int64_t n, float lr,
                            double wd, double beta1, double beta2, void* stream) {
  if (n < 0 || (n > 0 && (!param || !mom || !grad))) return GSQ_EINVAL;
  if (n == 0) return GSQ_OK;
  lion_flat_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
      param, mom, grad, n, lr, lion_const(wd, beta1, beta2));
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
