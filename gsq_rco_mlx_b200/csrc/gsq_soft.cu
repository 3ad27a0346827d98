// GSQ soft-quantized linear, elementwise side: the Gumbel-softmax soft weight (forward), and the
// fused per-step pass backward(step t) + Lion + forward(step t + 1) over the training state,
// argmax decode, and a flat Lion step.
//
// The forward stores the probabilities p of every draw (float32, exact), so the backward never
// regenerates noise: one pass per step reads logits, momentum, codes, the stored p and the
// weight gradients, and writes logits, momentum, the next step's p and the next step's soft
// weights as bf16 GEMM terms. Elementwise arithmetic uses explicit round-to-nearest intrinsics,
// so no multiply-add is contracted and every product and sum is rounded as a float32 array op.
#include <math.h>

#include "common.cuh"

namespace gsq {

template <int K>
struct SoftMath {
  // p = softmax((kappa * l + g) * (1 / tau)), sums and maxima in candidate order.
  __device__ __forceinline__ static void probs(const float l[K], const float g[K], float inv_tau,
                                               float kappa, float p[K]) {
    float y[K];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      y[k] = __fmul_rn(__fadd_rn(__fmul_rn(kappa, l[k]), g[k]), inv_tau);
      m = fmaxf(m, y[k]);
    }
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      y[k] = expf(__fsub_rn(y[k], m));
      sum = k == 0 ? y[0] : __fadd_rn(sum, y[k]);
    }
    const float inv = __frcp_rn(sum);
#pragma unroll
    for (int k = 0; k < K; ++k) p[k] = __fmul_rn(y[k], inv);
  }

  __device__ __forceinline__ static void candidates(int bits, int j0, float C[K]) {
    if (K == 4) {
#pragma unroll
      for (int k = 0; k < K; ++k) C[k] = (float)(k - 2);  // 2-bit grid [-2, -1, 0, 1]
    } else {
      const int top = (1 << bits) - 1;
#pragma unroll
      for (int k = 0; k < K; ++k) C[k] = grid_value(bits, min(max(j0 + k - 2, 0), top));
    }
  }

  __device__ __forceinline__ static void noise(const float* __restrict__ noise_r, int64_t d,
                                               int64_t i, const PhiloxKey& key, uint32_t step,
                                               uint32_t resample, float g[K]) {
    if (noise_r) {
#pragma unroll
      for (int k = 0; k < K; ++k) g[k] = noise_r[k * d + i];
    } else {
      gumbel_weight<K>(key, (uint32_t)i, step, resample, g);
    }
  }

  __device__ __forceinline__ static float value(const float p[K], const float C[K]) {
    float c = __fmul_rn(p[0], C[0]);
#pragma unroll
    for (int k = 1; k < K; ++k) c = __fadd_rn(c, __fmul_rn(p[k], C[k]));
    return c;
  }
};

// Output of one soft weight w = s c (- w_ref): float32 and/or three bf16 terms.
__device__ __forceinline__ void store_soft(float w, int64_t i, int64_t d, float* w_out,
                                           __nv_bfloat16* terms) {
  if (w_out) w_out[i] = w;
  if (terms) {
    __nv_bfloat16 h, m, l;
    split3_bf16(w, h, m, l);
    terms[i] = h;
    terms[d + i] = m;
    terms[2 * d + i] = l;
  }
}

template <int K>
__global__ void __launch_bounds__(256)
soft_fwd_kernel(const float* __restrict__ logits, const uint8_t* __restrict__ j0,
                const float* __restrict__ scales, const float* __restrict__ noise, NoiseKey nk,
                int out_f, int in_f, int G, int gs, int bits, float inv_tau, float kappa,
                const float* __restrict__ w_ref, float* __restrict__ w_out,
                __nv_bfloat16* __restrict__ terms, float* __restrict__ p_out) {
  const int64_t d = (int64_t)out_f * in_f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d;
       i += (int64_t)gridDim.x * blockDim.x) {
    float l[K], g[K], p[K], C[K];
#pragma unroll
    for (int k = 0; k < K; ++k) l[k] = logits[k * d + i];
    SoftMath<K>::noise(noise, d, i, nk.key, nk.step, nk.resample, g);
    SoftMath<K>::probs(l, g, inv_tau, kappa, p);
    SoftMath<K>::candidates(bits, K == 5 ? (int)j0[i] : 0, C);
    const int row = (int)(i / in_f), col = (int)(i - (int64_t)row * in_f);
    float w = __fmul_rn(scales[(int64_t)row * G + col / gs], SoftMath<K>::value(p, C));
    if (w_ref) w = __fsub_rn(w, w_ref[i]);
    store_soft(w, i, d, w_out, terms);
    if (p_out) {
#pragma unroll
      for (int k = 0; k < K; ++k) p_out[k * d + i] = p[k];
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

// x / R correctly rounded for R = 1 or 2 (halving is exact up to the rounding the division does).
template <int R>
__device__ __forceinline__ float div_by(float x) {
  static_assert(R == 1 || R == 2, "resample counts of the vectorised step");
  return R == 1 ? x : __fmul_rn(x, 0.5f);
}

struct StepArgs {
  float* logits;
  float* mom;
  const uint8_t* j0;
  float* scales;
  float* mom_s;
  float* probs;          // [R][K][d]: this step's p in, the next step's p out
  const float* grad_w;   // [R][d]
  int R, out_f, in_f, G, gs, bits;
  float kt;              // kappa_t / tau_t of this step
  float lr_l, lr_s;
  LionConst lc;
  int next;              // run the forward of the next step
  const float* noise;    // [R][K][d] host-supplied noise of the next step, or NULL
  PhiloxKey key;         // round keys of (seed, linear id)
  uint32_t next_step;
  float inv_tau1, kappa1;
  const float* w_ref;
  float* w_out;          // [R][d]
  __nv_bfloat16* terms;  // [R][3][d]
};

// One warp per (row, group): the group's weights are strided over the lanes (MAXW per lane).
// Backward of this step from the stored p: u_k = s G C_k, dL/dl = (kappa/tau) p (u - <p, u>),
// dL/ds = sum over the group of G c (warp reduction); the sums over resamples are divided by R;
// Lion on logits (per lane) and on the group scale (lane 0, broadcast); then the forward of the
// next step with the updated logits and scale.
template <int K, int MAXW>
__global__ void __launch_bounds__(256) soft_step_kernel(const StepArgs a) {
  const int64_t d = (int64_t)a.out_f * a.in_f;
  const int lane = threadIdx.x & 31;
  const int64_t n_units = (int64_t)a.out_f * a.G;
  const float fR = (float)a.R;
  for (int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; unit < n_units;
       unit += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int row = (int)(unit / a.G), grp = (int)(unit - (int64_t)row * a.G);
    const float s = a.scales[unit];
    const int c_begin = grp * a.gs, c_end = min(c_begin + a.gs, a.in_f);
    float C[MAXW][K], acc[MAXW][K];
#pragma unroll
    for (int t = 0; t < MAXW; ++t) {
      const int col = c_begin + lane + 32 * t;
      const int64_t i = (int64_t)row * a.in_f + min(col, c_end - 1);
      SoftMath<K>::candidates(a.bits, K == 5 ? (int)a.j0[i] : 0, C[t]);
    }
    float gsum = 0.f;
#pragma unroll 1
    for (int r = 0; r < a.R; ++r) {
      const float* p_r = a.probs + (int64_t)r * K * d;
      const float* g_r = a.grad_w + (int64_t)r * d;
      double part = 0.0;
#pragma unroll
      for (int t = 0; t < MAXW; ++t) {
        const int col = c_begin + lane + 32 * t;
        if (col >= c_end) continue;
        const int64_t i = (int64_t)row * a.in_f + col;
        float p[K];
#pragma unroll
        for (int k = 0; k < K; ++k) p[k] = p_r[k * d + i];
        const float Gr = g_r[i];
        part += (double)Gr * (double)SoftMath<K>::value(p, C[t]);
        const float sG = __fmul_rn(s, Gr);
        float u[K];
        float pu = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          u[k] = __fmul_rn(sG, C[t][k]);
          pu = k == 0 ? __fmul_rn(p[0], u[0]) : __fadd_rn(pu, __fmul_rn(p[k], u[k]));
        }
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const float gl = __fmul_rn(a.kt, __fmul_rn(p[k], __fsub_rn(u[k], pu)));
          acc[t][k] = r == 0 ? gl : __fadd_rn(acc[t][k], gl);
        }
      }
      const float gr = (float)warp_sum_d(part);
      gsum = r == 0 ? gr : __fadd_rn(gsum, gr);
    }
    // Lion on the group scale (lane 0), the new scale broadcast for the forward
    float s_new = s;
    if (lane == 0) {
      float mv = a.mom_s[unit];
      lion1(s_new, mv, __fdiv_rn(gsum, fR), a.lr_s, a.lc);
      a.scales[unit] = s_new;
      a.mom_s[unit] = mv;
    }
    s_new = __shfl_sync(0xffffffffu, s_new, 0);
#pragma unroll
    for (int t = 0; t < MAXW; ++t) {
      const int col = c_begin + lane + 32 * t;
      if (col >= c_end) continue;
      const int64_t i = (int64_t)row * a.in_f + col;
      float l[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        float pv = a.logits[k * d + i], mv = a.mom[k * d + i];
        lion1(pv, mv, __fdiv_rn(acc[t][k], fR), a.lr_l, a.lc);
        a.logits[k * d + i] = pv;
        a.mom[k * d + i] = mv;
        l[k] = pv;
      }
      if (!a.next) continue;
      const float wr = a.w_ref ? a.w_ref[i] : 0.f;
#pragma unroll 1
      for (int r = 0; r < a.R; ++r) {
        float g[K], p[K];
        SoftMath<K>::noise(a.noise ? a.noise + (int64_t)r * K * d : nullptr, d, i, a.key,
                           a.next_step, (uint32_t)r, g);
        SoftMath<K>::probs(l, g, a.inv_tau1, a.kappa1, p);
        float w = __fmul_rn(s_new, SoftMath<K>::value(p, C[t]));
        if (a.w_ref) w = __fsub_rn(w, wr);
        store_soft(w, i, d, a.w_out ? a.w_out + (int64_t)r * d : nullptr,
                   a.terms ? a.terms + (int64_t)r * 3 * d : nullptr);
        float* pn = a.probs + (int64_t)r * K * d;
#pragma unroll
        for (int k = 0; k < K; ++k) pn[k * d + i] = p[k];
      }
    }
  }
}

// Vectorised form of soft_step_kernel for group sizes that are multiples of 64 and a
// compile-time resample count: a warp owns one (row, group), each lane two adjacent columns of
// every 64-column chunk (8-byte loads and stores), and every input of a lane's two weights is
// loaded before any arithmetic, so each lane keeps ~2 (2K + R(K + 1) + 2) loads in flight.
template <int K, int R>
__global__ void __launch_bounds__(256, 3) soft_step_v2_kernel(const StepArgs a) {
  const int64_t d = (int64_t)a.out_f * a.in_f;
  const int lane = threadIdx.x & 31;
  const int64_t n_units = (int64_t)a.out_f * a.G;
  const int n_chunks = a.gs / 64;
  for (int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; unit < n_units;
       unit += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int row = (int)(unit / a.G), grp = (int)(unit - (int64_t)row * a.G);
    const float s = a.scales[unit];
    // pass 1: gradients of every chunk; the per-weight sums stay in registers only for one
    // chunk, so a chunk is re-read in pass 2 (Lion and the next forward)
    float gsum_r[R];
#pragma unroll
    for (int r = 0; r < R; ++r) gsum_r[r] = 0.f;
    double part[R];
#pragma unroll
    for (int r = 0; r < R; ++r) part[r] = 0.0;
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int col = grp * a.gs + ch * 64 + 2 * lane;
      if (col >= a.in_f) continue;  // in_f is a multiple of 64 on this path
      const int64_t i = (int64_t)row * a.in_f + col;
      float2 pv[R][K];
      float2 Gv[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int k = 0; k < K; ++k)
          pv[r][k] = *reinterpret_cast<const float2*>(a.probs + ((int64_t)r * K + k) * d + i);
        Gv[r] = *reinterpret_cast<const float2*>(a.grad_w + (int64_t)r * d + i);
      }
      const uchar2 jj = K == 5 ? *reinterpret_cast<const uchar2*>(a.j0 + i) : make_uchar2(0, 0);
      float C0[K], C1[K];
      SoftMath<K>::candidates(a.bits, jj.x, C0);
      SoftMath<K>::candidates(a.bits, jj.y, C1);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float p0[K], p1[K];
#pragma unroll
        for (int k = 0; k < K; ++k) { p0[k] = pv[r][k].x; p1[k] = pv[r][k].y; }
        part[r] += (double)Gv[r].x * (double)SoftMath<K>::value(p0, C0);
        part[r] += (double)Gv[r].y * (double)SoftMath<K>::value(p1, C1);
      }
    }
    float gsum = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float gr = (float)warp_sum_d(part[r]);
      gsum = r == 0 ? gr : __fadd_rn(gsum, gr);
    }
    float s_new = s;
    if (lane == 0) {
      float mv = a.mom_s[unit];
      lion1(s_new, mv, div_by<R>(gsum), a.lr_s, a.lc);
      a.scales[unit] = s_new;
      a.mom_s[unit] = mv;
    }
    s_new = __shfl_sync(0xffffffffu, s_new, 0);
    (void)gsum_r;
    // pass 2: logit gradients, Lion, next forward
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int col = grp * a.gs + ch * 64 + 2 * lane;
      if (col >= a.in_f) continue;
      const int64_t i = (int64_t)row * a.in_f + col;
      float2 lv[K], mv[K], pv[R][K];
      float2 Gv[R];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        lv[k] = *reinterpret_cast<const float2*>(a.logits + k * d + i);
        mv[k] = *reinterpret_cast<const float2*>(a.mom + k * d + i);
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int k = 0; k < K; ++k)
          pv[r][k] = *reinterpret_cast<const float2*>(a.probs + ((int64_t)r * K + k) * d + i);
        Gv[r] = *reinterpret_cast<const float2*>(a.grad_w + (int64_t)r * d + i);
      }
      const uchar2 jj = K == 5 ? *reinterpret_cast<const uchar2*>(a.j0 + i) : make_uchar2(0, 0);
      const float2 wr = a.w_ref && a.next ? *reinterpret_cast<const float2*>(a.w_ref + i)
                                          : make_float2(0.f, 0.f);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float C[K], acc[K], l[K], m[K];
        SoftMath<K>::candidates(a.bits, e ? jj.y : jj.x, C);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float p[K];
#pragma unroll
          for (int k = 0; k < K; ++k) p[k] = e ? pv[r][k].y : pv[r][k].x;
          const float sG = __fmul_rn(s, e ? Gv[r].y : Gv[r].x);
          float u[K];
          float pu = 0.f;
#pragma unroll
          for (int k = 0; k < K; ++k) {
            u[k] = __fmul_rn(sG, C[k]);
            pu = k == 0 ? __fmul_rn(p[0], u[0]) : __fadd_rn(pu, __fmul_rn(p[k], u[k]));
          }
#pragma unroll
          for (int k = 0; k < K; ++k) {
            const float gl = __fmul_rn(a.kt, __fmul_rn(p[k], __fsub_rn(u[k], pu)));
            acc[k] = r == 0 ? gl : __fadd_rn(acc[k], gl);
          }
        }
#pragma unroll
        for (int k = 0; k < K; ++k) {
          l[k] = e ? lv[k].y : lv[k].x;
          m[k] = e ? mv[k].y : mv[k].x;
          lion1(l[k], m[k], div_by<R>(acc[k]), a.lr_l, a.lc);
          if (e) { lv[k].y = l[k]; mv[k].y = m[k]; } else { lv[k].x = l[k]; mv[k].x = m[k]; }
        }
        if (a.next) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            float g[K], p[K];
            SoftMath<K>::noise(a.noise ? a.noise + (int64_t)r * K * d : nullptr, d, i + e, a.key,
                               a.next_step, (uint32_t)r, g);
            SoftMath<K>::probs(l, g, a.inv_tau1, a.kappa1, p);
#pragma unroll
            for (int k = 0; k < K; ++k) {
              if (e) pv[r][k].y = p[k]; else pv[r][k].x = p[k];
            }
            float w = __fmul_rn(s_new, SoftMath<K>::value(p, C));
            if (a.w_ref) w = __fsub_rn(w, e ? wr.y : wr.x);
            Gv[r].x = e ? Gv[r].x : w;  // reuse: slot x/y holds the new soft weight
            Gv[r].y = e ? w : Gv[r].y;
          }
        }
      }
#pragma unroll
      for (int k = 0; k < K; ++k) {
        *reinterpret_cast<float2*>(a.logits + k * d + i) = lv[k];
        *reinterpret_cast<float2*>(a.mom + k * d + i) = mv[k];
      }
      if (a.next) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
          for (int k = 0; k < K; ++k)
            *reinterpret_cast<float2*>(a.probs + ((int64_t)r * K + k) * d + i) = pv[r][k];
          if (a.w_out) *reinterpret_cast<float2*>(a.w_out + (int64_t)r * d + i) = Gv[r];
          if (a.terms) {
            __nv_bfloat16 h0, m0, l0, h1, m1, l1;
            split3_bf16(Gv[r].x, h0, m0, l0);
            split3_bf16(Gv[r].y, h1, m1, l1);
            __nv_bfloat16* tb = a.terms + (int64_t)r * 3 * d + i;
            *reinterpret_cast<__nv_bfloat162*>(tb) = __halves2bfloat162(h0, h1);
            *reinterpret_cast<__nv_bfloat162*>(tb + d) = __halves2bfloat162(m0, m1);
            *reinterpret_cast<__nv_bfloat162*>(tb + 2 * d) = __halves2bfloat162(l0, l1);
          }
        }
      }
    }
  }
}

// Ternary soft weights (1 bit, grid [-1, 0, 1]): two logit planes per weight, the mask lm and
// the sign lb, and four Gumbel draws g0..g3. m = sigmoid((2 kappa lm + (g1 - g0)) / tau) is the
// probability that the weight is active, v = sigmoid((2 kappa lb + (g3 - g2)) / tau) that its
// sign is +, and the soft value is c = m (2 v - 1). The stored probability planes are (m, v).
struct Ternary {
  __device__ __forceinline__ static float sigmoid(float z) {
    return __frcp_rn(__fadd_rn(1.f, expf(-z)));
  }
  __device__ __forceinline__ static void probs(float lm, float lb, const float g[4],
                                               float inv_tau, float two_kappa, float& m,
                                               float& v) {
    m = sigmoid(__fmul_rn(__fadd_rn(__fmul_rn(two_kappa, lm), __fsub_rn(g[1], g[0])), inv_tau));
    v = sigmoid(__fmul_rn(__fadd_rn(__fmul_rn(two_kappa, lb), __fsub_rn(g[3], g[2])), inv_tau));
  }
  __device__ __forceinline__ static float value(float m, float v) {
    return __fmul_rn(m, __fsub_rn(__fmul_rn(2.f, v), 1.f));
  }
  // one draw's dL/dlm and dL/dlb from sG = s dL/dw and kt2 = 2 kappa / tau:
  // dc/dlm = kt2 (2 v - 1) m (1 - m), dc/dlb = kt2 m 2 v (1 - v)
  __device__ __forceinline__ static void grads(float m, float v, float sG, float kt2, float& gm,
                                               float& gb) {
    const float b = __fsub_rn(__fmul_rn(2.f, v), 1.f);
    gm = __fmul_rn(kt2, __fmul_rn(__fmul_rn(sG, b), __fmul_rn(m, __fsub_rn(1.f, m))));
    gb = __fmul_rn(kt2, __fmul_rn(__fmul_rn(sG, m),
                                  __fmul_rn(2.f, __fmul_rn(v, __fsub_rn(1.f, v)))));
  }
  __device__ __forceinline__ static void noise(const float* __restrict__ noise_r, int64_t d,
                                               int64_t i, const PhiloxKey& key, uint32_t step,
                                               uint32_t resample, float g[4]) {
    if (noise_r) {
#pragma unroll
      for (int k = 0; k < 4; ++k) g[k] = noise_r[k * d + i];
    } else {
      gumbel_weight<4>(key, (uint32_t)i, step, resample, g);
    }
  }
};

__global__ void __launch_bounds__(256)
soft_fwd_ternary_kernel(const float* __restrict__ logits, const float* __restrict__ scales,
                        const float* __restrict__ noise, NoiseKey nk, int out_f, int in_f, int G,
                        int gs, float inv_tau, float two_kappa, const float* __restrict__ w_ref,
                        float* __restrict__ w_out, __nv_bfloat16* __restrict__ terms,
                        float* __restrict__ p_out) {
  const int64_t d = (int64_t)out_f * in_f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d;
       i += (int64_t)gridDim.x * blockDim.x) {
    float g[4], m, v;
    Ternary::noise(noise, d, i, nk.key, nk.step, nk.resample, g);
    Ternary::probs(logits[i], logits[d + i], g, inv_tau, two_kappa, m, v);
    const int row = (int)(i / in_f), col = (int)(i - (int64_t)row * in_f);
    float w = __fmul_rn(scales[(int64_t)row * G + col / gs], Ternary::value(m, v));
    if (w_ref) w = __fsub_rn(w, w_ref[i]);
    store_soft(w, i, d, w_out, terms);
    if (p_out) {
      p_out[i] = m;
      p_out[d + i] = v;
    }
  }
}

// The fused step for ternary weights, one warp per (row, group) with the group's columns strided
// over the lanes: pass 1 sums G c over the group and resamples (float64 warp sums, one float32
// sum per resample) and takes the Lion step of the group scale; pass 2 forms the mask and sign
// logit gradients of every draw from the stored (m, v), takes their Lion steps and runs the next
// step's forward with the new logits and scale.
__global__ void __launch_bounds__(256) soft_step_ternary_kernel(const StepArgs a) {
  const int64_t d = (int64_t)a.out_f * a.in_f;
  const int lane = threadIdx.x & 31;
  const int64_t n_units = (int64_t)a.out_f * a.G;
  const float fR = (float)a.R;
  const float kt2 = __fmul_rn(2.f, a.kt);
  const float two_kappa1 = __fmul_rn(2.f, a.kappa1);
  for (int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; unit < n_units;
       unit += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int row = (int)(unit / a.G), grp = (int)(unit - (int64_t)row * a.G);
    const float s = a.scales[unit];
    const int c_begin = grp * a.gs, c_end = min(c_begin + a.gs, a.in_f);
    float gsum = 0.f;
#pragma unroll 1
    for (int r = 0; r < a.R; ++r) {
      const float* p_r = a.probs + (int64_t)r * 2 * d;
      const float* g_r = a.grad_w + (int64_t)r * d;
      double part = 0.0;
      for (int col = c_begin + lane; col < c_end; col += 32) {
        const int64_t i = (int64_t)row * a.in_f + col;
        part += (double)g_r[i] * (double)Ternary::value(p_r[i], p_r[d + i]);
      }
      const float gr = (float)warp_sum_d(part);
      gsum = r == 0 ? gr : __fadd_rn(gsum, gr);
    }
    float s_new = s;
    if (lane == 0) {
      float mv = a.mom_s[unit];
      lion1(s_new, mv, __fdiv_rn(gsum, fR), a.lr_s, a.lc);
      a.scales[unit] = s_new;
      a.mom_s[unit] = mv;
    }
    s_new = __shfl_sync(0xffffffffu, s_new, 0);
    for (int col = c_begin + lane; col < c_end; col += 32) {
      const int64_t i = (int64_t)row * a.in_f + col;
      float am = 0.f, ab = 0.f;
#pragma unroll 1
      for (int r = 0; r < a.R; ++r) {
        const float* p_r = a.probs + (int64_t)r * 2 * d;
        float gm, gb;
        Ternary::grads(p_r[i], p_r[d + i], __fmul_rn(s, a.grad_w[(int64_t)r * d + i]), kt2, gm,
                       gb);
        am = r == 0 ? gm : __fadd_rn(am, gm);
        ab = r == 0 ? gb : __fadd_rn(ab, gb);
      }
      float lm = a.logits[i], mm = a.mom[i], lb = a.logits[d + i], mb = a.mom[d + i];
      lion1(lm, mm, __fdiv_rn(am, fR), a.lr_l, a.lc);
      lion1(lb, mb, __fdiv_rn(ab, fR), a.lr_l, a.lc);
      a.logits[i] = lm;
      a.mom[i] = mm;
      a.logits[d + i] = lb;
      a.mom[d + i] = mb;
      if (!a.next) continue;
      const float wr = a.w_ref ? a.w_ref[i] : 0.f;
#pragma unroll 1
      for (int r = 0; r < a.R; ++r) {
        float g[4], m, v;
        Ternary::noise(a.noise ? a.noise + (int64_t)r * 4 * d : nullptr, d, i, a.key,
                       a.next_step, (uint32_t)r, g);
        Ternary::probs(lm, lb, g, a.inv_tau1, two_kappa1, m, v);
        float w = __fmul_rn(s_new, Ternary::value(m, v));
        if (a.w_ref) w = __fsub_rn(w, wr);
        store_soft(w, i, d, a.w_out ? a.w_out + (int64_t)r * d : nullptr,
                   a.terms ? a.terms + (int64_t)r * 3 * d : nullptr);
        float* pn = a.probs + (int64_t)r * 2 * d;
        pn[i] = m;
        pn[d + i] = v;
      }
    }
  }
}

// Ternary decode (the mask and sign signs): code 1 (value 0) where lm < 0, else 2 (+1) where
// lb >= 0 and 0 (-1) where lb < 0.
__global__ void harden_ternary_kernel(const float* __restrict__ logits, int64_t d,
                                      uint8_t* __restrict__ codes) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d;
       i += (int64_t)gridDim.x * blockDim.x)
    codes[i] = logits[i] >= 0.f ? (logits[d + i] >= 0.f ? 2 : 0) : 1;
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

// logit planes per weight: ternary mask + sign, the 2-bit grid, the 5 local shifts
inline int n_logit_planes(int bits) {
  return bits == 1 ? 2 : bits == 2 ? 4 : (bits >= 3 && bits <= 7 ? 5 : 0);
}

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
                            float tau, float kappa, const float* w_ref, float* w_out,
                            void* w_terms, float* p_out, void* stream) {
  const int K = n_logit_planes(bits);
  if (K == 0) return GSQ_ENOTSUP;
  if (out_f <= 0 || in_f <= 0 || group_size <= 0 || !logits || !scales || (K == 5 && !j0) ||
      !(tau > 0.f))
    return GSQ_EINVAL;
  if ((int64_t)out_f * in_f > 0xFFFFFFFFll) return GSQ_EINVAL;  // Philox counter is 32-bit
  if (!w_out && !w_terms && !p_out) return GSQ_EINVAL;
  const int G = (in_f + group_size - 1) / group_size;
  const NoiseKey nk = make_noise_key(seed, linear_id, step, resample);
  const int64_t d = (int64_t)out_f * in_f;
  const float inv_tau = 1.0f / tau;  // IEEE division on the host
  cudaStream_t st = (cudaStream_t)stream;
  auto* terms = (__nv_bfloat16*)w_terms;
  if (K == 2)
    soft_fwd_ternary_kernel<<<grid_for(d, 256), 256, 0, st>>>(
        logits, scales, noise, nk, out_f, in_f, G, group_size, inv_tau, 2.0f * kappa, w_ref,
        w_out, terms, p_out);
  else if (K == 5)
    soft_fwd_kernel<5><<<grid_for(d, 256), 256, 0, st>>>(logits, j0, scales, noise, nk, out_f,
                                                        in_f, G, group_size, bits, inv_tau,
                                                        kappa, w_ref, w_out, terms, p_out);
  else
    soft_fwd_kernel<4><<<grid_for(d, 256), 256, 0, st>>>(logits, j0, scales, noise, nk, out_f,
                                                        in_f, G, group_size, bits, inv_tau,
                                                        kappa, w_ref, w_out, terms, p_out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_soft_step(float* logits, float* mom_logits, const uint8_t* j0, float* scales,
                             float* mom_scales, float* probs, const float* grad_w, int resamples,
                             int out_f, int in_f, int group_size, int bits, float tau,
                             float kappa, float lr_logits, float lr_scales, double wd,
                             double beta1, double beta2, int next, const float* noise_next,
                             uint64_t seed, uint32_t linear_id, uint32_t next_step,
                             float tau_next, float kappa_next, const float* w_ref,
                             float* w_out, void* w_terms, void* stream) {
  const int K = n_logit_planes(bits);
  if (K == 0) return GSQ_ENOTSUP;
  if (out_f <= 0 || in_f <= 0 || group_size <= 0 || resamples < 1 ||
      resamples > kMaxResamples || !logits || !mom_logits || !scales || !mom_scales ||
      !probs || !grad_w || (K == 5 && !j0) || !(tau > 0.f))
    return GSQ_EINVAL;
  if (next && (!(tau_next > 0.f) || (!w_out && !w_terms))) return GSQ_EINVAL;
  if ((int64_t)out_f * in_f > 0xFFFFFFFFll) return GSQ_EINVAL;
  const int per_lane = (group_size + 31) / 32;
  if (K != 2 && per_lane > 8) return GSQ_ENOTSUP;
  StepArgs a;
  a.logits = logits; a.mom = mom_logits; a.j0 = j0; a.scales = scales; a.mom_s = mom_scales;
  a.probs = probs; a.grad_w = grad_w;
  a.R = resamples; a.out_f = out_f; a.in_f = in_f;
  a.G = (in_f + group_size - 1) / group_size; a.gs = group_size; a.bits = bits;
  a.kt = kappa / tau;
  a.lr_l = lr_logits; a.lr_s = lr_scales;
  a.lc = lion_const(wd, beta1, beta2);
  a.next = next; a.noise = noise_next; a.key = philox_key(seed, linear_id);
  a.next_step = next_step;
  a.inv_tau1 = next ? 1.0f / tau_next : 0.f;
  a.kappa1 = kappa_next;
  a.w_ref = w_ref; a.w_out = w_out; a.terms = (__nv_bfloat16*)w_terms;
  const int64_t units = (int64_t)out_f * a.G;
  const unsigned grid = grid_for(units * 32, 256);
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 2) {
    soft_step_ternary_kernel<<<grid, 256, 0, st>>>(a);
    GSQ_CHECK_LAUNCH();
    return GSQ_OK;
  }
  // vectorised path: 64-column chunks, 8-byte aligned planes, resamples 1 or 2
  const bool vec = (group_size % 64 == 0) && (in_f % 64 == 0) && (resamples <= 2) &&
                   ((uintptr_t)logits % 8 == 0) && ((uintptr_t)mom_logits % 8 == 0) &&
                   ((uintptr_t)probs % 8 == 0) && ((uintptr_t)grad_w % 8 == 0) &&
                   (!w_ref || (uintptr_t)w_ref % 8 == 0) && (!w_out || (uintptr_t)w_out % 8 == 0) &&
                   (!w_terms || (uintptr_t)w_terms % 4 == 0) && ((uintptr_t)j0 % 2 == 0);
  if (vec) {
    if (K == 5 && resamples == 2) soft_step_v2_kernel<5, 2><<<grid, 256, 0, st>>>(a);
    else if (K == 5) soft_step_v2_kernel<5, 1><<<grid, 256, 0, st>>>(a);
    else if (resamples == 2) soft_step_v2_kernel<4, 2><<<grid, 256, 0, st>>>(a);
    else soft_step_v2_kernel<4, 1><<<grid, 256, 0, st>>>(a);
    GSQ_CHECK_LAUNCH();
    return GSQ_OK;
  }
#define GSQ_STEP_LAUNCH(KK, MW) soft_step_kernel<KK, MW><<<grid, 256, 0, st>>>(a)
  if (K == 5) {
    if (per_lane == 1) GSQ_STEP_LAUNCH(5, 1);
    else if (per_lane == 2) GSQ_STEP_LAUNCH(5, 2);
    else if (per_lane <= 4) GSQ_STEP_LAUNCH(5, 4);
    else GSQ_STEP_LAUNCH(5, 8);
  } else {
    if (per_lane == 1) GSQ_STEP_LAUNCH(4, 1);
    else if (per_lane == 2) GSQ_STEP_LAUNCH(4, 2);
    else if (per_lane <= 4) GSQ_STEP_LAUNCH(4, 4);
    else GSQ_STEP_LAUNCH(4, 8);
  }
#undef GSQ_STEP_LAUNCH
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_soft_bwd_lion(float* logits, float* mom_logits, const uint8_t* j0,
                                 float* scales, float* mom_scales, float* probs,
                                 const float* grad_w, int resamples, int out_f, int in_f,
                                 int group_size, int bits, float tau, float kappa,
                                 float lr_logits, float lr_scales, double wd, double beta1,
                                 double beta2, int next, const float* noise_next, uint64_t seed,
                                 uint32_t linear_id, uint32_t next_step, float tau_next,
                                 float kappa_next, const float* w_ref, float* w_out,
                                 void* w_terms, void* stream) {
  return gsq_soft_step(logits, mom_logits, j0, scales, mom_scales, probs, grad_w, resamples,
                       out_f, in_f, group_size, bits, tau, kappa, lr_logits, lr_scales, wd,
                       beta1, beta2, next, noise_next, seed, linear_id, next_step, tau_next,
                       kappa_next, w_ref, w_out, w_terms, stream);
}

extern "C" int gsq_harden(const float* logits, const uint8_t* j0, int out_f, int in_f, int bits,
                          uint8_t* codes, void* stream) {
  const int K = n_logit_planes(bits);
  if (K == 0) return GSQ_ENOTSUP;
  if (out_f <= 0 || in_f <= 0 || !logits || !codes || (K == 5 && !j0)) return GSQ_EINVAL;
  const int64_t d = (int64_t)out_f * in_f;
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 2)
    harden_ternary_kernel<<<grid_for(d, 256), 256, 0, st>>>(logits, d, codes);
  else if (K == 5)
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
