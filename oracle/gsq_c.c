/* Elementwise parts of the GSQ oracle in C (TEST INFRASTRUCTURE ONLY).
 *
 * The same arithmetic as the numpy restatement in oracle/gsq.py and oracle/philox.py, which
 * follows the reference egesabanci/gsq-rco-mlx:
 *   Philox Gumbel planes        oracle/philox.py (noise transform src/gsq_rco/gsq/staged.py:92-96)
 *   soft weight                 src/gsq_rco/gsq/staged.py:82-106, 271-298 (float32)
 *   soft backward               tests/oracles.py:340-344, local shift u_k = s * G * C_k (float64)
 *   Lion                        src/gsq_rco/gsq/lion.py:44-56 (float32)
 * It exists so that parity runs at full layer sizes (millions of weights, 200 steps) finish in
 * minutes; tests check it against the numpy restatement. Built with -ffp-contract=off so every
 * float32 product and sum rounds as numpy's does. Every function works on one range of its
 * index space [i0, i1), so that the Python side can split a call over host threads (ctypes
 * releases the interpreter lock during the call).
 */
#include <math.h>
#include <stdint.h>

static inline void philox10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n1 = (uint32_t)p1;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    const uint32_t n3 = (uint32_t)p0;
    c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

static inline float gumbel24(uint32_t b) {
  float u = ((float)b + 0.5f) * 5.9604644775390625e-08f; /* 2^-24 */
  const float lo = 1e-7f, hi = 1.0f - 1e-7f;
  if (u < lo) u = lo;
  if (u > hi) u = hi;
  return -logf(-logf(u));
}

/* out [K][d] float32: Gumbel noise of one draw (seed, linear, step, resample). */
void og_gumbel_planes(uint64_t seed, uint32_t linear_id, uint32_t step, uint32_t resample,
                      int64_t d, int K, float *out, int64_t i0, int64_t i1) {
  const uint32_t k0 = (uint32_t)seed;
  const uint32_t k1 = (uint32_t)(seed >> 32) ^ linear_id;
  for (int64_t i = i0; i < i1; ++i) {
    uint32_t c[4] = {(uint32_t)i, 0u, step, resample};
    philox10(c, k0, k1);
    for (int k = 0; k < K && k < 4; ++k) out[(int64_t)k * d + i] = gumbel24(c[k] >> 8);
    if (K > 4) {
      const uint32_t b = (c[0] & 255u) | ((c[1] & 255u) << 8) | ((c[2] & 255u) << 16);
      out[4 * d + i] = gumbel24(b);
    }
  }
}

/* Soft weight of one draw: p = softmax((kappa l + g) / tau) over the K candidates,
 * c = sum_k p_k C_k, w = s[row][col / gs] * c. logits, noise, Ckd, p: [K][d] float32;
 * scales [out][G] float32; w, c: [d] float32. */
void og_soft_weight(const float *logits, const float *noise, const float *Ckd,
                    const float *scales, int out_f, int in_f, int gs, int K, float tau,
                    float kappa, float *w, float *p, float *c, int64_t i0, int64_t i1) {
  const int64_t d = (int64_t)out_f * in_f;
  const int G = (in_f + gs - 1) / gs;
  const float inv_tau = 1.0f / tau;
  for (int64_t i = i0; i < i1; ++i) {
    float y[8];
    float mx = -INFINITY;
    for (int k = 0; k < K; ++k) {
      const float a = kappa * logits[(int64_t)k * d + i];
      const float b = a + noise[(int64_t)k * d + i];
      y[k] = b * inv_tau;
      if (y[k] > mx) mx = y[k];
    }
    float sum = 0.0f;
    for (int k = 0; k < K; ++k) {
      y[k] = expf(y[k] - mx);
      sum = sum + y[k];
    }
    const float inv = 1.0f / sum;
    float cc = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float pk = y[k] * inv;
      p[(int64_t)k * d + i] = pk;
      const float term = pk * Ckd[(int64_t)k * d + i];
      cc = (k == 0) ? term : cc + term;
    }
    c[i] = cc;
    const int64_t row = i / in_f, col = i % in_f;
    w[i] = scales[row * G + col / gs] * cc;
  }
}

/* Soft backward of one draw, added to float32 accumulators:
 *   u_k = s G C_k, dL/dl_k = (kappa / tau) p_k (u_k - <p, u>)   (float64, then float32)
 *   dL/ds[row][g] = sum over the group's columns of G c          (float64, then float32)
 * G [d] float64 = dL/dw_bar; glog_acc [K][d], gs_acc [out][G] float32. This function does
 * the logit part over weights [i0, i1); og_scale_grad_acc does the scale part. */
void og_soft_backward_acc(const double *Gr, const float *p, const float *Ckd, const float *c,
                          const float *scales, int out_f, int in_f, int gs, int K, double tau,
                          double kappa, float *glog_acc, float *gs_acc, int64_t i0, int64_t i1) {
  const int64_t d = (int64_t)out_f * in_f;
  const int G = (in_f + gs - 1) / gs;
  const double kt = kappa / tau;
  for (int64_t i = i0; i < i1; ++i) {
    const int64_t row = i / in_f, col = i % in_f;
    const double sG = (double)scales[row * G + col / gs] * Gr[i];
    double u[8], pu = 0.0;
    for (int k = 0; k < K; ++k) {
      u[k] = sG * (double)Ckd[(int64_t)k * d + i];
      const double t = (double)p[(int64_t)k * d + i] * u[k];
      pu = (k == 0) ? t : pu + t;
    }
    for (int k = 0; k < K; ++k) {
      const double pk = (double)p[(int64_t)k * d + i];
      const float g = (float)((kt * pk) * (u[k] - pu));
      glog_acc[(int64_t)k * d + i] = glog_acc[(int64_t)k * d + i] + g;
    }
  }
}

/* The scale part of og_soft_backward_acc over the (row, group) range [rg0, rg1). */
void og_scale_grad_acc(const double *Gr, const float *c, int out_f, int in_f, int gs,
                       float *gs_acc, int64_t rg0, int64_t rg1) {
  const int G = (in_f + gs - 1) / gs;
  for (int64_t rg = rg0; rg < rg1; ++rg) {
    const int64_t row = rg / G, g = rg % G;
    const int c0 = (int)g * gs, c1 = c0 + gs < in_f ? c0 + gs : in_f;
    double s = 0.0;
    for (int col = c0; col < c1; ++col) {
      const int64_t i = row * in_f + col;
      s += Gr[i] * (double)c[i];
    }
    gs_acc[rg] = gs_acc[rg] + (float)s;
  }
}

/* Lion in float32: u = sign(b1 m + (1 - b1) g); m <- b2 m + (1 - b2) g;
 * P <- P - lr (u + wd P). In place on P and M. */
void og_lion(float *P, float *M, const float *G, float lr, float wd, float b1,
             float one_minus_b1, float b2, float one_minus_b2, int64_t i0, int64_t i1) {
  for (int64_t i = i0; i < i1; ++i) {
    const float a = b1 * M[i];
    const float b = one_minus_b1 * G[i];
    const float mix = a + b;
    const float u = (mix > 0.0f) ? 1.0f : ((mix < 0.0f) ? -1.0f : 0.0f);
    const float dp = u + wd * P[i];
    P[i] = P[i] - lr * dp;
    const float m1 = b2 * M[i];
    const float m2 = one_minus_b2 * G[i];
    M[i] = m1 + m2;
  }
}
