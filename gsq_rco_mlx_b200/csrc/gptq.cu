// GPTQ on the GPU in float64: Hessian accumulation, factorization of the damped inverse
// Hessian into its upper Cholesky factor, the row-parallel blocked column sweep with signed
// group scales, dequantization and the calibration error 1/2 tr(D H D^T).
//
// Factorization: with J the exchange matrix, chol(J Hd J) = Lr gives Hd = (J Lr J)(J Lr J)^T
// with J Lr J upper, so Hd^-1 = U^T U with U = J Lr^-1 J. One Cholesky and one triangular
// inverse replace the reference's Cholesky, inverse, product and second Cholesky.
//
// Encoding arithmetic (rint of w / s, the error w - s q, the division by U_jj, the float32
// rounding of |s|) uses explicit round-to-nearest intrinsics, so codes follow the float64
// operations of the reference one rounding at a time.
#include <math.h>

#include "common.cuh"

namespace gsq {

constexpr int kCholNB = 32;    // Cholesky panel width
constexpr int kSweepRows = 16; // output rows per sweep CTA (one warp each)
constexpr int kMaxBlock = 128; // largest lazy-update block
constexpr int kMaxGroupPerLane = 8;  // group_size <= 256

// ------------------------------------------------------------------- Hessian ---------

__global__ void scale_f64_kernel(double* __restrict__ x, int64_t n, double a) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    x[i] *= a;
}

// ------------------------------------------------------------- factorization ---------

// dead[i] = (H_ii == 0); ws[0] = damp * mean(diag Hd) with dead diagonals set to 1.
__global__ void diag_prep_kernel(const double* __restrict__ H, int n, double damp,
                                 uint8_t* __restrict__ dead, double* __restrict__ ws) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double h = H[(int64_t)i * n + i];
    const bool dd = (h == 0.0);
    dead[i] = dd ? 1 : 0;
    s += dd ? 1.0 : h;
  }
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) ws[0] = damp * (v / (double)n);
  }
}

// A = J Hd J (lower triangle), Hd = H with dead diagonals 1 and the damping on the diagonal.
__global__ void reverse_damped_kernel(const double* __restrict__ H, int n,
                                      const uint8_t* __restrict__ dead,
                                      const double* __restrict__ ws, double* __restrict__ A) {
  const int64_t nn = (int64_t)n * n;
  const double add = ws[0];
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nn;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(e / n), j = (int)(e - (int64_t)i * n);
    if (j > i) { A[e] = 0.0; continue; }
    const int a = n - 1 - i, b = n - 1 - j;
    double v = H[(int64_t)a * n + b];
    if (a == b) v = (dead[a] ? 1.0 : v) + add;
    A[e] = v;
  }
}

// Unblocked Cholesky of the b x b diagonal block at (p, p), in shared memory.
__global__ void chol_diag_kernel(double* __restrict__ A, int n, int p, int b, int* info) {
  __shared__ double T[kCholNB][kCholNB + 1];
  const int tid = threadIdx.x;
  for (int e = tid; e < b * b; e += blockDim.x) {
    const int r = e / b, c = e % b;
    T[r][c] = (c <= r) ? A[(int64_t)(p + r) * n + p + c] : 0.0;
  }
  __syncthreads();
  for (int j = 0; j < b; ++j) {
    if (tid == 0) {
      double d = T[j][j];
      if (!(d > 0.0)) {
        if (info) atomicCAS(info, 0, p + j + 1);
        d = 1.0;
      }
      T[j][j] = sqrt(d);
    }
    __syncthreads();
    for (int r = j + 1 + tid; r < b; r += blockDim.x) T[r][j] = T[r][j] / T[j][j];
    __syncthreads();
    for (int e = tid; e < b * b; e += blockDim.x) {
      const int r = e / b, c = e % b;
      if (r > j && c > j && c <= r) T[r][c] -= T[r][j] * T[c][j];
    }
    __syncthreads();
  }
  for (int e = tid; e < b * b; e += blockDim.x) {
    const int r = e / b, c = e % b;
    if (c <= r) A[(int64_t)(p + r) * n + p + c] = T[r][c];
  }
}

// Panel below the diagonal block: rows r >= p + b solve x L11^T = a (forward substitution).
__global__ void chol_trsm_kernel(double* __restrict__ A, int n, int p, int b) {
  __shared__ double L[kCholNB][kCholNB + 1];
  for (int e = threadIdx.x; e < b * b; e += blockDim.x) {
    const int r = e / b, c = e % b;
    L[r][c] = (c <= r) ? A[(int64_t)(p + r) * n + p + c] : 0.0;
  }
  __syncthreads();
  const int r = p + b + blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  double x[kCholNB];
  double* row = A + (int64_t)r * n + p;
#pragma unroll
  for (int j = 0; j < kCholNB; ++j) {
    if (j >= b) break;
    double v = row[j];
    for (int k = 0; k < j; ++k) v -= x[k] * L[j][k];
    x[j] = v / L[j][j];
  }
#pragma unroll
  for (int j = 0; j < kCholNB; ++j) {
    if (j >= b) break;
    row[j] = x[j];
  }
}

// Inverse of each 64 x 64 diagonal block of the lower-triangular L (one CTA per block):
// X[b][b] = L[b][b]^-1 by forward substitution, one thread per column of the block.
constexpr int kInvNB = 64;

__global__ void tri_inv_diag_kernel(const double* __restrict__ L, int n, double* __restrict__ X) {
  __shared__ double Ls[kInvNB][kInvNB + 1];
  const int p = blockIdx.x * kInvNB;
  const int b = min(kInvNB, n - p);
  for (int e = threadIdx.x; e < b * b; e += blockDim.x) {
    const int r = e / b, c = e % b;
    Ls[r][c] = (c <= r) ? L[(int64_t)(p + r) * n + p + c] : 0.0;
  }
  __syncthreads();
  const int j = threadIdx.x;  // column of the inverse
  if (j < b) {
    double x[kInvNB];
#pragma unroll
    for (int i = 0; i < kInvNB; ++i) x[i] = 0.0;
#pragma unroll
    for (int i = 0; i < kInvNB; ++i) {
      if (i >= b) break;
      if (i < j) continue;
      double dot = (i == j) ? 1.0 : 0.0;
      for (int k = j; k < i; ++k) dot -= Ls[i][k] * x[k];
      x[i] = dot / Ls[i][i];
    }
#pragma unroll
    for (int i = 0; i < kInvNB; ++i) {
      if (i >= b) break;
      X[(int64_t)(p + i) * n + p + j] = (i >= j) ? x[i] : 0.0;
    }
  }
}

// U = J X J (reversed rows and columns): X lower-triangular -> U upper-triangular.
__global__ void reverse_both_kernel(const double* __restrict__ X, int n, double* __restrict__ U) {
  const int64_t nn = (int64_t)n * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nn;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int a = (int)(e / n), c = (int)(e - (int64_t)a * n);
    U[e] = (c >= a) ? X[(int64_t)(n - 1 - a) * n + (n - 1 - c)] : 0.0;
  }
}

// ---------------------------------------------------------------------- sweep ---------

__device__ __forceinline__ double grid_val_d(int bits, int code) {
  return bits == 1 ? (double)(code - 1) : (double)(code - (1 << (bits - 1)));
}

// gptq.py _encode: clip(rint(x / s), grid0, gridN) - grid0, a zero scale encodes x / 1.
__device__ __forceinline__ int encode_d(double x, double s, double g0, double gN) {
  const double ss = (s == 0.0) ? 1.0 : s;
  double q = rint(__ddiv_rn(x, ss));
  q = fmin(fmax(q, g0), gN);
  return (int)(q - g0);
}

__device__ __forceinline__ double sq_err_d(double x, double s, int bits, double g0, double gN) {
  const int c = encode_d(x, s, g0, gN);
  const double e = __dsub_rn(x, __dmul_rn(s, grid_val_d(bits, c)));
  return __dmul_rn(e, e);
}

__global__ void sweep_init_kernel(const float* __restrict__ W, const uint8_t* __restrict__ dead,
                                  int out_f, int in_f, double* __restrict__ Wk) {
  const int64_t d = (int64_t)out_f * in_f;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < d;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % in_f);
    Wk[e] = dead[c] ? 0.0 : (double)W[e];
  }
}

// One CTA = kSweepRows output rows, one warp per row. Shared memory: the U block (bs x bs),
// and per row the in-block weights W1 and errors E.
__global__ void __launch_bounds__(kSweepRows * 32)
gptq_sweep_kernel(const double* __restrict__ U, int out_f, int in_f, int bits, int gs, int bs,
                  int signed_scale, uint8_t* __restrict__ codes, float* __restrict__ scales,
                  double* __restrict__ Wk) {
  extern __shared__ double smem[];
  double* Ub = smem;                    // [bs][bs]
  double* W1 = Ub + bs * bs;            // [rows][bs]
  double* E = W1 + kSweepRows * bs;     // [rows][bs]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kSweepRows + warp;
  const bool live = r < out_f;
  const int G = (in_f + gs - 1) / gs;
  const double g0 = grid_val_d(bits, 0);
  const double gN = grid_val_d(bits, bits == 1 ? 2 : (1 << bits) - 1);
  const double gmax = fmax(fabs(g0), fabs(gN));
  double* w1 = W1 + warp * bs;
  double* e1 = E + warp * bs;
  double* wrow = Wk + (int64_t)(live ? r : 0) * in_f;
  double s_cur = 0.0;
  for (int i1 = 0; i1 < in_f; i1 += bs) {
    const int i2 = min(i1 + bs, in_f), nb = i2 - i1;
    for (int e = threadIdx.x; e < nb * nb; e += blockDim.x) {
      const int t = e / nb, c = e % nb;
      Ub[t * bs + c] = (c >= t) ? U[(int64_t)(i1 + t) * in_f + i1 + c] : 0.0;
    }
    if (live)
      for (int c = lane; c < nb; c += 32) {
        w1[c] = wrow[i1 + c];
        e1[c] = 0.0;
      }
    __syncthreads();
    if (live) {
      for (int i = 0; i < nb; ++i) {
        const int j = i1 + i;
        if (j % gs == 0) {
          // current weights of the group: in-block columns from W1, later columns from Wk minus
          // this block's errors pushed through U (the lazy update not yet applied)
          const int e_end = min(j + gs, in_f);
          double cur[kMaxGroupPerLane];
          double amax = 0.0;
#pragma unroll
          for (int t = 0; t < kMaxGroupPerLane; ++t) {
            const int c = j + lane + 32 * t;
            cur[t] = 0.0;
            if (c < e_end) {
              double v;
              if (c < i2) {
                v = w1[c - i1];
              } else {
                v = wrow[c];
                for (int q = 0; q < i; ++q) v -= e1[q] * U[(int64_t)(i1 + q) * in_f + c];
              }
              cur[t] = v;
              amax = fmax(amax, fabs(v));
            }
          }
          amax = warp_max_d(amax);
          double s = (double)__double2float_rn(__ddiv_rn(amax, gmax));
          if (signed_scale) {
            double ep = 0.0, en = 0.0;
#pragma unroll
            for (int t = 0; t < kMaxGroupPerLane; ++t) {
              if (j + lane + 32 * t < e_end) {
                ep += sq_err_d(cur[t], s, bits, g0, gN);
                en += sq_err_d(cur[t], -s, bits, g0, gN);
              }
            }
            ep = warp_sum_d(ep);
            en = warp_sum_d(en);
            if (en < ep) s = -s;
          }
          s_cur = s;
          if (lane == 0) scales[(int64_t)r * G + j / gs] = (float)s;
        }
        const double w = w1[i];
        const int q = encode_d(w, s_cur, g0, gN);
        const double err =
            __ddiv_rn(__dsub_rn(w, __dmul_rn(s_cur, grid_val_d(bits, q))), Ub[i * bs + i]);
        if (lane == 0) {
          codes[(int64_t)r * in_f + j] = (uint8_t)q;
          e1[i] = err;
        }
        for (int c = i + 1 + lane; c < nb; c += 32) w1[c] -= err * Ub[i * bs + c];
        __syncwarp();
      }
      // lazy update of the columns right of the block: Wk[r, i2:] -= E U[i1:i2, i2:]
      for (int c = i2 + lane; c < in_f; c += 32) {
        double acc = 0.0;
        for (int t = 0; t < nb; ++t) acc = fma(e1[t], U[(int64_t)(i1 + t) * in_f + c], acc);
        wrow[c] -= acc;
      }
    }
    __syncthreads();
  }
}

__global__ void dequant_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ sc,
                               int out_f, int in_f, int bits, int gs, float* __restrict__ wq) {
  const int64_t d = (int64_t)out_f * in_f;
  const int G = (in_f + gs - 1) / gs;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < d;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / in_f), c = (int)(e - (int64_t)r * in_f);
    wq[e] = __fmul_rn(sc[(int64_t)r * G + c / gs], grid_value(bits, codes[e]));
  }
}

__global__ void diff_f64_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                int64_t n, double* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (double)a[i] - (double)b[i];
}

__global__ void dot_partial_kernel(const double* __restrict__ x, const double* __restrict__ y,
                                   int64_t n, double* __restrict__ partials) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    s = fma(x[i], y[i], s);
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) partials[blockIdx.x] = v;
  }
}

__global__ void half_sum_kernel(const double* __restrict__ partials, int n, double* out) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += partials[i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) out[0] = 0.5 * v;
  }
}

inline unsigned blocks_for(int64_t n, int t) {
  int64_t b = (n + t - 1) / t;
  const int64_t cap = (int64_t)num_sms() * 32;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace gsq

using namespace gsq;

extern "C" int hessian_accum(const float* X, int64_t m, int k, double* H, int64_t n_prev,
                             void* stream) {
  if (m < 0 || k <= 0 || n_prev < 0 || !H || (m > 0 && !X)) return GSQ_EINVAL;
  if (m == 0) return GSQ_OK;
  if (m > 0x7FFFFFFF) return GSQ_EINVAL;
  const int64_t total = n_prev + m;
  const double beta = (double)n_prev / (double)total;
  const double alpha = 2.0 / (double)total;
  // H <- beta H + alpha X^T X: A(i, r) = X[r, i], B(r, j) = X[r, j]
  return gemm_simt<float, double>(k, k, (int)m, alpha, X, 1, k, X, k, 1, beta, H, k, 0,
                                  (cudaStream_t)stream);
}

extern "C" int gptq_factor(const double* H, int n, double damp, double* U, uint8_t* dead,
                           double* workspace, int* info, void* stream) {
  if (n <= 0 || !H || !U || !dead || !workspace || !info || !(damp >= 0.0)) return GSQ_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t nn = (int64_t)n * n;
  double* A = workspace;
  double* Xc = workspace + nn;
  double* scal = workspace + 2 * nn;
  if (cudaMemsetAsync(info, 0, sizeof(int), st) != cudaSuccess) return GSQ_ECUDA;
  diag_prep_kernel<<<1, 1024, 0, st>>>(H, n, damp, dead, scal);
  GSQ_CHECK_LAUNCH();
  reverse_damped_kernel<<<blocks_for(nn, 256), 256, 0, st>>>(H, n, dead, scal, A);
  GSQ_CHECK_LAUNCH();
  for (int p = 0; p < n; p += kCholNB) {
    const int b = min(kCholNB, n - p);
    chol_diag_kernel<<<1, 256, 0, st>>>(A, n, p, b, info);
    GSQ_CHECK_LAUNCH();
    const int rest = n - p - b;
    if (rest > 0) {
      chol_trsm_kernel<<<(rest + 127) / 128, 128, 0, st>>>(A, n, p, b);
      GSQ_CHECK_LAUNCH();
      // trailing lower triangle: A22 -= P P^T
      const double* P = A + (int64_t)(p + b) * n + p;
      const int rc = gemm_simt<double, double>(rest, rest, b, -1.0, P, n, 1, P, 1, n, 1.0,
                                               A + (int64_t)(p + b) * n + p + b, n, 1, st);
      if (rc != GSQ_OK) return rc;
    }
  }
  // X = L^-1, block lower-triangular: invert the 64 x 64 diagonal blocks, then merge pairs
  // of neighbouring blocks of width w: [[A, 0], [B, C]]^-1 has lower-left block
  // -C^-1 (B A^-1), two float64 GEMMs per pair (U serves as the temporary).
  if (cudaMemsetAsync(Xc, 0, sizeof(double) * nn, st) != cudaSuccess) return GSQ_ECUDA;
  tri_inv_diag_kernel<<<(n + kInvNB - 1) / kInvNB, kInvNB, 0, st>>>(A, n, Xc);
  GSQ_CHECK_LAUNCH();
  for (int w = kInvNB; w < n; w *= 2) {
    for (int p = 0; p + w < n; p += 2 * w) {
      const int wa = w, wc = min(w, n - p - w);
      const double* Bm = A + (int64_t)(p + w) * n + p;            // L21 [wc x wa]
      const double* Ainv = Xc + (int64_t)p * n + p;               // [wa x wa]
      const double* Cinv = Xc + (int64_t)(p + w) * n + p + w;     // [wc x wc]
      double* Tm = U;                                             // [wc x wa], ld wa
      double* X21 = Xc + (int64_t)(p + w) * n + p;                // [wc x wa]
      int rc = gemm_simt<double, double>(wc, wa, wa, 1.0, Bm, n, 1, Ainv, n, 1, 0.0, Tm, wa, 0,
                                         st);
      if (rc != GSQ_OK) return rc;
      rc = gemm_simt<double, double>(wc, wa, wc, -1.0, Cinv, n, 1, Tm, wa, 1, 0.0, X21, n, 0, st);
      if (rc != GSQ_OK) return rc;
    }
  }
  reverse_both_kernel<<<blocks_for(nn, 256), 256, 0, st>>>(Xc, n, U);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gptq_sweep(const float* W, const double* U, const uint8_t* dead, int out_f,
                          int in_f, int bits, int group_size, int block_size, int signed_scale,
                          uint8_t* codes, float* scales, double* Wwork, void* stream) {
  if (!W || !U || !dead || !codes || !scales || !Wwork || out_f <= 0 || in_f <= 0)
    return GSQ_EINVAL;
  if (bits < 1 || bits > 8 || group_size <= 0 || block_size <= 0) return GSQ_EINVAL;
  if (block_size > kMaxBlock || group_size > 32 * kMaxGroupPerLane) return GSQ_ENOTSUP;
  cudaStream_t st = (cudaStream_t)stream;
  sweep_init_kernel<<<blocks_for((int64_t)out_f * in_f, 256), 256, 0, st>>>(W, dead, out_f,
                                                                            in_f, Wwork);
  GSQ_CHECK_LAUNCH();
  const int bs = block_size;
  const size_t smem = sizeof(double) * ((size_t)bs * bs + 2 * (size_t)kSweepRows * bs);
  if (cudaFuncSetAttribute(gptq_sweep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return GSQ_ECUDA;
  gptq_sweep_kernel<<<(out_f + kSweepRows - 1) / kSweepRows, kSweepRows * 32, smem, st>>>(
      U, out_f, in_f, bits, group_size, bs, signed_scale, codes, scales, Wwork);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gptq_dequant(const uint8_t* codes, const float* scales, int out_f, int in_f,
                            int bits, int group_size, float* w_q, void* stream) {
  if (!codes || !scales || !w_q || out_f <= 0 || in_f <= 0 || bits < 1 || bits > 8 ||
      group_size <= 0)
    return GSQ_EINVAL;
  dequant_kernel<<<blocks_for((int64_t)out_f * in_f, 256), 256, 0, (cudaStream_t)stream>>>(
      codes, scales, out_f, in_f, bits, group_size, w_q);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gptq_err(const float* w_q, const float* W, const double* H, int out_f, int in_f,
                        double* err, double* workspace, void* stream) {
  if (!w_q || !W || !H || !err || !workspace || out_f <= 0 || in_f <= 0) return GSQ_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t d = (int64_t)out_f * in_f;
  double* D = workspace;
  double* T = workspace + d;
  double* partials = workspace + 2 * d;
  diff_f64_kernel<<<blocks_for(d, 256), 256, 0, st>>>(w_q, W, d, D);
  GSQ_CHECK_LAUNCH();
  const int rc = gemm_simt<double, double>(out_f, in_f, in_f, 1.0, D, in_f, 1, H, in_f, 1, 0.0,
                                           T, in_f, 0, st);
  if (rc != GSQ_OK) return rc;
  dot_partial_kernel<<<1024, 256, 0, st>>>(T, D, d, partials);
  GSQ_CHECK_LAUNCH();
  half_sum_kernel<<<1, 1024, 0, st>>>(partials, 1024, err);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
