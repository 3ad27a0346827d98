// CUDA-core GEMMs with arbitrary element strides (float32 and float64).
// The float64 instance carries GPTQ's factorization updates, lazy column updates and error
// term; the float32 instance is the first contraction of the GSQ step, kept as the
// reference-precision path next to the tensor-core engine.
#include "common.cuh"

namespace gsq {

template <typename TIn, typename T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
gemm_simt_kernel(int M, int N, int K, T alpha, const TIn* __restrict__ A, int64_t sam,
                 int64_t sak, const TIn* __restrict__ B, int64_t sbk, int64_t sbn, T beta,
                 T* __restrict__ C, int64_t ldc, int tri) {
  constexpr int NT = (BM / TM) * (BN / TN);
  __shared__ T As[BK][BM + 1];
  __shared__ T Bs[BK][BN + 1];
  const int bm = blockIdx.y * BM, bn = blockIdx.x * BN;
  if (tri && bn > bm + BM - 1) return;  // tile strictly above the diagonal
  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);
  T acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = T(0);
  const bool a_kfast = (sak == 1);
  const bool b_nfast = (sbn == 1);
  for (int k0 = 0; k0 < K; k0 += BK) {
    for (int e = tid; e < BM * BK; e += NT) {
      int mm, kk;
      if (a_kfast) { kk = e % BK; mm = e / BK; } else { mm = e % BM; kk = e / BM; }
      const int gm = bm + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? T(A[(int64_t)gm * sam + (int64_t)gk * sak]) : T(0);
    }
    for (int e = tid; e < BN * BK; e += NT) {
      int nn, kk;
      if (b_nfast) { nn = e % BN; kk = e / BN; } else { kk = e % BK; nn = e / BK; }
      const int gn = bn + nn, gk = k0 + kk;
      Bs[kk][nn] = (gn < N && gk < K) ? T(B[(int64_t)gk * sbk + (int64_t)gn * sbn]) : T(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      T a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int gm = bm + ty * TM + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int gn = bn + tx * TN + j;
      if (gn >= N || (tri && gn > gm)) continue;
      T* c = C + (int64_t)gm * ldc + gn;
      *c = (beta == T(0)) ? alpha * acc[i][j] : alpha * acc[i][j] + beta * (*c);
    }
  }
}

template <typename TIn, typename T>
int gemm_simt(int M, int N, int K, T alpha, const TIn* A, int64_t sam, int64_t sak, const TIn* B,
              int64_t sbk, int64_t sbn, T beta, T* C, int64_t ldc, int tri, cudaStream_t st) {
  if (M < 0 || N < 0 || K < 0 || (M > 0 && N > 0 && (!C || (K > 0 && (!A || !B)))))
    return GSQ_EINVAL;
  if (M == 0 || N == 0) return GSQ_OK;
  constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4;
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  if (grid.y > 65535) return GSQ_EINVAL;
  gemm_simt_kernel<TIn, T, BM, BN, BK, TM, TN><<<grid, (BM / TM) * (BN / TN), 0, st>>>(
      M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, ldc, tri);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

// Deterministic sum of squares: fixed grid of 1024 blocks, then one block.
__global__ void sumsq_partial_kernel(const float* __restrict__ x, int64_t n, double* partials) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const double v = (double)x[i];
    s = fma(v, v, s);
  }
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) partials[blockIdx.x] = v;
  }
}

__global__ void sum_partials_kernel(const double* __restrict__ partials, int n, double* out) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += partials[i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) out[0] = v;
  }
}

template int gemm_simt<float, double>(int, int, int, double, const float*, int64_t, int64_t,
                                      const float*, int64_t, int64_t, double, double*, int64_t,
                                      int, cudaStream_t);
template int gemm_simt<double, double>(int, int, int, double, const double*, int64_t, int64_t,
                                       const double*, int64_t, int64_t, double, double*,
                                       int64_t, int, cudaStream_t);

}  // namespace gsq

extern "C" int gsq_gemm_f32(int M, int N, int K, float alpha, const float* A, int64_t sam,
                            int64_t sak, const float* B, int64_t sbk, int64_t sbn, float beta,
                            float* C, int64_t ldc, void* stream) {
  return gsq::gemm_simt<float, float>(M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, ldc, 0,
                               (cudaStream_t)stream);
}

extern "C" int gsq_gemm_f64(int M, int N, int K, double alpha, const double* A, int64_t sam,
                            int64_t sak, const double* B, int64_t sbk, int64_t sbn, double beta,
                            double* C, int64_t ldc, int tri, void* stream) {
  return gsq::gemm_simt<double, double>(M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, ldc, tri,
                                (cudaStream_t)stream);
}

extern "C" int gsq_sumsq_f32(const float* x, int64_t n, double* partials, double* out,
                             void* stream) {
  if (n < 0 || !partials || !out || (n > 0 && !x)) return GSQ_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  gsq::sumsq_partial_kernel<<<1024, 256, 0, st>>>(x, n, partials);
  GSQ_CHECK_LAUNCH();
  gsq::sum_partials_kernel<<<1, 1024, 0, st>>>(partials, 1024, out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
