// Packed affine weights of the quantized-model eval (MLX "affine" layout, the export format of
// reference src/gsq_rco/gsq/export.py:60-90): per linear W [N][K],
//   words   u32 [N][K * bits / 32]   value k of a row at stream bits [k bits, (k + 1) bits),
//                                     least significant bit first, little-endian words
//   scales, biases [N][K / g]         bf16, f16 or f32
//   w[n][k] = scale[n][k / g] * q[n][k] + bias[n][k / g]
// evaluated in float32 (exact: a 16-bit scale times a code below 2^8 and a power-of-two multiple
// of the scale), then rounded to bf16 -- the bf16-dequantized dense weight of the reference's
// eval (src/gsq_rco/common/evaluate.py:35-78 on mlx-lm QuantizedLinear).
//
// Kernels:
//   qdequant_kernel  packed -> bf16 [N][ldw]: one thread per 32 values (bits words), an HBM
//                    stream; the prefill GEMM reads its output as the K-major B operand.
//   qgemv_kernel     Y [M][N] = X W^T for M <= 8 rows with the dequant fused into the weight
//                    load (MLX's matrix-vector form: per 32-value block s sum(x q) + bias
//                    sum(x), the weight never rounded): a warp per output column n, lanes over
//                    blocks, X staged in shared memory, warp-shuffle reduction.
#include <cuda_fp16.h>
#include <string.h>

#include "common.cuh"

namespace gsq {

constexpr int kQgemvMaxRows = 8;
constexpr size_t kQgemvSmemMax = 160 * 1024;

__device__ __forceinline__ float load_scale(const void* p, int64_t i, int dtype) {
  if (dtype == 0) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// The B words of one 32-value block (its stream bits are exactly B words, word-aligned).
template <int B>
__device__ __forceinline__ void load_words(const uint32_t* __restrict__ src, uint32_t w[B]) {
  if constexpr (B == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    w[0] = v.x; w[1] = v.y;
  } else if constexpr (B == 4 || B == 8) {
#pragma unroll
    for (int t = 0; t < B / 4; ++t) {
      const uint4 v = *reinterpret_cast<const uint4*>(src + 4 * t);
      w[4 * t] = v.x; w[4 * t + 1] = v.y; w[4 * t + 2] = v.z; w[4 * t + 3] = v.w;
    }
  } else if constexpr (B == 6) {
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      const uint2 v = *reinterpret_cast<const uint2*>(src + 2 * t);
      w[2 * t] = v.x; w[2 * t + 1] = v.y;
    }
  } else {
#pragma unroll
    for (int t = 0; t < B; ++t) w[t] = src[t];
  }
}

// Value j (< 32) of a block: stream bits [j B, j B + B) of the words.
template <int B>
__device__ __forceinline__ uint32_t code_at(const uint32_t w[B], int j) {
  const int bit = j * B, wi = bit >> 5, sh = bit & 31;
  const uint32_t lo = w[wi];
  const uint32_t hi = (sh + B > 32) ? w[wi + 1 < B ? wi + 1 : B - 1] : 0u;
  return __funnelshift_r(lo, hi, sh) & ((1u << B) - 1u);
}

template <int B>
__global__ void __launch_bounds__(256)
qdequant_kernel(const uint32_t* __restrict__ words, const void* __restrict__ scales,
                const void* __restrict__ biases, int sdtype, int N, int K, int gs,
                __nv_bfloat16* __restrict__ out, int64_t ldw) {
  const int nblk = K / 32, wpr = K / 32 * B, G = K / gs;
  const int64_t total = (int64_t)N * nblk;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(e / nblk), blk = (int)(e - (int64_t)n * nblk);
    uint32_t w[B];
    load_words<B>(words + (int64_t)n * wpr + (int64_t)blk * B, w);
    const int64_t gi = (int64_t)n * G + (blk * 32) / gs;
    const float s = load_scale(scales, gi, sdtype), b = load_scale(biases, gi, sdtype);
    __nv_bfloat16* o = out + (int64_t)n * ldw + blk * 32;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      __align__(16) __nv_bfloat16 t[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        t[j] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(s, (float)code_at<B>(w, 8 * v + j)), b));
      *reinterpret_cast<uint4*>(o + 8 * v) = *reinterpret_cast<const uint4*>(t);
    }
  }
}

// Y[m][n] = sum over 32-value blocks b of the row: s_b (sum_j x[m][32 b + j] q_j) + bias_b
// (sum_j x[m][32 b + j]), float32 -- MLX's quantized matrix-vector form (the weight s q + bias is
// never rounded; the code sums are exact integers times x). A warp per output column n, lanes
// over blocks (U blocks' words loaded before any arithmetic), codes turned into floats with the
// 2^23 exponent trick (float(q) = bits(0x4B000000 | q) - 2^23, no conversion unit), X staged in
// shared memory transposed per block position ([j / V][block][V], V values per vector load:
// consecutive lanes read consecutive vectors) as float32 (XF) or bf16, with per-block sums of X.
template <int B, int MR, int U, bool XF>
__global__ void __launch_bounds__(256)
qgemv_kernel(const __nv_bfloat16* __restrict__ X, int64_t ld_x, int M, int K,
             const uint32_t* __restrict__ words, const void* __restrict__ scales,
             const void* __restrict__ biases, int sdtype, int gs, int N, void* __restrict__ Y,
             int64_t ld_y, int y_f32) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int nblk = K / 32;
  float* xsum = reinterpret_cast<float*>(smem_raw);                  // [MR][nblk]
  unsigned char* xbase = smem_raw + (((size_t)MR * nblk * sizeof(float) + 15) & ~(size_t)15);
  constexpr int V = XF ? 4 : 8;                                      // values per 16-byte vector
  // staging: thread (m, b) moves block b of row m (32 values) and sums it
  for (int i = threadIdx.x; i < MR * nblk; i += blockDim.x) {
    const int m = i / nblk, b = i - m * nblk;
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 32 / 8; ++c) {
      uint4 raw = make_uint4(0u, 0u, 0u, 0u);
      if (m < M) raw = *reinterpret_cast<const uint4*>(X + (int64_t)m * ld_x + 32 * b + 8 * c);
      const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      float f[8];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 v = __bfloat1622float2(x2[t]);
        f[2 * t] = v.x;
        f[2 * t + 1] = v.y;
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) sum = __fadd_rn(sum, f[t]);
      if constexpr (XF) {
        float* xs = reinterpret_cast<float*>(xbase) + (size_t)m * K;
        *reinterpret_cast<float4*>(xs + ((size_t)(2 * c) * nblk + b) * 4) =
            make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4*>(xs + ((size_t)(2 * c + 1) * nblk + b) * 4) =
            make_float4(f[4], f[5], f[6], f[7]);
      } else {
        __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(xbase) + (size_t)m * K;
        *reinterpret_cast<uint4*>(xs + ((size_t)c * nblk + b) * 8) = raw;
      }
    }
    xsum[m * nblk + b] = sum;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int wpr = nblk * B, G = K / gs;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; n < N; n += warps) {
    float acc[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = 0.f;
    const uint32_t* wrow = words + (int64_t)n * wpr;
    for (int b0 = lane; b0 < nblk; b0 += 32 * U) {
      uint32_t w[U][B];
      float sc[U], bi[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int b = b0 + 32 * u;
        if (b < nblk) {
          load_words<B>(wrow + (int64_t)b * B, w[u]);
          const int64_t gi = (int64_t)n * G + (b * 32) / gs;
          sc[u] = load_scale(scales, gi, sdtype);
          bi[u] = load_scale(biases, gi, sdtype);
        } else {
#pragma unroll
          for (int t = 0; t < B; ++t) w[u][t] = 0u;
          sc[u] = 0.f;
          bi[u] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int b = b0 + 32 * u;
        if (b >= nblk) break;
        float dot[MR];
#pragma unroll
        for (int m = 0; m < MR; ++m) dot[m] = 0.f;
#pragma unroll
        for (int jv = 0; jv < 32 / V; ++jv) {
          float q[V];
#pragma unroll
          for (int t = 0; t < V; ++t)
            q[t] = __fsub_rn(__int_as_float(0x4B000000 | (int)code_at<B>(w[u], jv * V + t)),
                             8388608.f);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            float xv[V];
            if constexpr (XF) {
              const float4 v = *reinterpret_cast<const float4*>(
                  reinterpret_cast<const float*>(xbase) + (size_t)m * K +
                  ((size_t)jv * nblk + b) * 4);
              xv[0] = v.x; xv[1] = v.y; xv[2] = v.z; xv[3] = v.w;
            } else {
              const uint4 raw = *reinterpret_cast<const uint4*>(
                  reinterpret_cast<const __nv_bfloat16*>(xbase) + (size_t)m * K +
                  ((size_t)jv * nblk + b) * 8);
              const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
              for (int t = 0; t < V / 2; ++t) {
                const float2 f = __bfloat1622float2(x2[t]);
                xv[2 * t] = f.x;
                xv[2 * t + 1] = f.y;
              }
            }
#pragma unroll
            for (int t = 0; t < V; ++t) dot[m] = __fmaf_rn(xv[t], q[t], dot[m]);
          }
        }
#pragma unroll
        for (int m = 0; m < MR; ++m)
          acc[m] = __fmaf_rn(sc[u], dot[m], __fmaf_rn(bi[u], xsum[m * nblk + b], acc[m]));
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = warp_sum(acc[m]);
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        if (m >= M) break;
        if (y_f32)
          reinterpret_cast<float*>(Y)[(int64_t)m * ld_y + n] = acc[m];
        else
          reinterpret_cast<__nv_bfloat16*>(Y)[(int64_t)m * ld_y + n] = __float2bfloat16_rn(acc[m]);
      }
    }
  }
}

inline bool packed_args_ok(const void* words, const void* scales, const void* biases, int sdtype,
                           int N, int K, int bits, int gs) {
  if (!words || !scales || !biases || N <= 0 || K <= 0 || sdtype < 0 || sdtype > 2) return false;
  if (bits != 2 && bits != 3 && bits != 4 && bits != 5 && bits != 6 && bits != 8) return false;
  if (gs != 32 && gs != 64 && gs != 128) return false;
  if (K % gs) return false;
  const int align = bits == 4 || bits == 8 ? 16 : (bits == 2 || bits == 6 ? 8 : 4);
  if ((uintptr_t)words % align) return false;
  return true;
}

int qdequant_launch(const uint32_t* words, const void* scales, const void* biases, int sdtype,
                    int N, int K, int bits, int gs, __nv_bfloat16* out, int64_t ldw,
                    cudaStream_t st) {
  const int64_t total = (int64_t)N * (K / 32);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  const unsigned g = (unsigned)(blocks < 1 ? 1 : blocks);
#define GSQ_QDQ(BB) qdequant_kernel<BB><<<g, 256, 0, st>>>(words, scales, biases, sdtype, N, K, \
                                                               gs, out, ldw)
  switch (bits) {
    case 2: GSQ_QDQ(2); break;
    case 3: GSQ_QDQ(3); break;
    case 4: GSQ_QDQ(4); break;
    case 5: GSQ_QDQ(5); break;
    case 6: GSQ_QDQ(6); break;
    default: GSQ_QDQ(8); break;
  }
#undef GSQ_QDQ
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

inline size_t qgemv_smem(int MR, int K, bool xf) {
  return (((size_t)MR * (K / 32) * sizeof(float) + 15) & ~(size_t)15) + (size_t)MR * K * (xf ? 4 : 2);
}

template <int B>
int qgemv_launch_b(const __nv_bfloat16* X, int64_t ld_x, int M, int K, const uint32_t* words,
                   const void* scales, const void* biases, int sdtype, int gs, int N, void* Y,
                   int64_t ld_y, int y_f32, cudaStream_t st) {
  constexpr int U = B <= 4 ? 4 : 2;
  const int MR = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
  const bool xf = qgemv_smem(MR, K, true) <= kQgemvSmemMax;
  const size_t smem = qgemv_smem(MR, K, xf);
  if (smem > kQgemvSmemMax) return GSQ_ENOTSUP;
  int64_t blocks = ((int64_t)N * 32 + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  const unsigned g = (unsigned)(blocks < 1 ? 1 : blocks);
#define GSQ_QGEMV(RR, XX)                                                                    \
  do {                                                                                       \
    auto kern = qgemv_kernel<B, RR, U, XX>;                                                  \
    if (smem > 48 * 1024 &&                                                                  \
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != \
            cudaSuccess)                                                                     \
      return GSQ_ECUDA;                                                                      \
    kern<<<g, 256, smem, st>>>(X, ld_x, M, K, words, scales, biases, sdtype, gs, N, Y, ld_y, \
                               y_f32);                                                       \
  } while (0)
  if (xf) {
    if (MR == 1) GSQ_QGEMV(1, true);
    else if (MR == 2) GSQ_QGEMV(2, true);
    else if (MR == 4) GSQ_QGEMV(4, true);
    else GSQ_QGEMV(8, true);
  } else {
    if (MR == 1) GSQ_QGEMV(1, false);
    else if (MR == 2) GSQ_QGEMV(2, false);
    else if (MR == 4) GSQ_QGEMV(4, false);
    else GSQ_QGEMV(8, false);
  }
#undef GSQ_QGEMV
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

}  // namespace gsq

using namespace gsq;

extern "C" int qdequant_packed(const uint32_t* words, const void* scales, const void* biases,
                               int scale_dtype, int N, int K, int bits, int group_size,
                               void* out, int64_t ldw, void* stream) {
  if (!out || ldw < K || !packed_args_ok(words, scales, biases, scale_dtype, N, K, bits,
                                         group_size))
    return GSQ_EINVAL;
  if ((uintptr_t)out % 16 || ldw % 8) return GSQ_EINVAL;
  return qdequant_launch(words, scales, biases, scale_dtype, N, K, bits, group_size,
                         (__nv_bfloat16*)out, ldw, (cudaStream_t)stream);
}

extern "C" int qgemm_packed(const void* X, int M, int K, int64_t ld_x, const uint32_t* words,
                            const void* scales, const void* biases, int scale_dtype, int N,
                            int bits, int group_size, void* Y, int64_t ld_y, int y_f32,
                            void* workspace, int64_t workspace_bytes, int* err, void* stream) {
  if (!X || !Y || M <= 0 || ld_x < K || ld_y < N ||
      !packed_args_ok(words, scales, biases, scale_dtype, N, K, bits, group_size))
    return GSQ_EINVAL;
  if ((uintptr_t)X % 16 || ld_x % 8) return GSQ_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  const auto* x = (const __nv_bfloat16*)X;
  if (M <= kQgemvMaxRows) {
    switch (bits) {
      case 2: return qgemv_launch_b<2>(x, ld_x, M, K, words, scales, biases, scale_dtype,
                                       group_size, N, Y, ld_y, y_f32, st);
      case 3: return qgemv_launch_b<3>(x, ld_x, M, K, words, scales, biases, scale_dtype,
                                       group_size, N, Y, ld_y, y_f32, st);
      case 4: return qgemv_launch_b<4>(x, ld_x, M, K, words, scales, biases, scale_dtype,
                                       group_size, N, Y, ld_y, y_f32, st);
      case 5: return qgemv_launch_b<5>(x, ld_x, M, K, words, scales, biases, scale_dtype,
                                       group_size, N, Y, ld_y, y_f32, st);
      case 6: return qgemv_launch_b<6>(x, ld_x, M, K, words, scales, biases, scale_dtype,
                                       group_size, N, Y, ld_y, y_f32, st);
      default: return qgemv_launch_b<8>(x, ld_x, M, K, words, scales, biases, scale_dtype,
                                        group_size, N, Y, ld_y, y_f32, st);
    }
  }
  // prefill: dequantize into the workspace (bf16 [N][K], K-major), then the tensor-core GEMM
  if (!workspace || !err || workspace_bytes < (int64_t)N * K * 2 || (uintptr_t)workspace % 16)
    return GSQ_EINVAL;
  auto* wq = (__nv_bfloat16*)workspace;
  int s = qdequant_launch(words, scales, biases, scale_dtype, N, K, bits, group_size, wq, K, st);
  if (s != GSQ_OK) return s;
  gsq_gemm_desc d;
  memset(&d, 0, sizeof(d));
  d.M = M; d.N = N; d.K = K; d.batch = 1;
  d.a[0] = X; d.na = 1; d.lda = ld_x; d.a_rows = M;
  d.b[0] = wq; d.nb = 1; d.ldb = K; d.b_rows = N;
  d.order = 0; d.alpha = 1.f; d.beta = 0.f;
  if (y_f32) {
    d.C = (float*)Y; d.ldc = ld_y;
  } else {
    d.cs[0] = Y; d.ncs = 1; d.ldcs = ld_y;
  }
  d.err = err; d.bn = 128; d.split_k = 1;
  return gsq_gemm(&d, stream);
}
