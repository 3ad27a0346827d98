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
//                    load: a warp per output column n, lanes over 32-value blocks of the row,
//                    X staged in shared memory, warp-shuffle reduction.
#include <cuda_fp16.h>
#include <string.h>

#include "common.cuh"

namespace gsq {

constexpr int kQgemvMaxRows = 8;

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

// Y[m][n] = sum_k X[m][k] bf16(w[n][k]) for m < MR, float32 accumulation; out bf16 (rounded
// once) or float32. Dynamic shared memory: X as bf16 [MR][K].
template <int B, int MR>
__global__ void __launch_bounds__(256)
qgemv_kernel(const __nv_bfloat16* __restrict__ X, int64_t ld_x, int M, int K,
             const uint32_t* __restrict__ words, const void* __restrict__ scales,
             const void* __restrict__ biases, int sdtype, int gs, int N, void* __restrict__ Y,
             int64_t ld_y, int y_f32) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  const int nv = K / 8;
  for (int i = threadIdx.x; i < MR * nv; i += blockDim.x) {
    const int m = i / nv, c = i - m * nv;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (m < M) v = *reinterpret_cast<const uint4*>(X + (int64_t)m * ld_x + 8 * c);
    *reinterpret_cast<uint4*>(xs + (int64_t)m * K + 8 * c) = v;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nblk = K / 32, wpr = nblk * B, G = K / gs;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; n < N; n += warps) {
    float acc[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = 0.f;
    for (int blk = lane; blk < nblk; blk += 32) {
      uint32_t w[B];
      load_words<B>(words + (int64_t)n * wpr + (int64_t)blk * B, w);
      const int64_t gi = (int64_t)n * G + (blk * 32) / gs;
      const float s = load_scale(scales, gi, sdtype), b = load_scale(biases, gi, sdtype);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        float wf[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          wf[j] = bf16r_dev(__fadd_rn(__fmul_rn(s, (float)code_at<B>(w, 8 * v + j)), b));
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xs + (int64_t)m * K + blk * 32 + 8 * v);
          const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 xf = __bfloat1622float2(x2[j]);
            acc[m] = __fmaf_rn(xf.x, wf[2 * j], acc[m]);
            acc[m] = __fmaf_rn(xf.y, wf[2 * j + 1], acc[m]);
          }
        }
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

template <int B>
int qgemv_launch_b(const __nv_bfloat16* X, int64_t ld_x, int M, int K, const uint32_t* words,
                   const void* scales, const void* biases, int sdtype, int gs, int N, void* Y,
                   int64_t ld_y, int y_f32, cudaStream_t st) {
  const int MR = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
  const size_t smem = (size_t)MR * K * sizeof(__nv_bfloat16);
  int64_t blocks = ((int64_t)N * 32 + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  const unsigned g = (unsigned)(blocks < 1 ? 1 : blocks);
#define GSQ_QGEMV(RR)                                                                        \
  do {                                                                                       \
    auto kern = qgemv_kernel<B, RR>;                                                         \
    if (smem > 48 * 1024 &&                                                                  \
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != \
            cudaSuccess)                                                                     \
      return GSQ_ECUDA;                                                                      \
    kern<<<g, 256, smem, st>>>(X, ld_x, M, K, words, scales, biases, sdtype, gs, N, Y, ld_y, \
                               y_f32);                                                       \
  } while (0)
  if (MR == 1) GSQ_QGEMV(1);
  else if (MR == 2) GSQ_QGEMV(2);
  else if (MR == 4) GSQ_QGEMV(4);
  else GSQ_QGEMV(8);
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
    if ((size_t)kQgemvMaxRows * K * sizeof(__nv_bfloat16) > 200 * 1024) return GSQ_ENOTSUP;
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
