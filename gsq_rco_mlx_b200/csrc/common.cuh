// Shared device helpers of the GSQ / GPTQ / RCO kernels (sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gsq_rco_b200.h"

#define GSQ_CHECK_LAUNCH()                                     \
  do {                                                         \
    cudaError_t e_ = cudaGetLastError();                       \
    if (e_ != cudaSuccess) return GSQ_ECUDA;                   \
  } while (0)

namespace gsq {

// ---------------------------------------------------------------- Philox4x32-10 ---
// Salmon, Moraes, Dror, Shaw, SC'11. Ten rounds, Weyl key schedule. The ten round keys depend
// only on (seed, linear id), so the host computes them once per launch and the kernels read
// them from the parameter bank; a round is two 32x32->64 multiplies and two three-input XORs.
struct PhiloxKey {
  uint32_t k0[10], k1[10];
};

__host__ __device__ inline PhiloxKey philox_key(uint64_t seed, uint32_t linear_id) {
  PhiloxKey k;
  uint32_t a = (uint32_t)(seed & 0xFFFFFFFFull), b = (uint32_t)(seed >> 32) ^ linear_id;
  for (int r = 0; r < 10; ++r) {
    k.k0[r] = a;
    k.k1[r] = b;
    a += 0x9E3779B9u;
    b += 0xBB67AE85u;
  }
  return k;
}

__device__ __forceinline__ uint64_t mul_wide_u32(uint32_t a, uint32_t b) {
  uint64_t p;
  asm("mul.wide.u32 %0, %1, %2;" : "=l"(p) : "r"(a), "r"(b));
  return p;
}

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, const PhiloxKey& k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = mul_wide_u32(0xD2511F53u, c.x), p1 = mul_wide_u32(0xCD9E8D57u, c.z);
    c = make_uint4((uint32_t)(p1 >> 32) ^ c.y ^ k.k0[r], (uint32_t)p1,
                   (uint32_t)(p0 >> 32) ^ c.w ^ k.k1[r], (uint32_t)p0);
  }
  return c;
}

// Gumbel noise of one weight and draw: one Philox call (counter (i, 0, step, resample)),
// planes 0..3 from the high 24 bits of x0..x3, plane 4 from their low bytes.
struct NoiseKey {
  PhiloxKey key;
  uint32_t step, resample;
};

__host__ __device__ inline NoiseKey make_noise_key(uint64_t seed, uint32_t linear_id,
                                                   uint32_t step, uint32_t resample) {
  NoiseKey k;
  k.key = philox_key(seed, linear_id);
  k.step = step;
  k.resample = resample;
  return k;
}

// u = (b + 0.5) 2^-24 as one fused multiply-add (b < 2^24 converts exactly; scaling by a power
// of two commutes with rounding, so this equals rounding b + 0.5 and then scaling), clipped to
// [1e-7, 1 - 1e-7]; g = -log(-log u). The inner logarithm needs relative accuracy (-log u is as
// small as 1e-7 near u = 1) and is the accurate logf; the outer one, of E = -log u in
// [1e-7, 16.2], needs absolute accuracy only (g enters the softmax additively) and is the
// hardware base-2 logarithm (__log2f, absolute error about 2^-22 in log2 E) times ln 2: one
// special-function instruction instead of a second accurate logarithm, the soft passes' largest
// instruction count per weight.
__device__ __forceinline__ float gumbel_from_24(uint32_t b) {
  float u = __fmaf_rn((float)b, 5.9604644775390625e-08f, 2.98023223876953125e-08f);
  u = fminf(fmaxf(u, 1e-7f), 1.0f - 1e-7f);
  return __fmul_rn(-0.693147180559945309f, __log2f(-logf(u)));
}

template <int K>
__device__ __forceinline__ void gumbel_weight(const PhiloxKey& key, uint32_t i, uint32_t step,
                                              uint32_t resample, float g[K]) {
  const uint4 x = philox4x32_10(make_uint4(i, 0u, step, resample), key);
  g[0] = gumbel_from_24(x.x >> 8);
  g[1] = gumbel_from_24(x.y >> 8);
  g[2] = gumbel_from_24(x.z >> 8);
  g[3] = gumbel_from_24(x.w >> 8);
  if (K > 4) g[K - 1] = gumbel_from_24((x.x & 255u) | ((x.y & 255u) << 8) | ((x.z & 255u) << 16));
}

// -------------------------------------------------------------------- bf16 split ---
// x = hi + mid + lo to float32 precision: each term is the bf16 rounding of the residual.
__device__ __forceinline__ void split3_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& mid,
                                            __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  const float r1 = __fsub_rn(x, __bfloat162float(hi));
  mid = __float2bfloat16_rn(r1);
  const float r2 = __fsub_rn(r1, __bfloat162float(mid));
  lo = __float2bfloat16_rn(r2);
}

__device__ __forceinline__ float bf16r_dev(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__host__ __device__ inline float grid_value(int bits, int code) {
  // quant.get_grid: arange(2^b) - 2^(b-1); ternary (bits 1) is [-1, 0, 1]
  return bits == 1 ? (float)(code - 1) : (float)(code - (1 << (bits - 1)));
}

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace gsq

namespace gsq {
template <typename TIn, typename T>
int gemm_simt(int M, int N, int K, T alpha, const TIn* A, int64_t sam, int64_t sak, const TIn* B,
              int64_t sbk, int64_t sbn, T beta, T* C, int64_t ldc, int tri, cudaStream_t st);
}  // namespace gsq
