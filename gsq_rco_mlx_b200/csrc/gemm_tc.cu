// Float32-faithful GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulator).
//
//   C[m, n] = alpha * sum_k A(m, k) B(n, k)        A, B given as 1..3 bf16 terms each,
//                                                   A = sum_i A_i, B = sum_j B_j (K-major)
// The products A_i B_j with i + j <= order are accumulated into one float32 TMEM accumulator
// (order 2 with three terms per side reproduces float32 operands to 2^-24; an exactly-bf16
// operand needs one term). One CTA computes one 128 x BN tile:
//   warp 0     TMA producer: for each 64-wide k-block, every term tile of A and B into one
//              pipeline stage (128-byte swizzle), completion counted on the stage's mbarrier
//   warp 1     TMEM allocator and MMA issuer: 4 UMMA K-steps x |products| per stage, then a
//              commit that frees the stage; a final commit publishes the accumulator
//   warps 2-5  epilogue: tcgen05.ld of their 32 TMEM lanes, then any of: float32 C
//              (alpha acc + beta C), C as bf16 terms, C^T as bf16 terms (the K-major operand
//              of a later reduction over m), and a per-tile sum of squares
// Every mbarrier wait is bounded; a timeout sets *err and the CTA unwinds, freeing its TMEM.
#include "tc_common.cuh"

namespace gsq {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kSmemBudget = 200 * 1024;

struct GemmParams {
  CUtensorMap tma_a[3];
  CUtensorMap tma_b[3];
  int M, N, K;
  int na, nb, order;
  float alpha, beta;
  float* C;
  int64_t ldc;
  __nv_bfloat16* cs[3];  // C as bf16 terms [M][ldcs]
  int ncs;
  int64_t ldcs;
  __nv_bfloat16* ct[3];  // C^T as bf16 terms [N][ldct]
  int nct;
  int64_t ldct;
  double* sq_partial;  // [tiles] sum of (alpha acc)^2 per tile
  int* err;
  int stages;
  int kb_per_chunk;  // k-blocks accumulated in TMEM before promotion to registers
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// TMEM columns: two buffers, each a "big" accumulator (the hi x hi products) and a "small"
// one (every other product, 2^8 smaller). Tensor-core accumulation into TMEM is not IEEE
// round-to-nearest; folding each chunk of k-blocks into float32 registers with IEEE adds
// keeps the error of the 3-term products at the level of a float32 GEMM.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full_bar[8];
  __shared__ uint64_t empty_bar[8];
  __shared__ uint64_t accf_bar[2];
  __shared__ uint64_t acce_bar[2];
  __shared__ uint32_t tmem_base;
  __shared__ double red[4];

  constexpr uint32_t kTileA = BM * BK * 2;  // bytes of one A term tile
  constexpr uint32_t kTileB = BN * BK * 2;
  constexpr uint32_t kCols = 4 * BN;        // 2 buffers x (big, small)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile_m = blockIdx.y * BM, tile_n = blockIdx.x * BN;
  const int S = p.stages;
  const uint32_t stage_bytes = p.na * kTileA + p.nb * kTileB;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int num_kb = (p.K + BK - 1) / BK;
  const int P = p.kb_per_chunk;
  const int n_chunks = (num_kb + P - 1) / P;
  const bool has_small = (p.na > 1 || p.nb > 1) && p.order > 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < p.na; ++i) tma_prefetch_desc(&p.tma_a[i]);
    for (int i = 0; i < p.nb; ++i) tma_prefetch_desc(&p.tma_b[i]);
  }
  if (warp == 1) tmem_alloc(&tmem_base, kCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (uint32_t)(kb / S) & 1u;
        if (!mbar_wait(&empty_bar[s], ph ^ 1u, p.err, 1)) break;
        uint8_t* st = smem + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(&full_bar[s], stage_bytes);
        for (int i = 0; i < p.na; ++i)
          tma_load_2d(st + i * kTileA, &p.tma_a[i], &full_bar[s], kb * BK, tile_m);
        for (int j = 0; j < p.nb; ++j)
          tma_load_2d(st + p.na * kTileA + j * kTileB, &p.tma_b[j], &full_bar[s], kb * BK,
                      tile_n);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN);
      bool ok = true;
      for (int c = 0; c < n_chunks && ok; ++c) {
        const int b = c & 1;
        if (!mbar_wait(&acce_bar[b], ((uint32_t)(c >> 1) & 1u) ^ 1u, p.err, 4)) break;
        fence_after_sync();
        const uint32_t big = tmem + (uint32_t)(b * 2 * BN), small = big + BN;
        bool big_init = false, small_init = false;
        const int kb_end = min(num_kb, (c + 1) * P);
        for (int kb = c * P; kb < kb_end; ++kb) {
          const int s = kb % S;
          const uint32_t ph = (uint32_t)(kb / S) & 1u;
          if (!mbar_wait(&full_bar[s], ph, p.err, 2)) { ok = false; break; }
          fence_after_sync();
          const uint32_t st = smem_u32(smem + (size_t)s * stage_bytes);
          for (int i = 0; i < p.na; ++i) {
            for (int j = 0; j < p.nb; ++j) {
              if (i + j > p.order) continue;
              const uint32_t a0 = st + i * kTileA;
              const uint32_t b0 = st + p.na * kTileA + j * kTileB;
              const bool to_big = (i + j == 0);
              const uint32_t d = to_big ? big : small;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k) {
                const uint32_t acc = to_big ? (uint32_t)big_init : (uint32_t)small_init;
                umma_bf16(d, umma_desc_k_sw128(a0 + k * 32), umma_desc_k_sw128(b0 + k * 32),
                          idesc, acc);
                if (to_big) big_init = true; else small_init = true;
              }
            }
          }
          umma_commit(&empty_bar[s]);
        }
        umma_commit(&accf_bar[b]);
      }
    }
  } else {
    // epilogue warps 2..5: TMEM lanes 32 * (warp % 4) .. + 31, one output row per thread
    const int q = warp & 3;
    const int row = tile_m + q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float acc[BN];
#pragma unroll
    for (int t = 0; t < BN; ++t) acc[t] = 0.f;
    bool ok = true;
    for (int c = 0; c < n_chunks; ++c) {
      const int b = c & 1;
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&accf_bar[b], (uint32_t)(c >> 1) & 1u,
                                                   p.err, 3));
      if (!ok) break;
      fence_after_sync();
      const uint32_t big = tmem + lane_off + (uint32_t)(b * 2 * BN), small = big + BN;
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(big + (uint32_t)c0, v);
        if (has_small) {
          float w[16];
          tmem_ld16(small + (uint32_t)c0, w);
#pragma unroll
          for (int t = 0; t < 16; ++t) acc[c0 + t] = __fadd_rn(acc[c0 + t], __fadd_rn(v[t], w[t]));
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t) acc[c0 + t] = __fadd_rn(acc[c0 + t], v[t]);
        }
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[b]);
    }
    double sq = 0.0;
    if (ok && row < p.M) {
#pragma unroll
      for (int t = 0; t < BN; ++t) {
        const int col = tile_n + t;
        if (col < p.N) {
          float x = __fmul_rn(p.alpha, acc[t]);
          if (p.C) {
            float* cp = p.C + (int64_t)row * p.ldc + col;
            if (p.beta != 0.f) x = __fadd_rn(x, __fmul_rn(p.beta, *cp));
            *cp = x;
          }
          if (p.sq_partial) sq += (double)x * (double)x;
          if (p.ncs > 0 || p.nct > 0) {
            __nv_bfloat16 h[3];
            split3_bf16(x, h[0], h[1], h[2]);
            for (int i = 0; i < p.ncs; ++i) p.cs[i][(int64_t)row * p.ldcs + col] = h[i];
            for (int i = 0; i < p.nct; ++i) p.ct[i][(int64_t)col * p.ldct + row] = h[i];
          }
        }
      }
    }
    if (p.sq_partial) {
      sq = warp_sum_d(sq);
      if (lane == 0) red[q] = sq;
    }
  }
  fence_before_sync();
  __syncthreads();
  if (p.sq_partial && threadIdx.x == 0)
    p.sq_partial[blockIdx.y * gridDim.x + blockIdx.x] = red[0] + red[1] + red[2] + red[3];
  if (warp == 1) {
    fence_after_sync();
    tmem_dealloc(tmem, kCols);
  }
}

// ------------------------------------------------------------------------ host side ---

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)f;
  }
  return fn;
}

// bf16 matrix [rows][ld] (cols valid), box = box_rows x 64, 128-byte swizzle, zero OOB fill.
static bool make_map(CUtensorMap* m, const void* base, int rows, int cols, int64_t ld,
                     int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || ((uintptr_t)base & 15) || ((ld * 2) & 15) || rows <= 0 || cols <= 0)
    return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
static int launch(GemmParams& p, cudaStream_t st) {
  const uint32_t stage_bytes = p.na * BM * BK * 2 + p.nb * BN * BK * 2;
  int S = (int)(kSmemBudget / stage_bytes);
  if (S > 8) S = 8;
  if (S < 2) return GSQ_ENOTSUP;
  p.stages = S;
  int products = 0;
  for (int i = 0; i < p.na; ++i)
    for (int j = 0; j < p.nb; ++j) products += (i + j <= p.order);
  p.kb_per_chunk = products >= 3 ? 1 : (products == 2 ? 2 : 4);
  const size_t smem = (size_t)S * stage_bytes + 1024;
  if (cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return GSQ_ECUDA;
  dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM);
  gemm_tc_kernel<BN><<<grid, kThreads, smem, st>>>(p);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

}  // namespace tc
}  // namespace gsq

using namespace gsq;

extern "C" int gsq_gemm_tc(int M, int N, int K, const void* const* a_terms, int na, int64_t lda,
                           const void* const* b_terms, int nb, int64_t ldb, int order,
                           float alpha, float* C, int64_t ldc, float beta, void* const* c_terms,
                           int ncs, int64_t ldcs, void* const* ct_terms, int nct, int64_t ldct,
                           double* sq_partial, int* err, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0 || na < 1 || na > 3 || nb < 1 || nb > 3 || order < 0 ||
      !a_terms || !b_terms || !err || ncs < 0 || ncs > 3 || nct < 0 || nct > 3 ||
      (ncs > 0 && !c_terms) || (nct > 0 && !ct_terms))
    return GSQ_EINVAL;
  if (!C && ncs == 0 && nct == 0 && !sq_partial) return GSQ_EINVAL;
  if (lda < K || ldb < K || (C && ldc < N) || (ncs > 0 && ldcs < N) || (nct > 0 && ldct < M))
    return GSQ_EINVAL;
  tc::GemmParams p;
  memset(&p, 0, sizeof(p));
  const int BN = 128;
  for (int i = 0; i < na; ++i)
    if (!tc::make_map(&p.tma_a[i], a_terms[i], M, K, lda, tc::BM)) return GSQ_EINVAL;
  for (int j = 0; j < nb; ++j)
    if (!tc::make_map(&p.tma_b[j], b_terms[j], N, K, ldb, BN)) return GSQ_EINVAL;
  p.M = M; p.N = N; p.K = K;
  p.na = na; p.nb = nb; p.order = order;
  p.alpha = alpha; p.beta = beta;
  p.C = C; p.ldc = ldc;
  for (int i = 0; i < ncs; ++i) p.cs[i] = (__nv_bfloat16*)c_terms[i];
  p.ncs = ncs; p.ldcs = ldcs;
  for (int i = 0; i < nct; ++i) p.ct[i] = (__nv_bfloat16*)ct_terms[i];
  p.nct = nct; p.ldct = ldct;
  p.sq_partial = sq_partial;
  p.err = err;
  return tc::launch<128>(p, (cudaStream_t)stream);
}

// fp32 [rows][ld_in] -> up to three bf16 terms, optionally transposed ([cols][ld_out]).
namespace gsq {
__global__ void split_f32_kernel(const float* __restrict__ x, int rows, int cols, int64_t ld_in,
                                 __nv_bfloat16* __restrict__ t0, __nv_bfloat16* __restrict__ t1,
                                 __nv_bfloat16* __restrict__ t2, int64_t ld_out) {
  const int64_t n = (int64_t)rows * cols;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / cols), c = (int)(e - (int64_t)r * cols);
    __nv_bfloat16 h, m, l;
    split3_bf16(x[(int64_t)r * ld_in + c], h, m, l);
    const int64_t o = (int64_t)r * ld_out + c;
    t0[o] = h;
    if (t1) t1[o] = m;
    if (t2) t2[o] = l;
  }
}

// transposed: 32 x 32 tiles through shared memory
__global__ void split_f32_t_kernel(const float* __restrict__ x, int rows, int cols,
                                   int64_t ld_in, __nv_bfloat16* __restrict__ t0,
                                   __nv_bfloat16* __restrict__ t1,
                                   __nv_bfloat16* __restrict__ t2, int64_t ld_out) {
  __shared__ float S[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int rr = threadIdx.y; rr < 32; rr += 8) {
    const int r = r0 + rr, c = c0 + threadIdx.x;
    S[rr][threadIdx.x] = (r < rows && c < cols) ? x[(int64_t)r * ld_in + c] : 0.f;
  }
  __syncthreads();
  for (int cc = threadIdx.y; cc < 32; cc += 8) {
    const int c = c0 + cc, r = r0 + threadIdx.x;
    if (c < cols && r < rows) {
      __nv_bfloat16 h, m, l;
      split3_bf16(S[threadIdx.x][cc], h, m, l);
      const int64_t o = (int64_t)c * ld_out + r;
      t0[o] = h;
      if (t1) t1[o] = m;
      if (t2) t2[o] = l;
    }
  }
}
}  // namespace gsq

extern "C" int gsq_split_bf16(const float* x, int rows, int cols, int64_t ld_in, int transpose,
                              void* t0, void* t1, void* t2, int64_t ld_out, void* stream) {
  if (!x || !t0 || rows <= 0 || cols <= 0 || ld_in < cols ||
      ld_out < (transpose ? rows : cols))
    return GSQ_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  if (transpose) {
    dim3 g((cols + 31) / 32, (rows + 31) / 32);
    split_f32_t_kernel<<<g, dim3(32, 8), 0, st>>>(x, rows, cols, ld_in, (__nv_bfloat16*)t0,
                                                  (__nv_bfloat16*)t1, (__nv_bfloat16*)t2, ld_out);
  } else {
    const int64_t n = (int64_t)rows * cols;
    int64_t b = (n + 255) / 256;
    if (b > (int64_t)num_sms() * 16) b = (int64_t)num_sms() * 16;
    split_f32_kernel<<<(unsigned)b, 256, 0, st>>>(x, rows, cols, ld_in, (__nv_bfloat16*)t0,
                                                  (__nv_bfloat16*)t1, (__nv_bfloat16*)t2, ld_out);
  }
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
