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
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSmemBudget = 200 * 1024;

struct GemmParams {
  CUtensorMap tma_a[3];
  CUtensorMap tma_b[3];
  int M, N, K;
  int na, nb, order;
  float alpha, beta;
  float* C;
  int64_t ldc;
  int c_vec;             // C rows 16-byte aligned: float4 stores
  __nv_bfloat16* cs[3];  // C as bf16 terms [M][ldcs], ldcs % 8 == 0
  int ncs;
  int64_t ldcs;
  __nv_bfloat16* ct[3];  // C^T as bf16 terms [N][ldct], ldct % 8 == 0, ldct >= pad8(M)
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

__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
}

// TMEM columns: two buffers, each a "big" accumulator (the hi x hi products) and a "small"
// one (every other product, 2^8 smaller). Tensor-core accumulation into TMEM is not IEEE
// round-to-nearest; folding each chunk of k-blocks into float32 registers with IEEE adds
// keeps the error of the 3-term products at the level of a float32 GEMM. Eight epilogue warps
// fold: warp w reads TMEM lanes 32 (w % 4) .. + 31 (one output row per thread) and 64 of the
// tile's 128 columns.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full_bar[8];
  __shared__ uint64_t empty_bar[8];
  __shared__ uint64_t accf_bar[2];
  __shared__ uint64_t acce_bar[2];
  __shared__ uint32_t tmem_base;
  __shared__ double red[kEpiWarps];

  constexpr uint32_t kTileA = BM * BK * 2;  // bytes of one A term tile
  constexpr uint32_t kTileB = BN * BK * 2;
  constexpr uint32_t kCols = 4 * BN;        // 2 buffers x (big, small)
  constexpr int kHalf = BN / 2;             // columns per epilogue warp
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
      mbar_init(&acce_bar[b], kEpiWarps);
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
    const int ew = warp - 2;                  // epilogue warp 0..7
    const int q = warp & 3;                   // TMEM lane quadrant (hardware rule: warp % 4)
    const int h = ew >> 2;                    // column half of the tile
    const int r_loc = q * 32 + lane;
    const int row = tile_m + r_loc;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float acc[kHalf];
#pragma unroll
    for (int t = 0; t < kHalf; ++t) acc[t] = 0.f;
    bool ok = true;
    for (int c = 0; c < n_chunks; ++c) {
      const int b = c & 1;
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&accf_bar[b], (uint32_t)(c >> 1) & 1u,
                                                   p.err, 3));
      if (!ok) break;
      fence_after_sync();
      const uint32_t big = tmem + lane_off + (uint32_t)(b * 2 * BN + h * kHalf);
      const uint32_t small = big + BN;
#pragma unroll
      for (int c0 = 0; c0 < kHalf; c0 += 32) {
        uint32_t v[32], w[32];
        tmem_ld32_nowait(big + (uint32_t)c0, v);
        if (has_small) tmem_ld32_nowait(small + (uint32_t)c0, w);
        tmem_wait_ld();
        if (has_small) {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            acc[c0 + t] = __fadd_rn(acc[c0 + t],
                                    __fadd_rn(__uint_as_float(v[t]), __uint_as_float(w[t])));
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) acc[c0 + t] = __fadd_rn(acc[c0 + t], __uint_as_float(v[t]));
        }
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[b]);
    }
    // ---- outputs (the pipeline stages are idle now: every MMA and TMA load has completed)
    const bool live = ok && row < p.M;
    const int n0 = tile_n + h * kHalf;
    double sq = 0.0;
#pragma unroll
    for (int t = 0; t < kHalf; ++t) acc[t] = __fmul_rn(p.alpha, acc[t]);
    if (live && p.C) {
      float* crow = p.C + (int64_t)row * p.ldc + n0;
      if (p.c_vec && n0 + kHalf <= p.N) {
#pragma unroll
        for (int t = 0; t < kHalf; t += 4) {
          float4 x = make_float4(acc[t], acc[t + 1], acc[t + 2], acc[t + 3]);
          if (p.beta != 0.f) {
            const float4 o = *reinterpret_cast<const float4*>(crow + t);
            x.x = __fadd_rn(x.x, __fmul_rn(p.beta, o.x));
            x.y = __fadd_rn(x.y, __fmul_rn(p.beta, o.y));
            x.z = __fadd_rn(x.z, __fmul_rn(p.beta, o.z));
            x.w = __fadd_rn(x.w, __fmul_rn(p.beta, o.w));
          }
          *reinterpret_cast<float4*>(crow + t) = x;
          acc[t] = x.x; acc[t + 1] = x.y; acc[t + 2] = x.z; acc[t + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int t = 0; t < kHalf; ++t) {
          if (n0 + t < p.N) {
            float x = acc[t];
            if (p.beta != 0.f) x = __fadd_rn(x, __fmul_rn(p.beta, crow[t]));
            crow[t] = x;
            acc[t] = x;
          }
        }
      }
    }
    if (live && p.sq_partial) {
#pragma unroll
      for (int t = 0; t < kHalf; ++t)
        if (n0 + t < p.N) sq += (double)acc[t] * (double)acc[t];
    }
    if (live && p.ncs > 0) {
      // row-major terms straight from registers, 16-byte stores (8 bf16)
#pragma unroll
      for (int t = 0; t < kHalf; t += 8) {
        if (n0 + t >= p.N) break;
        __align__(16) __nv_bfloat16 hv[3][8];
#pragma unroll
        for (int u = 0; u < 8; ++u) split3_bf16(acc[t + u], hv[0][u], hv[1][u], hv[2][u]);
        for (int i = 0; i < p.ncs; ++i)
          *reinterpret_cast<uint4*>(p.cs[i] + (int64_t)row * p.ldcs + n0 + t) =
              *reinterpret_cast<const uint4*>(hv[i]);
      }
    }
    if (p.nct > 0) {
      // transposed terms: stage [term][n][m] bf16 tiles in shared memory, then 16-byte
      // coalesced row stores of C^T
      __nv_bfloat16* T = reinterpret_cast<__nv_bfloat16*>(smem);
#pragma unroll
      for (int t = 0; t < kHalf; ++t) {
        __nv_bfloat16 hv[3];
        split3_bf16(live ? acc[t] : 0.f, hv[0], hv[1], hv[2]);
        const int n_loc = h * kHalf + t;
        for (int i = 0; i < p.nct; ++i) T[(i * BN + n_loc) * BM + r_loc] = hv[i];
      }
      epi_sync();
      const int tid = threadIdx.x - 64;
      const int chunks = p.nct * BN * (BM / 8);
      for (int e = tid; e < chunks; e += 32 * kEpiWarps) {
        const int i = e / (BN * (BM / 8));
        const int rem = e - i * (BN * (BM / 8));
        const int n_loc = rem / (BM / 8), m8 = (rem % (BM / 8)) * 8;
        const int n = tile_n + n_loc, m = tile_m + m8;
        if (n < p.N && m < p.M && ok)
          *reinterpret_cast<uint4*>(p.ct[i] + (int64_t)n * p.ldct + m) =
              *reinterpret_cast<const uint4*>(T + (i * BN + n_loc) * BM + m8);
      }
    }
    if (p.sq_partial) {
      sq = warp_sum_d(sq);
      if (lane == 0) red[ew] = sq;
    }
  }
  fence_before_sync();
  __syncthreads();
  if (p.sq_partial && threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < kEpiWarps; ++i) t += red[i];
    p.sq_partial[blockIdx.y * gridDim.x + blockIdx.x] = t;
  }
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
  if (lda < K || ldb < K || (C && ldc < N) || (ncs > 0 && (ldcs < N || (ldcs & 7))) ||
      (nct > 0 && (ldct < ((M + 7) / 8) * 8 || (ldct & 7))))
    return GSQ_EINVAL;
  for (int i = 0; i < ncs; ++i)
    if ((uintptr_t)c_terms[i] & 15) return GSQ_EINVAL;
  for (int i = 0; i < nct; ++i)
    if ((uintptr_t)ct_terms[i] & 15) return GSQ_EINVAL;
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
  p.c_vec = (C && ((uintptr_t)C & 15) == 0 && (ldc & 3) == 0) ? 1 : 0;
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
