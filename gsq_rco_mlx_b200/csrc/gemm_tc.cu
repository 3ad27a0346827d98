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

enum Epi {
  EPI_PLAIN = 0,
  EPI_RESID = 1,
  EPI_SWIGLU_FWD = 2,
  EPI_SWIGLU_BWD = 3,
  EPI_BF16 = 4,        // bf16 chain: x = bf16(acc); x = bf16(x + bias); x = bf16(resid + x)
  EPI_SWIGLU_BF16 = 5  // bf16 SwiGLU: g, u = bf16(acc); bf16(bf16(g bf16(sigmoid(g))) u)
};

struct Aff {
  int div;
  int64_t s1, s2;
  __device__ __forceinline__ int64_t at(int z) const {
    return (int64_t)(z / div) * s1 + (int64_t)(z % div) * s2;
  }
};

struct GemmParams {
  CUtensorMap tma_a[3];
  CUtensorMap tma_b[3];
  CUtensorMap tma_b2[3];
  int M, N, K;
  int na, nb, order, causal, dual_b;
  float alpha, beta;
  float* C;
  int64_t ldc;
  int c_vec;
  __nv_bfloat16* cs[3];
  int ncs;
  int64_t ldcs;
  __nv_bfloat16* ct[3];
  int nct;
  int64_t ldct;
  int64_t ct_up_rows;
  double* sq_partial;
  const float* bias;
  const __nv_bfloat16* resid;
  const __nv_bfloat16* target;
  int64_t ld_rt;
  float out_scale;
  float* aux0;
  float* aux1;
  int64_t ld_aux;
  Aff a_off, b_off, c_off, t_row, t_col;
  int* err;
  int stages;
  int kb_per_chunk;
  int skip_upper;  // output tiles entirely above the diagonal (n >= m) are not computed
  int row_period;  // epi 1: rows with (row % row_period) == 0 have a zero residual
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
}

__device__ __forceinline__ float sigmoid_f(float x) {
  return __frcp_rn(__fadd_rn(1.0f, expf(-x)));
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One 128 x BN output tile per CTA (grid z = batch). TMEM: two buffers of a "big" accumulator
// (the hi x hi products) and a "small" one (every other product, 2^8 smaller); tensor-core
// accumulation into TMEM is not IEEE round-to-nearest, so every chunk of k-blocks is folded into
// float32 registers with IEEE adds. Eight epilogue warps fold and finish: warp w reads TMEM lanes
// 32 (w % 4) .. + 31 (one output row per thread) and the 32-column chunks j with j % 2 == w / 4
// of the tile (for the SwiGLU forward this pairs gate column c with up column c + 64).
template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full_bar[8];
  __shared__ uint64_t empty_bar[8];
  __shared__ uint64_t accf_bar[2];
  __shared__ uint64_t acce_bar[2];
  __shared__ uint32_t tmem_base;
  __shared__ double red[kEpiWarps];

  constexpr uint32_t kTileA = BM * BK * 2;
  constexpr uint32_t kTileB = BN * BK * 2;
  constexpr uint32_t kCols = 4 * BN;
  constexpr int kAcc = BN / 2;   // accumulator columns per epilogue thread
  constexpr int kNC = BN / 64;   // 32-column chunks per epilogue thread
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int z = blockIdx.z;
  const int tile_m = blockIdx.y * BM, tile_n = blockIdx.x * BN;
  if (p.skip_upper && tile_n >= tile_m + BM) return;  // uniform across the CTA
  const int S = p.stages;
  const uint32_t stage_bytes = p.na * kTileA + p.nb * kTileB;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  // k-block range: causal 1 = lower-triangular A (k < end of this row tile), causal 2 =
  // upper-triangular A (k >= start of this row tile)
  const int kb_total = (p.K + BK - 1) / BK;
  const int kb0 = p.causal == 2 ? min(tile_m / BK, kb_total - 1) : 0;
  const int kb1 = p.causal == 1 ? min(kb_total, (tile_m + BM + BK - 1) / BK) : kb_total;
  const int num_kb = kb1 - kb0;
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
    for (int i = 0; i < p.nb; ++i) {
      tma_prefetch_desc(&p.tma_b[i]);
      if (p.dual_b) tma_prefetch_desc(&p.tma_b2[i]);
    }
  }
  if (warp == 1) tmem_alloc(&tmem_base, kCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      const int a_row = tile_m + (int)p.a_off.at(z);
      const int b_row = (p.dual_b ? tile_n / 2 : tile_n) + (int)p.b_off.at(z);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (uint32_t)(kb / S) & 1u;
        if (!mbar_wait(&empty_bar[s], ph ^ 1u, p.err, 1)) break;
        uint8_t* st = smem + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(&full_bar[s], stage_bytes);
        for (int i = 0; i < p.na; ++i)
          tma_load_2d(st + i * kTileA, &p.tma_a[i], &full_bar[s], (kb0 + kb) * BK, a_row);
        for (int j = 0; j < p.nb; ++j) {
          uint8_t* bt = st + p.na * kTileA + j * kTileB;
          if (p.dual_b) {
            tma_load_2d(bt, &p.tma_b[j], &full_bar[s], (kb0 + kb) * BK, b_row);
            tma_load_2d(bt + kTileB / 2, &p.tma_b2[j], &full_bar[s], (kb0 + kb) * BK, b_row);
          } else {
            tma_load_2d(bt, &p.tma_b[j], &full_bar[s], (kb0 + kb) * BK, b_row);
          }
        }
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
    const int ew = warp - 2;
    const int q = warp & 3;
    const int h = ew >> 2;
    const int r_loc = q * 32 + lane;
    const int row = tile_m + r_loc;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float acc[kAcc];
#pragma unroll
    for (int t = 0; t < kAcc; ++t) acc[t] = 0.f;
    bool ok = true;
    for (int c = 0; c < n_chunks; ++c) {
      const int b = c & 1;
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&accf_bar[b], (uint32_t)(c >> 1) & 1u,
                                                   p.err, 3));
      if (!ok) break;
      fence_after_sync();
#pragma unroll
      for (int jc = 0; jc < kNC; ++jc) {
        const uint32_t col = (uint32_t)(64 * jc + 32 * h);
        const uint32_t big = tmem + lane_off + (uint32_t)(b * 2 * BN) + col;
        uint32_t v[32], w[32];
        tmem_ld32_nowait(big, v);
        if (has_small) tmem_ld32_nowait(big + BN, w);
        tmem_wait_ld();
        if (has_small) {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            acc[32 * jc + t] = __fadd_rn(acc[32 * jc + t],
                                         __fadd_rn(__uint_as_float(v[t]), __uint_as_float(w[t])));
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            acc[32 * jc + t] = __fadd_rn(acc[32 * jc + t], __uint_as_float(v[t]));
        }
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[b]);
    }
    // ---------------------------------------------------------------- outputs ---
    // (the pipeline stages are idle: every MMA and every TMA load has completed)
    const bool live = ok && row < p.M;
    const int64_t coff = p.c_off.at(z);
    double sq = 0.0;
    // column of accumulator slot t: n_of(t) = tile_n + 64 (t / 32) + 32 h + t % 32
#pragma unroll
    for (int t = 0; t < kAcc; ++t) acc[t] = __fmul_rn(p.alpha, acc[t]);
    if (EPI == EPI_PLAIN || EPI == EPI_RESID || EPI == EPI_BF16) {
#pragma unroll
      for (int jc = 0; jc < kNC; ++jc) {
        const int n0 = tile_n + 64 * jc + 32 * h;
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int n = n0 + t;
          float x = acc[32 * jc + t];
          if (EPI == EPI_BF16) {
            x = bf16r(x);
            if (p.bias && n < p.N) x = bf16r(__fadd_rn(x, p.bias[n]));
            if (p.resid && live && n < p.N)
              x = bf16r(__fadd_rn(__bfloat162float(p.resid[coff + (int64_t)row * p.ld_rt + n]), x));
            acc[32 * jc + t] = x;
            continue;
          }
          if (p.bias && n < p.N) x = __fadd_rn(x, p.bias[n]);
          if (EPI == EPI_RESID && live && n < p.N) {
            const int64_t o = coff + (int64_t)row * p.ld_rt + n;
            if (p.resid) x = __fadd_rn(x, __bfloat162float(p.resid[o]));
            x = __fsub_rn(x, __bfloat162float(p.target[o]));
            if (p.row_period > 0 && (row % p.row_period) == 0) x = 0.f;
            sq += (double)x * (double)x;
            x = __fmul_rn(p.out_scale, x);
          }
          acc[32 * jc + t] = x;
        }
        if (live && p.C) {
          float* crow = p.C + coff + (int64_t)row * p.ldc + n0;
          if (p.c_vec && n0 + 32 <= p.N) {
#pragma unroll
            for (int t = 0; t < 32; t += 4) {
              float4 x = make_float4(acc[32 * jc + t], acc[32 * jc + t + 1], acc[32 * jc + t + 2],
                                     acc[32 * jc + t + 3]);
              if (EPI == EPI_PLAIN && p.beta != 0.f) {
                const float4 o = *reinterpret_cast<const float4*>(crow + t);
                x.x = __fadd_rn(x.x, __fmul_rn(p.beta, o.x));
                x.y = __fadd_rn(x.y, __fmul_rn(p.beta, o.y));
                x.z = __fadd_rn(x.z, __fmul_rn(p.beta, o.z));
                x.w = __fadd_rn(x.w, __fmul_rn(p.beta, o.w));
                acc[32 * jc + t] = x.x; acc[32 * jc + t + 1] = x.y;
                acc[32 * jc + t + 2] = x.z; acc[32 * jc + t + 3] = x.w;
              }
              *reinterpret_cast<float4*>(crow + t) = x;
            }
          } else {
#pragma unroll
            for (int t = 0; t < 32; ++t) {
              if (n0 + t < p.N) {
                float x = acc[32 * jc + t];
                if (EPI == EPI_PLAIN && p.beta != 0.f) {
                  x = __fadd_rn(x, __fmul_rn(p.beta, crow[t]));
                  acc[32 * jc + t] = x;
                }
                crow[t] = x;
              }
            }
          }
        }
        if (EPI == EPI_PLAIN && live && p.sq_partial) {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (n0 + t < p.N) sq += (double)acc[32 * jc + t] * (double)acc[32 * jc + t];
        }
      }
    } else if (EPI == EPI_SWIGLU_BF16) {
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const float g = bf16r(acc[t]), u = bf16r(acc[32 + t]);
        acc[t] = bf16r(__fmul_rn(bf16r(__fmul_rn(g, bf16r(sigmoid_f(g)))), u));
      }
    } else if (EPI == EPI_SWIGLU_FWD) {
      // slots [0, 32): gate of column j = tile_n / 2 + 32 h + t; slots [32, 64): up of the same j
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const int j = tile_n / 2 + 32 * h + t;
        const float g = acc[t], u = acc[32 + t];
        if (live && j < p.N / 2) {
          const int64_t o = coff + (int64_t)row * p.ld_aux + j;
          p.aux0[o] = g;
          p.aux1[o] = u;
        }
        acc[t] = __fmul_rn(__fmul_rn(g, sigmoid_f(g)), u);  // silu(g) * u
      }
    } else {  // EPI_SWIGLU_BWD: slots hold dd = dL/d(silu(g) u) of column n
#pragma unroll
      for (int jc = 0; jc < kNC; ++jc) {
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int n = tile_n + 64 * jc + 32 * h + t;
          float dg = 0.f, du = 0.f;
          if (live && n < p.N) {
            const int64_t o = coff + (int64_t)row * p.ld_aux + n;
            const float g = p.aux0[o], u = p.aux1[o];
            const float sg = sigmoid_f(g);
            const float dd = acc[32 * jc + t];
            du = __fmul_rn(dd, __fmul_rn(g, sg));
            // d(g sigmoid(g))/dg = sigmoid(g) + g sigmoid(g) (1 - sigmoid(g))
            const float dsil = __fadd_rn(sg, __fmul_rn(g, __fmul_rn(sg, __fsub_rn(1.0f, sg))));
            dg = __fmul_rn(__fmul_rn(dd, u), dsil);
          }
          acc[32 * jc + t] = dg;
          // du is staged right away below (transposed); keep dg in acc
          if (p.nct > 0) {
            __nv_bfloat16 hv[3];
            split3_bf16(du, hv[0], hv[1], hv[2]);
            __nv_bfloat16* T = reinterpret_cast<__nv_bfloat16*>(smem);
            const int n_loc = 64 * jc + 32 * h + t;
            for (int i = 0; i < p.nct; ++i)
              T[((p.nct + i) * BN + n_loc) * BM + r_loc] = live ? hv[i] : __float2bfloat16_rn(0.f);
          }
        }
      }
    }
    // ---- bf16 term outputs
    const int n_out_cols = EPI == EPI_SWIGLU_FWD ? 32 * kNC / 2 : 0;  // (unused marker)
    (void)n_out_cols;
    constexpr bool kHalfOut = (EPI == EPI_SWIGLU_FWD || EPI == EPI_SWIGLU_BF16);
    if (EPI != EPI_SWIGLU_BWD) {
      if (live && p.ncs > 0) {
        const int nch = kHalfOut ? 1 : kNC;
        for (int jc = 0; jc < nch; ++jc) {
          const int n0 = kHalfOut ? tile_n / 2 + 32 * h : tile_n + 64 * jc + 32 * h;
          const int n_lim = kHalfOut ? p.N / 2 : p.N;
#pragma unroll
          for (int t = 0; t < 32; t += 8) {
            if (n0 + t >= n_lim) break;
            __align__(16) __nv_bfloat16 hv[3][8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              split3_bf16(acc[32 * jc + t + u], hv[0][u], hv[1][u], hv[2][u]);
            for (int i = 0; i < p.ncs; ++i)
              *reinterpret_cast<uint4*>(p.cs[i] + coff + (int64_t)row * p.ldcs + n0 + t) =
                  *reinterpret_cast<const uint4*>(hv[i]);
          }
        }
      }
    }
    if (p.nct > 0) {
      // transposed terms: stage [plane][term][n_loc][m_loc] bf16 in shared memory, then 16-byte
      // coalesced row stores of C^T (plane 1: the up-gradient rows of the SwiGLU backward)
      __nv_bfloat16* T = reinterpret_cast<__nv_bfloat16*>(smem);
      const int rows_t = kHalfOut ? BN / 2 : BN;
      const int planes = EPI == EPI_SWIGLU_BWD ? 2 : 1;
      if (kHalfOut) {
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          __nv_bfloat16 hv[3];
          split3_bf16(live ? acc[t] : 0.f, hv[0], hv[1], hv[2]);
          const int n_loc = 32 * h + t;
          for (int i = 0; i < p.nct; ++i) T[(i * rows_t + n_loc) * BM + r_loc] = hv[i];
        }
      } else {
#pragma unroll
        for (int jc = 0; jc < kNC; ++jc) {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            __nv_bfloat16 hv[3];
            split3_bf16(live ? acc[32 * jc + t] : 0.f, hv[0], hv[1], hv[2]);
            const int n_loc = 64 * jc + 32 * h + t;
            for (int i = 0; i < p.nct; ++i) T[(i * rows_t + n_loc) * BM + r_loc] = hv[i];
          }
        }
      }
      epi_sync();
      const int tid = threadIdx.x - 64;
      const int n_first = kHalfOut ? tile_n / 2 : tile_n;
      const int n_lim = kHalfOut ? p.N / 2 : p.N;
      const int64_t r_base = p.t_row.at(z), c_base = p.t_col.at(z);
      const int per_plane = p.nct * rows_t * (BM / 8);
      for (int e = tid; e < planes * per_plane; e += 32 * kEpiWarps) {
        const int pl = e / per_plane;
        const int rem0 = e - pl * per_plane;
        const int i = rem0 / (rows_t * (BM / 8));
        const int rem = rem0 - i * (rows_t * (BM / 8));
        const int n_loc = rem / (BM / 8), m8 = (rem % (BM / 8)) * 8;
        const int n = n_first + n_loc, m = tile_m + m8;
        if (n < n_lim && m < p.M && ok)
          *reinterpret_cast<uint4*>(p.ct[i] + (r_base + n + (pl ? p.ct_up_rows : 0)) * p.ldct +
                                    c_base + m) =
              *reinterpret_cast<const uint4*>(T + ((pl * p.nct + i) * rows_t + n_loc) * BM + m8);
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
    p.sq_partial[((int64_t)z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x] = t;
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
static bool make_map(CUtensorMap* m, const void* base, int64_t rows, int cols, int64_t ld,
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

template <int BN, int EPI>
static int launch(GemmParams& p, int batch, cudaStream_t st) {
  const uint32_t stage_bytes = p.na * BM * BK * 2 + p.nb * BN * BK * 2;
  int S = (int)(kSmemBudget / stage_bytes);
  if (S > 8) S = 8;
  if (S < 2) return GSQ_ENOTSUP;
  p.stages = S;
  // the transposed-term staging reuses the pipeline stages
  const int rows_t = (EPI == EPI_SWIGLU_FWD || EPI == EPI_SWIGLU_BF16) ? BN / 2 : BN;
  const size_t stage_need = (size_t)(EPI == EPI_SWIGLU_BWD ? 2 : 1) * p.nct * rows_t * BM * 2;
  if (stage_need > (size_t)S * stage_bytes) return GSQ_ENOTSUP;
  int products = 0;
  for (int i = 0; i < p.na; ++i)
    for (int j = 0; j < p.nb; ++j) products += (i + j <= p.order);
  p.kb_per_chunk = products >= 3 ? 1 : (products == 2 ? 2 : 4);
  const size_t smem = (size_t)S * stage_bytes + 1024;
  static bool attr_set[2][6] = {{false}};
  bool& done = attr_set[BN == 128][EPI];
  if (!done) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBudget + 1024) != cudaSuccess)
      return GSQ_ECUDA;
    done = true;
  }
  dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, batch);
  gemm_tc_kernel<BN, EPI><<<grid, kThreads, smem, st>>>(p);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

}  // namespace tc
}  // namespace gsq

using namespace gsq;

static tc::Aff to_aff(int div, int64_t s1, int64_t s2) {
  tc::Aff a;
  a.div = div > 0 ? div : 1;
  a.s1 = s1;
  a.s2 = s2;
  return a;
}

extern "C" int gsq_gemm(const gsq_gemm_desc* d, void* stream) {
  if (!d) return GSQ_EINVAL;
  const int M = d->M, N = d->N, K = d->K;
  if (M <= 0 || N <= 0 || K <= 0 || d->batch < 1 || d->batch > 65535 || d->na < 1 ||
      d->na > 3 || d->nb < 1 || d->nb > 3 || d->order < 0 || !d->err || d->ncs < 0 ||
      d->ncs > 3 || d->nct < 0 || d->nct > 3 || d->epi < 0 || d->epi > 5)
    return GSQ_EINVAL;
  if (d->bn != 64 && d->bn != 128) return GSQ_EINVAL;
  const int epi = d->epi;
  if (!d->C && d->ncs == 0 && d->nct == 0 && !d->sq_partial) return GSQ_EINVAL;
  if (d->lda < K || d->ldb < K || (d->C && d->ldc < ((epi == 2 || epi == 5) ? N / 2 : N)))
    return GSQ_EINVAL;
  if (d->ncs > 0 && (d->ldcs & 7)) return GSQ_EINVAL;
  if (d->nct > 0 && (d->ldct & 7)) return GSQ_EINVAL;
  for (int i = 0; i < d->ncs; ++i)
    if (!d->cs[i] || ((uintptr_t)d->cs[i] & 15)) return GSQ_EINVAL;
  for (int i = 0; i < d->nct; ++i)
    if (!d->ct[i] || ((uintptr_t)d->ct[i] & 15)) return GSQ_EINVAL;
  if (epi == 1 && !d->target) return GSQ_EINVAL;
  if ((epi == 2 || epi == 3) && (!d->aux0 || !d->aux1 || d->bn != 128)) return GSQ_EINVAL;
  if ((epi == 2 || epi == 5) && (!d->b2[0] || (N % 128) != 0 || d->bn != 128)) return GSQ_EINVAL;
  if (d->causal < 0 || d->causal > 2 || (d->causal && d->K < M)) return GSQ_EINVAL;
  tc::GemmParams p;
  memset(&p, 0, sizeof(p));
  const int BN = d->bn;
  const bool dual = (epi == 2 || epi == 5);
  const int b_box = dual ? BN / 2 : BN;
  for (int i = 0; i < d->na; ++i)
    if (!tc::make_map(&p.tma_a[i], d->a[i], d->a_rows, K, d->lda, tc::BM)) return GSQ_EINVAL;
  for (int j = 0; j < d->nb; ++j) {
    if (!tc::make_map(&p.tma_b[j], d->b[j], d->b_rows, K, d->ldb, b_box)) return GSQ_EINVAL;
    if (dual && !tc::make_map(&p.tma_b2[j], d->b2[j], d->b_rows, K, d->ldb, b_box))
      return GSQ_EINVAL;
  }
  p.M = M; p.N = N; p.K = K;
  p.na = d->na; p.nb = d->nb; p.order = d->order; p.causal = d->causal;
  p.dual_b = dual;
  p.skip_upper = d->skip_upper;
  p.row_period = d->row_period;
  p.alpha = d->alpha; p.beta = d->beta;
  p.C = d->C; p.ldc = d->ldc;
  p.c_vec = (d->C && ((uintptr_t)d->C & 15) == 0 && (d->ldc & 3) == 0 &&
             ((d->c_s1 | d->c_s2) & 3) == 0) ? 1 : 0;
  for (int i = 0; i < d->ncs; ++i) p.cs[i] = (__nv_bfloat16*)d->cs[i];
  p.ncs = d->ncs; p.ldcs = d->ldcs;
  for (int i = 0; i < d->nct; ++i) p.ct[i] = (__nv_bfloat16*)d->ct[i];
  p.nct = d->nct; p.ldct = d->ldct; p.ct_up_rows = d->ct_up_rows;
  p.sq_partial = d->sq_partial;
  p.bias = d->bias;
  p.resid = (const __nv_bfloat16*)d->resid;
  p.target = (const __nv_bfloat16*)d->target;
  p.ld_rt = d->ld_rt;
  p.out_scale = d->out_scale;
  p.aux0 = d->aux0; p.aux1 = d->aux1; p.ld_aux = d->ld_aux;
  p.a_off = to_aff(d->a_div, d->a_s1, d->a_s2);
  p.b_off = to_aff(d->b_div, d->b_s1, d->b_s2);
  p.c_off = to_aff(d->c_div, d->c_s1, d->c_s2);
  p.t_row = to_aff(d->t_div, d->t_r1, d->t_r2);
  p.t_col = to_aff(d->t_div, d->t_c1, d->t_c2);
  p.err = d->err;
  cudaStream_t st = (cudaStream_t)stream;
  if (BN == 64) {
    if (epi == 0) return tc::launch<64, 0>(p, d->batch, st);
    if (epi == 1) return tc::launch<64, 1>(p, d->batch, st);
    if (epi == 4) return tc::launch<64, 4>(p, d->batch, st);
    return GSQ_EINVAL;
  }
  switch (epi) {
    case 0: return tc::launch<128, 0>(p, d->batch, st);
    case 1: return tc::launch<128, 1>(p, d->batch, st);
    case 2: return tc::launch<128, 2>(p, d->batch, st);
    case 3: return tc::launch<128, 3>(p, d->batch, st);
    case 4: return tc::launch<128, 4>(p, d->batch, st);
    default: return tc::launch<128, 5>(p, d->batch, st);
  }
}

// The single-GEMM form (no batching, plain epilogue).
extern "C" int gsq_gemm_tc(int M, int N, int K, const void* const* a_terms, int na, int64_t lda,
                           const void* const* b_terms, int nb, int64_t ldb, int order,
                           float alpha, float* C, int64_t ldc, float beta, void* const* c_terms,
                           int ncs, int64_t ldcs, void* const* ct_terms, int nct, int64_t ldct,
                           double* sq_partial, int* err, void* stream) {
  if (!a_terms || !b_terms || na < 1 || na > 3 || nb < 1 || nb > 3 || ncs < 0 || ncs > 3 ||
      nct < 0 || nct > 3 || (ncs > 0 && !c_terms) || (nct > 0 && !ct_terms))
    return GSQ_EINVAL;
  if ((nct > 0 && ldct < ((M + 7) / 8) * 8) || (ncs > 0 && ldcs < N)) return GSQ_EINVAL;
  gsq_gemm_desc d;
  memset(&d, 0, sizeof(d));
  d.M = M; d.N = N; d.K = K; d.batch = 1;
  for (int i = 0; i < na; ++i) d.a[i] = a_terms[i];
  d.na = na; d.lda = lda; d.a_rows = M;
  for (int j = 0; j < nb; ++j) d.b[j] = b_terms[j];
  d.nb = nb; d.ldb = ldb; d.b_rows = N;
  d.order = order; d.alpha = alpha; d.beta = beta;
  d.C = C; d.ldc = ldc;
  for (int i = 0; i < ncs; ++i) d.cs[i] = c_terms[i];
  d.ncs = ncs; d.ldcs = ldcs;
  for (int i = 0; i < nct; ++i) d.ct[i] = ct_terms[i];
  d.nct = nct; d.ldct = ldct;
  d.sq_partial = sq_partial; d.err = err; d.bn = 128;
  return gsq_gemm(&d, stream);
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
