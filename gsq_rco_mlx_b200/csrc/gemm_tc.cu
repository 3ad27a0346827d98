// Float32-faithful GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulator).
//
//   C[m, n] = alpha * sum_k A(m, k) B(n, k)        A, B given as 1..3 bf16 terms each,
//                                                   A = sum_i A_i, B = sum_j B_j (K-major)
// The products A_i B_j with i + j <= order are accumulated on the tensor cores (order 2 with
// three terms per side reproduces float32 operands to 2^-24; an exactly-bf16 operand needs one
// term). Persistent kernel: one CTA per SM walks the 128 x BN output tiles (batch z, row tile m,
// column tile n) in a static round-robin order. Within a batch the tile index runs along the
// dimension of the smaller operand first (m fastest when B is the larger operand, n fastest
// when A is): the CTAs that run at the same time then share the tiles of the larger operand,
// so it crosses from DRAM once while the smaller one stays in L2. Roles:
//   warp 0     TMA producer: for each 64-wide k-block, every term tile of A and B into one
//              pipeline stage (128-byte swizzle), completion counted on the stage's mbarrier
//   warp 1     TMEM allocator and MMA issuer
//   warps 2-9  epilogue: fold the accumulators into float32 registers, then the fused outputs
// Tensor-core accumulation into TMEM is not IEEE round-to-nearest. The hi x hi products ("big")
// therefore go to a ring of chunk accumulators that the epilogue folds into registers with IEEE
// adds after every chunk of k-blocks; the other products ("small", 2^8 smaller and less) stay in
// one of two per-tile accumulators for the whole k-range. The ring lets the MMAs of the next tile
// run while the epilogue is still writing the outputs of this one.
// Outputs leave through a per-warp 32 x 32 shared-memory transpose: row-major outputs as
// coalesced row segments, transposed outputs (C^T as bf16 terms: the K-major operand of a later
// reduction over m) as coalesced column segments.
// Every mbarrier wait is bounded; a timeout sets *err and every role winds down without further
// waits on its partners, the MMA issuer waits (bounded) for its last MMAs and the producer for
// its copies in flight, and the CTA frees its TMEM.
#include <new>

#include "tc_common.cuh"

namespace gsq {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStgLd = 33;                                   // staging row stride (floats)
constexpr uint32_t kStgBytes = kEpiWarps * 32 * kStgLd * 4;  // one 32 x 32 tile per warp
constexpr uint32_t kTmaBuf = 4096;                           // one TMA-store staging buffer
constexpr uint32_t kSmemMax = 232448 - 1024;  // dynamic opt-in: 227 KB less the static 1 KB
constexpr uint32_t kPipeBudget = 192 * 1024;                 // pipeline stages
constexpr int kMaxStages = 8;
constexpr int kMaxBig = 8;
constexpr uint32_t kTmemCols = 512;

enum Epi {
  EPI_PLAIN = 0,
  EPI_RESID = 1,
  EPI_SWIGLU_FWD = 2,
  EPI_SWIGLU_BWD = 3,
  EPI_BF16 = 4,        // bf16 chain: x = bf16(acc); x = bf16(x + bias); x = bf16(resid + x)
  EPI_SWIGLU_BF16 = 5,  // bf16 SwiGLU: g, u = bf16(acc); bf16(bf16(g bf16(sigmoid(g))) u)
  EPI_SWIGLU_BWD_BF16 = 6  // its backward with bf16 cotangents (dd = bf16(acc), g, u from aux)
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
  int n_big;       // chunk accumulators in the TMEM ring
  int tiles_m, tiles_n;
  int n_fast;  // tile order: n fastest (A the larger operand) instead of m fastest
  int causal_order;  // causal products: longest k-ranges first, in a snake over the CTAs
  int small_bufs;    // 1 or 2 TMEM accumulators for a tile's cross products (see launch)
  int64_t total_tiles;
  int skip_upper;  // output tiles entirely above the diagonal (n >= m) are not computed
  int row_period;  // epi 1: rows with (row % row_period) == 0 have a zero residual
  // two-element (8-byte float / 4-byte bf16) accesses are aligned for these outputs
  int pair_c, pair_cs, pair_ct, pair_aux, pair_rt;
  int splits, kb_split;  // split-K: parts of kb_split k-blocks, partials into ws [part][M][N]
  float* ws;
  // row-major outputs through TMA stores (EPI_PLAIN / EPI_BF16 without transposed outputs):
  // C float32 or the cs bf16 terms as 32 x 32 boxes, 3-D (x, y, batch) or 4-D (x, y, z % div,
  // z / div) maps
  CUtensorMap tma_c;
  CUtensorMap tma_cs[3];
  CUtensorMap tma_ct[3];   // C^T terms, 3-D (x = row, y = output column, batch)
  CUtensorMap tma_aux[2];  // SwiGLU g / u rows
  int tma_out, out_rank, tma_bufs;  // tma_bufs: 4 KB staging buffers per epilogue warp (1..3)
  int tma_bf16_only;                  // every box is bf16 (2 KB): no C / aux float32 boxes
  int a_mn, b_mn;  // MN-major operands: 64 x 64 boxes (MN inner) at +8 KB per 64 MN indices
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

struct TileInfo {
  int z, ks, tile_m, tile_n, kb0, nkb;
  int64_t part;  // index of the tile's sum-of-squares partial
};

// Tile L of the round-robin order; false for a tile that skip_upper leaves out. The k-block
// range: causal 1 = lower-triangular A (k < end of this row tile), causal 2 = upper-triangular A
// (k >= start of this row tile).
// Causal products (causal_order): the tiles of a row level (one row tile of every batch and
// column tile) have the same k-range, so the order takes the levels from the longest k-range
// to the shortest, and the CTAs walk the rounds of gridDim.x tiles alternately forwards and
// backwards (a snake): a CTA that took a long tile in one round takes a short one in the next,
// which bounds the causal tail (static round-robin otherwise leaves some CTAs 40 % above the
// mean at the attention products' 16 row tiles).
template <int BN>
__device__ __forceinline__ bool tile_at(const GemmParams& p, int64_t L, TileInfo& t) {
  int my, nx;
  if (p.causal_order) {
    const int64_t G = gridDim.x;
    const int64_t r = L / G, pos = L - r * G;
    const int64_t c = min(G, p.total_tiles - r * G);
    const int64_t idx = r * G + ((r & 1) ? c - 1 - pos : pos);
    const int64_t width = p.total_tiles / p.tiles_m;  // batch x tiles_n tiles per level
    const int level = (int)(idx / width);
    const int64_t rem = idx - (int64_t)level * width;
    t.z = (int)(rem / p.tiles_n);
    t.ks = 0;
    nx = (int)(rem - (int64_t)t.z * p.tiles_n);
    my = p.causal == 1 ? p.tiles_m - 1 - level : level;
  } else {
    const int64_t per = (int64_t)p.tiles_m * p.tiles_n;
    const int64_t zk = L / per;
    t.z = (int)(zk / p.splits);
    t.ks = (int)(zk - (int64_t)t.z * p.splits);
    const int rem = (int)(L - zk * per);
    my = p.n_fast ? rem / p.tiles_n : rem % p.tiles_m;
    nx = p.n_fast ? rem % p.tiles_n : rem / p.tiles_m;
  }
  t.tile_m = my * BM;
  t.tile_n = nx * BN;
  if (p.skip_upper && t.tile_n >= t.tile_m + BM) return false;
  const int kb_total = (p.K + BK - 1) / BK;
  t.kb0 = p.causal == 2 ? min(t.tile_m / BK, kb_total - 1) : 0;
  const int kb1 = p.causal == 1 ? min(kb_total, (t.tile_m + BM + BK - 1) / BK) : kb_total;
  t.nkb = kb1 - t.kb0;
  if (p.splits > 1) {
    t.kb0 += t.ks * p.kb_split;
    t.nkb = min(p.kb_split, t.nkb - t.ks * p.kb_split);
  }
  t.part = ((int64_t)t.z * p.tiles_m + my) * p.tiles_n + nx;
  return true;
}

// ------------------------------------------------------------- epilogue helpers ---

// This lane's row of 32 values into row `lane` of the warp's staging tile.
__device__ __forceinline__ void stage_put(float* stg, int lane, const float* v) {
#pragma unroll
  for (int t = 0; t < 32; ++t) stg[lane * kStgLd + t] = v[t];
  __syncwarp();
}

__device__ __forceinline__ void load_bf2(const __nv_bfloat16* ptr, bool two, bool pair, float& a,
                                         float& b) {
  if (two && pair) {
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(ptr);
    a = __low2float(v);
    b = __high2float(v);
  } else {
    a = __bfloat162float(ptr[0]);
    b = two ? __bfloat162float(ptr[1]) : 0.f;
  }
}

__device__ __forceinline__ void load_f2(const float* ptr, bool two, bool pair, float& a,
                                        float& b) {
  if (two && pair) {
    const float2 v = *reinterpret_cast<const float2*>(ptr);
    a = v.x;
    b = v.y;
  } else {
    a = ptr[0];
    b = two ? ptr[1] : 0.f;
  }
}

__device__ __forceinline__ void store_f2(float* ptr, float a, float b, bool two, bool pair) {
  if (two && pair) {
    *reinterpret_cast<float2*>(ptr) = make_float2(a, b);
  } else {
    ptr[0] = a;
    if (two) ptr[1] = b;
  }
}

// x0, x1 (consecutive elements) as n_terms bf16 terms at terms[i] + off
__device__ __forceinline__ void store_terms2(__nv_bfloat16* const* terms, int n_terms, int64_t off,
                                             float x0, float x1, bool two, bool pair) {
  __nv_bfloat16 h0[3], h1[3];
  split3_bf16(x0, h0[0], h0[1], h0[2]);
  split3_bf16(x1, h1[0], h1[1], h1[2]);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (i < n_terms) {
      __nv_bfloat16* ptr = terms[i] + off;
      if (two && pair) {
        *reinterpret_cast<__nv_bfloat162*>(ptr) = __halves2bfloat162(h0[i], h1[i]);
      } else {
        ptr[0] = h0[i];
        if (two) ptr[1] = h1[i];
      }
    }
  }
}

// Columns c of the staging tile (rows m of the output band) as rows n0 + c of C^T:
// ct[i][(r_base + up + n0 + c) * ldct + c_base + row0 + m], n0 + c < n_lim, row0 + m < M.
__device__ __forceinline__ void transposed_pass(const GemmParams& p, const TileInfo& t,
                                                const float* stg, int lane, int n0, int n_lim,
                                                int row0, int64_t up) {
  const int64_t r_base = p.t_row.at(t.z) + up, c_base = p.t_col.at(t.z);
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    const int c = 2 * i + (lane >> 4), m = 2 * (lane & 15);
    const int n = n0 + c, row = row0 + m;
    if (n < n_lim && row < p.M) {
      const float x0 = stg[m * kStgLd + c], x1 = stg[(m + 1) * kStgLd + c];
      store_terms2(p.ct, p.nct, (r_base + n) * p.ldct + c_base + row, x0, x1, row + 1 < p.M,
                   p.pair_ct != 0);
    }
  }
}

// ----------------------------------------------------------------- TMA box epilogue ---
// The outputs of one tile as 32 x 32 boxes written by the TMA unit (tma_out). Epilogue warp
// (q, h) holds, per 32-column group, rows row0 + lane (lane = row) and 32 consecutive columns in
// registers; a box is staged in the warp's ring of 4 KB buffers in the store's swizzled layout
// and stored by one lane, one bulk group per buffer. Row-major float32 boxes (128-byte rows:
// 16-byte chunk c of row r at c ^ (r % 8)), row-major bf16 boxes (64-byte rows: chunk c at
// c ^ ((r / 2) % 4)) and transposed bf16 boxes (box row = output column) are all written without
// shared-memory bank conflicts. The TMA unit clips rows and columns outside the output.
struct BoxRing {
  uint8_t* base;
  int nbuf, bsize, cur, used;  // nbuf buffers of bsize bytes (4096, or 2048 for bf16 boxes only)
};

__device__ __forceinline__ void ring_wait(int nbuf) {
  if (nbuf >= 3) bulk_wait_read<2>();
  else if (nbuf == 2) bulk_wait_read<1>();
  else bulk_wait_read<0>();
}

// Room for a box of `bytes` (2048 or 4096): a full buffer is committed, and a fresh buffer is
// used only once the group that last read it is done.
__device__ __forceinline__ uint8_t* ring_slot(BoxRing& r, int bytes, int lane) {
  if (r.used + bytes > r.bsize) {
    if (lane == 0) bulk_commit();
    r.cur = r.cur + 1 == r.nbuf ? 0 : r.cur + 1;
    r.used = 0;
  }
  if (r.used == 0) {
    if (lane == 0) ring_wait(r.nbuf);
    __syncwarp();
  }
  uint8_t* b = r.base + r.cur * r.bsize + r.used;
  r.used += bytes;
  return b;
}

__device__ __forceinline__ void ring_flush(BoxRing& r, int lane) {
  if (r.used) {
    if (lane == 0) bulk_commit();
    r.cur = r.cur + 1 == r.nbuf ? 0 : r.cur + 1;
    r.used = 0;
  }
}

// The terms of x = t0 + t1 + t2 (to float32 precision) are peeled one at a time: the next term
// is bf16(v) and v keeps the exact remainder v - t (split3_bf16 step by step). `last` skips the
// remainder after the final term.
__device__ __forceinline__ uint32_t peel2(float& v0, float& v1, bool last) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
  if (!last) {
    const float2 f = __bfloat1622float2(h);
    v0 = __fsub_rn(v0, f.x);
    v1 = __fsub_rn(v1, f.y);
  }
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ __nv_bfloat16 peel1(float& v, bool last) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  if (!last) v = __fsub_rn(v, __bfloat162float(h));
  return h;
}

__device__ __forceinline__ void box_put_f32(uint8_t* buf, int lane, const float* v) {
  float* f = reinterpret_cast<float*>(buf) + lane * 32;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<float4*>(f + ((c ^ (lane & 7)) << 2)) =
        make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// the next bf16 term of v (peeled in place)
__device__ __forceinline__ void box_put_bf16(uint8_t* buf, int lane, float* v, bool last) {
  uint8_t* row = buf + lane * 64;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 o;
    o.x = peel2(v[8 * c], v[8 * c + 1], last);
    o.y = peel2(v[8 * c + 2], v[8 * c + 3], last);
    o.z = peel2(v[8 * c + 4], v[8 * c + 5], last);
    o.w = peel2(v[8 * c + 6], v[8 * c + 7], last);
    *reinterpret_cast<uint4*>(row + ((c ^ ((lane >> 1) & 3)) << 4)) = o;
  }
}

// bf16 term `term` of v, v unchanged (the earlier terms are peeled from a copy of each chunk)
__device__ __forceinline__ void box_put_bf16_keep(uint8_t* buf, int lane, const float* v,
                                                  int term) {
  uint8_t* row = buf + lane * 64;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = v[8 * c + j];
    for (int k = 0; k < term; ++k) {
#pragma unroll
      for (int j = 0; j < 8; j += 2) peel2(r[j], r[j + 1], false);
    }
    uint4 o;
    o.x = peel2(r[0], r[1], true);
    o.y = peel2(r[2], r[3], true);
    o.z = peel2(r[4], r[5], true);
    o.w = peel2(r[6], r[7], true);
    *reinterpret_cast<uint4*>(row + ((c ^ ((lane >> 1) & 3)) << 4)) = o;
  }
}

// transposed: box row u (output column n0 + u), box column lane (output row row0 + lane)
__device__ __forceinline__ void box_put_bf16_t(uint8_t* buf, int lane, float* v, bool last) {
  const int c = lane >> 3, e = (lane & 7) * 2;
#pragma unroll
  for (int u = 0; u < 32; ++u)
    *reinterpret_cast<__nv_bfloat16*>(buf + u * 64 + ((c ^ ((u >> 1) & 3)) << 4) + e) =
        peel1(v[u], last);
}

__device__ __forceinline__ void box_store(const CUtensorMap* map, const uint8_t* buf, int rank,
                                          int x, int y, int zr, int zq, int lane) {
  fence_proxy_async_shared();
  __syncwarp();
  if (lane == 0) {
    if (rank == 3) tma_store_3d(map, buf, x, y, zq);
    else tma_store_4d(map, buf, x, y, zr, zq);
  }
}

// Row-major output (map of the C layout) of the values v of columns col0 .. col0 + 31
__device__ __forceinline__ void out_rows_f32(BoxRing& r, const GemmParams& p,
                                             const CUtensorMap* map, const float* v, int col0,
                                             int row0, int zr, int zq, int lane) {
  uint8_t* b = ring_slot(r, 4096, lane);
  box_put_f32(b, lane, v);
  if (row0 < p.M) box_store(map, b, p.out_rank, col0, row0, zr, zq, lane);
}

// Row-major bf16 terms of v (v is consumed: it holds the last remainder afterwards)
__device__ __forceinline__ void out_rows_terms(BoxRing& r, const GemmParams& p, float* v,
                                               int nterms, int col0, int row0, int zr, int zq,
                                               int lane) {
  for (int i = 0; i < nterms; ++i) {
    uint8_t* b = ring_slot(r, 2048, lane);
    box_put_bf16(b, lane, v, i + 1 == nterms);
    if (row0 < p.M) box_store(&p.tma_cs[i], b, p.out_rank, col0, row0, zr, zq, lane);
  }
}

// C^T terms: output rows up + col0 .. (of batch z), columns row0 .. (v is consumed)
__device__ __forceinline__ void out_cols_terms(BoxRing& r, const GemmParams& p, float* v,
                                               int col0, int up, int row0, int z, int lane) {
  for (int i = 0; i < p.nct; ++i) {
    uint8_t* b = ring_slot(r, 2048, lane);
    box_put_bf16_t(b, lane, v, i + 1 == p.nct);
    if (row0 < p.M) box_store(&p.tma_ct[i], b, 3, row0, up + col0, 0, z, lane);
  }
}

// Both term layouts of v: when the transposed terms follow, the row-major ones leave v as it is
// (a single term never changes it)
__device__ __forceinline__ void out_terms(BoxRing& r, const GemmParams& p, float* v, int nterms,
                                          int col0, int up, int row0, int zr, int zq, int z,
                                          int lane) {
  if (p.nct && nterms > 1) {
    for (int i = 0; i < nterms; ++i) {
      uint8_t* b = ring_slot(r, 2048, lane);
      box_put_bf16_keep(b, lane, v, i);
      if (row0 < p.M) box_store(&p.tma_cs[i], b, p.out_rank, col0 + up, row0, zr, zq, lane);
    }
  } else if (nterms) {
    out_rows_terms(r, p, v, nterms, col0 + up, row0, zr, zq, lane);
  }
  if (p.nct) out_cols_terms(r, p, v, col0, up, row0, z, lane);
}

// 8 consecutive values of a row segment (columns c .. c + 7 of 32): one 16-byte load where the
// segment is whole, else per element; 0 outside the output.
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* ptr, bool ok, int nvalid, int c,
                                          float* r) {
  if (ok && nvalid >= 32) {
    const uint4 raw = *reinterpret_cast<const uint4*>(ptr + c);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(b2[j]);
      r[2 * j] = f.x;
      r[2 * j + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = (ok && c + j < nvalid) ? __bfloat162float(ptr[c + j]) : 0.f;
  }
}

__device__ __forceinline__ void load8_f32(const float* ptr, bool ok, int nvalid, int c, float* r) {
  if (ok && nvalid >= 32) {
    const float4 f0 = *reinterpret_cast<const float4*>(ptr + c);
    const float4 f1 = *reinterpret_cast<const float4*>(ptr + c + 4);
    r[0] = f0.x; r[1] = f0.y; r[2] = f0.z; r[3] = f0.w;
    r[4] = f1.x; r[5] = f1.y; r[6] = f1.z; r[7] = f1.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = (ok && c + j < nvalid) ? ptr[c + j] : 0.f;
  }
}

// The row inputs that the epilogue of this warp's part of tile t reads (SwiGLU-backward g and u,
// residual and target rows), fetched into L2 while the tile's MMAs run: the epilogue's loads of
// one 32-column group then wait on L2 rather than on HBM. Only addresses inside the inputs.
template <int BN, int EPI>
__device__ __forceinline__ void prefetch_row_inputs(const GemmParams& p, const TileInfo& t,
                                                    int lane, int q, int h) {
  constexpr bool kBwd = EPI == EPI_SWIGLU_BWD || EPI == EPI_SWIGLU_BWD_BF16;
  if (!kBwd && EPI != EPI_RESID && EPI != EPI_BF16) return;
  const int row = t.tile_m + 32 * q + lane;
  if (row >= p.M) return;
  const int64_t coff = p.c_off.at(t.z);
#pragma unroll
  for (int jc = 0; jc < BN / 64; ++jc) {
    const int n0 = t.tile_n + 64 * jc + 32 * h;
    if (n0 >= p.N) break;
    const int last = min(31, p.N - 1 - n0);
    if (kBwd) {
      const float* gp = p.aux0 + coff + (int64_t)row * p.ld_aux + n0;
      const float* up = p.aux1 + coff + (int64_t)row * p.ld_aux + n0;
      prefetch_l2(gp);
      prefetch_l2(gp + last);
      prefetch_l2(up);
      prefetch_l2(up + last);
    } else {
      const int64_t off = coff + (int64_t)row * p.ld_rt + n0;
      if (p.resid) {
        prefetch_l2(p.resid + off);
        prefetch_l2(p.resid + off + last);
      }
      if (EPI == EPI_RESID) {
        prefetch_l2(p.target + off);
        prefetch_l2(p.target + off + last);
      }
    }
  }
}

// bias[n0 + c .. n0 + c + 7] (0 at columns >= n0 + nvalid); one float4 pair when the 32
// columns are all inside and the bias is 16-byte aligned
__device__ __forceinline__ void load8_bias(const float* bias, int n0, int nvalid, int c,
                                           float* r) {
  if (nvalid >= 32 && ((uintptr_t)bias & 15) == 0) {
    const float4 f0 = *reinterpret_cast<const float4*>(bias + n0 + c);
    const float4 f1 = *reinterpret_cast<const float4*>(bias + n0 + c + 4);
    r[0] = f0.x; r[1] = f0.y; r[2] = f0.z; r[3] = f0.w;
    r[4] = f1.x; r[5] = f1.y; r[6] = f1.z; r[7] = f1.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = c + j < nvalid ? bias[n0 + c + j] : 0.f;
  }
}

template <int BN, int EPI>
__device__ __forceinline__ double epilogue_tma(const GemmParams& p, const TileInfo& t, float* acc,
                                               BoxRing& ring, int lane, int q, int h) {
  constexpr int kNC = BN / 64;
  constexpr bool kDual = EPI == EPI_SWIGLU_FWD || EPI == EPI_SWIGLU_BF16;
  const int row0 = t.tile_m + 32 * q, row = row0 + lane;
  const bool row_ok = row < p.M;
  const int zr = t.z % p.c_off.div, zq = t.z / p.c_off.div;
  const int64_t coff = p.c_off.at(t.z);
  double sq = 0.0;
#pragma unroll
  for (int i = 0; i < BN / 2; ++i) acc[i] = __fmul_rn(p.alpha, acc[i]);
  constexpr int kGroups = kDual ? 1 : kNC;
  const int nlim = kDual ? p.N / 2 : p.N;
#pragma unroll
  for (int jc = 0; jc < kGroups; ++jc) {
    const int n0 = kDual ? t.tile_n / 2 + 32 * h : t.tile_n + 64 * jc + 32 * h;
    if (n0 >= nlim) continue;
    const int nvalid = nlim - n0;
    float* a = acc + 32 * jc;
    if (EPI == EPI_SWIGLU_FWD || EPI == EPI_SWIGLU_BF16) {
      if (EPI == EPI_SWIGLU_BF16) {
#pragma unroll
        for (int u = 0; u < 64; ++u) a[u] = bf16r(a[u]);
      }
      if (p.aux0) {
        out_rows_f32(ring, p, &p.tma_aux[0], a, n0, row0, zr, zq, lane);
        out_rows_f32(ring, p, &p.tma_aux[1], a + 32, n0, row0, zr, zq, lane);
      }
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const float g = a[u], uu = a[32 + u];
        a[u] = EPI == EPI_SWIGLU_FWD ? __fmul_rn(__fmul_rn(g, sigmoid_f(g)), uu)
                                     : bf16r(__fmul_rn(bf16r(__fmul_rn(g, bf16r(sigmoid_f(g)))),
                                                       uu));
      }
      out_terms(ring, p, a, p.ncs, n0, 0, row0, zr, zq, t.z, lane);
    } else if (EPI == EPI_SWIGLU_BWD || EPI == EPI_SWIGLU_BWD_BF16) {
      const float* gp = p.aux0 + coff + (int64_t)row * p.ld_aux + n0;
      const float* up = p.aux1 + coff + (int64_t)row * p.ld_aux + n0;
      float du[32];
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        float g[8], u[8];
        load8_f32(gp, row_ok, nvalid, c, g);
        load8_f32(up, row_ok, nvalid, c, u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int e = c + j;
          if (EPI == EPI_SWIGLU_BWD) {
            const float sg = sigmoid_f(g[j]);
            const float dd = a[e];
            du[e] = __fmul_rn(dd, __fmul_rn(g[j], sg));
            const float dsil =
                __fadd_rn(sg, __fmul_rn(g[j], __fmul_rn(sg, __fsub_rn(1.0f, sg))));
            a[e] = __fmul_rn(__fmul_rn(dd, u[j]), dsil);
          } else {
            const float dd = bf16r(a[e]);
            const float sf = sigmoid_f(g[j]);
            const float sb = bf16r(sf);
            const float av = bf16r(__fmul_rn(g[j], sb));
            du[e] = bf16r(__fmul_rn(dd, av));
            const float da = bf16r(__fmul_rn(dd, u[j]));
            const float ds = bf16r(__fmul_rn(da, g[j]));
            a[e] = bf16r(__fadd_rn(__fmul_rn(da, sb),
                                   __fmul_rn(ds, __fmul_rn(sf, __fsub_rn(1.0f, sf)))));
          }
          const bool live = row_ok && e < nvalid;
          a[e] = live ? a[e] : 0.f;
          du[e] = live ? du[e] : 0.f;
        }
      }
      // row-major [dg | du]: columns n and n + ct_up_rows; transposed: rows n and n + ct_up_rows
      const int nt = p.ncs == 0 ? 0 : (EPI == EPI_SWIGLU_BWD_BF16 ? 1 : p.ncs);
      out_terms(ring, p, a, nt, n0, 0, row0, zr, zq, t.z, lane);
      out_terms(ring, p, du, nt, n0, (int)p.ct_up_rows, row0, zr, zq, t.z, lane);
    } else {
      // EPI_PLAIN, EPI_RESID, EPI_BF16. Every optional input is one uniform branch around a
      // loop over the group (never a test per element): bias values arrive 8 at a time (0
      // beyond the output's columns), residual and target rows through load8_bf16.
      const bool hb = p.bias != nullptr, hr = p.resid != nullptr;
      const __nv_bfloat16* rp = p.resid + coff + (int64_t)row * p.ld_rt + n0;
      if (EPI == EPI_BF16) {
        // x = bf16(acc); x = bf16(x + bias); x = bf16(resid + x). With neither input and only
        // single-term bf16 outputs the rounding is left to the output conversion, which rounds
        // the same way.
        if (hb || hr || p.C || p.sq_partial || p.ncs > 1 || p.nct > 1) {
#pragma unroll
          for (int u = 0; u < 32; ++u) a[u] = bf16r(a[u]);
        }
        if (hb) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float b[8];
            load8_bias(p.bias, n0, nvalid, c, b);
#pragma unroll
            for (int j = 0; j < 8; ++j) a[c + j] = bf16r(__fadd_rn(a[c + j], b[j]));
          }
        }
        if (hr) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float r[8];
            load8_bf16(rp, row_ok, nvalid, c, r);
#pragma unroll
            for (int j = 0; j < 8; ++j) a[c + j] = bf16r(__fadd_rn(r[j], a[c + j]));
          }
        }
      } else if (EPI == EPI_RESID) {
        const __nv_bfloat16* tp = p.target + coff + (int64_t)row * p.ld_rt + n0;
        const bool live = row_ok && !(p.row_period > 0 && (row % p.row_period) == 0);
        if (hb) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float b[8];
            load8_bias(p.bias, n0, nvalid, c, b);
#pragma unroll
            for (int j = 0; j < 8; ++j) a[c + j] = __fadd_rn(a[c + j], b[j]);
          }
        }
        if (hr) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float r[8];
            load8_bf16(rp, row_ok, nvalid, c, r);
#pragma unroll
            for (int j = 0; j < 8; ++j) a[c + j] = __fadd_rn(a[c + j], r[j]);
          }
        }
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          float tg[8];
          load8_bf16(tp, row_ok, nvalid, c, tg);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int u = c + j;
            const float x = (live && u < nvalid) ? __fsub_rn(a[u], tg[j]) : 0.f;
            sq = fma((double)x, (double)x, sq);
            a[u] = __fmul_rn(p.out_scale, x);
          }
        }
      } else if (hb) {
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          float b[8];
          load8_bias(p.bias, n0, nvalid, c, b);
#pragma unroll
          for (int j = 0; j < 8; ++j) a[c + j] = __fadd_rn(a[c + j], b[j]);
        }
      }
      if (EPI != EPI_RESID && p.sq_partial && row_ok) {
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const double v = u < nvalid ? (double)a[u] : 0.0;
          sq = fma(v, v, sq);
        }
      }
      if (p.C) out_rows_f32(ring, p, &p.tma_c, a, n0, row0, zr, zq, lane);
      if (p.nct && !row_ok) {
        // transposed values outside the output are zero (the consumer's padding rows); the
        // TMA unit clips these rows of the row-major boxes
#pragma unroll
        for (int u = 0; u < 32; ++u) a[u] = 0.f;
      }
      out_terms(ring, p, a, p.ncs, n0, 0, row0, zr, zq, t.z, lane);
    }
    ring_flush(ring, lane);
  }
  return sq;
}

// The fused outputs of one tile from the folded accumulator. Epilogue warp (q, h) holds rows
// tile_m + 32 q + lane and the 32-column groups jc (columns tile_n + 64 jc + 32 h + t); for the
// SwiGLU forward, slots [0, 32) are the gate and [32, 64) the up projection of the output
// columns tile_n / 2 + 32 h + t.
template <int BN, int EPI>
__device__ __forceinline__ double epilogue_out(const GemmParams& p, const TileInfo& t, float* acc,
                                               float* stg, int lane, int q, int h) {
  constexpr int kNC = BN / 64;
  const int64_t coff = p.c_off.at(t.z);
  const int row0 = t.tile_m + 32 * q;
  double sq = 0.0;
  if (EPI == EPI_PLAIN && p.splits > 1) {  // split-K partial: raw sums into the workspace
    float* W = p.ws + (int64_t)t.ks * p.M * p.N;
#pragma unroll
    for (int jc = 0; jc < kNC; ++jc) {
      const int n0 = t.tile_n + 64 * jc + 32 * h;
      stage_put(stg, lane, acc + 32 * jc);
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
        const int row = row0 + r, n = n0 + c;
        if (row < p.M && n < p.N)
          store_f2(W + (int64_t)row * p.N + n, stg[r * kStgLd + c], stg[r * kStgLd + c + 1],
                   n + 1 < p.N, (p.N & 1) == 0);
      }
      __syncwarp();
    }
    return 0.0;
  }
#pragma unroll
  for (int i = 0; i < BN / 2; ++i) acc[i] = __fmul_rn(p.alpha, acc[i]);

  if (EPI == EPI_PLAIN || EPI == EPI_RESID || EPI == EPI_BF16) {
#pragma unroll
    for (int jc = 0; jc < kNC; ++jc) {
      const int n0 = t.tile_n + 64 * jc + 32 * h;
      float* a = acc + 32 * jc;
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int n = n0 + u;
        float x = a[u];
        if (EPI == EPI_BF16) {
          x = bf16r(x);
          if (p.bias && n < p.N) x = bf16r(__fadd_rn(x, p.bias[n]));
        } else if (p.bias && n < p.N) {
          x = __fadd_rn(x, p.bias[n]);
        }
        a[u] = x;
      }
      stage_put(stg, lane, a);
#pragma unroll 2
      for (int i = 0; i < 16; ++i) {
        const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
        const int row = row0 + r, n = n0 + c;
        float* sp = stg + r * kStgLd + c;
        float x0 = sp[0], x1 = sp[1];
        const bool in0 = row < p.M && n < p.N, in1 = in0 && n + 1 < p.N;
        if (in0) {
          if (EPI == EPI_PLAIN) {
            if (p.beta != 0.f && p.C) {
              float c0, c1;
              load_f2(p.C + coff + (int64_t)row * p.ldc + n, in1, p.pair_c != 0, c0, c1);
              x0 = __fadd_rn(x0, __fmul_rn(p.beta, c0));
              x1 = __fadd_rn(x1, __fmul_rn(p.beta, c1));
            }
            if (p.sq_partial) {
              sq += (double)x0 * (double)x0;
              if (in1) sq += (double)x1 * (double)x1;
            }
          } else {
            const int64_t o = coff + (int64_t)row * p.ld_rt + n;
            float r0 = 0.f, r1 = 0.f;
            if (p.resid) load_bf2(p.resid + o, in1, p.pair_rt != 0, r0, r1);
            if (EPI == EPI_RESID) {
              float t0, t1;
              load_bf2(p.target + o, in1, p.pair_rt != 0, t0, t1);
              if (p.resid) {
                x0 = __fadd_rn(x0, r0);
                x1 = __fadd_rn(x1, r1);
              }
              x0 = __fsub_rn(x0, t0);
              x1 = __fsub_rn(x1, t1);
              if (p.row_period > 0 && (row % p.row_period) == 0) {
                x0 = 0.f;
                x1 = 0.f;
              }
              sq += (double)x0 * (double)x0;
              if (in1) sq += (double)x1 * (double)x1;
              x0 = __fmul_rn(p.out_scale, x0);
              x1 = __fmul_rn(p.out_scale, x1);
            } else if (p.resid) {
              x0 = bf16r(__fadd_rn(r0, x0));
              x1 = bf16r(__fadd_rn(r1, x1));
            }
          }
          if (p.C) store_f2(p.C + coff + (int64_t)row * p.ldc + n, x0, x1, in1, p.pair_c != 0);
          if (p.ncs > 0)
            store_terms2(p.cs, p.ncs, coff + (int64_t)row * p.ldcs + n, x0, x1, in1,
                         p.pair_cs != 0);
        }
        if (p.nct > 0) {
          sp[0] = x0;
          sp[1] = x1;
        }
      }
      if (p.nct > 0) {
        __syncwarp();
        transposed_pass(p, t, stg, lane, n0, p.N, row0, 0);
      }
      __syncwarp();
    }
  } else if (EPI == EPI_SWIGLU_FWD || EPI == EPI_SWIGLU_BF16) {
    const int n0 = t.tile_n / 2 + 32 * h, nl = p.N / 2;
    if (EPI == EPI_SWIGLU_FWD) {
      // g and u (float32, row-major) for the backward
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        stage_put(stg, lane, acc + 32 * part);
        float* dst = part ? p.aux1 : p.aux0;
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
          const int row = row0 + r, j = n0 + c;
          if (row < p.M && j < nl)
            store_f2(dst + coff + (int64_t)row * p.ld_aux + j, stg[r * kStgLd + c],
                     stg[r * kStgLd + c + 1], j + 1 < nl, p.pair_aux != 0);
        }
        __syncwarp();
      }
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const float g = acc[u], uu = acc[32 + u];
        acc[u] = __fmul_rn(__fmul_rn(g, sigmoid_f(g)), uu);  // silu(g) * u
      }
    } else {
#pragma unroll
      for (int u = 0; u < 64; ++u) acc[u] = bf16r(acc[u]);
      if (p.aux0) {
        // bf16 g and u (float32 storage) for the backward
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          stage_put(stg, lane, acc + 32 * part);
          float* dst = part ? p.aux1 : p.aux0;
#pragma unroll 4
          for (int i = 0; i < 16; ++i) {
            const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
            const int row = row0 + r, j = n0 + c;
            if (row < p.M && j < nl)
              store_f2(dst + coff + (int64_t)row * p.ld_aux + j, stg[r * kStgLd + c],
                       stg[r * kStgLd + c + 1], j + 1 < nl, p.pair_aux != 0);
          }
          __syncwarp();
        }
      }
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const float g = acc[u], uu = acc[32 + u];
        acc[u] = bf16r(__fmul_rn(bf16r(__fmul_rn(g, bf16r(sigmoid_f(g)))), uu));
      }
    }
    stage_put(stg, lane, acc);
    if (p.ncs > 0) {
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
        const int row = row0 + r, j = n0 + c;
        if (row < p.M && j < nl)
          store_terms2(p.cs, p.ncs, coff + (int64_t)row * p.ldcs + j, stg[r * kStgLd + c],
                       stg[r * kStgLd + c + 1], j + 1 < nl, p.pair_cs != 0);
      }
    }
    if (p.nct > 0) transposed_pass(p, t, stg, lane, n0, nl, row0, 0);
    __syncwarp();
  } else if (EPI == EPI_SWIGLU_BWD_BF16) {
    // slots hold the cotangent of d = bf16(a u) (a = bf16(g s), s = bf16(sigmoid g)) of column n;
    // with g, u (bf16 values) from aux: du = bf16(dd a), da = bf16(dd u), ds = bf16(da g),
    // dg = bf16(da s + ds sigmoid(g) (1 - sigmoid(g))). dg / du go out as row terms at columns n
    // and n + ct_up_rows, and transposed at rows n and n + ct_up_rows.
#pragma unroll
    for (int jc = 0; jc < kNC; ++jc) {
      const int n0 = t.tile_n + 64 * jc + 32 * h;
      stage_put(stg, lane, acc + 32 * jc);
      float du_keep[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
        const int row = row0 + r, n = n0 + c;
        float* sp = stg + r * kStgLd + c;
        float dg[2] = {0.f, 0.f}, du[2] = {0.f, 0.f};
        const bool in0 = row < p.M && n < p.N, in1 = in0 && n + 1 < p.N;
        if (in0) {
          const int64_t o = coff + (int64_t)row * p.ld_aux + n;
          float g[2], u[2];
          load_f2(p.aux0 + o, in1, p.pair_aux != 0, g[0], g[1]);
          load_f2(p.aux1 + o, in1, p.pair_aux != 0, u[0], u[1]);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float dd = bf16r(sp[e]);
            const float sf = sigmoid_f(g[e]);
            const float sb = bf16r(sf);
            const float a = bf16r(__fmul_rn(g[e], sb));
            du[e] = bf16r(__fmul_rn(dd, a));
            const float da = bf16r(__fmul_rn(dd, u[e]));
            const float ds = bf16r(__fmul_rn(da, g[e]));
            dg[e] = bf16r(__fadd_rn(__fmul_rn(da, sb),
                                    __fmul_rn(ds, __fmul_rn(sf, __fsub_rn(1.0f, sf)))));
          }
          if (p.ncs > 0) {
            const int64_t oc = coff + (int64_t)row * p.ldcs + n;
            store_terms2(p.cs, 1, oc, dg[0], dg[1], in1, p.pair_cs != 0);
            store_terms2(p.cs, 1, oc + p.ct_up_rows, du[0], du[1], in1, p.pair_cs != 0);
          }
        }
        sp[0] = dg[0];
        sp[1] = dg[1];
        du_keep[2 * i] = du[0];
        du_keep[2 * i + 1] = du[1];
      }
      __syncwarp();
      if (p.nct > 0) transposed_pass(p, t, stg, lane, n0, p.N, row0, 0);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
        stg[r * kStgLd + c] = du_keep[2 * i];
        stg[r * kStgLd + c + 1] = du_keep[2 * i + 1];
      }
      __syncwarp();
      if (p.nct > 0) transposed_pass(p, t, stg, lane, n0, p.N, row0, p.ct_up_rows);
      __syncwarp();
    }
  } else {  // EPI_SWIGLU_BWD: slots hold dd = dL/d(silu(g) u) of column n; dL/dg and dL/du go
            // out transposed (planes 0 and 1 of the C^T terms)
#pragma unroll
    for (int jc = 0; jc < kNC; ++jc) {
      const int n0 = t.tile_n + 64 * jc + 32 * h;
      stage_put(stg, lane, acc + 32 * jc);
      float du_keep[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
        const int row = row0 + r, n = n0 + c;
        float* sp = stg + r * kStgLd + c;
        float dg[2] = {0.f, 0.f}, du[2] = {0.f, 0.f};
        const bool in0 = row < p.M && n < p.N, in1 = in0 && n + 1 < p.N;
        if (in0) {
          const int64_t o = coff + (int64_t)row * p.ld_aux + n;
          float g[2], u[2];
          load_f2(p.aux0 + o, in1, p.pair_aux != 0, g[0], g[1]);
          load_f2(p.aux1 + o, in1, p.pair_aux != 0, u[0], u[1]);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float sg = sigmoid_f(g[e]);
            const float dd = sp[e];
            du[e] = __fmul_rn(dd, __fmul_rn(g[e], sg));
            // d(g sigmoid(g))/dg = sigmoid(g) + g sigmoid(g) (1 - sigmoid(g))
            const float dsil =
                __fadd_rn(sg, __fmul_rn(g[e], __fmul_rn(sg, __fsub_rn(1.0f, sg))));
            dg[e] = __fmul_rn(__fmul_rn(dd, u[e]), dsil);
          }
        }
        sp[0] = dg[0];
        sp[1] = dg[1];
        du_keep[2 * i] = du[0];
        du_keep[2 * i + 1] = du[1];
      }
      __syncwarp();
      if (p.nct > 0) transposed_pass(p, t, stg, lane, n0, p.N, row0, 0);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = 2 * i + (lane >> 4), c = 2 * (lane & 15);
        stg[r * kStgLd + c] = du_keep[2 * i];
        stg[r * kStgLd + c + 1] = du_keep[2 * i + 1];
      }
      __syncwarp();
      if (p.nct > 0) transposed_pass(p, t, stg, lane, n0, p.N, row0, p.ct_up_rows);
      __syncwarp();
    }
  }
  return sq;
}

// 4 K=16 steps of one 64-wide k-block into accumulator d: the shared-memory descriptors advance
// by 32 bytes (2 in the start-address field) per step; the first step accumulates if acc_first.
__device__ __forceinline__ void umma4(uint32_t d, uint64_t a, uint64_t b, uint64_t sa,
                                      uint64_t sb, uint32_t idesc, uint32_t acc_first) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %4, 0;\n\t"
      "setp.eq.b32 p1, %3, %3;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %6, %3, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %8, %3, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %9, %10, %3, p1;\n\t}"
      ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc_first), "l"(a + sa), "l"(b + sb),
        "l"(a + 2 * sa), "l"(b + 2 * sb), "l"(a + 3 * sa), "l"(b + 3 * sb));
}

// The products of one k-block for NA x NBT bf16 terms of order <= 2 (hi x hi into big, the rest
// into small); A term i at ad + i*1024, B term j at bd + j*tb in the descriptor's address field;
// sa / sb: the address step of one K = 16 slice (32 B K-major, 2 KB MN-major).
template <int NA, int NBT>
__device__ __forceinline__ void issue_kb(uint64_t ad, uint64_t bd, uint32_t tb, uint64_t sa,
                                         uint64_t sb, uint32_t big, uint32_t small,
                                         uint32_t idesc, uint32_t big_acc, uint32_t small_acc) {
  umma4(big, ad, bd, sa, sb, idesc, big_acc);
  if (NA == 1 && NBT == 3) {
    umma4(small, ad, bd + tb, sa, sb, idesc, small_acc);
    umma4(small, ad, bd + 2 * tb, sa, sb, idesc, 1u);
  } else if (NA == 3 && NBT == 1) {
    umma4(small, ad + 1024, bd, sa, sb, idesc, small_acc);
    umma4(small, ad + 2048, bd, sa, sb, idesc, 1u);
  } else if (NA == 3 && NBT == 3) {
    umma4(small, ad, bd + tb, sa, sb, idesc, small_acc);
    umma4(small, ad + 1024, bd, sa, sb, idesc, 1u);
    umma4(small, ad, bd + 2 * tb, sa, sb, idesc, 1u);
    umma4(small, ad + 1024, bd + tb, sa, sb, idesc, 1u);
    umma4(small, ad + 2048, bd, sa, sb, idesc, 1u);
  }
}

// --------------------------------------------------------------------------- kernel ---
template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full_bar[kMaxStages];
  __shared__ uint64_t empty_bar[kMaxStages];
  __shared__ uint64_t bigf_bar[kMaxBig];   // chunk accumulator ready
  __shared__ uint64_t bige_bar[kMaxBig];   // chunk accumulator folded
  __shared__ uint64_t smf_bar[2];          // tile "small" accumulator ready
  __shared__ uint64_t sme_bar[2];          // tile "small" accumulator folded
  __shared__ uint64_t done_bar;
  __shared__ uint32_t tmem_base;
  __shared__ double red[kEpiWarps];

  constexpr uint32_t kTileA = BM * BK * 2;
  constexpr uint32_t kTileB = BN * BK * 2;
  constexpr int kAcc = BN / 2;  // accumulator columns per epilogue thread
  constexpr int kNC = BN / 64;  // 32-column groups per epilogue thread
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages, NB = p.n_big, P = p.kb_per_chunk;
  const uint32_t stage_bytes = p.na * kTileA + p.nb * kTileB;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const bool has_small = (p.na > 1 || p.nb > 1) && p.order > 0;
  const uint32_t small_col = (uint32_t)(NB * BN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&bigf_bar[b], 1);
      mbar_init(&bige_bar[b], kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&smf_bar[b], 1);
      mbar_init(&sme_bar[b], kEpiWarps);
    }
    mbar_init(&done_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < p.na; ++i) tma_prefetch_desc(&p.tma_a[i]);
    for (int i = 0; i < p.nb; ++i) {
      tma_prefetch_desc(&p.tma_b[i]);
      if (p.dual_b) tma_prefetch_desc(&p.tma_b2[i]);
    }
  }
  if (warp == 1) tmem_alloc(&tmem_base, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, issued = 0;
      bool ok = true;
      for (int64_t L = blockIdx.x; L < p.total_tiles && ok; L += gridDim.x) {
        TileInfo t;
        if (!tile_at<BN>(p, L, t)) continue;
        const int a_row = t.tile_m + (int)p.a_off.at(t.z);
        const int b_row = (p.dual_b ? t.tile_n / 2 : t.tile_n) + (int)p.b_off.at(t.z);
        for (int kb = 0; kb < t.nkb; ++kb) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, p.err, 1)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + (size_t)s * stage_bytes;
          mbar_arrive_expect_tx(&full_bar[s], stage_bytes);
          const int kx = (t.kb0 + kb) * BK;
          for (int i = 0; i < p.na; ++i) {
            if (p.a_mn) {  // two 64 (M) x 64 (K) boxes of the [K][M] operand (batch rows at a_off)
              const int ky = kx + (int)p.a_off.at(t.z);
              tma_load_2d(st + i * kTileA, &p.tma_a[i], &full_bar[s], t.tile_m, ky);
              tma_load_2d(st + i * kTileA + 8192, &p.tma_a[i], &full_bar[s], t.tile_m + 64, ky);
            } else {
              tma_load_2d(st + i * kTileA, &p.tma_a[i], &full_bar[s], kx, a_row);
            }
          }
          for (int j = 0; j < p.nb; ++j) {
            uint8_t* bt = st + p.na * kTileA + j * kTileB;
            if (p.b_mn) {
#pragma unroll
              for (int bb = 0; bb < BN / 64; ++bb)
                tma_load_2d(bt + bb * 8192, &p.tma_b[j], &full_bar[s], t.tile_n + 64 * bb, kx);
            } else if (p.dual_b) {
              tma_load_2d(bt, &p.tma_b[j], &full_bar[s], kx, b_row);
              tma_load_2d(bt + kTileB / 2, &p.tma_b2[j], &full_bar[s], kx, b_row);
            } else {
              tma_load_2d(bt, &p.tma_b[j], &full_bar[s], kx, b_row);
            }
          }
          ++issued;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // let the copies still in flight land before the CTA exits (bounded waits)
        const uint32_t n = issued < (uint32_t)S ? issued : (uint32_t)S;
        for (uint32_t j = 0; j < n; ++j) {
          if (--s < 0) {
            s = S - 1;
            ph ^= 1u;
          }
          mbar_wait(&full_bar[s], ph, nullptr, 6);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN) | ((uint32_t)p.a_mn << 15) |
                             ((uint32_t)p.b_mn << 16);
      const uint64_t sa = p.a_mn ? 128u : 2u, sb = p.b_mn ? 128u : 2u;
      // term configurations with a compile-time product list (order 2); others: generic loop
      const int cfg = (p.na == 1 && p.nb == 1) ? 1
                    : (p.order != 2) ? 0
                    : (p.na == 1 && p.nb == 3) ? 2 : (p.na == 3 && p.nb == 1) ? 3
                    : (p.na == 3 && p.nb == 3) ? 4 : 0;
      int s = 0, bs = 0;
      uint32_t ph = 0, bph = 0, tcount = 0;
      bool ok = true, any = false;
      for (int64_t L = blockIdx.x; L < p.total_tiles && ok; L += gridDim.x) {
        TileInfo t;
        if (!tile_at<BN>(p, L, t)) continue;
        const uint32_t tb = p.small_bufs == 2 ? (tcount & 1u) : 0u;
        const uint32_t tph = p.small_bufs == 2 ? ((tcount >> 1) & 1u) : (tcount & 1u);
        ++tcount;
        const uint32_t small = tmem + small_col + tb * (uint32_t)BN;
        if (has_small) {
          if (!mbar_wait(&sme_bar[tb], tph ^ 1u, p.err, 5)) break;
          fence_after_sync();
        }
        bool small_init = false;
        for (int c0 = 0; c0 < t.nkb && ok; c0 += P) {
          if (!mbar_wait(&bige_bar[bs], bph ^ 1u, p.err, 4)) {
            ok = false;
            break;
          }
          fence_after_sync();
          const uint32_t big = tmem + (uint32_t)(bs * BN);
          bool big_init = false;
          const int c1 = min(t.nkb, c0 + P);
          for (int kb = c0; kb < c1; ++kb) {
            if (!mbar_wait(&full_bar[s], ph, p.err, 2)) {
              ok = false;
              break;
            }
            fence_after_sync();
            const uint32_t st = smem_u32(smem + (size_t)s * stage_bytes);
            if (cfg != 0) {  // compile-time product lists: few instructions between UMMAs
              const uint32_t sb_addr = st + p.na * kTileA;
              const uint64_t ad = p.a_mn ? umma_desc_mn_sw128(st) : umma_desc_k_sw128(st);
              const uint64_t bd = p.b_mn ? umma_desc_mn_sw128(sb_addr) : umma_desc_k_sw128(sb_addr);
              const uint32_t tb = kTileB >> 4;
              const uint32_t ba = big_init ? 1u : 0u, sm = small_init ? 1u : 0u;
              if (cfg == 1) issue_kb<1, 1>(ad, bd, tb, sa, sb, big, small, idesc, ba, sm);
              else if (cfg == 2) issue_kb<1, 3>(ad, bd, tb, sa, sb, big, small, idesc, ba, sm);
              else if (cfg == 3) issue_kb<3, 1>(ad, bd, tb, sa, sb, big, small, idesc, ba, sm);
              else issue_kb<3, 3>(ad, bd, tb, sa, sb, big, small, idesc, ba, sm);
              big_init = true;
              if (cfg != 1) small_init = true;
            } else
            for (int i = 0; i < p.na; ++i) {
              for (int j = 0; j < p.nb; ++j) {
                if (i + j > p.order) continue;
                const uint32_t a0 = st + i * kTileA;
                const uint32_t b0 = st + p.na * kTileA + j * kTileB;
                const bool to_big = (i + j == 0);
                const uint32_t d = to_big ? big : small;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                  const uint32_t accum = to_big ? (uint32_t)big_init : (uint32_t)small_init;
                  const uint64_t da = p.a_mn ? umma_desc_mn_sw128(a0) + k * sa
                                             : umma_desc_k_sw128(a0) + k * sa;
                  const uint64_t db = p.b_mn ? umma_desc_mn_sw128(b0) + k * sb
                                             : umma_desc_k_sw128(b0) + k * sb;
                  umma_bf16(d, da, db, idesc, accum);
                  if (to_big) big_init = true; else small_init = true;
                }
              }
            }
            umma_commit(&empty_bar[s]);
            any = true;
            if (++s == S) {
              s = 0;
              ph ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(&bigf_bar[bs]);
          if (++bs == NB) {
            bs = 0;
            bph ^= 1u;
          }
        }
        if (ok && has_small) umma_commit(&smf_bar[tb]);
      }
      if (any) {  // every MMA issued here has completed before the TMEM is freed
        umma_commit(&done_bar);
        mbar_wait(&done_bar, 0, nullptr, 7);
      }
    }
  } else {
    const int ew = warp - 2;
    const int q = warp & 3;  // TMEM lane quadrant of this warp
    const int h = ew >> 2;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float* stg = reinterpret_cast<float*>(smem + (size_t)S * stage_bytes) + ew * (32 * kStgLd);
    BoxRing ring;
    ring.base = smem + (size_t)S * stage_bytes + (size_t)ew * p.tma_bufs * kTmaBuf;
    ring.nbuf = p.tma_bufs;
    ring.bsize = (int)kTmaBuf;
    if (p.tma_bufs == 1 && p.tma_bf16_only) {  // one 4 KB area as two 2 KB buffers
      ring.nbuf = 2;
      ring.bsize = (int)kTmaBuf / 2;
    }
    ring.cur = 0;
    ring.used = 0;
    int bs = 0;
    uint32_t bph = 0, tcount = 0;
    bool ok = true;
    // after a timeout the loop still runs to the end (skipping every wait and output), so that
    // all eight warps take the same named-barrier steps
    for (int64_t L = blockIdx.x; L < p.total_tiles; L += gridDim.x) {
      TileInfo t;
      if (!tile_at<BN>(p, L, t)) continue;
      const uint32_t tb = p.small_bufs == 2 ? (tcount & 1u) : 0u;
      const uint32_t tph = p.small_bufs == 2 ? ((tcount >> 1) & 1u) : (tcount & 1u);
      ++tcount;
      prefetch_row_inputs<BN, EPI>(p, t, lane, q, h);
      float acc[kAcc];
#pragma unroll
      for (int u = 0; u < kAcc; ++u) acc[u] = 0.f;
      for (int c0 = 0; c0 < t.nkb; c0 += P) {
        if (ok) ok = mbar_wait(&bigf_bar[bs], bph, p.err, 3);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          fence_after_sync();
          uint32_t v[kNC][32];
#pragma unroll
          for (int jc = 0; jc < kNC; ++jc)
            tmem_ld32_nowait(tmem + lane_off + (uint32_t)(bs * BN + 64 * jc + 32 * h), v[jc]);
          tmem_wait_ld();
#pragma unroll
          for (int jc = 0; jc < kNC; ++jc)
#pragma unroll
            for (int u = 0; u < 32; ++u)
              acc[32 * jc + u] = __fadd_rn(acc[32 * jc + u], __uint_as_float(v[jc][u]));
          fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bige_bar[bs]);
        }
        if (++bs == NB) {
          bs = 0;
          bph ^= 1u;
        }
      }
      if (has_small) {
        if (ok) ok = mbar_wait(&smf_bar[tb], tph, p.err, 3);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          fence_after_sync();
          uint32_t v[kNC][32];
#pragma unroll
          for (int jc = 0; jc < kNC; ++jc)
            tmem_ld32_nowait(tmem + lane_off + small_col + tb * (uint32_t)BN +
                                 (uint32_t)(64 * jc + 32 * h),
                             v[jc]);
          tmem_wait_ld();
#pragma unroll
          for (int jc = 0; jc < kNC; ++jc)
#pragma unroll
            for (int u = 0; u < 32; ++u)
              acc[32 * jc + u] = __fadd_rn(acc[32 * jc + u], __uint_as_float(v[jc][u]));
          fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sme_bar[tb]);
        }
      }
      double sq = 0.0;
      if (ok) {
        if (p.tma_out)
          sq = epilogue_tma<BN, EPI>(p, t, acc, ring, lane, q, h);
        else
          sq = epilogue_out<BN, EPI>(p, t, acc, stg, lane, q, h);
      }
      if (p.sq_partial) {
        sq = warp_sum_d(sq);
        if (lane == 0) red[ew] = sq;
        epi_sync();
        if (ew == 0 && lane == 0 && ok) {
          double tot = 0.0;
          for (int i = 0; i < kEpiWarps; ++i) tot += red[i];
          p.sq_partial[t.part] = tot;
        }
        epi_sync();
      }
    }
    if (p.tma_out) {  // the boxes' global writes are done before the CTA exits
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
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

// Output map of the TMA-store epilogue: [nz][div][M][ld] view (element strides ld, s2, s1) with
// 32 x 32 boxes; float32 rows of 128 B (128-byte swizzle) or bf16 rows of 64 B (64-byte).
static bool make_out_map(CUtensorMap* m, const void* base, bool f32, int N, int M, int64_t ld,
                         int div, int64_t s1, int64_t s2, int batch, int* rank) {
  EncodeTiledFn fn = encode_fn();
  const int64_t e = f32 ? 4 : 2;
  if (!fn || !base || ((uintptr_t)base & 15) || ((ld * e) & 15) || ((s1 * e) & 15) ||
      ((s2 * e) & 15))
    return false;
  const int nz = (batch + div - 1) / div;
  cuuint32_t box[4] = {32, 32, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                     : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (div == 1) {
    cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)nz};
    cuuint64_t strides[2] = {(cuuint64_t)(ld * e),
                             (cuuint64_t)((s1 > 0 ? s1 : ld * M) * e)};
    *rank = 3;
    return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  if (s1 <= 0 || s2 <= 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)div, (cuuint64_t)nz};
  cuuint64_t strides[3] = {(cuuint64_t)(ld * e), (cuuint64_t)(s2 * e), (cuuint64_t)(s1 * e)};
  *rank = 4;
  return fn(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI>
static int launch(GemmParams& p, int batch, cudaStream_t st) {
  const uint32_t stage_bytes = p.na * BM * BK * 2 + p.nb * BN * BK * 2;
  int S = (int)(kPipeBudget / stage_bytes);
  if (p.tma_out) {  // TMA-store staging: two buffers per warp where two stages still fit, else one
    p.tma_bufs = 0;
    for (int bufs = 3; bufs >= 1 && !p.tma_bufs; --bufs) {
      const int sb = (int)((kSmemMax - 1024 - kEpiWarps * bufs * kTmaBuf) / stage_bytes);
      if (sb >= 2) {
        p.tma_bufs = bufs;
        S = sb < S ? sb : S;
      }
    }
    if (!p.tma_bufs) p.tma_out = 0;
  }
  if (S > kMaxStages) S = kMaxStages;
  if (S < 2) return GSQ_ENOTSUP;
  p.stages = S;
  int products = 0;
  for (int i = 0; i < p.na; ++i)
    for (int j = 0; j < p.nb; ++j) products += (i + j <= p.order);
  p.kb_per_chunk = products >= 3 ? 2 : 4;
  // a bf16-output product of bf16 operands (the bf16 model's chain epilogues) folds its TMEM
  // chunks every 8 k-blocks: its float32 sum is rounded to bf16 once, and K <= 512 (the
  // attention products) needs no fold at all; the TMEM accumulation error grows with the
  // chunk length, so long reductions (the head gradient over the vocabulary) keep folding
  if (products == 1 && (EPI == EPI_BF16 || EPI == EPI_SWIGLU_BF16 || EPI == EPI_SWIGLU_BWD_BF16))
    p.kb_per_chunk = 8;
  const bool has_small = (p.na > 1 || p.nb > 1) && p.order > 0;
  // cross-product ("small") accumulators: two let the next tile's MMAs start before the
  // epilogue has read this tile's; one leaves a further chunk slot to the hi x hi ring, so the
  // MMAs run further ahead while the epilogue writes a tile's outputs
  if (p.small_bufs != 1) p.small_bufs = 2;
  int nbig = (int)((kTmemCols - (has_small ? (uint32_t)p.small_bufs * BN : 0u)) / BN);
  p.n_big = nbig > kMaxBig ? kMaxBig : nbig;
  p.tiles_m = (p.M + BM - 1) / BM;
  p.tiles_n = (p.N + BN - 1) / BN;
  p.total_tiles = (int64_t)p.tiles_m * p.tiles_n * batch * p.splits;
  // single products: walk along the smaller operand first (its bytes M x K x na vs N x K x nb)
  p.n_fast = (batch == 1 && p.splits == 1 && !p.skip_upper && p.causal == 0 &&
              (int64_t)p.M * p.na > (int64_t)p.N * p.nb) ? 1 : 0;
  p.causal_order = (p.causal != 0 && p.splits == 1 && !p.skip_upper) ? 1 : 0;
  const size_t smem = 1024 + (size_t)S * stage_bytes +
                      (p.tma_out ? (size_t)kEpiWarps * p.tma_bufs * kTmaBuf : (size_t)kStgBytes);
  static bool attr_set[2][7] = {{false}};
  bool& done = attr_set[BN == 128][EPI];
  if (!done) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemMax) !=
        cudaSuccess)
      return GSQ_ECUDA;
    done = true;
  }
  if (smem > kSmemMax) return GSQ_ENOTSUP;
  const int64_t g = p.total_tiles < num_sms() ? p.total_tiles : num_sms();
  gemm_tc_kernel<BN, EPI><<<(unsigned)g, kThreads, smem, st>>>(p);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

// C = alpha sum_s ws[s] + beta C (sum in part order), float32 [M][ldc]
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N,
                                     float alpha, float beta, float* __restrict__ C, int64_t ldc) {
  const int64_t n_el = (int64_t)M * N;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_el;
       e += (int64_t)gridDim.x * blockDim.x) {
    float v = ws[e];
    for (int s = 1; s < splits; ++s) v = __fadd_rn(v, ws[(int64_t)s * n_el + e]);
    const int r = (int)(e / N), c = (int)(e - (int64_t)r * N);
    float* cp = C + (int64_t)r * ldc + c;
    float x = __fmul_rn(alpha, v);
    if (beta != 0.f) x = __fadd_rn(x, __fmul_rn(beta, *cp));
    *cp = x;
  }
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

// A checked, ready-to-launch GEMM: the kernel parameters (tensor maps encoded) and what the
// launch needs besides them.
struct GemmPlan {
  tc::GemmParams p;
  int epi, bn, batch;
  int M, N;
  float alpha, beta;
  float* C;
  int64_t ldc;
};

static int gemm_prepare(const gsq_gemm_desc* d, GemmPlan* plan) {
  if (!d || !plan) return GSQ_EINVAL;
  const int M = d->M, N = d->N, K = d->K;
  if (M <= 0 || N <= 0 || K <= 0 || d->batch < 1 || d->batch > 65535 || d->na < 1 ||
      d->na > 3 || d->nb < 1 || d->nb > 3 || d->order < 0 || !d->err || d->ncs < 0 ||
      d->ncs > 3 || d->nct < 0 || d->nct > 3 || d->epi < 0 || d->epi > 6)
    return GSQ_EINVAL;
  if (d->bn != 64 && d->bn != 128) return GSQ_EINVAL;
  const int epi = d->epi;
  if (!d->C && d->ncs == 0 && d->nct == 0 && !d->sq_partial) return GSQ_EINVAL;
  const int amn = d->a_major != 0, bmn = d->b_major != 0;
  if (d->a_major < 0 || d->a_major > 1 || d->b_major < 0 || d->b_major > 1) return GSQ_EINVAL;
  if ((amn ? (d->lda < M || d->a_rows < K) : d->lda < K) ||
      (bmn ? (d->ldb < N || d->b_rows < K) : d->ldb < K) ||
      (d->C && d->ldc < ((epi == 2 || epi == 5) ? N / 2 : N)))
    return GSQ_EINVAL;
  // MN-major operands: B is one product (no batch offsets, no causal range) and not paired
  // with b2; a batched or causal MN-major A moves its batch offsets along its K rows, so K is
  // whole k-blocks there (no box reaches into the next batch's rows)
  if (bmn && (d->batch != 1 || d->causal)) return GSQ_EINVAL;
  if (amn && (d->batch != 1 || d->causal) && (K % tc::BK) != 0) return GSQ_EINVAL;
  if (bmn && (epi == 2 || epi == 5)) return GSQ_EINVAL;
  if (d->ncs > 0 && (d->ldcs & 7)) return GSQ_EINVAL;
  if (d->nct > 0 && (d->ldct & 7)) return GSQ_EINVAL;
  for (int i = 0; i < d->ncs; ++i)
    if (!d->cs[i] || ((uintptr_t)d->cs[i] & 15)) return GSQ_EINVAL;
  for (int i = 0; i < d->nct; ++i)
    if (!d->ct[i] || ((uintptr_t)d->ct[i] & 15)) return GSQ_EINVAL;
  if (epi == 1 && !d->target) return GSQ_EINVAL;
  if ((epi == 2 || epi == 3 || epi == 6) && (!d->aux0 || !d->aux1 || (d->bn != 128 && epi != 3)))
    return GSQ_EINVAL;
  if (epi == 5 && (!d->aux0) != (!d->aux1)) return GSQ_EINVAL;
  if (epi == 6 && (d->ncs > 1 || d->nct > 1)) return GSQ_EINVAL;
  if ((epi == 2 || epi == 5) && (!d->b2[0] || (N % 128) != 0 || d->bn != 128)) return GSQ_EINVAL;
  if (d->causal < 0 || d->causal > 2 || (d->causal && d->K < M)) return GSQ_EINVAL;
  const int splits = d->split_k > 1 ? d->split_k : 1;
  if (splits > 1 && (epi != 0 || d->batch != 1 || d->causal || !d->C || d->bias || d->ncs ||
                     d->nct || d->sq_partial || !d->workspace || ((uintptr_t)d->workspace & 7)))
    return GSQ_EINVAL;
  tc::GemmParams p;
  memset(&p, 0, sizeof(p));
  const int BN = d->bn;
  const bool dual = (epi == 2 || epi == 5);
  const int b_box = dual ? BN / 2 : BN;
  for (int i = 0; i < d->na; ++i) {
    const bool ok = amn ? tc::make_map(&p.tma_a[i], d->a[i], d->a_rows, M, d->lda, 64)
                        : tc::make_map(&p.tma_a[i], d->a[i], d->a_rows, K, d->lda, tc::BM);
    if (!ok) return GSQ_EINVAL;
  }
  p.a_mn = amn;
  if (d->small_bufs < 0 || d->small_bufs > 2) return GSQ_EINVAL;
  // default: the epilogues that read row inputs and write several outputs per element (residual
  // loss, SwiGLU forward / backward) keep one cross-product accumulator and give its TMEM to
  // the hi x hi ring (measured 1-6 % faster, warm); the others keep two
  p.small_bufs = d->small_bufs ? d->small_bufs : ((epi >= 1 && epi <= 3) ? 1 : 2);
  p.b_mn = bmn;
  for (int j = 0; j < d->nb; ++j) {
    const bool ok = bmn ? tc::make_map(&p.tma_b[j], d->b[j], d->b_rows, N, d->ldb, 64)
                        : tc::make_map(&p.tma_b[j], d->b[j], d->b_rows, K, d->ldb, b_box);
    if (!ok) return GSQ_EINVAL;
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
  {
    const int kb_total = (K + tc::BK - 1) / tc::BK;
    const int per = (kb_total + splits - 1) / splits;
    p.kb_split = per;
    p.splits = (kb_total + per - 1) / per;  // every part non-empty
    p.ws = d->workspace;
  }
  const bool c_even = ((d->c_s1 | d->c_s2) & 1) == 0;
  p.pair_c = (d->C && ((uintptr_t)d->C & 7) == 0 && (d->ldc & 1) == 0 && c_even) ? 1 : 0;
  p.pair_cs = ((d->ldcs & 1) == 0 && c_even) ? 1 : 0;
  p.pair_ct = ((d->ldct & 1) == 0 && ((d->t_c1 | d->t_c2) & 1) == 0) ? 1 : 0;
  p.pair_aux = (((uintptr_t)d->aux0 & 7) == 0 && ((uintptr_t)d->aux1 & 7) == 0 &&
                (d->ld_aux & 1) == 0 && c_even) ? 1 : 0;
  p.pair_rt = (((uintptr_t)d->resid & 3) == 0 && ((uintptr_t)d->target & 3) == 0 &&
               (d->ld_rt & 1) == 0 && c_even) ? 1 : 0;
  // TMA box epilogue: every output of the tile as 32 x 32 boxes (row-major C / cs / aux, the
  // transposed ct terms); falls back to the per-element stores where a layout does not fit.
  if (p.splits == 1 && !(epi == 0 && d->beta != 0.f && d->C)) {
    const int div = p.c_off.div;
    const bool dual = (epi == 2 || epi == 5), bwd = (epi == 3 || epi == 6);
    const int n_rows_out = dual ? N / 2 : (bwd ? (int)d->ct_up_rows + N : N);
    const bool c_ok = ((d->c_s1 | d->c_s2) & 7) == 0;
    bool ok = c_ok;
    int rank = 3;
    if (ok && bwd && (N % 32) != 0) ok = false;
    if (ok && (d->resid || d->target) &&
        ((((uintptr_t)d->resid | (uintptr_t)d->target) & 15) || (d->ld_rt & 7)))
      ok = false;
    if (ok && bwd && ((((uintptr_t)d->aux0 | (uintptr_t)d->aux1) & 15) || (d->ld_aux & 3)))
      ok = false;
    if (ok && d->C && !dual && !bwd)
      ok = tc::make_out_map(&p.tma_c, d->C, true, N, M, d->ldc, div, d->c_s1, d->c_s2,
                            d->batch, &rank);
    for (int i = 0; i < d->ncs && ok; ++i)
      ok = tc::make_out_map(&p.tma_cs[i], d->cs[i], false, n_rows_out, M, d->ldcs, div,
                            d->c_s1, d->c_s2, d->batch, &rank);
    if (ok && dual && d->aux0)
      ok = tc::make_out_map(&p.tma_aux[0], d->aux0, true, N / 2, M, d->ld_aux, div, d->c_s1,
                            d->c_s2, d->batch, &rank) &&
           tc::make_out_map(&p.tma_aux[1], d->aux1, true, N / 2, M, d->ld_aux, div, d->c_s1,
                            d->c_s2, d->batch, &rank);
    if (ok && d->nct > 0) {
      // C^T as [batch][rows][ldct] (x = output row m, y = output column): plain row offsets only
      const bool t_ok = d->t_c1 == 0 && d->t_c2 == 0 && (d->batch == 1 || d->t_div <= 1);
      const int ct_rows = bwd ? (int)d->ct_up_rows + N : (dual ? N / 2 : N);
      const int64_t zs = d->batch > 1 ? d->t_r1 : (int64_t)ct_rows;
      int r3 = 3;
      ok = t_ok && zs > 0;
      for (int i = 0; i < d->nct && ok; ++i)
        ok = tc::make_out_map(&p.tma_ct[i], d->ct[i], false, M, ct_rows, d->ldct, 1,
                              zs * d->ldct, 0, d->batch, &r3);
    }
    if (ok) {
      p.tma_out = 1;
      p.out_rank = rank;
      p.tma_bf16_only = !((d->C && !dual && !bwd) || (dual && d->aux0));
    }
  }
  // the row-major outputs of the float32 SwiGLU backward exist only in the box epilogue
  if (epi == 3 && d->ncs > 0 && !p.tma_out) return GSQ_ENOTSUP;
  if (BN == 64 && p.splits == 1 && epi != 0 && epi != 1 && epi != 3 && epi != 4)
    return GSQ_EINVAL;
  plan->p = p;
  plan->epi = epi;
  plan->bn = BN;
  plan->batch = d->batch;
  plan->M = M;
  plan->N = N;
  plan->alpha = d->alpha;
  plan->beta = d->beta;
  plan->C = d->C;
  plan->ldc = d->ldc;
  return GSQ_OK;
}

static int gemm_launch(const GemmPlan& plan, cudaStream_t st) {
  tc::GemmParams p = plan.p;  // launch() fills in the per-launch configuration
  const int BN = plan.bn, epi = plan.epi;
  if (p.splits > 1) {
    const int rc = BN == 64 ? tc::launch<64, 0>(p, 1, st) : tc::launch<128, 0>(p, 1, st);
    if (rc != GSQ_OK) return rc;
    const int64_t n_el = (int64_t)plan.M * plan.N;
    int64_t blocks = (n_el + 255) / 256;
    if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
    tc::splitk_reduce_kernel<<<(unsigned)blocks, 256, 0, st>>>(
        p.ws, p.splits, plan.M, plan.N, plan.alpha, plan.beta, plan.C, plan.ldc);
    GSQ_CHECK_LAUNCH();
    return GSQ_OK;
  }
  if (BN == 64) {
    if (epi == 0) return tc::launch<64, 0>(p, plan.batch, st);
    if (epi == 1) return tc::launch<64, 1>(p, plan.batch, st);
    if (epi == 4) return tc::launch<64, 4>(p, plan.batch, st);
    if (epi == 3) return tc::launch<64, 3>(p, plan.batch, st);
    return GSQ_EINVAL;
  }
  switch (epi) {
    case 0: return tc::launch<128, 0>(p, plan.batch, st);
    case 1: return tc::launch<128, 1>(p, plan.batch, st);
    case 2: return tc::launch<128, 2>(p, plan.batch, st);
    case 3: return tc::launch<128, 3>(p, plan.batch, st);
    case 4: return tc::launch<128, 4>(p, plan.batch, st);
    case 5: return tc::launch<128, 5>(p, plan.batch, st);
    default: return tc::launch<128, 6>(p, plan.batch, st);
  }
}

extern "C" int gsq_gemm(const gsq_gemm_desc* d, void* stream) {
  GemmPlan plan;
  const int rc = gemm_prepare(d, &plan);
  if (rc != GSQ_OK) return rc;
  return gemm_launch(plan, (cudaStream_t)stream);
}

extern "C" int gsq_gemm_plan_create(const gsq_gemm_desc* d, void** plan) {
  if (!d || !plan) return GSQ_EINVAL;
  *plan = nullptr;
  GemmPlan* g = new (std::nothrow) GemmPlan;
  if (!g) return GSQ_ECUDA;
  const int rc = gemm_prepare(d, g);
  if (rc != GSQ_OK) {
    delete g;
    return rc;
  }
  *plan = g;
  return GSQ_OK;
}

extern "C" int gsq_gemm_plan_run(const void* plan, void* stream) {
  if (!plan) return GSQ_EINVAL;
  return gemm_launch(*static_cast<const GemmPlan*>(plan), (cudaStream_t)stream);
}

extern "C" int gsq_gemm_plan_destroy(void* plan) {
  delete static_cast<GemmPlan*>(plan);
  return GSQ_OK;
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
