// Operand staging of the GSQ step: gather the micro-batch rows (positions 1.. of the chosen
// calibration sequences) and split them into bf16 terms in both the row-major layout (the
// K-major A operand of the forward residual GEMM) and the transposed layout (the K-major B
// operand of the weight-gradient GEMM, reduction over rows), in one pass; plus a float64
// sum used for the per-tile loss partials.
#include "common.cuh"

namespace gsq {

template <typename TS>
__global__ void gather_split_kernel(const TS* __restrict__ x, int64_t ld_x,
                                    const int32_t* __restrict__ seq, int per_seq,
                                    int64_t seq_stride, int offset, int rows, int cols,
                                    int n_terms, __nv_bfloat16* __restrict__ t0,
                                    __nv_bfloat16* __restrict__ t1,
                                    __nv_bfloat16* __restrict__ t2, int64_t ld_t,
                                    __nv_bfloat16* __restrict__ u0,
                                    __nv_bfloat16* __restrict__ u1,
                                    __nv_bfloat16* __restrict__ u2, int64_t ld_u) {
  __shared__ float S[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int rr = threadIdx.y; rr < 32; rr += 8) {
    const int r = r0 + rr, c = c0 + threadIdx.x;
    float v = 0.f;
    if (r < rows && c < cols) {
      const int64_t src = (int64_t)seq[r / per_seq] * seq_stride + offset + (r % per_seq);
      v = (float)x[src * ld_x + c];
      if (t0) {
        __nv_bfloat16 h, m, l;
        split3_bf16(v, h, m, l);
        const int64_t o = (int64_t)r * ld_t + c;
        t0[o] = h;
        if (n_terms > 1) t1[o] = m;
        if (n_terms > 2) t2[o] = l;
      }
    }
    S[rr][threadIdx.x] = v;
  }
  __syncthreads();
  if (!u0) return;
  for (int cc = threadIdx.y; cc < 32; cc += 8) {
    const int c = c0 + cc, r = r0 + threadIdx.x;
    if (c < cols && r < rows) {
      __nv_bfloat16 h, m, l;
      split3_bf16(S[threadIdx.x][cc], h, m, l);
      const int64_t o = (int64_t)c * ld_u + r;
      u0[o] = h;
      if (n_terms > 1) u1[o] = m;
      if (n_terms > 2) u2[o] = l;
    }
  }
}

// The row-major terms alone (no transposed copy): one thread per 8 consecutive columns of a
// gathered row, 16-byte loads and stores. Needs cols, ld_x and ld_t multiples of 8 and 16-byte
// aligned rows.
template <typename TS>
__global__ void gather_rows_kernel(const TS* __restrict__ x, int64_t ld_x,
                                   const int32_t* __restrict__ seq, int per_seq,
                                   int64_t seq_stride, int offset, int rows, int cols,
                                   int n_terms, __nv_bfloat16* __restrict__ t0,
                                   __nv_bfloat16* __restrict__ t1,
                                   __nv_bfloat16* __restrict__ t2, int64_t ld_t) {
  const int per_row = cols / 8;
  const int64_t n = (int64_t)rows * per_row;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / per_row), c = (int)(e - (int64_t)r * per_row) * 8;
    const int64_t src = (int64_t)seq[r / per_seq] * seq_stride + offset + (r % per_seq);
    float v[8];
    if (sizeof(TS) == 2) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + src * ld_x + c);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b2[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
    } else {
      const float4* f4 = reinterpret_cast<const float4*>(x + src * ld_x + c);
      const float4 a = f4[0], b = f4[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    __align__(16) __nv_bfloat16 h[3][8];
#pragma unroll
    for (int j = 0; j < 8; ++j) split3_bf16(v[j], h[0][j], h[1][j], h[2][j]);
    const int64_t o = (int64_t)r * ld_t + c;
    *reinterpret_cast<uint4*>(t0 + o) = *reinterpret_cast<const uint4*>(h[0]);
    if (n_terms > 1) *reinterpret_cast<uint4*>(t1 + o) = *reinterpret_cast<const uint4*>(h[1]);
    if (n_terms > 2) *reinterpret_cast<uint4*>(t2 + o) = *reinterpret_cast<const uint4*>(h[2]);
  }
}

__global__ void sum_f64_kernel(const double* __restrict__ x, int n, double* out) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) out[0] = v;
  }
}

// Block partials of sum (t0 + t1 + t2)[r, c] * G[r, c] over a [rows][cols] matrix held as bf16
// terms (t1 / t2 may be null), products and sums in float64; one partial per block. Blocks take
// whole rows; with cols, ld_t and ld_g multiples of 8 (16-byte rows) a thread reads 8 columns
// per step (one 16-byte load per term, two per G).
__global__ void __launch_bounds__(256)
dot_terms_kernel(const __nv_bfloat16* __restrict__ t0, const __nv_bfloat16* __restrict__ t1,
                 const __nv_bfloat16* __restrict__ t2, int64_t ld_t, const float* __restrict__ G,
                 int64_t ld_g, int rows, int cols, int vec, double* __restrict__ partials) {
  __shared__ double sh[8];
  double s = 0.0;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* a0 = t0 + (int64_t)r * ld_t;
    const __nv_bfloat16* a1 = t1 ? t1 + (int64_t)r * ld_t : nullptr;
    const __nv_bfloat16* a2 = t2 ? t2 + (int64_t)r * ld_t : nullptr;
    const float* g = G + (int64_t)r * ld_g;
    if (vec) {
      for (int c = 8 * threadIdx.x; c < cols; c += 8 * blockDim.x) {
        const uint4 u0 = *reinterpret_cast<const uint4*>(a0 + c);
        const uint4 u1 = a1 ? *reinterpret_cast<const uint4*>(a1 + c) : make_uint4(0, 0, 0, 0);
        const uint4 u2 = a2 ? *reinterpret_cast<const uint4*>(a2 + c) : make_uint4(0, 0, 0, 0);
        const float4 g0 = *reinterpret_cast<const float4*>(g + c);
        const float4 g1 = *reinterpret_cast<const float4*>(g + c + 4);
        const __nv_bfloat16* b0 = reinterpret_cast<const __nv_bfloat16*>(&u0);
        const __nv_bfloat16* b1 = reinterpret_cast<const __nv_bfloat16*>(&u1);
        const __nv_bfloat16* b2 = reinterpret_cast<const __nv_bfloat16*>(&u2);
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float d = __bfloat162float(b0[j]);
          if (a1) d = __fadd_rn(d, __bfloat162float(b1[j]));
          if (a2) d = __fadd_rn(d, __bfloat162float(b2[j]));
          s += (double)d * (double)gv[j];
        }
      }
    } else {
      for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float d = __bfloat162float(a0[c]);
        if (a1) d = __fadd_rn(d, __bfloat162float(a1[c]));
        if (a2) d = __fadd_rn(d, __bfloat162float(a2[c]));
        s += (double)d * (double)g[c];
      }
    }
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

// out[0] = scale * sum of partials[0..n) (one block, fixed order: deterministic)
__global__ void scaled_sum_f64_kernel(const double* __restrict__ x, int n, double scale,
                                      double* out) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) out[0] = scale * v;
  }
}

// out[z][c][r] = in[z][r][c] for bf16 matrices [rows][ld_in] -> [cols][ld_out]: 64 x 64 tiles
// through shared memory, 16-byte row segments in and out when the strides allow (vec), single
// elements otherwise. skip_upper: tiles whose 128-column block lies strictly above their 128-row
// block (a causal matrix's zeros) are neither read nor written; a causal consumer that reduces
// from the 128-aligned start of each 128-row tile never reads their transposed copies.
__global__ void __launch_bounds__(256)
transpose_bf16_kernel(const __nv_bfloat16* __restrict__ in, int rows, int cols, int64_t ld_in,
                      int64_t bs_in, __nv_bfloat16* __restrict__ out, int64_t ld_out,
                      int64_t bs_out, int vec_in, int vec_out, int skip_upper) {
  __shared__ __align__(16) __nv_bfloat16 S[64][72];
  const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  if (skip_upper && (c0 >> 7) > (r0 >> 7)) return;
  const __nv_bfloat16* src = in + (int64_t)blockIdx.z * bs_in;
  __nv_bfloat16* dst = out + (int64_t)blockIdx.z * bs_out;
  const int t = threadIdx.x;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int r = (t >> 3) + 32 * p, c8 = (t & 7) * 8;
    const int gr = r0 + r, gc = c0 + c8;
    __align__(16) __nv_bfloat16 v[8];
    if (vec_in && gr < rows && gc + 8 <= cols) {
      *reinterpret_cast<uint4*>(v) = *reinterpret_cast<const uint4*>(src + (int64_t)gr * ld_in + gc);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        v[k] = (gr < rows && gc + k < cols) ? src[(int64_t)gr * ld_in + gc + k]
                                            : __float2bfloat16_rn(0.f);
    }
    *reinterpret_cast<uint4*>(&S[r][c8]) = *reinterpret_cast<const uint4*>(v);
  }
  __syncthreads();
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int c = (t >> 3) + 32 * p, r8 = (t & 7) * 8;
    const int gc = c0 + c, gr = r0 + r8;
    if (gc >= cols) continue;
    __align__(16) __nv_bfloat16 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = S[r8 + k][c];
    __nv_bfloat16* o = dst + (int64_t)gc * ld_out + gr;
    if (vec_out && gr + 8 <= rows) {
      *reinterpret_cast<uint4*>(o) = *reinterpret_cast<const uint4*>(v);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (gr + k < rows) o[k] = v[k];
    }
  }
}

// dV of a kv head = sum of the dV of its `rep` query heads, written as three bf16 terms
// transposed: in float32 [S * nh][T][64] (z = s * nh + h), out[kv * 64 + d][s * T + t].
__global__ void head_group_sum_t_kernel(const float* __restrict__ dv, int S, int nh, int rep, int T,
                                        __nv_bfloat16* __restrict__ o0, __nv_bfloat16* __restrict__ o1,
                                        __nv_bfloat16* __restrict__ o2, int64_t ld_o) {
  __shared__ float tile[32][33];
  const int nkv = nh / rep;
  const int sk = blockIdx.z;  // s * nkv + kv
  const int s = sk / nkv, kv = sk % nkv;
  const int t0 = blockIdx.y * 32, d0 = blockIdx.x * 32;
  for (int tt = threadIdx.y; tt < 32; tt += 8) {
    const int t = t0 + tt, dd = d0 + threadIdx.x;
    float acc = 0.f;
    if (t < T && dd < 64)
      for (int r = 0; r < rep; ++r) {
        const int64_t z = (int64_t)s * nh + kv * rep + r;
        acc = __fadd_rn(acc, dv[(z * T + t) * 64 + dd]);
      }
    tile[tt][threadIdx.x] = acc;
  }
  __syncthreads();
  for (int di = threadIdx.y; di < 32; di += 8) {
    const int dd = d0 + di, t = t0 + threadIdx.x;
    if (dd < 64 && t < T) {
      __nv_bfloat16 h, m, l;
      split3_bf16(tile[threadIdx.x][di], h, m, l);
      const int64_t o = (int64_t)(kv * 64 + dd) * ld_o + (int64_t)s * T + t;
      o0[o] = h; o1[o] = m; o2[o] = l;
    }
  }
}

}  // namespace gsq

using namespace gsq;

extern "C" int gsq_transpose_bf16(const void* in, int rows, int cols, int64_t ld_in, int64_t bs_in,
                                  void* out, int64_t ld_out, int64_t bs_out, int batch,
                                  int skip_upper, void* stream) {
  if (!in || !out || rows <= 0 || cols <= 0 || batch <= 0 || ld_in < cols || ld_out < rows ||
      batch > 65535)
    return GSQ_EINVAL;
  const int vec_in = ((uintptr_t)in % 16 == 0 && ld_in % 8 == 0 && bs_in % 8 == 0) ? 1 : 0;
  const int vec_out = ((uintptr_t)out % 16 == 0 && ld_out % 8 == 0 && bs_out % 8 == 0) ? 1 : 0;
  dim3 g((cols + 63) / 64, (rows + 63) / 64, batch);
  transpose_bf16_kernel<<<g, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)in, rows, cols, ld_in, bs_in, (__nv_bfloat16*)out, ld_out, bs_out,
      vec_in, vec_out, skip_upper ? 1 : 0);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_head_group_sum_t(const float* dv, int S, int nh, int rep, int T, void* o0,
                                    void* o1, void* o2, int64_t ld_o, void* stream) {
  if (!dv || !o0 || !o1 || !o2 || S <= 0 || nh <= 0 || rep <= 0 || nh % rep || T <= 0 ||
      ld_o < (int64_t)S * T)
    return GSQ_EINVAL;
  dim3 g(2, (T + 31) / 32, S * (nh / rep));
  head_group_sum_t_kernel<<<g, dim3(32, 8), 0, (cudaStream_t)stream>>>(
      dv, S, nh, rep, T, (__nv_bfloat16*)o0, (__nv_bfloat16*)o1, (__nv_bfloat16*)o2, ld_o);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_gather_split(const void* x, int src_bf16, int64_t ld_x, const int32_t* seq,
                                int per_seq, int64_t seq_stride, int offset, int rows, int cols,
                                int n_terms, void* const* row_terms, int64_t ld_t,
                                void* const* col_terms, int64_t ld_u, void* stream) {
  if (!x || !seq || per_seq <= 0 || rows <= 0 || cols <= 0 || n_terms < 1 || n_terms > 3 ||
      ld_x < cols || (!row_terms && !col_terms) || (row_terms && ld_t < cols) ||
      (col_terms && ld_u < rows))
    return GSQ_EINVAL;
  __nv_bfloat16* t[3] = {nullptr, nullptr, nullptr};
  __nv_bfloat16* u[3] = {nullptr, nullptr, nullptr};
  for (int i = 0; i < n_terms; ++i) {
    if (row_terms) t[i] = (__nv_bfloat16*)row_terms[i];
    if (col_terms) u[i] = (__nv_bfloat16*)col_terms[i];
  }
  cudaStream_t st = (cudaStream_t)stream;
  bool vec = !col_terms && cols % 8 == 0 && ld_x % 8 == 0 && ld_t % 8 == 0 &&
             ((uintptr_t)x & 15) == 0;
  for (int i = 0; i < n_terms; ++i) vec = vec && ((uintptr_t)t[i] & 15) == 0;
  if (vec) {
    const int64_t n = (int64_t)rows * (cols / 8);
    int64_t nb = (n + 255) / 256;
    if (nb > 65535) nb = 65535;
    if (src_bf16)
      gather_rows_kernel<__nv_bfloat16><<<(unsigned)nb, 256, 0, st>>>(
          (const __nv_bfloat16*)x, ld_x, seq, per_seq, seq_stride, offset, rows, cols, n_terms,
          t[0], t[1], t[2], ld_t);
    else
      gather_rows_kernel<float><<<(unsigned)nb, 256, 0, st>>>(
          (const float*)x, ld_x, seq, per_seq, seq_stride, offset, rows, cols, n_terms, t[0],
          t[1], t[2], ld_t);
    GSQ_CHECK_LAUNCH();
    return GSQ_OK;
  }
  dim3 g((cols + 31) / 32, (rows + 31) / 32);
  if (src_bf16)
    gather_split_kernel<__nv_bfloat16><<<g, dim3(32, 8), 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)x, ld_x, seq, per_seq, seq_stride, offset, rows, cols, n_terms,
        t[0], t[1], t[2], ld_t, u[0], u[1], u[2], ld_u);
  else
    gather_split_kernel<float><<<g, dim3(32, 8), 0, (cudaStream_t)stream>>>(
        (const float*)x, ld_x, seq, per_seq, seq_stride, offset, rows, cols, n_terms, t[0], t[1],
        t[2], ld_t, u[0], u[1], u[2], ld_u);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_dot_terms(const void* t0, const void* t1, const void* t2, int64_t ld_t,
                             const float* G, int64_t ld_g, int rows, int cols, double scale,
                             double* partials, double* out, void* stream) {
  if (!t0 || !G || !partials || !out || rows <= 0 || cols <= 0 || ld_t < cols || ld_g < cols)
    return GSQ_EINVAL;
  const uintptr_t al = (uintptr_t)t0 | (uintptr_t)t1 | (uintptr_t)t2 | (uintptr_t)G;
  const int vec = ((cols | ld_t | ld_g) & 7) == 0 && (al & 15) == 0;
  const int blocks = rows < 1024 ? rows : 1024;
  cudaStream_t st = (cudaStream_t)stream;
  dot_terms_kernel<<<blocks, 256, 0, st>>>(
      (const __nv_bfloat16*)t0, (const __nv_bfloat16*)t1, (const __nv_bfloat16*)t2, ld_t, G,
      ld_g, rows, cols, vec, partials);
  GSQ_CHECK_LAUNCH();
  scaled_sum_f64_kernel<<<1, 256, 0, st>>>(partials, blocks, scale, out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_sum_f64(const double* x, int n, double* out, void* stream) {
  if (!x || !out || n <= 0) return GSQ_EINVAL;
  sum_f64_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(x, n, out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
