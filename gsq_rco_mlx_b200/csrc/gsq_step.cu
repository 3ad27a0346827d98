// Operand staging of the GSQ step: gather the micro-batch rows (positions 1.. of the chosen
// calibration sequences) and split them into bf16 terms in both the row-major layout (the
// K-major A operand of the forward residual GEMM) and the transposed layout (the K-major B
// operand of the weight-gradient GEMM, reduction over rows), in one pass; plus a float64
// sum used for the per-tile loss partials.
#include "common.cuh"

namespace gsq {

__global__ void gather_split_kernel(const float* __restrict__ x, int64_t ld_x,
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
      v = x[src * ld_x + c];
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

}  // namespace gsq

using namespace gsq;

extern "C" int gsq_gather_split(const float* x, int64_t ld_x, const int32_t* seq, int per_seq,
                                int64_t seq_stride, int offset, int rows, int cols, int n_terms,
                                void* const* row_terms, int64_t ld_t, void* const* col_terms,
                                int64_t ld_u, void* stream) {
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
  dim3 g((cols + 31) / 32, (rows + 31) / 32);
  gather_split_kernel<<<g, dim3(32, 8), 0, (cudaStream_t)stream>>>(
      x, ld_x, seq, per_seq, seq_stride, offset, rows, cols, n_terms, t[0], t[1], t[2], ld_t,
      u[0], u[1], u[2], ld_u);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

extern "C" int gsq_sum_f64(const double* x, int n, double* out, void* stream) {
  if (!x || !out || n <= 0) return GSQ_EINVAL;
  sum_f64_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(x, n, out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
