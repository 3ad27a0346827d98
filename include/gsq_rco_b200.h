/* gsq_rco_b200.h: C ABI of the B200 (sm_100a) kernels behind the GSQ / GPTQ / RCO hot path.
 *
 * The reference (egesabanci/gsq-rco-mlx) is pure Python: its "boundary" is its module API.
 * Each entry point below replaces the reference function cited beside it; the Python
 * package gsq_rco_mlx_b200 binds them through ctypes and keeps the reference's names,
 * argument meaning and error behaviour.
 *
 * Conventions
 *   - Every pointer is DEVICE memory unless stated otherwise; sizes are element counts.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Calls are asynchronous.
 *   - Return value: GSQ_OK (0) or a nonzero status; a bad argument never launches a kernel.
 *     Kernels never trap: device-side failures (e.g. a non-positive-definite Hessian) are
 *     reported through a device `info` word that the caller reads back.
 *   - Row-major everywhere. GSQ logits and their momentum are plane-major [K][d]
 *     (K = 5 local-shift candidates for 3..7 bits, K = 4 grid values for 2 bits),
 *     d = out_f * in_f, weight index i = row * in_f + col. Group scales are [out_f][G],
 *     G = ceil(in_f / group_size).
 */
#ifndef GSQ_RCO_B200_H
#define GSQ_RCO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  GSQ_OK = 0,
  GSQ_EINVAL = 1,   /* bad argument or size */
  GSQ_ECUDA = 2,    /* CUDA launch / runtime error */
  GSQ_ETIMEOUT = 3, /* a bounded device wait gave up */
  GSQ_ENOTSUP = 4   /* valid request that this build does not implement */
};

/* ABI revision of this header; bumps on any signature change. */
int gsq_abi_version(void);
/* Static, human-readable text of a status code. */
const char *gsq_status_string(int status);

/* ------------------------------------------------------------------ GSQ ---------- */

/* Soft weight of one Gumbel-softmax draw (the forward of the first step of a stage):
 *   p = softmax((kappa * l + g) * (1 / tau)) over the K candidates, c = sum_k p_k C_k,
 *   w_bar[o, i] = scales[o, i / group_size] * c,  out = w_bar - w_ref (w_ref may be NULL).
 * C_k = grid[clip(j0 + k - 2)] (bits 3..7) or grid[k] (bits 2). Gumbel g comes from `noise`
 * ([K][d] float32, host-supplied) or, if noise == NULL, from one Philox4x32-10 call per
 * weight with key (seed, linear_id) and counter (i, 0, step, resample): plane k < 4 from the
 * high 24 bits of word k, plane 4 from the low bytes of words 0..2; g = -log(-log u) with
 * u = (bits + 0.5) 2^-24 clipped to [1e-7, 1 - 1e-7].
 * Outputs (at least one): w_out float32 [out_f][in_f]; w_terms bf16 [3][out_f][in_f] with
 * out == t0 + t1 + t2 to float32 precision (the GEMM operand); p_out float32 [K][d].
 * bits 1 (ternary, grid [-1, 0, 1]): logits are the two planes [2][d] (mask lm, sign lb), the
 * Gumbel planes are four [4][d] (all four Philox words' high 24 bits), and
 *   m = sigmoid((2 kappa lm + (g1 - g0)) * (1 / tau)),  v = sigmoid((2 kappa lb + (g3 - g2)) * (1 / tau)),
 *   c = m (2 v - 1);  p_out holds the planes (m, v); j0 is unused.
 * Replaces: src/gsq_rco/gsq/staged.py:271-298 (_Linear.soft) with :82-84 (_gs_softmax),
 * :87-89 (_binary_gs), :92-96 (_gumbel), :99-106 (_grid_rows, _shift_rows), :109-115
 * (_ternary_rows); the residual of staged.py:327. */
int gsq_soft_fwd(const float *logits, const uint8_t *j0, const float *scales, const float *noise,
                 uint64_t seed, uint32_t linear_id, uint32_t step, uint32_t resample,
                 int out_f, int in_f, int group_size, int bits, float tau, float kappa,
                 const float *w_ref, float *w_out, void *w_terms, float *p_out, void *stream);

/* One fused pass per GSQ step over the training state of a linear:
 *   backward of this step from the stored probabilities probs [R][K][d] and the weight
 *   gradients grad_w [R][out_f][in_f] (dL/dw_bar per resample):
 *     u_k = s G C_k,  dL/dl = (kappa / tau) p (u - <p, u>),  dL/ds = sum over the group of G c,
 *   summed over the R resamples and divided by R; one Lion step
 *     m' = b1 m + (1 - b1) g;  p <- p - lr (sign(m') + wd p);  m <- b2 m + (1 - b2) g
 *   on logits/mom_logits (lr_logits) and scales/mom_scales (lr_scales; 0 freezes them);
 *   then, if next != 0, the forward of step next_step with the updated state: new
 *   probabilities into probs (in place) and the soft weights (minus w_ref) into w_out
 *   [R][out_f][in_f] float32 and/or w_terms bf16 [R][3][out_f][in_f]. noise_next: host-supplied
 *   Gumbel planes [R][K][d] of the next step, or NULL for Philox (as gsq_soft_fwd).
 * bits 1 (ternary): probs holds the planes (m, v) per resample ([R][2][d]), noise_next is
 * [R][4][d], and the logit gradients are
 *   dL/dlm = (2 kappa / tau) s G (2 v - 1) m (1 - m),  dL/dlb = (2 kappa / tau) s G m 2 v (1 - v).
 * The betas and wd are the caller's float64 values, each of b, 1 - b, wd rounded to float32
 * once (MLX's treatment of Python scalars). resamples: 1..8; group_size <= 256 (any for bits 1).
 * Replaces: the MLX autodiff of staged.py:322-329 through :271-298, the resample average of
 * staged.py:383-390, lion_update src/gsq_rco/gsq/lion.py:44-56, and the next step's
 * _Linear.soft (staged.py:271-298). */
int gsq_soft_step(float *logits, float *mom_logits, const uint8_t *j0, float *scales,
                  float *mom_scales, float *probs, const float *grad_w, int resamples, int out_f,
                  int in_f, int group_size, int bits, float tau, float kappa, float lr_logits,
                  float lr_scales, double wd, double beta1, double beta2, int next,
                  const float *noise_next, uint64_t seed, uint32_t linear_id, uint32_t next_step,
                  float tau_next, float kappa_next, const float *w_ref, float *w_out,
                  void *w_terms, void *stream);

/* gsq_soft_step under the name the reference-facing contract gives the fused soft backward +
 * Lion step (+ the next step's forward): identical arguments, behaviour and status codes. */
int gsq_soft_bwd_lion(float *logits, float *mom_logits, const uint8_t *j0, float *scales,
                      float *mom_scales, float *probs, const float *grad_w, int resamples,
                      int out_f, int in_f, int group_size, int bits, float tau, float kappa,
                      float lr_logits, float lr_scales, double wd, double beta1, double beta2,
                      int next, const float *noise_next, uint64_t seed, uint32_t linear_id,
                      uint32_t next_step, float tau_next, float kappa_next, const float *w_ref,
                      float *w_out, void *w_terms, void *stream);

/* Argmax decode of trained logits to uint8 codes [out_f][in_f] (first maximum wins;
 * local shift clipped to the grid; ternary: code 1 (value 0) where lm < 0, else 2 (+1) where
 * lb >= 0 and 0 (-1) where lb < 0). Replaces staged.py:300-314 (_Linear.hard_codes) and
 * src/gsq_rco/gsq/quant.py:75-83 (local_shift_indices). */
int gsq_harden(const float *logits, const uint8_t *j0, int out_f, int in_f, int bits,
               uint8_t *codes, void *stream);

/* One Lion step on a flat float32 tensor. Replaces src/gsq_rco/gsq/lion.py:44-56. */
int gsq_lion_f32(float *param, float *mom, const float *grad, int64_t n, float lr, double wd,
                 double beta1, double beta2, void *stream);

/* ------------------------------------------------------------- contractions ------ */

/* C[m, n] = alpha * sum_k A(m, k) B(k, n) + beta * C[m, n], float32 CUDA-core GEMM with
 * arbitrary element strides: A(m, k) = A[m*sam + k*sak], B(k, n) = B[k*sbk + n*sbn].
 * Replaces the float32 products of staged.py:327 (X (W_bar - W)^T and its MLX backward). */
int gsq_gemm_f32(int M, int N, int K, float alpha, const float *A, int64_t sam, int64_t sak,
                 const float *B, int64_t sbk, int64_t sbn, float beta, float *C, int64_t ldc,
                 void *stream);

/* Same in float64; tri = 1 computes only the lower triangle n <= m of C.
 * Replaces the float64 products of src/gsq_rco/gsq/gptq.py:98,118,154,182,186. */
int gsq_gemm_f64(int M, int N, int K, double alpha, const double *A, int64_t sam, int64_t sak,
                 const double *B, int64_t sbk, int64_t sbn, double beta, double *C, int64_t ldc,
                 int tri, void *stream);

/* Descriptor of one (batched) tensor-core GEMM with a fused epilogue, gsq_gemm below.
 * Batch z of `batch`: A rows start at a_off(z), B rows at b_off(z), C / cs / resid / target /
 * aux elements at c_off(z), C^T rows / columns at t_row(z) / t_col(z), where an offset is
 * (z / div) * s1 + (z % div) * s2. a_rows / b_rows: total rows of the A / B matrices. */
typedef struct {
  int M, N, K, batch;
  const void *a[3];
  int na;
  int64_t lda;
  int64_t a_rows;
  const void *b[3];
  const void *b2[3]; /* SwiGLU forward: the "up" rows, paired with the "gate" rows of b */
  int nb;
  int64_t ldb;
  int64_t b_rows;
  int order, causal, epi, bn;
  float alpha, beta;
  float *C;
  int64_t ldc;
  void *cs[3];
  int ncs;
  int64_t ldcs;
  void *ct[3];
  int nct;
  int64_t ldct;
  int64_t ct_up_rows;
  double *sq_partial;
  const float *bias;
  const void *resid;
  const void *target;
  int64_t ld_rt;
  float out_scale;
  float *aux0;
  float *aux1;
  int64_t ld_aux;
  int a_div;
  int64_t a_s1, a_s2;
  int b_div;
  int64_t b_s1, b_s2;
  int c_div;
  int64_t c_s1, c_s2;
  int t_div;
  int64_t t_r1, t_r2, t_c1, t_c2;
  int *err;
  int skip_upper; /* skip output tiles with n >= m (all above the diagonal): causal scores */
  int row_period; /* epi 1: rows m with m % row_period == 0 get a zero residual (position 0) */
  /* split_k > 1 (epi 0, batch 1, C only: no bias / terms / sq_partial, not causal): the k-range
   * is cut into split_k contiguous parts whose partial products land in workspace
   * (float32, >= split_k * M * N) and are summed in part order, then C = alpha sum + beta C. */
  int split_k;
  float *workspace;
  /* operand layout: 0 = K-major (A [M][lda], B [N][ldb], the reduction index contiguous);
   * 1 = MN-major (A stored [K][lda] with the M index contiguous, B [K][ldb] with N contiguous:
   * a row-major activation used as its own transpose). An MN-major B needs batch 1, no causal
   * range and no SwiGLU pairing (b2); an MN-major A may be batched (a_off then moves along its
   * K rows) or causal when K is a multiple of 64. */
  int a_major, b_major;
  /* TMEM accumulators for a tile's cross products (the products below hi x hi) when there are
   * any: 2 lets the next tile's MMAs start before the epilogue has read this tile's; 1 gives
   * that TMEM to one more chunk of the hi x hi ring instead; 0 = 1 for epi 1, 2, 3 and 2 for
   * the others. Same results either way. */
  int small_bufs;
} gsq_gemm_desc;

/* Batched float32-faithful tensor-core GEMM with a fused epilogue (see gsq_gemm_tc for the
 * arithmetic). bn: tile width 64 or 128. causal: batch rows m only reduce over k < the end of
 * their 128-row tile (a causal probability matrix whose upper triangle is zero).
 * epi 0: x = alpha acc + bias[n] (+ beta C) -> C, cs terms, ct terms, per-tile sum of x^2.
 * epi 1: r = alpha acc + bias[n] + resid[m, n] - target[m, n] (bf16 resid / target, resid may
 *        be NULL); per-tile sum of r^2; x = out_scale r -> C, cs, ct (the stage-loss residual
 *        and its gradient).
 * epi 2: SwiGLU forward. B rows: 64-row blocks of b (gate) and b2 (up) interleaved per tile,
 *        N = 2 * width. g, u -> aux0, aux1 float32 [M][ld_aux]; silu(g) u -> cs, ct.
 * epi 3: SwiGLU backward. acc = dL/d(silu(g) u) of column n; with g, u from aux0 / aux1:
 *        dL/dg -> ct rows n, dL/du -> ct rows n + ct_up_rows.
 * epi 4: bf16 chain of a bf16 model: x = bf16(alpha acc); x = bf16(x + bias[n]) if bias;
 *        x = bf16(resid[m, n] + x) if resid -> C (float32 of the bf16 value), cs, ct (1 term
 *        each is the bf16 value itself).
 * epi 5: bf16 SwiGLU (b / b2 as in epi 2): g, u = bf16(acc); bf16(bf16(g bf16(sigmoid(g))) u)
 *        -> cs, ct; with aux0 / aux1 also g, u (bf16 values, float32 [M][ld_aux]).
 * epi 6: its backward with bf16 cotangents: dd = bf16(acc) of column n, g, u from aux0 / aux1;
 *        s = bf16(sigmoid g), a = bf16(g s): du = bf16(dd a), da = bf16(dd u), ds = bf16(da g),
 *        dg = bf16(da s + ds sigmoid(g)(1 - sigmoid(g))) -> cs (1 term) at columns n and
 *        n + ct_up_rows, ct (1 term) at rows n and n + ct_up_rows.
 * Replaces the block matmuls of src/gsq_rco/gsq/e2e.py:132-134,155,166,170,173 in the stage
 * losses of src/gsq_rco/gsq/staged.py:332-354 and their MLX backward. */
int gsq_gemm(const gsq_gemm_desc *desc, void *stream);

/* The same GEMM as a plan: gsq_gemm_plan_create checks desc and encodes its tensor maps once
 * (host memory only, no device allocation); gsq_gemm_plan_run launches it on a stream with the
 * buffers, shapes and scalars desc named at creation (they must stay valid and unmoved);
 * gsq_gemm_plan_destroy frees it. A step that repeats the same GEMMs on the same buffers pays
 * the descriptor checks and the tensor-map encoding once instead of at every launch. Same
 * results as gsq_gemm. */
int gsq_gemm_plan_create(const gsq_gemm_desc *desc, void **plan);
int gsq_gemm_plan_run(const void *plan, void *stream);
int gsq_gemm_plan_destroy(void *plan);

/* Float32-faithful tensor-core GEMM (tcgen05, TMEM accumulator, TMA-fed):
 *   C[m, n] = alpha * sum_k A(m, k) B(n, k) (+ beta * C[m, n])
 * A and B arrive as na / nb bf16 terms (A = sum_i A_i), each K-major [M][lda] / [N][ldb]
 * (lda, ldb multiples of 8, 16-byte aligned bases); the products A_i B_j with i + j <= order
 * are accumulated in float32 (three terms per side, order 2: float32 operands to 2^-24;
 * an exactly-bf16 operand needs one term). Epilogue outputs (each optional):
 *   C float32 [M][ldc];  c_terms: C as ncs bf16 terms [M][ldcs];
 *   ct_terms: C^T as nct bf16 terms [N][ldct] (the K-major operand of a reduction over m);
 *   sq_partial: float64 per 128 x 128 tile, the sum of C^2 (ceil(M/128) * ceil(N/128)).
 * err: device int, nonzero if a bounded wait timed out.
 * Replaces the float32 matmuls of staged.py:327 and their MLX backward, and the block
 * matmuls of src/gsq_rco/gsq/e2e.py:132-134,166,170,173 inside the stage losses. */
int gsq_gemm_tc(int M, int N, int K, const void *const *a_terms, int na, int64_t lda,
                const void *const *b_terms, int nb, int64_t ldb, int order, float alpha,
                float *C, int64_t ldc, float beta, void *const *c_terms, int ncs, int64_t ldcs,
                void *const *ct_terms, int nct, int64_t ldct, double *sq_partial, int *err,
                void *stream);

/* x float32 [rows][ld_in] -> bf16 terms t0 (+ t1, t2 if non-NULL) with x = t0 + t1 + t2 to
 * float32 precision; transpose = 1 writes [cols][ld_out]. */
int gsq_split_bf16(const float *x, int rows, int cols, int64_t ld_in, int transpose, void *t0,
                   void *t1, void *t2, int64_t ld_out, void *stream);

/* Micro-batch operand staging of the GSQ step: output row r is source row
 * seq[r / per_seq] * seq_stride + offset + r % per_seq of x float32 [.][ld_x] (positions 1..T-1
 * of the chosen sequences: per_seq = T - 1, seq_stride = T, offset = 1). Writes n_terms bf16
 * terms row-major [rows][ld_t] (row_terms) and/or transposed [cols][ld_u] (col_terms).
 * Replaces the micro-batch draw of staged.py:380 with _rows :128-130 (and _take :124-125). */
int gsq_gather_split(const void *x, int src_bf16, int64_t ld_x, const int32_t *seq, int per_seq,
                     int64_t seq_stride, int offset, int rows, int cols, int n_terms,
                     void *const *row_terms, int64_t ld_t, void *const *col_terms, int64_t ld_u,
                     void *stream);

/* out[z] = in[z]^T for bf16 matrices [rows][ld_in] (batch stride bs_in) -> [cols][ld_out].
 * skip_upper: input tiles whose 128-column block lies strictly above their 128-row block (a
 * causal matrix's zeros) are skipped and their transposed copies left unwritten (a causal
 * consumer reducing from the 128-aligned start of each 128-row tile never reads them). */
int gsq_transpose_bf16(const void *in, int rows, int cols, int64_t ld_in, int64_t bs_in, void *out,
                       int64_t ld_out, int64_t bs_out, int batch, int skip_upper, void *stream);

/* The value gradient of each kv head, summed over its rep query heads (GQA repeat of
 * src/gsq_rco/gsq/e2e.py:146-148, backward), as three bf16 terms transposed:
 * dv float32 [S * nh][T][64] -> o[kv * 64 + d][s * T + t]. */
int gsq_head_group_sum_t(const float *dv, int S, int nh, int rep, int T, void *o0, void *o1,
                         void *o2, int64_t ld_o, void *stream);

/* out[0] = scale * sum over r < rows, c < cols of (t0 + t1 + t2)[r][c] * G[r][c] for a matrix
 * held as bf16 terms (t1, t2 may be NULL; rows of ld_t elements) and a float32 G (rows of ld_g),
 * products and sums in float64, deterministic. partials: >= 1024 doubles. The qk-stage loss
 * mean((X D^T)^2) = sum D (D X^T X) / (M out) from D = w_bar - W and G = 2 D X^T X / (M out)
 * (src/gsq_rco/gsq/staged.py:327-328). */
int gsq_dot_terms(const void *t0, const void *t1, const void *t2, int64_t ld_t, const float *G,
                  int64_t ld_g, int rows, int cols, double scale, double *partials, double *out,
                  void *stream);

/* out[0] = sum of x[0..n) in float64 (one block; the loss from per-tile partials). */
int gsq_sum_f64(const double *x, int n, double *out, void *stream);

/* out[0] = sum_i x[i]^2 in float64 (deterministic two-pass). partials: >= 1024 doubles.
 * Replaces the mean of R^2 in staged.py:328 (the caller divides by the count). */
int gsq_sumsq_f32(const float *x, int64_t n, double *partials, double *out, void *stream);

/* ------------------------------------------------------------ decoder block -------- */

/* y = bf16((x * (1 / sqrt(mean(x^2) + eps))) * w) per row of x bf16 [rows][ld_x], H columns
 * (mean from a float64 sum of the float32 squares). y bf16 [rows][ld_y] and/or the transposed
 * yt bf16 [H][ld_yt]; zero_pos0 writes zeros to yt for rows r with r % seq_len == 0.
 * Replaces src/gsq_rco/gsq/e2e.py:90-93 (rmsnorm). */
int gsq_rmsnorm(const void *x, int64_t ld_x, const void *w, int rows, int H, float eps, void *y,
                int64_t ld_y, void *yt, int64_t ld_yt, int seq_len, int zero_pos0, void *stream);

/* Half-split rotary embedding of bf16 q or k x [S*T][ld_x] (nh heads of 64 at column h*64),
 * float32 [x1 c - x2 s, x1 s + x2 c] with cos / sin float32 [T][32], written as three bf16
 * terms head-major o[(s * nh + h) * T + t][64]. Replaces src/gsq_rco/gsq/e2e.py:96-108,145. */
int gsq_rope_split(const void *x, int64_t ld_x, int S, int T, int nh, const float *cosv,
                   const float *sinv, void *o0, void *o1, void *o2, void *stream);

/* Causal softmax of score rows S float32 [B*T][T] (keys <= query): P bf16 [B*T][T] with zeros
 * above the diagonal, and optionally PT bf16 [B][T][T] (P transposed per batch). Without PT
 * (and T % 4 == 0, 16-byte aligned S, 8-byte aligned P) each row is written only up to the
 * end of its 128-key block, the part the causal P V and transposed products read.
 * Replaces src/gsq_rco/gsq/e2e.py:149-154 (mask, softmax, cast to bf16). */
int gsq_softmax_causal(const float *S, int B, int T, void *P, void *PT, void *stream);

/* Row window of the causal softmax (data-parallel query rows): local row i of batch z is query
 * position row0 + i and sees keys k <= row0 + i of the cols stored (row0 + rows <= cols).
 * S float32 [B][rows][ld_s] -> P bf16 [B][rows][ld_p], masked keys k < cols written as 0; with
 * row0 == 0 and cols, ld_s, ld_p multiples of 4 (S 16-byte, P 8-byte aligned) the zeros stop at
 * the end of each query's 128-key block, as in gsq_softmax_causal (the causal P V product and
 * the causal transpose read no key beyond it). Same arithmetic as gsq_softmax_causal
 * (src/gsq_rco/gsq/e2e.py:149-155). */
int gsq_softmax_causal_rows(const float *S, int B, int rows, int cols, int64_t ld_s, int row0,
                            void *P, int64_t ld_p, void *stream);

/* out[r] = E[ids[r]] (bf16 rows of H). Replaces the embedding lookup of the calibration
 * stream (src/gsq_rco/gsq/pipeline.py's block inputs, e2e.py:64-74). */
int gsq_embed(const int32_t *ids, int64_t n, const void *E, int H, void *out, void *stream);

/* x[r][c] = 0 (bf16) for the columns c < cols with c % period == 0: position 0 of every
 * sequence in a transposed activation buffer (Hessians skip it, staged.py:14-15,128-130). */
int gsq_zero_cols(void *x, int rows, int64_t ld, int cols, int period, void *stream);

/* H <- beta H + alpha G, float64 H and float32 G of n elements (a Gram matrix accumulated by
 * the tensor cores folded into the float64 Hessian). Replaces gptq.py:97-100. */
int gsq_hess_accum(double *H, const float *G, int64_t n, double beta, double alpha, void *stream);

/* ------------------------------------------------------------------- GPTQ -------- */

/* Streaming Hessian H <- H * n_prev / (n_prev + m) + 2 / (n_prev + m) X^T X, float64 H
 * [k][k], float32 rows X [m][k]. Replaces src/gsq_rco/gsq/gptq.py:89-101
 * (hessian_from_inputs) and src/gsq_rco/gsq/staged.py:143-155 (hessian_add). */
int hessian_accum(const float *X, int64_t m, int k, double *H, int64_t n_prev, void *stream);

/* Upper factor U of (H + damp * mean(diag H) I)^-1 = U^T U, after the dead-input rule
 * (H_ii == 0 -> H_ii = 1, flagged in dead[i]). U [n][n] float64 (upper triangle; the strict
 * lower triangle is zero). workspace: 2*n*n + 64 doubles. info (device int): 0, or j + 1 if the
 * damped Hessian is not positive definite at column j.
 * Replaces src/gsq_rco/gsq/gptq.py:143-157 and _tri_inv_lower :104-120. */
int gptq_factor(const double *H, int n, double damp, double *U, uint8_t *dead,
                double *workspace, int *info, void *stream);

/* Blocked GPTQ column sweep with signed group scales and lazy block updates, every output
 * row independent. W float32 [out_f][in_f]; codes uint8 [out_f][in_f]; scales float32
 * [out_f][G]; Wwork float64 [out_f][in_f] scratch.
 * Replaces src/gsq_rco/gsq/gptq.py:159-182 with _encode :31-36 and _group_scales :43-51. */
int gptq_sweep(const float *W, const double *U, const uint8_t *dead, int out_f, int in_f,
               int bits, int group_size, int block_size, int signed_scale, uint8_t *codes,
               float *scales, double *Wwork, void *stream);

/* w_q[o, i] = scales[o, i / group_size] * grid[codes[o, i]] (float32).
 * Replaces src/gsq_rco/gsq/gptq.py:63-73 and src/gsq_rco/rco/database.py:244-256. */
int gptq_dequant(const uint8_t *codes, const float *scales, int out_f, int in_f, int bits,
                 int group_size, float *w_q, void *stream);

/* err[0] = 1/2 tr(D H D^T), D = w_q - W (float64). workspace: 2*out_f*in_f + 1024 doubles.
 * Replaces src/gsq_rco/gsq/gptq.py:184-186. */
int gptq_err(const float *w_q, const float *W, const double *H, int out_f, int in_f,
             double *err, double *workspace, void *stream);

/* --------------------------------------------------------------------- RCO -------- */

/* Exact multiple-choice knapsack DP, one CTA per instance (Gumbel sample):
 * maximise sum_i s[i, k_i] subject to sum_i step[i, k_i] <= budget, float64 values, strict
 * '>' (lowest option keeps ties), backtrack from the smallest budget reaching the optimum.
 * scores [n_inst][N][K] float64, step [N][K] int64 (w_i * c_k), choice_ws uint8
 * [n_inst][N][budget + 1] scratch, z_out int32 [n_inst][N] chosen option per group.
 * The two DP rows live in shared memory when 2 * (budget + 1) doubles fit (budget <= 13823);
 * larger budgets use dp_ws float64 [n_inst][2][budget + 1] (may be NULL otherwise).
 * step entries must be >= 0. An instance with a negative step entry, or with no assignment
 * whose cost fits the budget, gets z_out = -1 in all N entries (nothing is read outside the
 * instance's table).
 * Replaces src/gsq_rco/rco/manifold.py:304-334 (_mckp_dp). */
int mckp_dp_f64(const double *scores, const int64_t *step, int n_inst, int N, int K,
                int64_t budget, uint8_t *choice_ws, double *dp_ws, int32_t *z_out,
                void *stream);

/* Allocation-free variant of mckp_dp_f64, for callers that cannot allocate device memory
 * (a runtime that owns every device byte through its own pool, a host language binding
 * without a CUDA allocator). No counterpart in the reference, whose DP runs in numpy.
 * The choice table lives in a fixed 16 MiB array inside the library (every GPU that loads the
 * library holds it until exit); the DP rows live in shared memory. Limits: budget <= 13823 and
 * n_inst * N * (budget + 1) <= 16 MiB, else GSQ_EINVAL. The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress): make it before any stream capture. The
 * address is kept for the life of the process, so do not call this across a cudaDeviceReset
 * of that device. Calls share the array: calls whose kernels overlap on one GPU race, so serialise them.
 * Nothing is allocated or freed. Same results as mckp_dp_f64 (z_out = -1 as there). */
int mckp_dp_f64_noalloc(const double *scores, const int64_t *step, int n_inst, int N, int K,
                        int64_t budget, int32_t *z_out, void *stream);

/* ------------------------------------------------------------ RCO objective -------- */

/* Row pass of the tied-embedding KL head (src/gsq_rco/common/evaluate.py:111-151,
 * kl_value_and_grad_hidden / _kl_chunk_value_grad): zq, zr bf16 [n][ld] logits (bf16(h E^T) of the
 * quantized and the reference stream, V = vocabulary, V % 8 == 0, 16-byte aligned rows). Per
 * row: lse = logsumexp(z) (float32, float64 sum of exp), q = exp(zq - lse_q),
 * p = exp(zr - lse_r), kl_rows[r] = sum p (zr - lse_r - zq + lse_q) (float64), D = bf16(q - p)
 * [n][ld_d] (the logit gradient; dKL/dh_q = D E by a tensor-core GEMM). lse: optional float32
 * [n][2] (lse_q, lse_r). The logit GEMMs and D E run through gsq_gemm (epi 4). */
int gsq_kl_rows(const void *zq, const void *zr, int n, int V, int64_t ld, void *D, int64_t ld_d,
                double *kl_rows, float *lse, void *stream);

/* The RCO objective's KL head, forward and backward, over n rows in chunks of <= chunk rows:
 * per chunk zq = bf16(h_q E^T) and zr = bf16(h_ref E^T) (tensor-core GEMMs, bf16-chain
 * epilogue), kl_rows[r] = KL(p_ref || p_q) and D = bf16(q - p) (gsq_kl_rows), grad =
 * bf16(D E) (tensor-core GEMM against ET); then total[0] = the float64 sum of kl_rows.
 * h_q, h_ref bf16 [n][H]; E bf16 [V][H]; ET bf16 [H][ld_et] (E transposed); zq, zr, D bf16
 * work buffers [chunk][V]; kl_rows float64 [n]; grad bf16 [n][H], the gradient of the sum (the
 * mean's is grad / n: gsq_div_bf16). err: the GEMMs' device error word (zeroed by the caller,
 * nonzero after a bounded wait gave up). H, V and ld_et multiples of 8, ld_et >= V. The
 * launches and their order are those of the library's Python KL head (rco/kl.py).
 * Replaces src/gsq_rco/common/evaluate.py:111-151 (kl_value_and_grad_hidden with its 64-row
 * chunks, :28-33 the tied-embedding logits). */
int kl_head_fwd_bwd(const void *h_q, const void *h_ref, int n, int H, const void *E,
                    const void *ET, int64_t ld_et, int V, int chunk, void *zq, void *zr, void *D,
                    double *kl_rows, double *total, void *grad, int *err, void *stream);

/* w bf16 [out][in] = bf16(scales[r][c / gs] * grid[codes[r, c]]): a database candidate
 * assembled in the model dtype (src/gsq_rco/rco/database.py:244-256, allocate.py:117). */
int gsq_dequant_bf16(const uint8_t *codes, const float *scales, int out_f, int in_f, int bits,
                     int group_size, void *w, void *stream);

/* x = bf16(f32(x) / divisor) for n bf16 elements (the head gradient's mean over positions,
 * evaluate.py:150). */
int gsq_div_bf16(void *x, int64_t n, float divisor, void *stream);

/* Straight-through upstream of one linear (src/gsq_rco/rco/allocate.py:169-174, _dots):
 * out[k] = sum G * (f32(bf16(scales_k[r][c / gs] * grid_k[codes_k[r, c]])) - f32(W[r, c])) in
 * float64 for the K <= 8 database options (codes_k uint8 [out][in], scales_k float32
 * [out][ceil(in / gs)], bits_k in 1..8). G float32 [out][in] = dL/dW, W bf16 [out][in] the
 * reference weight. partials: >= max_blocks * K doubles. */
int ste_dots(const float *G, const void *W, int out_f, int in_f, int group_size, int K,
             const uint8_t *const *codes, const float *const *scales, const int *bits,
             double *partials, int max_blocks, double *out, void *stream);

/* ------------------------------------------------ decoder block backward (RCO) ------ */
/* The per-layer vjp of the RCO objective (src/gsq_rco/rco/allocate.py:156-167): cotangents of
 * bf16 forward tensors are rounded to bf16, float32 ones (scores, RoPE'd q / k) stay float32. */

/* out = bf16(resid + bf16(dx)) with dx the cotangent of x for the RMSNorm y = (x inv) w
 * (e2e.py:90-93), inv = 1 / sqrt(mean x^2 + eps) in float64; resid may be NULL. bf16 rows. */
int gsq_rmsnorm_bwd(const void *x, int64_t ld_x, const void *w, const void *dy, int64_t ld_dy,
                    const void *resid, int64_t ld_r, void *out, int64_t ld_o, int rows, int H,
                    double eps, void *stream);

/* dS = scale Pf (dP - sum_k dP Pf) of the causal softmax Pf = softmax(S) (recomputed from the
 * float32 scores S [B*T][T] as gsq_softmax_causal does), dP bf16 [B*T][ld_p]; dS as three bf16
 * terms [B*T][ld_o] (zeros for keys > query). e2e.py:149-155 backward. */
int gsq_softmax_bwd(const float *S, const void *dP, int B, int T, int64_t ld_p, void *o0,
                    void *o1, void *o2, int64_t ld_o, float scale, void *stream);

/* RoPE backward (e2e.py:103-108): dy float32 [(s nh + h) T + t][ld_i] (64 per head) ->
 * bf16(rotation^T dy) at out[s T + t][col0 + h 64 + d]. */
int gsq_rope_bwd(const float *dy, int64_t ld_i, int S, int T, int nh, const float *cosv,
                 const float *sinv, void *out, int64_t ld_o, int col0, void *stream);

/* GQA cotangent sum (e2e.py:146-148 backward): in float32 [(s nh + h) T + t][ld_i] summed over
 * the rep query heads of each kv head -> out_f float32 [(s nkv + kv) T + t][64] and / or out_b
 * bf16 at [s T + t][col0 + kv 64 + d] (ld_o). */
int gsq_group_sum(const float *in, int64_t ld_i, int S, int nh, int rep, int T, float *out_f,
                  void *out_b, int64_t ld_o, int col0, void *stream);

/* Group-scale gradient of a stored-form linear with fixed codes (App-H scale fine-tune,
 * src/gsq_rco/gsq/staged.py:555-634): out[r][g] = sum over the columns c of group g of
 * G[r][c] grid[code[r][c]], G float32 [out_f][in_f] the weight gradient, out float32
 * [out_f][ceil(in_f / group_size)] (float64 sums). */
int gsq_scale_grad(const float *G, const uint8_t *codes, int out_f, int in_f, int bits,
                   int group_size, float *out, void *stream);

/* ---- packed quantized-model eval (MLX affine export format) ----
 * A packed linear W [N][K] (src/gsq_rco/gsq/export.py:60-90, pack_codes / to_mlx_affine):
 * words u32 [N][K bits / 32], value k of row n at stream bits [k bits, (k + 1) bits), least
 * significant bit first, little-endian words; scales and biases [N][K / group_size] of
 * scale_dtype 0 = bf16, 1 = f16, 2 = f32; w = scale q + bias (float32, exact), rounded to bf16.
 * bits in {2, 3, 4, 5, 6, 8}, group_size in {32, 64, 128} dividing K; words aligned to 16 bytes
 * (bits 4, 8), 8 bytes (2, 6) or 4 bytes (3, 5). */

/* out bf16 [N][ldw] = the bf16 dense weight (ldw % 8 == 0, 16-byte aligned): the dequant of
 * mx.dequantize (export.py:87-90 inverse) as one HBM stream. */
int qdequant_packed(const uint32_t *words, const void *scales, const void *biases,
                    int scale_dtype, int N, int K, int bits, int group_size, void *out,
                    int64_t ldw, void *stream);

/* Y [M][ld_y] = X W^T (X bf16 [M][ld_x], 16-byte aligned, ld_x % 8 == 0; Y bf16 rounded once,
 * or float32 if y_f32), float32 accumulation: the QuantizedLinear matmul of mlx-lm under
 * evaluate.py:35-78, in MLX's two forms. M <= 8 (matrix-vector): one fused kernel reads the
 * packed words once (HBM stream) and forms, per 32-value block, s sum(x q) + bias sum(x) -- the
 * weight s q + bias is never rounded. M > 8 (matrix-matrix): the weight is dequantized to bf16
 * into workspace (>= N K 2 bytes, 16-byte aligned) and the tensor-core GEMM reads it (err:
 * device int for its bounded waits). */
int qgemm_packed(const void *X, int M, int K, int64_t ld_x, const uint32_t *words,
                 const void *scales, const void *biases, int scale_dtype, int N, int bits,
                 int group_size, void *Y, int64_t ld_y, int y_f32, void *workspace,
                 int64_t workspace_bytes, int *err, void *stream);

/* Next-token NLL rows (evaluate.py:35-52, nll_from_hidden): z bf16 [n][ld] logits (V % 8 == 0,
 * 16-byte aligned rows), nll[r] = logsumexp(z_r) - z_r[targets[r]] (float32 logsumexp with a
 * float64 sum of exp, as gsq_kl_rows); targets[r] < 0: row not scored (0); >= V: NaN. */
int gsq_nll_rows(const void *z, int n, int V, int64_t ld, const int32_t *targets, double *nll,
                 void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GSQ_RCO_B200_H */
