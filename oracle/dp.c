/* Exact multiple-choice knapsack DP: plain-C restatement (oracle). TEST INFRASTRUCTURE ONLY.
 *
 * Follows egesabanci/gsq-rco-mlx src/gsq_rco/rco/manifold.py:304-334 (_mckp_dp):
 *   dp[b] = best value with total cost <= b (float64), -inf where nothing fits;
 *   per (group i, option k): cand = dp[b - c_ik] + s_ik replaces new[b] only if strictly
 *   greater, so the lowest option index keeps ties; the backtrack starts at the smallest
 *   budget whose value reaches dp[B] (the cheapest optimum).
 * Built by oracle/Makefile into oracle/_build/libdp_oracle.so; called through ctypes by the
 * tests and by bench.py's CPU baseline only.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* s [N*K] row-major float64, step [N*K] int64 costs, choice scratch [N*(B+1)] uint8,
 * z_out [N] chosen option per group. Returns 0 on success, 1 on bad arguments. */
int oracle_mckp_dp(const double *s, const int64_t *step, int N, int K, int64_t B,
                   uint8_t *choice, int32_t *z_out) {
  if (N < 1 || K < 1 || K > 255 || B < 0) return 1;
  double *dp = (double *)malloc(sizeof(double) * (size_t)(B + 1));
  double *nw = (double *)malloc(sizeof(double) * (size_t)(B + 1));
  if (!dp || !nw) { free(dp); free(nw); return 1; }
  for (int64_t b = 0; b <= B; ++b) dp[b] = 0.0;
  for (int i = 0; i < N; ++i) {
    uint8_t *ch = choice + (size_t)i * (size_t)(B + 1);
    for (int64_t b = 0; b <= B; ++b) { nw[b] = -INFINITY; ch[b] = 0; }
    for (int k = 0; k < K; ++k) {
      int64_t c = step[(size_t)i * K + k];
      if (c > B) continue;
      double sv = s[(size_t)i * K + k];
      for (int64_t b = c; b <= B; ++b) {
        double cand = dp[b - c] + sv;
        if (cand > nw[b]) { nw[b] = cand; ch[b] = (uint8_t)k; }
      }
    }
    double *t = dp; dp = nw; nw = t;
  }
  int64_t b = 0;
  while (b < B && !(dp[b] >= dp[B])) ++b;
  for (int i = N - 1; i >= 0; --i) {
    int k = choice[(size_t)i * (size_t)(B + 1) + (size_t)b];
    z_out[i] = k;
    b -= step[(size_t)i * K + k];
  }
  free(dp); free(nw);
  return 0;
}
