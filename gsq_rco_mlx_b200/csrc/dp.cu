// Exact multiple-choice knapsack DP (the RCO decode), one CTA per instance.
//
// dp[b] = best value of the groups so far with total cost <= b; a group's row is built from
// the previous row, each thread owning a fixed set of budgets, so the K options of a group
// are folded in registers with a strict '>' in option order (the lowest option keeps ties).
// The two rows live in shared memory (float64) when they fit; the choice table streams to
// global memory with coalesced byte stores. The backtrack starts at the smallest budget whose
// value reaches dp[B] (the cheapest optimum).
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace gsq {

constexpr int kDPThreads = 1024;
constexpr int64_t kDPSmemBudget = 13823;  // 2 * (B + 1) doubles <= 216 KiB

__global__ void __launch_bounds__(kDPThreads)
mckp_dp_kernel(const double* __restrict__ scores, const int64_t* __restrict__ step, int N, int K,
               int64_t B, uint8_t* __restrict__ choice_all, double* __restrict__ dp_glob,
               int32_t* __restrict__ z_all) {
  extern __shared__ double dsm[];
  __shared__ int64_t s_best;
  __shared__ int s_bad;
  const int inst = blockIdx.x;
  const double* s = scores + (int64_t)inst * N * K;
  uint8_t* choice = choice_all + (int64_t)inst * N * (B + 1);
  int32_t* z = z_all + (int64_t)inst * N;
  double* cur = dp_glob ? dp_glob + (int64_t)inst * 2 * (B + 1) : dsm;
  double* nxt = cur + (B + 1);
  // A negative cost would index cur[] past its end: refuse the instance (z = -1).
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int64_t e = threadIdx.x; e < (int64_t)N * K; e += blockDim.x)
    if (step[e] < 0) s_bad = 1;
  __syncthreads();
  if (s_bad) {
    for (int i = threadIdx.x; i < N; i += blockDim.x) z[i] = -1;
    return;
  }
  for (int64_t b = threadIdx.x; b <= B; b += blockDim.x) cur[b] = 0.0;
  __syncthreads();
  for (int i = 0; i < N; ++i) {
    const double* si = s + (int64_t)i * K;
    const int64_t* ci = step + (int64_t)i * K;
    uint8_t* chi = choice + (int64_t)i * (B + 1);
    for (int64_t b = threadIdx.x; b <= B; b += blockDim.x) {
      double best = -INFINITY;
      int arg = 0;
      for (int k = 0; k < K; ++k) {
        const int64_t c = ci[k];
        if (c > b) continue;
        const double cand = cur[b - c] + si[k];
        if (cand > best) { best = cand; arg = k; }
      }
      nxt[b] = best;
      chi[b] = (uint8_t)arg;
    }
    __syncthreads();
    double* t = cur; cur = nxt; nxt = t;
  }
  // No assignment fits the budget: dp[B] stayed -inf. Report it (z = -1), no backtrack.
  const double target = cur[B];
  if (target == -INFINITY) {
    for (int i = threadIdx.x; i < N; i += blockDim.x) z[i] = -1;
    return;
  }
  // smallest b with dp[b] >= dp[B]
  if (threadIdx.x == 0) s_best = B;
  __syncthreads();
  int64_t mine = B;
  for (int64_t b = threadIdx.x; b <= B; b += blockDim.x)
    if (cur[b] >= target) { mine = b; break; }
  atomicMin((unsigned long long*)&s_best, (unsigned long long)mine);
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t b = s_best;
    int i = N - 1;
    for (; i >= 0; --i) {
      const int k = choice[(int64_t)i * (B + 1) + b];
      const int64_t c = step[(int64_t)i * K + k];
      if (c > b) break;  // cannot happen on a finite optimum; never read below row start
      z[i] = k;
      b -= c;
    }
    if (i >= 0)
      for (int j = 0; j < N; ++j) z[j] = -1;
  }
}

}  // namespace gsq

using namespace gsq;

extern "C" int mckp_dp_f64(const double* scores, const int64_t* step, int n_inst, int N, int K,
                           int64_t budget, uint8_t* choice_ws, double* dp_ws, int32_t* z_out,
                           void* stream) {
  if (!scores || !step || !choice_ws || !z_out || n_inst < 1 || N < 1 || K < 1 || K > 255 ||
      budget < 0)
    return GSQ_EINVAL;
  const bool in_smem = budget <= kDPSmemBudget;
  if (!in_smem && !dp_ws) return GSQ_EINVAL;
  const size_t smem = in_smem ? sizeof(double) * 2 * (size_t)(budget + 1) : 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(mckp_dp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return GSQ_ECUDA;
  mckp_dp_kernel<<<n_inst, kDPThreads, smem, st>>>(scores, step, N, K, budget, choice_ws,
                                                   in_smem ? nullptr : dp_ws, z_out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}

// ------------------------------------------------------------- allocation-free variant ---
// Some callers cannot allocate device memory: a runtime that owns every device byte through
// its own pool, or a host language whose binding has no CUDA allocator. For them the DP's
// scratch (the choice table) lives in this fixed array, which every GPU that loads the
// library holds until the process exits. Calls share it and it keeps the last call's
// contents: two calls whose kernels overlap on the same GPU (e.g. on different streams) race
// on it, so a caller serialises them.
namespace gsq {

constexpr size_t kStaticChoiceBytes = 16u << 20;  // 16 MiB: n_inst * N * (budget + 1) bytes
static __device__ __align__(256) uint8_t g_dp_choice_scratch[kStaticChoiceBytes];

constexpr int kMaxDevices = 64;
static void* g_dp_choice_addr[kMaxDevices] = {nullptr};
static std::mutex g_dp_choice_mu;

// Device address of the array on the current device; the first call on a device looks it up
// (host code must not use the symbol itself: on the host it is only a stand-in).
static int static_choice_addr(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GSQ_ECUDA;
  std::lock_guard<std::mutex> lock(g_dp_choice_mu);
  if (!g_dp_choice_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dp_choice_scratch) != cudaSuccess || !p) return GSQ_ECUDA;
    g_dp_choice_addr[dev] = p;
  }
  *out = g_dp_choice_addr[dev];
  return GSQ_OK;
}

}  // namespace gsq

extern "C" int mckp_dp_f64_noalloc(const double* scores, const int64_t* step, int n_inst, int N,
                                   int K, int64_t budget, int32_t* z_out, void* stream) {
  if (!scores || !step || !z_out || n_inst < 1 || N < 1 || K < 1 || K > 255 || budget < 0)
    return GSQ_EINVAL;
  // limits of this variant: the DP rows in shared memory, the choice table in the fixed array
  if (budget > kDPSmemBudget) return GSQ_EINVAL;
  if ((uint64_t)n_inst * (uint64_t)N * (uint64_t)(budget + 1) > kStaticChoiceBytes)
    return GSQ_EINVAL;
  void* choice = nullptr;
  const int rc = static_choice_addr(&choice);
  if (rc != GSQ_OK) return rc;
  const size_t smem = sizeof(double) * 2 * (size_t)(budget + 1);
  cudaStream_t st = (cudaStream_t)stream;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(mckp_dp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return GSQ_ECUDA;
  // every choice entry of every group is written before the backtrack reads it, so the
  // contents left by an earlier call need no clearing
  mckp_dp_kernel<<<n_inst, kDPThreads, smem, st>>>(scores, step, N, K, budget,
                                                   (uint8_t*)choice, nullptr, z_out);
  GSQ_CHECK_LAUNCH();
  return GSQ_OK;
}
