// Decode route counters, updated on the device so a captured CUDA graph keeps
// counting at every replay.
//
// Replaces RouteStats.count (engine/src/vllm/model_executor/layers/fused_moe/
// experts/nvfp4_8r_stats.py:81-98), which is nine torch ops per call, with one
// launch of one CTA.  Per layer the caller owns
//   stat       int64 [5]      calls, routes, HOST routes, distinct HOST experts
//                             of the call (summed), WARM routes
//   gap_hist   int64 [7]      HOST routes by rounds since their expert's last
//                             HOST use: <= 1, 2, <= 4, <= 16, <= 64, <= 256, more/never
//   routes     int64 [E]      routes per expert
//   last_round int32 [E + 1]  round of each expert's last HOST use (-2^30 never);
//                             entry E takes the writes of the non-HOST routes
// The round of a call is stat[0] before it.  All gaps of a call are taken
// before any last round moves (one barrier), as the reference's vector ops do.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/b200moe.h"
#include "common.cuh"

namespace b200moe {
namespace {

constexpr int kStatsThreads = 512;
constexpr int32_t kNever = -(1 << 30);

__device__ __forceinline__ int gap_bucket(int64_t gap) {
  // the first edge >= gap (edges 1, 2, 4, 16, 64, 256), 6 past the last
  return gap <= 1 ? 0 : gap <= 2 ? 1 : gap <= 4 ? 2 : gap <= 16 ? 3 : gap <= 64 ? 4 : gap <= 256 ? 5 : 6;
}

__global__ void __launch_bounds__(kStatsThreads) route_stats_kernel(const int32_t* __restrict__ ids, int n, int E,
                                                                    const uint8_t* __restrict__ is_host,
                                                                    const uint8_t* __restrict__ is_warm, int64_t* stat,
                                                                    int64_t* gap_hist, int64_t* routes,
                                                                    int32_t* last_round, uint32_t* err) {
  __shared__ int s_hist[7];
  __shared__ int s_host, s_warm, s_bad, s_distinct;
  const int t = threadIdx.x;
  if (t < 7) s_hist[t] = 0;
  if (t == 0) s_host = s_warm = s_bad = s_distinct = 0;
  __syncthreads();
  const int64_t r = stat[0];
  int host = 0, warm = 0, bad = 0;
  for (int i = t; i < n; i += blockDim.x) {
    const int e = ids[i];
    if (e < 0 || e >= E) {
      ++bad;
      continue;
    }
    if (is_host[e]) {
      ++host;
      atomicAdd(&s_hist[gap_bucket(r - int64_t(last_round[e]))], 1);
    }
    warm += is_warm[e] ? 1 : 0;
    atomicAdd(reinterpret_cast<unsigned long long*>(&routes[e]), 1ull);
  }
  __syncthreads();  // every gap is read before a last round moves
  bool other = false;
  for (int i = t; i < n; i += blockDim.x) {
    const int e = ids[i];
    if (e < 0 || e >= E) continue;
    if (is_host[e])
      last_round[e] = int32_t(r);
    else
      other = true;
  }
  if (other) last_round[E] = kNever;
  if (host) atomicAdd(&s_host, host);
  if (warm) atomicAdd(&s_warm, warm);
  if (bad) atomicAdd(&s_bad, bad);
  __syncthreads();
  int distinct = 0;
  for (int e = t; e < E; e += blockDim.x) distinct += last_round[e] == int32_t(r) ? 1 : 0;
  if (distinct) atomicAdd(&s_distinct, distinct);
  __syncthreads();
  if (t < 7 && s_hist[t]) gap_hist[t] += s_hist[t];
  if (t == 0) {
    if (s_bad) set_error(err, kErrBounds);
    stat[1] += n - s_bad;
    stat[2] += s_host;
    stat[3] += s_distinct;
    stat[4] += s_warm;
    stat[0] = r + 1;
  }
}

}  // namespace
}  // namespace b200moe

extern "C" int b200moe_route_stats(void* stream, const int32_t* topk_ids, int n, int num_experts,
                                   const uint8_t* is_host, const uint8_t* is_warm, int64_t* stat, int64_t* gap_hist,
                                   int64_t* routes, int32_t* last_round, uint32_t* err) {
  using namespace b200moe;
  if (!topk_ids || !is_host || !is_warm || !stat || !gap_hist || !routes || !last_round || !err || n < 0 ||
      num_experts < 1)
    return B200MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(stat) | reinterpret_cast<uintptr_t>(gap_hist) |
       reinterpret_cast<uintptr_t>(routes)) & 7)
    return B200MOE_ERR_ALIGN;
  route_stats_kernel<<<1, kStatsThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      topk_ids, n, num_experts, is_host, is_warm, stat, gap_hist, routes, last_round, err);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}
