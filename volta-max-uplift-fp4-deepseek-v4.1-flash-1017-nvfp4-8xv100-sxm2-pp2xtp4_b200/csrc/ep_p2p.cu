// Expert-parallel exchange over NVLink peer memory: no NCCL call and no host
// round trip, so a whole expert-parallel step can sit in one CUDA graph.
//
// The reference has no expert parallelism (engine/patches/gguf_moe.patch:57-58);
// this is the B200 form of configs[4]'s dispatch / combine.  Every rank owns
// one device allocation that all ranks map through CUDA IPC (cudaMalloc +
// cudaIpcOpenMemHandle; no multicast object):
//
//   mbox     int32: per source rank data_flag and ret_flag ([2][world]), then
//            two row-reservation counters (one per epoch parity)
//   eid      int32 [R_cap]: expert id of each received route
//   home     int32 [R_cap]: (home rank << 24) | route index at home
//   rows     fp16 [R_cap][H]: received activation rows, R_cap = world * S_max
//   y2home   fp16 [S_max][H]: y2 rows of this rank's own routes, written by owners
//
// One step (all ranks, same order; flags carry a per-step epoch kept on the
// device, so no host value changes between steps):
//   push:    a warp per route reserves a row in its owner's buffer with one
//            system-scope atomic on the owner's counter of this epoch (no rank
//            waits for another's counts), stores the route's f16 row, expert
//            id and home there; the last CTA raises data_flag on every rank;
//   (the owner runs its experts on the received rows: b200moe_ep_forward,
//   whose route-plan launch first waits for every rank's data_flag and takes
//   the rows received from the counter, resetting both counters)
//   return:  store each received route's y2 row into its home rank's y2home;
//            the last CTA raises ret_flag on every rank;
//   combine: wait for every rank's ret_flag, then out[t] = residual[t] + the
//            slot-order sum of fma(f32(y2), w) -- the single-GPU combine.
// A rank pushes step s + 1 only after its combine of step s saw every owner's
// return, which each owner raises after its plan of step s read and reset the
// counters: no reservation of step s + 1 can land before that reset.  Rows
// land in reservation order, which varies from run to run; every route's row
// is computed on its own (top-1 rows, per-column MMA sums), so the results do
// not depend on it.  Flags are written with st.release.sys after a system
// fence and read with ld.acquire.sys; every wait is bounded by kWaitLimitNs and
// sets kErrTimeout.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace b200moe {

constexpr int kEpMaxWorld = 16;

struct EpP2P {
  int world, rank, H;
  int k, S, num_experts;
  const void* x;
  int x_bf16;
  const int32_t* ids;
  const int32_t* perm;
  const int32_t* owner;
  int r_cap;  // rows of every rank's receive buffer
  uint8_t* peer[kEpMaxWorld];
  size_t off_mbox, off_eid, off_home, off_rows, off_y2home;
  int* epoch;    // local: epoch of the step in flight (advanced by push)
  int* done;     // local: finished CTAs of the current kernel
  int32_t* recv;  // local [3]: rows received, then {0, rows}
  uint32_t* err;
};

__device__ __forceinline__ int* mbox_of(const EpP2P& a, int r) {
  return reinterpret_cast<int*>(a.peer[r] + a.off_mbox);
}

// mbox words: data flags [0, W), return flags [W, 2W), reservation counters [2W, 2W + 2)
__device__ __forceinline__ int* resv_of(const EpP2P& a, int r, int e) { return mbox_of(a, r) + 2 * a.world + (e & 1); }

// The last CTA to finish raises flag slot `which` (0 data, 1 ret) for this
// rank on every rank.
__device__ __forceinline__ void last_cta_signal(const EpP2P& a, int which, int e, bool advance_epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(a.done, 1) == int(gridDim.x) - 1) {
      __threadfence_system();
      const int W = a.world;
      for (int r = 0; r < W; ++r) st_release_sys(mbox_of(a, r) + which * W + a.rank, e);
      *a.done = 0;
      if (advance_epoch) *a.epoch = e;
    }
  }
}

__global__ void __launch_bounds__(256) ep_push_kernel(const EpP2P a) {
  const int W = a.world;
  const int e = *a.epoch + 1;
  // one warp per route: its owner and row reserved once, then the row's 16-byte
  // pieces (H / 8 of them) four at a time per lane
  const int lane = threadIdx.x & 31;
  const int warps = int(gridDim.x * blockDim.x) >> 5;
  const int chunks = a.H / 8;
  for (int route = int(blockIdx.x * blockDim.x + threadIdx.x) >> 5; route < a.S; route += warps) {
    const int id = a.ids[route];
    const int dst = (id >= 0 && id < a.num_experts) ? a.owner[id] : -1;
    if (dst < 0 || dst >= W) {  // no owner: never sent, contributes 0 in the combine
      if (lane == 0) set_error(a.err, kErrBounds);
      continue;
    }
    int row = 0;
    if (lane == 0) row = atomicAdd_system(resv_of(a, dst, e), 1);
    row = __shfl_sync(0xffffffffu, row, 0);
    if (row >= a.r_cap) {
      if (lane == 0) set_error(a.err, kErrRange);
      continue;
    }
    const uint16_t* src = static_cast<const uint16_t*>(a.x) + int64_t(route / a.k) * a.H;
    uint8_t* base = a.peer[dst];
    uint4* drow = reinterpret_cast<uint4*>(base + a.off_rows + int64_t(row) * a.H * 2);
    for (int c0 = lane; c0 < chunks; c0 += 32 * 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + 32 * u;
        if (c < chunks) v[u] = *reinterpret_cast<const uint4*>(src + 8 * c);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + 32 * u;
        if (c >= chunks) continue;
        if (a.x_bf16) {
          const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __half2 h = __floats2half2_rn(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xFFFF0000u));
            o[j] = *reinterpret_cast<const uint32_t*>(&h);
          }
          v[u] = make_uint4(o[0], o[1], o[2], o[3]);
        }
        drow[c] = v[u];
      }
    }
    if (lane == 0) {
      reinterpret_cast<int*>(base + a.off_eid)[row] = id;
      reinterpret_cast<int*>(base + a.off_home)[row] = (a.rank << 24) | route;
    }
  }
  last_cta_signal(a, 0, e, true);
}

__global__ void __launch_bounds__(256) ep_return_kernel(const EpP2P a, const __half* __restrict__ y2) {
  const int e = *a.epoch;
  const int n = a.recv[0];
  const int chunks = a.H / 8;
  const int* home = reinterpret_cast<const int*>(a.peer[a.rank] + a.off_home);
  // one warp per received row: its home looked up once, the row four 16-byte pieces at a time per lane
  const int lane = threadIdx.x & 31;
  const int warps = int(gridDim.x * blockDim.x) >> 5;
  for (int row = int(blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n; row += warps) {
    const int h = home[row];
    const int hr = h >> 24, hp = h & 0xFFFFFF;
    if (hr < 0 || hr >= a.world) {
      if (lane == 0) set_error(a.err, kErrBounds);
      continue;
    }
    const uint4* srow = reinterpret_cast<const uint4*>(y2 + int64_t(row) * a.H);
    uint4* drow = reinterpret_cast<uint4*>(a.peer[hr] + a.off_y2home + int64_t(hp) * a.H * 2);
    for (int c0 = lane; c0 < chunks; c0 += 32 * 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + 32 * u < chunks) v[u] = srow[c0 + 32 * u];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + 32 * u < chunks) drow[c0 + 32 * u] = v[u];
    }
  }
  last_cta_signal(a, 1, e, false);
}

__global__ void __launch_bounds__(256) ep_combine_p2p_kernel(const EpP2P a, const float* __restrict__ w, int T,
                                                           const float* __restrict__ residual, float* __restrict__ out) {
  __shared__ int s_ok;
  const int W = a.world, e = *a.epoch;
  if (threadIdx.x == 0) s_ok = wait_flags(mbox_of(a, a.rank) + W, W, e, a.err);
  __syncthreads();
  if (!s_ok) return;
  const __half* y2 = reinterpret_cast<const __half*>(a.peer[a.rank] + a.off_y2home);
  const int per_row = a.H / 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(T) * per_row;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / per_row), c = int(i % per_row) * 4;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    for (int slot = 0; slot < a.k; ++slot) {
      const int route = t * a.k + slot;
      const int id = a.ids[route];
      if (id < 0 || id >= a.num_experts) continue;  // no owner: contributes 0 (flagged by the plan)
      const int o = a.owner[id];
      if (o < 0 || o >= W) continue;
      const float wr = w[route];
      const uint2 v = __ldcg(reinterpret_cast<const uint2*>(y2 + int64_t(route) * a.H + c));
      const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
      const float2 q = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
      s0 = __fmaf_rn(p.x, wr, s0);
      s1 = __fmaf_rn(p.y, wr, s1);
      s2 = __fmaf_rn(q.x, wr, s2);
      s3 = __fmaf_rn(q.y, wr, s3);
    }
    float4 o4 = make_float4(s0, s1, s2, s3);
    if (residual) {
      const float4 r = *reinterpret_cast<const float4*>(residual + int64_t(t) * a.H + c);
      o4.x += r.x;
      o4.y += r.y;
      o4.z += r.z;
      o4.w += r.w;
    }
    *reinterpret_cast<float4*>(out + int64_t(t) * a.H + c) = o4;
  }
}

}  // namespace b200moe

using namespace b200moe;

struct b200moe_ep {
  int device = 0, world = 1, rank = 0, H = 0, max_routes = 0, r_cap = 0;
  uint8_t* shared = nullptr;  // this rank's IPC-shared allocation
  size_t off_mbox = 0, off_eid = 0, off_home = 0, off_rows = 0, off_y2home = 0, shared_bytes = 0;
  uint8_t* peer[kEpMaxWorld] = {};
  bool opened[kEpMaxWorld] = {};
  // local (not shared)
  int* epoch = nullptr;
  int* done = nullptr;
  int32_t* recv = nullptr;
  uint32_t* err = nullptr;
  __half* y2 = nullptr;  // the local experts' y2 rows [r_cap][H]
  int grid = 148;
};

namespace {

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

struct EpDeviceGuard {
  int prev = -1;
  explicit EpDeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~EpDeviceGuard() {
    int cur;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

void ep_free(b200moe_ep* E) {
  for (int r = 0; r < kEpMaxWorld; ++r)
    if (E->opened[r]) cudaIpcCloseMemHandle(E->peer[r]);
  void* ptrs[] = {E->shared, E->epoch, E->done, E->recv, E->err, E->y2};
  for (void* p : ptrs)
    if (p) cudaFree(p);
}

EpP2P ep_args(const b200moe_ep* E) {
  EpP2P a{};
  a.world = E->world;
  a.rank = E->rank;
  a.H = E->H;
  a.r_cap = E->r_cap;
  for (int r = 0; r < E->world; ++r) a.peer[r] = E->peer[r];
  a.off_mbox = E->off_mbox;
  a.off_eid = E->off_eid;
  a.off_home = E->off_home;
  a.off_rows = E->off_rows;
  a.off_y2home = E->off_y2home;
  a.epoch = E->epoch;
  a.done = E->done;
  a.recv = E->recv;
  a.err = E->err;
  return a;
}

bool connected(const b200moe_ep* E) {
  for (int r = 0; r < E->world; ++r)
    if (!E->peer[r]) return false;
  return true;
}

}  // namespace

extern "C" {

int b200moe_ep_create(int device, int world, int rank, int hidden, int max_routes, b200moe_ep** out) {
  if (!out || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world || hidden < 8 || hidden % 8 ||
      max_routes < 1 || int64_t(world) * max_routes >= (1 << 24))
    return B200MOE_ERR_INVALID_ARG;
  EpDeviceGuard guard(device);
  auto* E = new b200moe_ep();
  E->device = device;
  E->world = world;
  E->rank = rank;
  E->H = hidden;
  E->max_routes = max_routes;
  E->r_cap = world * max_routes;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    delete E;
    return B200MOE_ERR_CUDA;
  }
  E->grid = prop.multiProcessorCount;
  size_t o = 0;
  E->off_mbox = o;
  o += up256(size_t(2 * world + 2) * 4);
  E->off_eid = o;
  o += up256(size_t(E->r_cap) * 4);
  E->off_home = o;
  o += up256(size_t(E->r_cap) * 4);
  E->off_rows = o;
  o += up256(size_t(E->r_cap) * hidden * 2);
  E->off_y2home = o;
  o += up256(size_t(max_routes) * hidden * 2);
  E->shared_bytes = o;
  bool ok = cudaMalloc(&E->shared, o) == cudaSuccess &&
            cudaMalloc(&E->epoch, 4) == cudaSuccess && cudaMalloc(&E->done, 4) == cudaSuccess &&
            cudaMalloc(&E->recv, 16) == cudaSuccess && cudaMalloc(&E->err, 4) == cudaSuccess &&
            cudaMalloc(&E->y2, size_t(E->r_cap) * hidden * 2) == cudaSuccess;
  ok = ok && cudaMemset(E->shared, 0, E->off_eid) == cudaSuccess && cudaMemset(E->epoch, 0, 4) == cudaSuccess &&
       cudaMemset(E->done, 0, 4) == cudaSuccess && cudaMemset(E->recv, 0, 16) == cudaSuccess &&
       cudaMemset(E->err, 0, 4) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  if (!ok) {
    ep_free(E);
    delete E;
    return B200MOE_ERR_NOMEM;
  }
  E->peer[rank] = E->shared;
  *out = E;
  return B200MOE_OK;
}

// The CUDA IPC handle (64 bytes) of this rank's shared allocation.
int b200moe_ep_ipc_handle(b200moe_ep* E, void* handle) {
  if (!E || !handle) return B200MOE_ERR_INVALID_ARG;
  EpDeviceGuard guard(E->device);
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, E->shared) != cudaSuccess) return B200MOE_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return B200MOE_OK;
}

// Map every other rank's allocation from the handles of all ranks (world x 64 bytes).
int b200moe_ep_connect(b200moe_ep* E, const void* handles) {
  if (!E || !handles) return B200MOE_ERR_INVALID_ARG;
  EpDeviceGuard guard(E->device);
  for (int r = 0; r < E->world; ++r) {
    if (r == E->rank || E->opened[r]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + size_t(r) * sizeof(h), sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return B200MOE_ERR_CUDA;
    E->peer[r] = static_cast<uint8_t*>(p);
    E->opened[r] = true;
  }
  return B200MOE_OK;
}

int b200moe_ep_destroy(b200moe_ep* E) {
  if (!E) return B200MOE_ERR_INVALID_ARG;
  EpDeviceGuard guard(E->device);
  cudaDeviceSynchronize();
  ep_free(E);
  delete E;
  return B200MOE_OK;
}

// Receive side for b200moe_forward_rows: rows (fp16 [max_rows][H]), expert
// ids, the device count of rows received, {0, rows}, and the local y2 buffer.
int b200moe_ep_recv_buffers(b200moe_ep* E, void** rows, int32_t** expert_ids, int32_t** n_valid,
                            int32_t** row_range, void** y2, int* max_rows) {
  if (!E || !rows || !expert_ids || !n_valid || !row_range || !y2 || !max_rows) return B200MOE_ERR_INVALID_ARG;
  *rows = E->shared + E->off_rows;
  *expert_ids = reinterpret_cast<int32_t*>(E->shared + E->off_eid);
  *n_valid = E->recv;
  *row_range = E->recv + 1;
  *y2 = E->y2;
  *max_rows = E->r_cap;
  return B200MOE_OK;
}

// Store this rank's T*k routes into their owners' buffers (one launch; the
// owners' b200moe_ep_forward waits for every rank's push).
int b200moe_ep_push(b200moe_ep* E, void* stream, const void* x, int x_dtype, const int32_t* ids, int T, int k,
                    int num_experts, const int32_t* owner_of_expert) {
  if (!E || !x || !ids || !owner_of_expert || T < 1 || k < 1 || num_experts < E->world) return B200MOE_ERR_INVALID_ARG;
  if (x_dtype != B200MOE_F16 && x_dtype != B200MOE_BF16) return B200MOE_ERR_DTYPE;
  if (int64_t(T) * k > E->max_routes) return B200MOE_ERR_RANGE;
  if (reinterpret_cast<uintptr_t>(x) & 15) return B200MOE_ERR_ALIGN;
  if (!connected(E)) return B200MOE_ERR_STATE;
  EpDeviceGuard guard(E->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int S = T * k;
  EpP2P a = ep_args(E);
  a.k = k;
  a.S = S;
  a.num_experts = num_experts;
  a.x = x;
  a.x_bf16 = x_dtype == B200MOE_BF16;
  a.ids = ids;
  a.owner = owner_of_expert;
  const int blocks = std::min(std::max((S + 7) / 8, 1), E->grid * 2);  // a warp per route
  ep_push_kernel<<<blocks, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

}  // extern "C"

// What b200moe_ep_forward's route plan needs to receive a step: the data flags
// of every rank (this rank's mbox), the epoch, the reservation counters and the
// receive count it writes.
int b200moe::ep_recv_wait(const b200moe_ep* E, EpRecvWait* w) {
  if (!E || !w || !connected(E)) return B200MOE_ERR_STATE;
  int* mbox = reinterpret_cast<int*>(E->shared + E->off_mbox);
  w->flags = mbox;
  w->n_flags = E->world;
  w->epoch = E->epoch;
  w->resv = mbox + 2 * E->world;
  w->out = E->recv;
  w->rows = E->shared + E->off_rows;
  w->expert_ids = reinterpret_cast<const int32_t*>(E->shared + E->off_eid);
  w->y2 = E->y2;
  w->max_rows = E->r_cap;
  w->device = E->device;
  return B200MOE_OK;
}

int b200moe::ep_return_targets(const b200moe_ep* E, EpReturn* r) {
  if (!E || !r || !connected(E) || E->world > kEpMaxPeers) return B200MOE_ERR_STATE;
  *r = EpReturn{};
  r->home = reinterpret_cast<const int32_t*>(E->shared + E->off_home);
  for (int i = 0; i < E->world; ++i) r->peer[i] = E->peer[i];
  r->off_y2home = int64_t(E->off_y2home);
  r->off_mbox = int64_t(E->off_mbox);
  r->world = E->world;
  r->rank = E->rank;
  r->epoch = E->epoch;
  r->done = E->done;
  return B200MOE_OK;
}

extern "C" {

// Return the local experts' y2 rows (the buffer of b200moe_ep_recv_buffers) to their home ranks.
int b200moe_ep_return(b200moe_ep* E, void* stream) {
  if (!E) return B200MOE_ERR_INVALID_ARG;
  if (!connected(E)) return B200MOE_ERR_STATE;
  EpDeviceGuard guard(E->device);
  EpP2P a = ep_args(E);
  const int blocks = std::min(std::max((E->r_cap + 7) / 8, 1), E->grid * 2);  // a warp per row received
  ep_return_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(a, E->y2);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

// out[t] = residual[t] (optional) + slot-order sum of fma(f32(y2), w) over this rank's routes.
int b200moe_ep_combine_p2p(b200moe_ep* E, void* stream, const int32_t* ids, const float* topk_weights, int T,
                           int k, int num_experts, const int32_t* owner_of_expert, const float* residual,
                           float* out) {
  if (!E || !ids || !topk_weights || !owner_of_expert || !out || T < 1 || k < 1 || E->H % 4)
    return B200MOE_ERR_INVALID_ARG;
  if (int64_t(T) * k > E->max_routes) return B200MOE_ERR_RANGE;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (residual && (reinterpret_cast<uintptr_t>(residual) & 15)))
    return B200MOE_ERR_ALIGN;
  if (!connected(E)) return B200MOE_ERR_STATE;
  EpDeviceGuard guard(E->device);
  EpP2P a = ep_args(E);
  a.k = k;
  a.num_experts = num_experts;
  a.ids = ids;
  a.owner = owner_of_expert;
  const int64_t work = int64_t(T) * (E->H / 4);
  const int blocks = int(std::min<int64_t>(std::max<int64_t>((work + 255) / 256, 1), int64_t(E->grid) * 4));
  ep_combine_p2p_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(a, topk_weights, T, residual, out);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

// Synchronize the stream; the number of routes received in the last step and
// (up to max) their expert ids, copied to host memory.
int b200moe_ep_received(b200moe_ep* E, void* stream, int32_t* n, int32_t* expert_ids, int max) {
  if (!E || !n || (max > 0 && !expert_ids)) return B200MOE_ERR_INVALID_ARG;
  EpDeviceGuard guard(E->device);
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return B200MOE_ERR_CUDA;
  if (cudaMemcpy(n, E->recv, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return B200MOE_ERR_CUDA;
  const int c = std::min(std::max(*n, 0), max);
  if (c > 0 && cudaMemcpy(expert_ids, E->shared + E->off_eid, size_t(c) * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return B200MOE_ERR_CUDA;
  return B200MOE_OK;
}

// Synchronize the stream and map the exchange's error bits to a status (then clear them).
int b200moe_ep_check_errors(b200moe_ep* E, void* stream, uint32_t* bits) {
  if (!E) return B200MOE_ERR_INVALID_ARG;
  EpDeviceGuard guard(E->device);
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return B200MOE_ERR_CUDA;
  uint32_t e = 0;
  if (cudaMemcpy(&e, E->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return B200MOE_ERR_CUDA;
  if (e && cudaMemset(E->err, 0, 4) != cudaSuccess) return B200MOE_ERR_CUDA;
  if (bits) *bits = e;
  if (e & kErrBounds) return B200MOE_ERR_BOUNDS;
  if (e & kErrTimeout) return B200MOE_ERR_TIMEOUT;
  if (e & kErrRange) return B200MOE_ERR_RANGE;
  return B200MOE_OK;
}

}  // extern "C"
