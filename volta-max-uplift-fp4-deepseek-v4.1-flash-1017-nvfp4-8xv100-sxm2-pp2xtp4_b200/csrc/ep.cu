// Expert-parallel dispatch and combine kernels (the exchange itself is NCCL
// all-to-all, issued by the host through torch.distributed).
//
// The reference has no expert parallelism (engine/patches/gguf_moe.patch:57-58:
// "nvfp4_8r experts take global ids (no EP)"); its tier placement becomes the
// ownership of contiguous expert-id ranges by GPU here.
//
//   dispatch: stable counting sort of this GPU's routes by owner rank (the
//     route-plan kernel with key = owner rank), per-rank counts, and the f16
//     activation row, expert id and sorted position of every route;
//   owner:    its local experts run the routes with k = 1 and weight 1.0, so the
//     layer's output rows are exactly the fp16 y2 rows (f32_to_f16 copies them);
//   combine:  out[t] = residual[t] + sum over slots, in slot order, of
//     fma(f32(y2[route]), w[route]) -- the single-GPU combine's arithmetic.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace b200moe {

// send_experts[p] = ids[perm[p]], route_pos[perm[p]] = p; a route whose id
// has no owner (the plan kernel sorted it last and flagged BOUNDS) is never
// sent and gets route_pos -1, which the combine skips.
__global__ void ep_meta_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ perm, int S,
                               int num_experts, const int32_t* __restrict__ owner, int world,
                               int32_t* __restrict__ send_experts, int32_t* __restrict__ route_pos) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < S; p += gridDim.x * blockDim.x) {
    const int r = perm[p];
    const int e = ids[r];
    const bool ok = e >= 0 && e < num_experts && owner[e] >= 0 && owner[e] < world;
    send_experts[p] = ok ? e : -1;
    route_pos[r] = ok ? p : -1;
  }
}

// One block per token row chunk: thread handles 4 consecutive hidden columns.
__global__ void ep_combine_kernel(const __half* __restrict__ y2, const int32_t* __restrict__ route_pos,
                                  const float* __restrict__ w, int T, int k, int H, const float* __restrict__ residual,
                                  float* __restrict__ out) {
  const int per_row = H / 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(T) * per_row;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / per_row), c = int(i % per_row) * 4;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    for (int slot = 0; slot < k; ++slot) {
      const int route = t * k + slot;
      const int pos = route_pos[route];
      if (pos < 0) continue;  // route without an expert contributes 0
      const float wr = w[route];
      const uint2 v = *reinterpret_cast<const uint2*>(y2 + int64_t(pos) * H + c);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
      s0 = __fmaf_rn(a.x, wr, s0);
      s1 = __fmaf_rn(a.y, wr, s1);
      s2 = __fmaf_rn(b.x, wr, s2);
      s3 = __fmaf_rn(b.y, wr, s3);
    }
    float4 o = make_float4(s0, s1, s2, s3);
    if (residual) {
      const float4 r = *reinterpret_cast<const float4*>(residual + int64_t(t) * H + c);
      o.x += r.x;
      o.y += r.y;
      o.z += r.z;
      o.w += r.w;
    }
    *reinterpret_cast<float4*>(out + int64_t(t) * H + c) = o;
  }
}

__global__ void f32_to_f16_kernel(const float4* __restrict__ x, int64_t n4, uint2* __restrict__ y) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    const float4 v = x[i];
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    y[i] = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  }
}

static int blocks_for(int64_t n, int threads, int cap = 148 * 16) {
  int64_t b = (n + threads - 1) / threads;
  return int(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace b200moe

using namespace b200moe;

// Workspace of b200moe_ep_dispatch: perm [S] + chunks + counts, in bytes.
extern "C" size_t b200moe_ep_workspace_bytes(int max_routes, int world) {
  return size_t(max_routes) * 4 + size_t(max_routes + world) * sizeof(Chunk) + 256 + size_t(world) * 4 + 1024;
}

extern "C" int b200moe_ep_dispatch(void* stream, const void* x, int x_dtype, const int32_t* ids, int T, int k,
                                   int num_experts, int world, const int32_t* owner_of_expert, int H, void* send_rows,
                                   int32_t* send_experts, int32_t* route_pos, int32_t* send_counts, void* workspace,
                                   size_t workspace_bytes, uint32_t* err) {
  if (!x || !ids || !owner_of_expert || !send_rows || !send_experts || !route_pos || !send_counts || !workspace ||
      T < 1 || k < 1 || world < 1 || world > 1024 || num_experts < world || H < 8 || H % 8)
    return B200MOE_ERR_INVALID_ARG;
  if (x_dtype != B200MOE_F16 && x_dtype != B200MOE_BF16) return B200MOE_ERR_DTYPE;
  const int S = T * k;
  if (workspace_bytes < b200moe_ep_workspace_bytes(S, world)) return B200MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(send_rows) & 15)) return B200MOE_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* perm = reinterpret_cast<int32_t*>(ws);
  Chunk* chunks = reinterpret_cast<Chunk*>(ws + ((size_t(S) * 4 + 255) / 256) * 256);
  int32_t* n_chunks = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(chunks) + size_t(S + world) * sizeof(Chunk));
  PlanArgs p{};
  p.ids = ids;
  p.n = S;
  p.num_experts = num_experts;
  p.key_of_expert = owner_of_expert;  // key = owner rank
  p.n_keys = world;
  p.perm = perm;
  p.n_banks = 1;
  p.key_lo[0] = 0;
  p.key_hi[0] = world;
  p.rc[0] = S;
  p.max_chunks[0] = S + world;
  p.chunks[0] = chunks;
  p.n_chunks = n_chunks;
  p.key_counts = send_counts;
  p.err = err;
  if (launch_plan(s, p)) return B200MOE_ERR_CUDA;
  if (launch_gather_rows(s, x, x_dtype == B200MOE_BF16, perm, S, k, H, send_rows)) return B200MOE_ERR_CUDA;
  ep_meta_kernel<<<blocks_for(S, 256), 256, 0, s>>>(ids, perm, S, num_experts, owner_of_expert, world,
                                                    send_experts, route_pos);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

extern "C" int b200moe_ep_combine(void* stream, const void* y2, const int32_t* route_pos, const float* topk_weights,
                                  int T, int k, int H, const float* residual, float* out) {
  if (!y2 || !route_pos || !topk_weights || !out || T < 1 || k < 1 || H < 4 || H % 4) return B200MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(y2) & 7) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (residual && (reinterpret_cast<uintptr_t>(residual) & 15)))
    return B200MOE_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ep_combine_kernel<<<blocks_for(int64_t(T) * (H / 4), 256), 256, 0, s>>>(
      static_cast<const __half*>(y2), route_pos, topk_weights, T, k, H, residual, out);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

extern "C" int b200moe_f32_to_f16(void* stream, const float* x, int64_t n, void* y) {
  if (!x || !y || n < 0 || n % 4) return B200MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 7)) return B200MOE_ERR_ALIGN;
  if (n == 0) return B200MOE_OK;
  f32_to_f16_kernel<<<blocks_for(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(x), n / 4, static_cast<uint2*>(y));
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

extern "C" int b200moe_gate(void* stream, const float* logits, int T, int num_experts, int top_k, int32_t* ids,
                            float* weights, uint32_t* err) {
  if (!logits || !ids || !weights || T < 1 || num_experts < 1 || num_experts > 1024 || top_k < 1 || top_k > 16 ||
      top_k > num_experts)
    return B200MOE_ERR_INVALID_ARG;
  if (launch_gating(static_cast<cudaStream_t>(stream), logits, T, num_experts, top_k, ids, weights, err))
    return B200MOE_ERR_CUDA;
  return B200MOE_OK;
}
