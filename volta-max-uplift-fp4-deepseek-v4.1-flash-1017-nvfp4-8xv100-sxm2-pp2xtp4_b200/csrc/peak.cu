// Dense tensor-core peaks of this GPU, measured with the same tcgen05.mma
// kinds the expert kernels issue: one persistent CTA per SM issues
// back-to-back MMAs on operands that stay in shared memory (zeros), so the
// launch time is the tensor pipe's own.  The roofline denominators of the
// prefill and decode kernels (FP4 block-scaled, FP8, f16) come from here; the
// bf16 figure of the pool's cuBLAS measurement is the cross-check of kind 0.
//
// Kinds (M = 128, one CTA group):
//   0  kind::f16, f16 x f16 -> f32, N 256, K 16 per MMA
//   1  kind::f8f6f4, E4M3 x E4M3 -> f32, N 256, K 32
//   2  kind::mxf4nvf4.block16, E2M1 x E2M1, UE4M3 scale per 16 -> f32, N 128, K 64
//   3  kind::mxf4nvf4.block32, E2M1 x E2M1, UE8M0 scale per 32 -> f32, N 128, K 64
//   4  kind::f16 at N 128 (the block-scaled kinds' N, for comparison)
// Every MMA reads 32 bytes per operand row: four MMAs walk one 128-byte
// swizzled row of A (128 rows) and B (N rows).
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace b200moe {
namespace {

constexpr int kPeakThreads = 128;

struct PeakDevice {  // makes `device` current for the call, restores the caller's
  int prev = -1;
  explicit PeakDevice(int d) {
    cudaGetDevice(&prev);
    cudaSetDevice(d);
  }
  ~PeakDevice() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
constexpr uint32_t kPeakCols = 512;

__device__ __forceinline__ uint64_t peak_desc_sw128(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}
__device__ __forceinline__ uint64_t peak_desc_sf(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(128 >> 4) << 32) | (uint64_t(1) << 46);
}

template <int KIND>
struct PeakKind {
  static constexpr int N = (KIND == 0 || KIND == 1) ? 256 : 128;
  static constexpr int K = KIND == 0 || KIND == 4 ? 16 : KIND == 1 ? 32 : 64;  // per MMA
  static constexpr uint32_t kMN = (uint32_t(N >> 3) << 17) | (uint32_t(128 >> 4) << 24);
  static constexpr uint32_t kIdesc = KIND == 0 || KIND == 4 ? ((1u << 4) | kMN)          // f16 in, f32 out
                                     : KIND == 1           ? ((1u << 4) | kMN)          // E4M3 (0) in, f32 out
                                     : KIND == 2           ? ((1u << 7) | (1u << 10) | kMN)
                                                           : ((1u << 7) | (1u << 10) | (1u << 23) | kMN);
};

template <int KIND>
__device__ __forceinline__ void peak_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t sfa, uint32_t sfb,
                                         uint32_t acc) {
  constexpr uint32_t idesc = PeakKind<KIND>::kIdesc;
  if constexpr (KIND == 0 || KIND == 4)
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::
                     "r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
  else if constexpr (KIND == 1)
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p; }" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
  else if constexpr (KIND == 2)
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p; }" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb));
  else
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p; }" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb));
}

template <int KIND>
constexpr size_t peak_smem() {
  return 1024 + 128 * 128 + size_t(PeakKind<KIND>::N) * 128 + 2 * 512 + 64;
}

template <int KIND>
__global__ void __launch_bounds__(kPeakThreads, 1) mma_peak_kernel(int iters, uint32_t* err) {
  constexpr int N = PeakKind<KIND>::N;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - smem_u32(smem_raw));
  uint8_t* a_tile = base;
  uint8_t* b_tile = a_tile + 128 * 128;
  uint8_t* sf = b_tile + N * 128;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sf + 2 * 512);
  __shared__ uint32_t tmem_sh;
  // zero operands and scales (the products are zeros: the timing does not depend on values)
  for (int i = threadIdx.x; i < (128 * 128 + N * 128 + 2 * 512) / 16; i += kPeakThreads)
    reinterpret_cast<uint4*>(a_tile)[i] = make_uint4(0, 0, 0, 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                 "r"(kPeakCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_sh;
  if (threadIdx.x == 0) {
    const uint32_t sfa = tmem + 256, sfb = tmem + 260;
    if (KIND == 2 || KIND == 3) {
      asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfa), "l"(peak_desc_sf(smem_u32(sf))));
      asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfb),
                   "l"(peak_desc_sf(smem_u32(sf + 512))));
    }
    const uint32_t a0 = smem_u32(a_tile), b0 = smem_u32(b_tile);
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        peak_mma<KIND>(tmem, peak_desc_sw128(a0 + 32 * j), peak_desc_sw128(b0 + 32 * j), sfa, sfb, (it | j) != 0);
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
    mbar_wait(bar, 0, err);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (threadIdx.x < 32)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPeakCols));
}

template <int KIND>
int run_peak(int grid, int iters, cudaStream_t s, uint32_t* err) {
  constexpr size_t smem = peak_smem<KIND>();
  if (cudaFuncSetAttribute(mma_peak_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
      cudaSuccess)
    return B200MOE_ERR_CUDA;
  mma_peak_kernel<KIND><<<grid, kPeakThreads, smem, s>>>(iters, err);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

}  // namespace
}  // namespace b200moe

using namespace b200moe;

extern "C" int b200moe_mma_peak(int device, int kind, int iters, float* tflops, float* ms) {
  if (kind < 0 || kind > 4 || iters < 1 || iters > (1 << 24) || !tflops || !ms) return B200MOE_ERR_INVALID_ARG;
  PeakDevice guard(device);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return B200MOE_ERR_CUDA;
  const int grid = prop.multiProcessorCount;
  uint32_t* err = nullptr;
  if (cudaMalloc(&err, 4) != cudaSuccess) return B200MOE_ERR_NOMEM;
  cudaStream_t s = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  int st = B200MOE_OK;
  if (cudaMemset(err, 0, 4) != cudaSuccess || cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess)
    st = B200MOE_ERR_CUDA;
  auto launch = [&](int n) {
    switch (kind) {
      case 0: return run_peak<0>(grid, n, s, err);
      case 1: return run_peak<1>(grid, n, s, err);
      case 2: return run_peak<2>(grid, n, s, err);
      case 3: return run_peak<3>(grid, n, s, err);
      default: return run_peak<4>(grid, n, s, err);
    }
  };
  if (st == B200MOE_OK) st = launch(std::max(1, iters / 8));  // warm-up (clocks, module load)
  if (st == B200MOE_OK && (cudaEventRecord(e0, s) != cudaSuccess)) st = B200MOE_ERR_CUDA;
  if (st == B200MOE_OK) st = launch(iters);
  if (st == B200MOE_OK && (cudaEventRecord(e1, s) != cudaSuccess || cudaEventSynchronize(e1) != cudaSuccess))
    st = B200MOE_ERR_CUDA;
  uint32_t bits = 0;
  if (st == B200MOE_OK && cudaMemcpy(&bits, err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) st = B200MOE_ERR_CUDA;
  if (st == B200MOE_OK && bits) st = B200MOE_ERR_TIMEOUT;
  float t = 0.f;
  if (st == B200MOE_OK && cudaEventElapsedTime(&t, e0, e1) != cudaSuccess) st = B200MOE_ERR_CUDA;
  if (st == B200MOE_OK) {
    const int n = (kind == 0 || kind == 1) ? 256 : 128;
    const int k = (kind == 0 || kind == 4) ? 16 : kind == 1 ? 32 : 64;
    const double flops = 2.0 * 128 * n * k * 4.0 * double(iters) * grid;
    *ms = t;
    *tflops = float(flops / (double(t) * 1e-3) / 1e12);
  }
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (s) cudaStreamDestroy(s);
  cudaFree(err);
  return st;
}
