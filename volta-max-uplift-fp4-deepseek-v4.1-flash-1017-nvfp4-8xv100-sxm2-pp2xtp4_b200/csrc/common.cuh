// Shared device helpers of the B200 routed-MoE library (sm_100a only).
//
// Every spin-wait here is bounded by the global timer: a wait that runs out
// records an error code in the caller's error word and returns false, so a
// logic error surfaces as a status instead of a hung GPU.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "../../include/b200moe.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library is written for sm_100a (B200) only"
#endif

namespace b200moe {

// Error word bits written by kernels (OR-ed; the host maps them to a status).
enum : uint32_t {
  kErrBounds = 1u << 0,   // an id, slot, offset or count outside its range
  kErrTimeout = 1u << 1,  // a bounded wait ran out
  kErrFormat = 1u << 2,   // a packed value the format forbids (E4M3 NaN, E8M0 255)
  kErrRange = 1u << 3,    // a value outside what the kernel layout can hold
};

// Bound of every spin-wait, in nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void set_error(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

// Programmatic dependent launch.  The kernels of the forward chain (gating,
// route plan, planes, expert GEMMs, combine) are launched with programmatic
// stream serialization, so a launch may be scheduled, and run its set-up
// (barriers, TMEM, tensor maps), while the previous one finishes.  Each such
// kernel calls pdl_wait() in every thread before it reads or writes memory
// that an earlier launch of the stream touches, and before any early return:
// the wait ends when the previous grid has completed with its writes visible,
// so the completion of any grid of the chain implies that of every earlier
// one.  pdl_trigger() lets the stream's next launch be scheduled: the small
// kernels call it right after their wait, the expert GEMMs only at their end
// (measured on B200: CTAs of the next launch waiting beside a GEMM's for its
// whole run slowed the configs[1] decode step by 1-2 %, while a trigger at
// the end saved 3 us of the 64 us M = 1 step).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Whether chain launches carry the programmatic attribute (B200MOE_PDL=0 turns it off).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("B200MOE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Launch a chain kernel (one that calls pdl_wait() as above) on stream s.
template <typename... P, typename... A>
inline cudaError_t launch_chain_attr(bool pdl, void (*kernel)(P...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t s, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
}
template <typename... P, typename... A>
inline cudaError_t launch_chain(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                A&&... args) {
  return launch_chain_attr(pdl_enabled(), kernel, grid, block, smem, s, static_cast<A&&>(args)...);
}

// System-scope acquire load / release store (flags written over NVLink by peer GPUs).
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until flags[0..n) have all reached epoch e (monotonic counters), at
// most kWaitLimitNs; false (and kErrTimeout) when the bound runs out.
__device__ __forceinline__ bool wait_flags(const int* flags, int n, int e, uint32_t* err) {
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    bool ok = true;
    for (int i = 0; i < n; ++i) ok = ok && (ld_acquire_sys(flags + i) - e) >= 0;
    if (ok) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      set_error(err, kErrTimeout);
      return false;
    }
    __nanosleep(128);
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait with a suspend-time hint: a warp whose phase is not complete sleeps
// (up to 1 ms) until it completes instead of spinning on the issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity; false (and an error bit) after the limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 3u) == 3u && global_timer_ns() - t0 > kWaitLimitNs) {
      set_error(err, kErrTimeout);
      return false;
    }
  }
}

// ------------------------------------------------------- bulk async copies
// Global -> shared, completion counted on an mbarrier in bytes.  Both addresses
// 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 eviction hint for data that is read once (expert weights).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void bulk_g2s_hint(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
      "%2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ------------------------------------------------------------ conversions
// Byte B of `word` (two E2M1 values, low nibble = lower half) -> f16x2.  Exact.
template <int B>
__device__ __forceinline__ uint32_t e2m1x2_byte(uint32_t word) {
  uint32_t out;
  if constexpr (B == 0)
    asm("{ .reg .b8 b0, b1, b2, b3; mov.b32 {b0, b1, b2, b3}, %1; cvt.rn.f16x2.e2m1x2 %0, b0; }"
        : "=r"(out)
        : "r"(word));
  else if constexpr (B == 1)
    asm("{ .reg .b8 b0, b1, b2, b3; mov.b32 {b0, b1, b2, b3}, %1; cvt.rn.f16x2.e2m1x2 %0, b1; }"
        : "=r"(out)
        : "r"(word));
  else if constexpr (B == 2)
    asm("{ .reg .b8 b0, b1, b2, b3; mov.b32 {b0, b1, b2, b3}, %1; cvt.rn.f16x2.e2m1x2 %0, b2; }"
        : "=r"(out)
        : "r"(word));
  else
    asm("{ .reg .b8 b0, b1, b2, b3; mov.b32 {b0, b1, b2, b3}, %1; cvt.rn.f16x2.e2m1x2 %0, b3; }"
        : "=r"(out)
        : "r"(word));
  return out;
}

// Four bytes of E2M1 pairs (8 values, low nibble first) -> four f16x2, each
// multiplied by the f16x2 scale s2: one unpack for the whole word.  Exact when
// value x scale is representable in f16 (always for the E4M3 / rebased E8M0 scales).
__device__ __forceinline__ void e2m1x8_scaled(uint32_t w, uint32_t s2, uint32_t (&o)[4]) {
  asm("{ .reg .b8 b0, b1, b2, b3; .reg .b32 h0, h1, h2, h3;\n"
      " mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 h0, b0;\n cvt.rn.f16x2.e2m1x2 h1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 h2, b2;\n cvt.rn.f16x2.e2m1x2 h3, b3;\n"
      " mul.rn.f16x2 %0, h0, %5;\n mul.rn.f16x2 %1, h1, %5;\n"
      " mul.rn.f16x2 %2, h2, %5;\n mul.rn.f16x2 %3, h3, %5; }"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w), "r"(s2));
}

// Two E4M3 bytes (low byte = lower half) -> f16x2.  Exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t out;
  uint16_t v = static_cast<uint16_t>(two_bytes);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(v));
  return out;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Broadcast the low / high half of an f16x2 to both halves.
__device__ __forceinline__ uint32_t lo_half2(uint32_t v) { return __byte_perm(v, 0, 0x1010); }
__device__ __forceinline__ uint32_t hi_half2(uint32_t v) { return __byte_perm(v, 0, 0x3232); }

// --------------------------------------------------------------- tensor core
// D += A (16x16, row) * B (16x8, col), f16 inputs, f32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D += A (16x32, row) * B (32x8, col), int8 inputs, s32 accumulate.
__device__ __forceinline__ void mma_16832_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D += A . B on m16n8k16 s8 x s8 -> s32: a0 = row g, a1 = row g + 8, each K
// 4t..4t+3; b = K 4t..4t+3 of column g (g = lane / 4, t = lane % 4).
__device__ __forceinline__ void mma_16816_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(b));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// Named barrier among `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace b200moe
