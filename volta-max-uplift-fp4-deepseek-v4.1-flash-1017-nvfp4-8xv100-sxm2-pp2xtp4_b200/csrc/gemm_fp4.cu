// Block-scaled FP4 expert GEMM on the 5th-generation tensor cores: the FP4
// weights go from HBM to shared memory to tcgen05.mma.kind::mxf4nvf4 (E2M1
// operands; E4M3 scale per 16 for NVFP4, E8M0 per 32 for MXFP4, read by the
// tensor core from TMEM) without any conversion on the SM.  Used for every
// decode launch of the FP4 bank, and for prefills below 4,096 routes, of a
// layer created with prefill_gemm = 2 (longer prefills run the tcgen05 f16
// GEMM over the same weight units).
//
// Replaces the reference's QPN launches (engine/.../experts/nvfp4_8r_native.py:929-944,
// prefill RB2/RB4 at :1039-1075) and, in the W13 epilogue, its SwiGLU.
//
// Activations.  The block-scaled FP4 kind takes FP4 on both sides, so each
// activation row x is written as four E2M1 planes, x ~ g * sum_p s_pb * q_p:
// plane p quantizes the residual of the planes before it, with a block scale
// s_pb (E4M3 per 16, or a power of two per 32 for MXFP4) and one FP32 factor g
// per row (NVFP4: its amax over 6 * 448, so plane 0's block scales use E4M3's
// range and the later ones stay inside it; MXFP4: 1).  Each plane cuts the
// error about ten times; four planes leave ~1e-4 relative on the layer's
// inputs (the fp16 activations of the reference are ~5e-4).  The planes are
// stored route-major (row 4 * position + p), so the RC routes of a chunk are
// 4 RC consecutive rows: one TMA box is the MMA's B operand (N = 4 RC, column
// 4n + p), one MMA per 64-wide K step covers every plane of every route, and
// the epilogue sums a route's four columns times g.
//
// Tiles.  An item is a chunk of <= RC routes of one expert (RC = 4, 8 or 16
// by the call's size) x one weight unit row of two 128-row tiles (W13: 128
// gate rows and the 128 matching up rows, so a TMEM lane holds a gate and its
// up value; W2: two adjacent row tiles), two MMAs into two accumulators.  Per
// 256-wide K tile the producer loads the 36 KB weight unit (codes already in
// the 128-byte swizzled order, scales pre-blocked) with one bulk copy, the
// chunk's plane rows with one TMA box and their scales with one bulk copy; the
// MMA thread copies the scales into TMEM (tcgen05.cp 32x128b.warpx4) and issues
// four MMAs (K = 64) per accumulator; four epilogue warps (one TMEM lane
// quarter each = 32 weight rows) finish the item: W13 forms fp16 y13, the
// limited SwiGLU and the SwiGLU row's amax (for its W2 planes), W2 the fp16 y2
// rows; the weighted combine is one launch after W2.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "fp4_device.cuh"
#include "internal.h"
#include "layout.cuh"

namespace b200moe {
namespace {

// Where W2 writes the fp16 y2 row of a route, column col: the layer's y2 by
// route index, or (fused expert-parallel return) the home rank's y2home row,
// code = (home rank << 24) | route index at home; null for a bad home rank.
__device__ __forceinline__ __half* y2_row(const Fp4Args& a, int code, int col) {
  if (!a.ep.home) return reinterpret_cast<__half*>(a.y2) + int64_t(code) * a.H + col;
  const int hr = code >> 24, hp = code & 0xFFFFFF;
  if (hr < 0 || hr >= a.ep.world) {
    set_error(a.err, kErrBounds);
    return nullptr;
  }
  return reinterpret_cast<__half*>(a.ep.peer[hr] + a.ep.off_y2home) + int64_t(hp) * a.H + col;
}

template <int EPI, int TILES, int RC, int MX>
__global__ void __launch_bounds__(kThreads, 1)
    fp4_gemm_kernel(const Fp4Args a, const __grid_constant__ CUtensorMap map_x) {
  static_assert(EPI == 1 || TILES == 2, "W13 items pair a gate tile with its up tile");
  using St = Fp4Stage<TILES, RC, MX>;
  constexpr int kRC = St::kRC, kN = St::kN;
  constexpr int kStages = St::kStages, kStage = St::kBytes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* stages = smem_raw + (base_u32 - smem_u32(smem_raw));
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + kStages * kStage);
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* sf_full = acc_empty + 2;     // [kStages] the stage's scales are in TMEM (copier commit)
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  volatile int* abort_ptr = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_full[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
    abort_flag = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base_sh;
  pdl_wait();  // the plan, planes and (W2) SwiGLU rows of the launches before are complete
  const int n_kt = a.K / 256;
  const int n_ks = a.K / 64;
  const int n_items = a.n_chunks[a.bank] * a.n_rt;
  // the next item's chunk is loaded one item ahead: its latency never stalls a role
  auto chunk_of_item = [&](int item) {
    Chunk c{};
    c.slot = -1;
    if (item < n_items) c = a.chunks[item / a.n_rt];
    return c;
  };
  auto item_ok = [&](const Chunk& ch) {
    return ch.slot >= 0 && ch.slot < a.n_slots && ch.count >= 1 && ch.count <= kRC && ch.begin >= 0 &&
           ch.begin + ch.count <= a.S;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
      uint32_t g = 0, issued = 0, parity = 0;
      Chunk next = chunk_of_item(blockIdx.x);
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int ci = item / a.n_rt;
        const Chunk ch = next;
        next = chunk_of_item(item + gridDim.x);
        if (!item_ok(ch)) {
          set_error(a.err, kErrBounds);
          continue;
        }
        const int rt = item % a.n_rt;
        const uint8_t* wu = a.wt + (int64_t(ch.slot) * a.n_rt + rt) * n_kt * St::kUnit;
        const uint8_t* sf_b = a.sfb + int64_t(ci) * n_ks * 512;
        for (int kt = 0; kt < n_kt; ++kt, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1u;
          if (*abort_ptr || !mbar_wait(&empty[s], ph ^ 1u, a.err)) {
            *abort_ptr = 1;
            break;
          }
          uint8_t* st = stages + s * kStage;
          const uint32_t bytes = uint32_t(kStage);
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_g2s_hint(st, wu + int64_t(kt) * St::kUnit, St::kUnit, &full[s], pol);  // codes + scales
          tma_2d(st + St::kOffB, &map_x, kt * 128, ch.begin * kP, &full[s]);  // the chunk's routes x planes
          bulk_g2s(st + St::kOffSFB, sf_b + kt * kSFBytes, kSFBytes, &full[s]);
          issued |= 1u << s;
          parity = (parity & ~(1u << s)) | (ph << s);
        }
        if (*abort_ptr) break;
      }
      // no copy may be in flight when the CTA exits
      for (int s = 0; s < kStages; ++s)
        if (issued & (1u << s)) mbar_wait(&full[s], (parity >> s) & 1u, a.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t g = 0, acc_i = 0, last_b = 0, last_ph = 0;
      bool committed = false;
      Chunk next = chunk_of_item(blockIdx.x);
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const Chunk ch = next;
        next = chunk_of_item(item + gridDim.x);
        if (!item_ok(ch)) continue;
        const uint32_t b = St::kAccBufs == 2 ? (acc_i & 1u) : 0u;
        const uint32_t bph = St::kAccBufs == 2 ? ((acc_i >> 1) & 1u) : (acc_i & 1u);
        if (*abort_ptr || !mbar_wait(&acc_empty[b], bph ^ 1u, a.err)) {
          *abort_ptr = 1;
          break;
        }
        fence_after();
        const uint32_t dg = tmem + b * St::kAccCols, du = dg + kN;
        bool ok = true;
        for (int kt = 0; kt < n_kt; ++kt, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1u;
          // the stage's operands (producer) and its scales in TMEM (copier warp)
          if (*abort_ptr || !mbar_wait(&full[s], ph, a.err) || !mbar_wait(&sf_full[s], ph, a.err)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t st = smem_u32(stages + s * kStage);
          const uint32_t sfg = tmem + kSfCol + s * St::kSfCols, sfu = sfg + 16, sfb = sfg + St::kSfB;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t acc = (kt | j) != 0;
            const uint64_t bdesc = desc_sw128(st + St::kOffB + 32 * j);
            mma_fp4<MX>(dg, desc_sw128(st + St::kOffAG + 32 * j), bdesc, sfg + 4 * j, sfb + 4 * j, acc, St::kIdesc);
            if (TILES == 2)
              mma_fp4<MX>(du, desc_sw128(st + St::kOffAU + 32 * j), bdesc, sfu + 4 * j, sfb + 4 * j, acc, St::kIdesc);
          }
          commit_to(&empty[s]);
        }
        commit_to(&acc_full[b]);  // a partial item too, so its MMAs can be waited for
        committed = true;
        last_b = b;
        last_ph = bph;
        ++acc_i;
        if (!ok) {
          *abort_ptr = 1;
          break;
        }
      }
      if (committed) mbar_wait(&acc_full[last_b], last_ph, a.err);
    }
  } else if (warp == 6) {
    // ------------------------------------------------------------ scale copier
    // the stage's block scales (weight tiles, activation planes) into its TMEM columns, committed to
    // sf_full[s]: issued from a thread of their own, the 12 copies of a stage overlap the MMA thread's
    // issue of the previous stage (one thread issuing both took ~0.84 us per 36 KB stage on B200,
    // under the HBM rate of an SM at small batches)
    if (lane == 0) {
      uint32_t g = 0, issued = 0, parity = 0;
      for (int item = blockIdx.x; item < n_items && !*abort_ptr; item += gridDim.x) {
        const Chunk ch = chunk_of_item(item);
        if (!item_ok(ch)) continue;
        for (int kt = 0; kt < n_kt; ++kt, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1u;
          if (*abort_ptr || !mbar_wait(&full[s], ph, a.err)) {
            *abort_ptr = 1;
            break;
          }
          fence_after();
          const uint32_t st = smem_u32(stages + s * kStage);
          const uint32_t sfg = tmem + kSfCol + s * St::kSfCols, sfu = sfg + 16, sfb = sfg + St::kSfB;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sf_copy(sfg + 4 * j, st + St::kOffSFG + 512 * j);
            if (TILES == 2) sf_copy(sfu + 4 * j, st + St::kOffSFU + 512 * j);
            sf_copy(sfb + 4 * j, st + St::kOffSFB + 512 * j);
          }
          commit_to(&sf_full[s]);
          issued |= 1u << s;
          parity = (parity & ~(1u << s)) | (ph << s);
        }
      }
      // no copy may be in flight when TMEM is freed
      for (int s = 0; s < kStages; ++s)
        if (issued & (1u << s)) mbar_wait(&sf_full[s], (parity >> s) & 1u, a.err);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter .. : weight rows of this warp
    const int row = quarter * 32 + lane;
    uint32_t acc_i = 0;
    Chunk next = chunk_of_item(blockIdx.x);
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const Chunk ch = next;
      next = chunk_of_item(item + gridDim.x);
      if (!item_ok(ch)) continue;
      const int rt = item % a.n_rt;
      // per-route data and scales, loaded while the MMAs run: lane n holds route n's
      const float* gl = a.globals ? a.globals + ch.slot * 3 : nullptr;
      const float gw0 = gl ? gl[EPI == 0 ? 0 : 2] : 1.f, gw1 = (gl && EPI == 0) ? gl[1] : 1.f;
      float gx_l = 0.f;
      int route_l = 0;
      if (lane < ch.count) {
        gx_l = __ldg(a.gx + ch.begin + lane);
        if (EPI == 1) route_l = a.perm[ch.begin + lane];
        if (EPI == 1 && a.ep.home) route_l = a.ep.home[route_l];  // fused return: (home rank << 24) | route
      }
      const uint32_t b = St::kAccBufs == 2 ? (acc_i & 1u) : 0u;
      const uint32_t bph = St::kAccBufs == 2 ? ((acc_i >> 1) & 1u) : (acc_i & 1u);
      bool ok = !*abort_ptr && mbar_wait(&acc_full[b], bph, a.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        *abort_ptr = 1;
        break;
      }
      fence_after();
      const uint32_t lanes = uint32_t(quarter * 32) << 16;
      if constexpr (kN > 64) {
        // one accumulator buffer: read it four routes (16 columns per tile) at a time and hand it back to
        // the MMA thread as soon as the last slice is in registers
        const uint32_t acc0 = tmem + lanes + b * St::kAccCols;
        const int n_slices = (ch.count + 3) / 4;
        for (int sl = 0; sl < n_slices; ++sl) {
          float s0[16], s1[16];
          tmem_ld16(acc0 + sl * 16, s0);
          tmem_ld16(acc0 + kN + sl * 16, s1);  // up / second tile
          if (sl == n_slices - 1) {
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int n = sl * 4 + j;
            if (n >= ch.count) break;
            float v0 = 0.f, v1 = 0.f;
#pragma unroll
            for (int p = 0; p < kP; ++p) {
              v0 += s0[j * kP + p];
              v1 += s1[j * kP + p];
            }
            const float gx = __shfl_sync(0xffffffffu, gx_l, n);
            if (EPI == 0) {
              const int pos = ch.begin + n;
              const float gh = __half2float(__float2half_rn(v0 * gx * gw0));
              const float uh = __half2float(__float2half_rn(v1 * gx * gw1));
              const __half h = swiglu1(gh, uh, a.limit);
              a.inter[int64_t(pos) * a.inter_stride + rt * 128 + row] = h;
              float hm = fabsf(__half2float(h));
#pragma unroll
              for (int o = 16; o; o >>= 1) hm = fmaxf(hm, __shfl_xor_sync(0xffffffffu, hm, o));
              if (lane == 0) atomicMax(a.rowmax + pos, __float_as_uint(hm));
            } else {
              const int route = __shfl_sync(0xffffffffu, route_l, n);
              __half* yrow = y2_row(a, route, rt * 256 + row);
              if (yrow) {
                yrow[0] = __float2half_rn(v0 * gx * gw0);
                yrow[128] = __float2half_rn(v1 * gx * gw0);
              }
            }
          }
        }
        ++acc_i;
        continue;
      }
      float d0[kN], d1[TILES == 2 ? kN : 1];
#pragma unroll
      for (int c = 0; c < kN; c += 16) tmem_ld16(tmem + lanes + b * St::kAccCols + c, d0 + c);
      if (TILES == 2) {
#pragma unroll
        for (int c = 0; c < kN; c += 16)
          tmem_ld16(tmem + lanes + b * St::kAccCols + kN + c, d1 + c);  // up / second tile
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // the accumulator is in registers now
      if (EPI == 0) {
#pragma unroll
        for (int n = 0; n < kRC; ++n) {
          if (n >= ch.count) break;
          const int pos = ch.begin + n;
          float gs = 0.f, us = 0.f;
#pragma unroll
          for (int p = 0; p < kP; ++p) {
            gs += d0[n * kP + p];
            us += d1[n * kP + p];
          }
          const float gx = __shfl_sync(0xffffffffu, gx_l, n);
          const float gh = __half2float(__float2half_rn(gs * gx * gw0));
          const float uh = __half2float(__float2half_rn(us * gx * gw1));
          const __half h = swiglu1(gh, uh, a.limit);
          a.inter[int64_t(pos) * a.inter_stride + rt * 128 + row] = h;
          float hm = fabsf(__half2float(h));  // the row's amax for its W2 planes
#pragma unroll
          for (int o = 16; o; o >>= 1) hm = fmaxf(hm, __shfl_xor_sync(0xffffffffu, hm, o));
          if (lane == 0) atomicMax(a.rowmax + pos, __float_as_uint(hm));
        }
      } else {
        // fp16 y2 rows (unweighted, by route index); the slot-order combine
        // runs after the W2 launches of both banks
#pragma unroll
        for (int n = 0; n < kRC; ++n) {
          if (n >= ch.count) break;
          const int route = __shfl_sync(0xffffffffu, route_l, n);
          const float gx = __shfl_sync(0xffffffffu, gx_l, n);
          __half* yrow = y2_row(a, route, rt * (128 * TILES) + row);
          if (!yrow) continue;
          float v = 0.f;
#pragma unroll
          for (int p = 0; p < kP; ++p) v += d0[n * kP + p];
          yrow[0] = __float2half_rn(v * gx * gw0);
          if (TILES == 2) {
            float v1 = 0.f;
#pragma unroll
            for (int p = 0; p < kP; ++p) v1 += d1[n * kP + p];
            yrow[128] = __float2half_rn(v1 * gx * gw0);
          }
        }
        if (a.counters) {
          // fused combine (small decode calls): each route stored counts once per 32-column tile of this
          // warp (rt * 4 TILES + 4 h + quarter); the warp that completes a token's tile sums the token's
          // routes in slot order, the separate combine's arithmetic (a route without an expert has a zero
          // y2 row and weight, both written by the route plan, which also counts it)
          __threadfence();
          __syncwarp();
          const int tiles = a.H / 32;
#pragma unroll 1
          for (int n = 0; n < ch.count; ++n) {
            const int tok = __shfl_sync(0xffffffffu, route_l, n) / a.top_k;
#pragma unroll
            for (int h = 0; h < TILES; ++h) {
              const int tile = rt * (4 * TILES) + 4 * h + quarter;
              int* cp = a.counters + int64_t(tok) * tiles + tile;
              int done = 0;
              if (lane == 0) done = atomicAdd(cp, 1) == a.top_k - 1;
              if (__shfl_sync(0xffffffffu, done, 0)) {
                __threadfence();
                const int col = tile * 32 + lane;
                float sum = 0.f;
                for (int slot = 0; slot < a.top_k; ++slot) {
                  const int r = tok * a.top_k + slot;
                  const float y = __half2float(__ushort_as_half(
                      __ldcg(reinterpret_cast<const unsigned short*>(a.y2) + int64_t(r) * a.H + col)));
                  sum = __fmaf_rn(y, __ldcg(a.w_eff + r), sum);
                }
                a.out[int64_t(tok) * a.H + col] = sum;
                if (lane == 0) *cp = 0;
              }
            }
          }
        }
      }
      ++acc_i;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  pdl_trigger();  // the next launch may take this SM (and its TMEM) now
  if (EPI == 1 && a.ep.home && threadIdx.x == 0) {
    // fused return: once every CTA's y2 stores are visible, the last CTA raises this rank's return flag
    // on every rank (the combines wait for them)
    __threadfence_system();
    if (atomicAdd(a.ep.done, 1) == int(gridDim.x) - 1) {
      __threadfence_system();
      const int e = *a.ep.epoch;
      for (int r = 0; r < a.ep.world; ++r)
        st_release_sys(reinterpret_cast<int*>(a.ep.peer[r] + a.ep.off_mbox) + a.ep.world + a.ep.rank, e);
      *a.ep.done = 0;
    }
  }
}

// ---------------------------------------------------------------- plane kernel
// planes_row (fp4_device.cuh) over the bank's rows: a CTA per (row, 1024-wide
// slice); W13 (BY_TOKEN) takes the token rows of x, W2 the SwiGLU rows.
template <int BY_TOKEN, int BF16, int MX>
__global__ void __launch_bounds__(kPlaneThreads) fp4_planes_kernel(
    const uint16_t* __restrict__ src, int64_t src_stride, int K, const int32_t* __restrict__ inv, int top_k,
    const int32_t* __restrict__ chunk_of, int bank, const int32_t* __restrict__ bank_range, int n_tokens,
    uint32_t* rowmax, uint8_t* planes, int plane_rows, uint8_t* sfb, float* gx) {
  __shared__ PlaneScratch sm;
  pdl_wait();
  pdl_trigger();
  const int lo = bank_range[2 * bank], hi = bank_range[2 * bank + 1];
  const int rows = BY_TOKEN ? n_tokens : hi - lo;
  for (int ri = blockIdx.x; ri < rows; ri += gridDim.x)
    planes_row<BY_TOKEN, BF16, MX>(sm, src, src_stride, K, inv, top_k, chunk_of, lo, hi, ri, rowmax, planes, sfb, gx);
}

// --------------------------------------------------------------- combine
// out[t] = sum over slots, in slot order, of fma(f32(y2[route]), w[route]):
// the fused combine's arithmetic, with a route that has no expert (sorted
// past the last bank, inv[route] >= end) taken as a zero row.  Thread: 8
// consecutive columns of a token (one 16-byte load per route).
__global__ void fp4_combine_kernel(const __half* __restrict__ y2, const int32_t* __restrict__ inv,
                                   const int32_t* __restrict__ bank_range, int n_banks, const float* __restrict__ w,
                                   int T, int k, int H, float* __restrict__ out) {
  const int per_row = H / 8;  // 8 columns (one 16-byte load of y2) per thread
  pdl_wait();
  pdl_trigger();
  const int end = bank_range[2 * (n_banks - 1) + 1];
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(T) * per_row;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / per_row), c = int(i % per_row) * 8;
    float sum[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) sum[e] = 0.f;
    // eight slots at a time: their positions and weights, then their rows, are loaded before the first add
    for (int s0 = 0; s0 < k; s0 += 8) {
      const int ns = min(8, k - s0);
      int pos[8];
      float wr[8];
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < ns) {
          pos[j] = inv[t * k + s0 + j];
          wr[j] = w[t * k + s0 + j];
        }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = make_uint4(0u, 0u, 0u, 0u);
        if (j < ns && pos[j] < end) v[j] = *reinterpret_cast<const uint4*>(y2 + int64_t(t * k + s0 + j) * H + c);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= ns) break;
        const uint32_t h[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[e]));
          sum[2 * e] = __fmaf_rn(f.x, wr[j], sum[2 * e]);
          sum[2 * e + 1] = __fmaf_rn(f.y, wr[j], sum[2 * e + 1]);
        }
      }
    }
    float4* o = reinterpret_cast<float4*>(out + int64_t(t) * H + c);
    o[0] = make_float4(sum[0], sum[1], sum[2], sum[3]);
    o[1] = make_float4(sum[4], sum[5], sum[6], sum[7]);
  }
}

// --------------------------------------------------------------- prepack
// FP4 codes [slot][rows][K/2] and block scales [slot][rows][K/VS] (NVFP4: E4M3
// per 16, MXFP4: E8M0 per 32) -> weight units [slot][rt][kt], one bulk copy
// each: the unit's tiles (W13: the gate tile, rows rt * 128 .. of W1, then the
// up tile, the same rows of W3; W2: rows rt * 256 .. and rt * 256 + 128 ..) of
// 128 rows x 128 bytes of codes in the 128-byte swizzled order the MMA reads
// (16-byte chunk c of row r at r * 128 + ((c ^ (r & 7)) << 4)), then per tile
// its four 512-byte scale blocks, one per 64-wide K step q (byte m0 * 16 +
// m1 * 4 + s of block q = the scale of row m1 * 32 + m0, K block 4 q + s for
// NVFP4, 2 q + s for MXFP4, whose bytes 2 and 3 stay zero).
// MXFP4 (globals given): a nonzero block whose exponent falls outside the f16
// range of its projection's rebase (global 2^(emax - 140)) is flagged
// B200MOE_ERR_RANGE, as the decode bank's prepack does: the tcgen05 prefill
// dequantizes to f16 with that rebase.
template <int MX>
__global__ void fp4_tile_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales, int n_slots,
                                int rows_per_slot, int K, int n_tiles, int n_rt, int rt_rows, int tile_rows,
                                const float* __restrict__ globals, int proj0, uint32_t* err,
                                uint8_t* __restrict__ out) {
  const int n_kt = K / 256;
  const int64_t unit_bytes = int64_t(n_tiles) * (kATile + kSFBytes);
  const int64_t n_units = int64_t(n_slots) * n_rt * n_kt;
  for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
    const int kt = int(u % n_kt), rt = int((u / n_kt) % n_rt);
    const int64_t slot = u / (int64_t(n_kt) * n_rt);
    uint8_t* dst = out + u * unit_bytes;
    for (int j = 0; j < n_tiles; ++j) {
      const int64_t row0 = slot * rows_per_slot + int64_t(rt) * rt_rows + int64_t(j) * tile_rows;
      for (int i = threadIdx.x; i < 128 * 8; i += blockDim.x) {
        const int r = i >> 3, c = i & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(codes + (row0 + r) * (K / 2) + kt * 128 + c * 16);
        *reinterpret_cast<uint4*>(dst + j * kATile + r * 128 + ((c ^ (r & 7)) << 4)) = v;
      }
      for (int i = threadIdx.x; i < 128 * 4; i += blockDim.x) {
        const int r = i >> 2, q = i & 3;
        const uint32_t v =
            MX ? uint32_t(*reinterpret_cast<const uint16_t*>(scales + (row0 + r) * (K / 32) + kt * 8 + q * 2))
               : *reinterpret_cast<const uint32_t*>(scales + (row0 + r) * (K / 16) + kt * 16 + q * 4);
        if (MX && globals) {
          const int proj = proj0 + (proj0 == 0 ? j : 0);  // W13: tile 0 = W1, tile 1 = W3; W2: 2
          int gexp;
          frexpf(globals[slot * 3 + proj], &gexp);
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const uint4 cw = *reinterpret_cast<const uint4*>(codes + (row0 + r) * (K / 2) + kt * 128 + (2 * q + b) * 16);
            const bool zero = ((cw.x | cw.y | cw.z | cw.w) & 0x77777777u) == 0;
            const int f = int((v >> (8 * b)) & 255u) - 127 - (gexp - 1) + 15;
            if (!zero && (f < 1 || f > 30)) set_error(err, kErrRange);
          }
        }
        *reinterpret_cast<uint32_t*>(dst + n_tiles * kATile + j * kSFBytes + q * 512 + (r & 31) * 16 + (r >> 5) * 4) = v;
      }
    }
  }
}

template <int EPI, int TILES, int RC, int MX>
int launch_fp4_one(cudaStream_t s, const Fp4Args& a, const void* map_x, int grid) {
  const size_t smem = Fp4Stage<TILES, RC, MX>::kSmem;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return -1;
  if (!(attr_set.load() >> dev & 1)) {
    if (cudaFuncSetAttribute(fp4_gemm_kernel<EPI, TILES, RC, MX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(smem)) !=
        cudaSuccess)
      return -1;
    attr_set.fetch_or(uint64_t(1) << dev);
  }
  return launch_chain(fp4_gemm_kernel<EPI, TILES, RC, MX>, dim3(grid), dim3(kThreads), smem, s, a,
                      *static_cast<const CUtensorMap*>(map_x)) == cudaSuccess
             ? 0
             : -1;
}

template <int MX>
int launch_fp4_rc(cudaStream_t s, int epi, int rc, const Fp4Args& a, const void* map_x, int grid) {
  switch (rc) {
    case 4:
      return epi == 0 ? launch_fp4_one<0, 2, 4, MX>(s, a, map_x, grid) : launch_fp4_one<1, 2, 4, MX>(s, a, map_x, grid);
    case 8:
      return epi == 0 ? launch_fp4_one<0, 2, 8, MX>(s, a, map_x, grid) : launch_fp4_one<1, 2, 8, MX>(s, a, map_x, grid);
    case 16:
      return epi == 0 ? launch_fp4_one<0, 2, 16, MX>(s, a, map_x, grid)
                      : launch_fp4_one<1, 2, 16, MX>(s, a, map_x, grid);
    case 32:
      return epi == 0 ? launch_fp4_one<0, 2, 32, MX>(s, a, map_x, grid)
                      : launch_fp4_one<1, 2, 32, MX>(s, a, map_x, grid);
    default: return -1;
  }
}

}  // namespace

int launch_fp4_gemm(cudaStream_t s, int epi, int rc, bool mx, const Fp4Args& a, const void* map_x, int grid) {
  // W2 items take two adjacent 128-row tiles, as W13 items take a gate and an up tile
  return mx ? launch_fp4_rc<1>(s, epi, rc, a, map_x, grid) : launch_fp4_rc<0>(s, epi, rc, a, map_x, grid);
}

int launch_fp4_planes(cudaStream_t s, bool by_token, bool bf16, bool mx, const void* src, int64_t src_stride, int K,
                      const int32_t* inv, int top_k, const int32_t* chunk_of, int bank,
                      const int32_t* bank_range, int max_rows, uint32_t* rowmax, uint8_t* planes, int plane_rows,
                      uint8_t* sfb, float* gx) {
  // max_rows: the token rows (by_token) or the bound on the bank's positions
  if (K % 256 || top_k > 32) return -1;
  const dim3 grid(std::max(1, std::min(max_rows, 148 * 8)), (K + kSlice - 1) / kSlice);
  const uint16_t* x = static_cast<const uint16_t*>(src);
  auto kernel = by_token ? (bf16 ? (mx ? fp4_planes_kernel<1, 1, 1> : fp4_planes_kernel<1, 1, 0>)
                                 : (mx ? fp4_planes_kernel<1, 0, 1> : fp4_planes_kernel<1, 0, 0>))
                         : (mx ? fp4_planes_kernel<0, 0, 1> : fp4_planes_kernel<0, 0, 0>);
  if (!by_token && bf16) return -1;  // SwiGLU rows are fp16
  return launch_chain(kernel, grid, dim3(kPlaneThreads), 0, s, x, src_stride, K, inv, top_k, chunk_of, bank,
                      bank_range, by_token ? max_rows : 0, rowmax, planes, plane_rows, sfb, gx) == cudaSuccess
             ? 0
             : -1;
}

int launch_route_combine(cudaStream_t s, const __half* y2, const int32_t* inv, const int32_t* bank_range,
                         int n_banks, const float* w, int T, int k, int H, float* out) {
  if (H % 8 || T < 1) return -1;
  const int64_t n = int64_t(T) * (H / 8);
  const int blocks = int(std::min<int64_t>((n + 255) / 256, 148 * 16));
  return launch_chain(fp4_combine_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, s, y2, inv, bank_range, n_banks,
                      w, T, k, H, out) == cudaSuccess
             ? 0
             : -1;
}

int launch_fp4_tile(cudaStream_t s, bool mx, const uint8_t* codes, const uint8_t* scales, int n_slots,
                    int rows_per_slot, int K, bool gate_up, const float* globals, uint32_t* err, uint8_t* out) {
  // W13 (gate_up): tile 0 = rows rt * 128 .. of W1, tile 1 the same rows of W3;
  // W2: tiles 0 and 1 = rows rt * 256 .. and rt * 256 + 128 ..
  if (K % 256 || rows_per_slot % 256 || n_slots < 1) return -1;
  const int n_rt = rows_per_slot / 256;
  const int64_t units = int64_t(n_slots) * n_rt * (K / 256);
  const int blocks = int(std::min<int64_t>(units, 148 * 8));
  auto kernel = mx ? fp4_tile_kernel<1> : fp4_tile_kernel<0>;
  kernel<<<blocks, 256, 0, s>>>(codes, scales, n_slots, rows_per_slot, K, 2, n_rt, gate_up ? 128 : 256,
                                gate_up ? rows_per_slot / 2 : 128, globals, gate_up ? 0 : 2, err, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace b200moe
