// Block-scaled FP4 expert GEMM on the 5th-generation tensor cores: the
// NVFP4 weights go from HBM to shared memory to tcgen05.mma.kind::mxf4nvf4
// (E2M1 operands, E4M3 scale per 16 along K, read by the tensor core from
// TMEM) without any conversion on the SM.  Used for every launch of the FP4
// bank (decode and prefill) of a layer created with prefill_gemm = 2.
//
// Replaces the reference's QPN launches (engine/.../experts/nvfp4_8r_native.py:929-944,
// prefill RB2/RB4 at :1039-1075) and, in the epilogues, its SwiGLU and
// weighted reduce, as the other expert kernels here do.
//
// Activations.  The block-scaled FP4 kind takes FP4 on both sides, so each
// activation row x is written as four E2M1 planes, x ~ sum_p g_p * s_pb * q_p:
// plane p quantizes the residual of the planes before it, with an E4M3 scale
// s_pb per 16 elements and an FP32 factor g_p per row and plane (its amax over
// 6 * 448, so the block scales use E4M3's range).  Each plane cuts the error
// about ten times; four planes leave ~1e-4 relative on the layer's inputs
// (the fp16 activations of the reference are ~5e-4).  The planes are four
// groups of 16 rows of the MMA's B operand (N = 64): one MMA per 64-wide K
// step covers every plane of every route of the chunk, and the epilogue sums
// the four columns of a route with their g_p.
//
// Tiles.  An item is a chunk of <= 16 routes of one expert x a tile of 128
// weight rows (W13: 128 gate rows and the 128 matching up rows, two MMAs into
// two accumulators, so a TMEM lane holds a gate and its up value).  Per 256-wide
// K tile the producer warp loads by TMA the weight tile(s) [128 rows x 128 B,
// 128-byte swizzle] and the four activation planes [16 rows x 128 B each],
// and by bulk copy the pre-blocked scales (4 x 512 B per operand); the MMA
// thread copies the scales into TMEM (tcgen05.cp 32x128b.warpx4) and issues
// four MMAs (K = 64) per accumulator; four epilogue warps (one TMEM lane
// quarter each = 32 weight rows) finish the item: W13 forms fp16 y13 and the
// limited SwiGLU, W2 the fp16 y2 rows and the slot-order combine.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "internal.h"
#include "layout.cuh"

namespace b200moe {
namespace {

constexpr int kP = kFp4Planes;             // activation planes
constexpr int kRC = kFp4TcRoutes;          // routes per chunk
constexpr int kN = kP * kRC;               // MMA N = 64
constexpr int kATile = 128 * 128;          // weight tile: 128 rows x 256 FP4 = 16 KB
constexpr int kBTile = kN * 128;           // activation tile: 64 rows x 256 FP4 = 8 KB
constexpr int kSFBytes = 4 * 512;          // the scale blocks of one 256-wide K tile
constexpr int kOffAG = 0, kOffAU = kATile, kOffB = 2 * kATile;
constexpr int kOffSFG = 2 * kATile + kBTile, kOffSFU = kOffSFG + kSFBytes, kOffSFB = kOffSFU + kSFBytes;
constexpr int kStage = kOffSFB + kSFBytes;  // 46 KB
constexpr int kStages = 4;
constexpr int kThreads = 6 * 32;           // producer, MMA, 4 epilogue warps
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfCol = 256;           // per stage: SFA gate 16, SFA up 16, SFB 16 columns
constexpr uint32_t kSfStageCols = 48;      // own columns per stage: a copy never lands under an MMA in flight
static_assert(kSfCol + kStages * kSfStageCols <= kTmemCols, "TMEM columns");
// kind::mxf4nvf4 block16: A and B E2M1 (1), K-major, N = 64, M = 128, scales UE4M3
constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | (uint32_t(kN >> 3) << 17) | (uint32_t(128 >> 4) << 24);

__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}
// a 512-byte scale block: K-major, no swizzle, 8-row core matrices of 16 B rows 128 B apart
__device__ __forceinline__ uint64_t desc_sf(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(128 >> 4) << 32) | (uint64_t(1) << 46);
}

__device__ __forceinline__ void sf_copy(uint32_t tcol, uint32_t smem) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tcol), "l"(desc_sf(smem)));
}

__device__ __forceinline__ void mma_fp4(uint32_t d, uint64_t a, uint64_t b, uint32_t sfa, uint32_t sfb,
                                        uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p; }" ::"r"(d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate), "r"(sfa), "r"(sfb));
}

__device__ __forceinline__ void commit_to(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ __half swiglu1(float g, float u, float limit) {
  g = g > limit ? limit : g;
  u = u > limit ? limit : u;
  u = u < -limit ? -limit : u;
  return __float2half_rn(__fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u));
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    fp4_gemm_kernel(const Fp4Args a, const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* stages = smem_raw + (base_u32 - smem_u32(smem_raw));
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + kStages * kStage);
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  volatile int* abort_ptr = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
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
  const int n_kt = a.K / 256;
  const int n_ks = a.K / 64;
  const int n_items = a.n_chunks[a.bank] * a.n_rt;
  auto item_ok = [&](const Chunk& ch) {
    return ch.slot >= 0 && ch.slot < a.n_slots && ch.count >= 1 && ch.count <= kRC && ch.begin >= 0 &&
           ch.begin + ch.count <= a.S;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t g = 0, issued = 0, parity = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int ci = item / a.n_rt;
        const Chunk ch = a.chunks[ci];
        if (!item_ok(ch)) {
          set_error(a.err, kErrBounds);
          continue;
        }
        const int rt = item % a.n_rt;
        const int row_g = ch.slot * a.rows_per_slot + rt * 128;
        const uint8_t* sf_g = a.sfa + (int64_t(ch.slot) * a.rb_per_slot + rt) * n_ks * 512;
        const uint8_t* sf_u = sf_g + int64_t(a.up_rb) * n_ks * 512;
        const uint8_t* sf_b = a.sfb + int64_t(ci) * n_ks * 512;
        for (int kt = 0; kt < n_kt; ++kt, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1u;
          if (*abort_ptr || !mbar_wait(&empty[s], ph ^ 1u, a.err)) {
            *abort_ptr = 1;
            break;
          }
          uint8_t* st = stages + s * kStage;
          const uint32_t bytes = uint32_t((EPI == 0 ? 2 : 1) * (kATile + kSFBytes) + kBTile + kSFBytes);
          mbar_arrive_expect_tx(&full[s], bytes);
          tma_2d(st + kOffAG, &map_w, kt * 128, row_g, &full[s]);
          bulk_g2s_hint(st + kOffSFG, sf_g + kt * kSFBytes, kSFBytes, &full[s], pol);
          if (EPI == 0) {
            tma_2d(st + kOffAU, &map_w, kt * 128, row_g + a.up_rb * 128, &full[s]);
            bulk_g2s_hint(st + kOffSFU, sf_u + kt * kSFBytes, kSFBytes, &full[s], pol);
          }
#pragma unroll
          for (int p = 0; p < kP; ++p) tma_2d(st + kOffB + p * kRC * 128, &map_x, kt * 128, p * a.plane_rows + ch.begin, &full[s]);
          bulk_g2s(st + kOffSFB, sf_b + kt * kSFBytes, kSFBytes, &full[s]);
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
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const Chunk ch = a.chunks[item / a.n_rt];
        if (!item_ok(ch)) continue;
        const uint32_t b = acc_i & 1u, bph = (acc_i >> 1) & 1u;
        if (*abort_ptr || !mbar_wait(&acc_empty[b], bph ^ 1u, a.err)) {
          *abort_ptr = 1;
          break;
        }
        fence_after();
        const uint32_t dg = tmem + b * 128, du = dg + 64;
        bool ok = true;
        for (int kt = 0; kt < n_kt; ++kt, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1u;
          if (*abort_ptr || !mbar_wait(&full[s], ph, a.err)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t st = smem_u32(stages + s * kStage);
          const uint32_t sfg = tmem + kSfCol + s * kSfStageCols, sfu = sfg + 16, sfb = sfg + 32;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sf_copy(sfg + 4 * j, st + kOffSFG + 512 * j);
            if (EPI == 0) sf_copy(sfu + 4 * j, st + kOffSFU + 512 * j);
            sf_copy(sfb + 4 * j, st + kOffSFB + 512 * j);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t acc = (kt | j) != 0;
            mma_fp4(dg, desc_sw128(st + kOffAG + 32 * j), desc_sw128(st + kOffB + 32 * j), sfg + 4 * j, sfb + 4 * j, acc);
            if (EPI == 0)
              mma_fp4(du, desc_sw128(st + kOffAU + 32 * j), desc_sw128(st + kOffB + 32 * j), sfu + 4 * j, sfb + 4 * j,
                      acc);
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
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter .. : weight rows of this warp
    const int row = quarter * 32 + lane;
    uint32_t acc_i = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const Chunk ch = a.chunks[item / a.n_rt];
      if (!item_ok(ch)) continue;
      const int rt = item % a.n_rt;
      const uint32_t b = acc_i & 1u, bph = (acc_i >> 1) & 1u;
      bool ok = !*abort_ptr && mbar_wait(&acc_full[b], bph, a.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        *abort_ptr = 1;
        break;
      }
      fence_after();
      const uint32_t lanes = uint32_t(quarter * 32) << 16;
      const float* gl = a.globals ? a.globals + ch.slot * 3 : nullptr;
      float d0[kN], d1[EPI == 0 ? kN : 1];
#pragma unroll
      for (int c = 0; c < kN; c += 16) tmem_ld16(tmem + lanes + b * 128 + c, d0 + c);
      if (EPI == 0) {
#pragma unroll
        for (int c = 0; c < kN; c += 16) tmem_ld16(tmem + lanes + b * 128 + 64 + c, d1 + c);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // the accumulator is in registers now
      if (EPI == 0) {
        const float g1 = gl ? gl[0] : 1.f, g3 = gl ? gl[1] : 1.f;
#pragma unroll
        for (int n = 0; n < kRC; ++n) {
          if (n >= ch.count) break;
          const int pos = ch.begin + n;
          float gs = 0.f, us = 0.f;
#pragma unroll
          for (int p = 0; p < kP; ++p) {
            const float gx = __ldg(a.gx + int64_t(p) * a.plane_rows + pos);
            gs = fmaf(d0[p * kRC + n], gx, gs);
            us = fmaf(d1[p * kRC + n], gx, us);
          }
          const float gh = __half2float(__float2half_rn(gs * g1));
          const float uh = __half2float(__float2half_rn(us * g3));
          a.inter[int64_t(pos) * a.inter_stride + rt * 128 + row] = swiglu1(gh, uh, a.limit);
        }
      } else {
        const float g2 = gl ? gl[2] : 1.f;
        const int tile = rt * 4 + quarter;  // 32-row tile of the output row
#pragma unroll
        for (int n = 0; n < kRC; ++n) {
          if (n >= ch.count) break;
          const int pos = ch.begin + n;
          float v = 0.f;
#pragma unroll
          for (int p = 0; p < kP; ++p) v = fmaf(d0[p * kRC + n], __ldg(a.gx + int64_t(p) * a.plane_rows + pos), v);
          const int route = a.perm[pos];
          reinterpret_cast<__half*>(a.y2)[int64_t(route) * a.H + rt * 128 + row] = __float2half_rn(v * g2);
        }
        if (a.counters) {
          __threadfence();
          __syncwarp();
          for (int n = 0; n < ch.count; ++n) {
            const int route = a.perm[ch.begin + n];
            const int tok = route / a.top_k;
            int* cnt = a.counters + int64_t(tok) * (a.H / 32) + tile;
            int old = 0;
            if (lane == 0) old = atomicAdd(cnt, 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == a.top_k - 1) {  // the last route of (token, tile): slot-order sum
              __threadfence();
              const unsigned short* y2 = reinterpret_cast<const unsigned short*>(a.y2);
              const int orow = rt * 128 + row;
              float sum = 0.f;
              for (int slot = 0; slot < a.top_k; ++slot) {
                const int r2 = tok * a.top_k + slot;
                const float y = __half2float(__ushort_as_half(__ldcg(y2 + int64_t(r2) * a.H + orow)));
                sum = __fmaf_rn(y, __ldcg(a.w_eff + r2), sum);
              }
              a.out[int64_t(tok) * a.H + orow] = sum;
              if (lane == 0) *cnt = 0;
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
}

// ---------------------------------------------------------------- planes
// One CTA per sorted route position of the FP4 bank: the row (a token's x
// for W13, the route's SwiGLU row for W2) as kP E2M1 planes, their blocked
// scales in the chunk's SFB blocks (MMA row p * 16 + n) and g_p.
template <int SRC_TOKEN>
__global__ void __launch_bounds__(128) fp4_planes_kernel(const __half* __restrict__ src, int64_t src_stride, int K,
                                                         const int32_t* __restrict__ perm, int top_k,
                                                         const Chunk* __restrict__ chunks,
                                                         const int32_t* __restrict__ n_chunks, int bank,
                                                         const int32_t* __restrict__ bank_range, uint8_t* planes,
                                                         int plane_rows, uint8_t* sfb, float* gx) {
  constexpr int kMaxBlk = 4;  // 16-wide blocks per thread: K <= 128 * 16 * kMaxBlk
  __shared__ float red[4];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nb = K / 16, n_ks = K / 64;
  const int nch = n_chunks[bank];
  for (int pos = bank_range[2 * bank] + blockIdx.x; pos < bank_range[2 * bank + 1]; pos += gridDim.x) {
    // the chunk holding pos: chunks are in position order
    int lo = 0, hi = nch - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (chunks[mid].begin <= pos) lo = mid;
      else hi = mid - 1;
    }
    const int c = lo, n = pos - chunks[c].begin;
    const __half* row = src + (SRC_TOKEN ? int64_t(perm[pos] / top_k) : int64_t(pos)) * src_stride;
    float r[kMaxBlk][16];
#pragma unroll
    for (int i = 0; i < kMaxBlk; ++i) {
      const int blk = t + 128 * i;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (blk < nb) v = *reinterpret_cast<const uint4*>(row + blk * 16 + h * 8);
        const __half2* hv = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(hv[e]);
          r[i][h * 8 + 2 * e] = f.x;
          r[i][h * 8 + 2 * e + 1] = f.y;
        }
      }
    }
#pragma unroll 1
    for (int p = 0; p < kP; ++p) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxBlk; ++i)
#pragma unroll
        for (int e = 0; e < 16; ++e) m = fmaxf(m, fabsf(r[i][e]));
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) red[warp] = m;
      __syncthreads();
      const float amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
      __syncthreads();
      const float g = amax / (6.f * 448.f);
      const float inv_g = g > 0.f ? 1.f / g : 0.f;
      const int mrow = p * kRC + n, m0 = mrow & 31, m1 = mrow >> 5;
#pragma unroll
      for (int i = 0; i < kMaxBlk; ++i) {
        const int blk = t + 128 * i;
        if (blk >= nb) continue;
        float bm = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) bm = fmaxf(bm, fabsf(r[i][e]));
        const uint32_t sc = e4m3_encode(bm / 6.f * inv_g);
        const float scale = e4m3_value(sc) * g;
        const float inv = scale > 0.f ? 1.f / scale : 0.f;
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float v = r[i][e] * inv;
          const uint32_t code = e2m1_code(fabsf(v)) | (v < 0.f ? 8u : 0u);
          const float dq = (code & 8u ? -1.f : 1.f) * e2m1_mag(code) * scale;
          r[i][e] -= dq;
          w[e >> 3] |= code << (4 * (e & 7));
        }
        *reinterpret_cast<uint2*>(planes + (int64_t(p) * plane_rows + pos) * (K / 2) + blk * 8) = make_uint2(w[0], w[1]);
        sfb[(int64_t(c) * n_ks + (blk >> 2)) * 512 + m0 * 16 + m1 * 4 + (blk & 3)] = uint8_t(sc);
      }
      if (t == 0) gx[int64_t(p) * plane_rows + pos] = g;
    }
  }
}

// --------------------------------------------------------------- prepack
// NVFP4 scales [slot][rows][K/16] -> blocked [slot][rows/128][K/64][512]:
// byte m0 * 16 + m1 * 4 + s of block (rb, ks) = scale of row rb * 128 + m1 * 32 + m0, K block 4 ks + s.
__global__ void fp4_block_scales_kernel(const uint8_t* __restrict__ sc, int64_t n_rows, int K, uint8_t* __restrict__ out) {
  const int kb16 = K / 16, n_ks = K / 64;
  const int64_t total = n_rows * kb16;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / kb16;
    const int kb = int(i % kb16);
    const int64_t rb = r >> 7;
    const int m = int(r & 127), m0 = m & 31, m1 = m >> 5;
    out[(rb * n_ks + (kb >> 2)) * 512 + m0 * 16 + m1 * 4 + (kb & 3)] = sc[i];
  }
}

template <int EPI>
int launch_fp4_one(cudaStream_t s, const Fp4Args& a, const void* map_w, const void* map_x, int grid) {
  const size_t smem = 1024 + size_t(kStages) * kStage + 64 * 8;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return -1;
  if (!(attr_set.load() >> dev & 1)) {
    if (cudaFuncSetAttribute(fp4_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
        cudaSuccess)
      return -1;
    attr_set.fetch_or(uint64_t(1) << dev);
  }
  fp4_gemm_kernel<EPI><<<grid, kThreads, smem, s>>>(a, *static_cast<const CUtensorMap*>(map_w),
                                                    *static_cast<const CUtensorMap*>(map_x));
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace

int launch_fp4_gemm(cudaStream_t s, int epi, const Fp4Args& a, const void* map_w, const void* map_x, int grid) {
  return epi == 0 ? launch_fp4_one<0>(s, a, map_w, map_x, grid) : launch_fp4_one<1>(s, a, map_w, map_x, grid);
}

int launch_fp4_planes(cudaStream_t s, bool by_token, const __half* src, int64_t src_stride, int K,
                      const int32_t* perm, int top_k, const Chunk* chunks, const int32_t* n_chunks, int bank,
                      const int32_t* bank_range, int max_rows, uint8_t* planes, int plane_rows, uint8_t* sfb,
                      float* gx) {
  if (K % 256 || K > 128 * 16 * 4) return -1;
  const int blocks = std::max(1, std::min(max_rows, 148 * 16));
  if (by_token)
    fp4_planes_kernel<1><<<blocks, 128, 0, s>>>(src, src_stride, K, perm, top_k, chunks, n_chunks, bank, bank_range,
                                                planes, plane_rows, sfb, gx);
  else
    fp4_planes_kernel<0><<<blocks, 128, 0, s>>>(src, src_stride, K, perm, top_k, chunks, n_chunks, bank, bank_range,
                                                planes, plane_rows, sfb, gx);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_fp4_block_scales(cudaStream_t s, const uint8_t* scales, int64_t n_rows, int K, uint8_t* out) {
  if (n_rows % 128 || K % 64) return -1;
  const int64_t total = n_rows * (K / 16);
  const int blocks = int(std::min<int64_t>((total + 255) / 256, 148 * 32));
  fp4_block_scales_kernel<<<std::max(blocks, 1), 256, 0, s>>>(scales, n_rows, K, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace b200moe
