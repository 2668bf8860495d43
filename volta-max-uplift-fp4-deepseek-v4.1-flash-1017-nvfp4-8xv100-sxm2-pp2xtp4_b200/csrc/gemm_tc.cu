// Prefill expert GEMM on the 5th-generation tensor cores (tcgen05, TMEM).
//
// Replaces the reference's prefill QPN launches (RB2 / RB4,
// engine/kernels/prefill-rb4/qpn_rb4_append.cu:12-89; engine/.../experts/nvfp4_8r_native.py:1039-1075)
// and, fused into the epilogues, its SwiGLU and weighted reduce.
//
// One persistent CTA per SM walks items = (token tile of <= 128 routes of one
// expert) x (row tile of 256 weight rows).  D[tokens x rows] = X . W^T with the
// routes as the MMA's M (128) and the weight rows as its N (256).  Per 64-wide K block:
//   warp 0 (producer): TMA tensor load of the permuted fp16 token tile
//     [128 rows x 64 K, 128B swizzle] into a 5-deep ring, and bulk loads of the
//     packed FP4 units (one per 128-wide K, shared by two K blocks);
//   warps 2-9 (dequant): FP4 codes x block scale -> f16 (exact) written in the
//     UMMA K-major 128B-swizzle layout, then fence.proxy.async;
//   warp 1 (MMA): one thread issues 4 x tcgen05.mma.kind::f16 (M128 N256 K16)
//     into a TMEM accumulator (two buffers, 512 columns) and commits;
//   warps 10-13 (epilogue): tcgen05.ld (one TMEM lane = one route), then
//     W13: columns 0-127 are 128 gate rows and 128-255 the matching up rows,
//     so each thread forms fp16 y13 and the limited SwiGLU of its own route;
//     W2: the fp16 y2 rows of its route (the weighted combine is one launch
//     after W2: fused here its atomics and re-reads stalled the epilogue).
// Every wait is bounded; after an abort the roles drain in-flight copies and
// MMAs before TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "layout.cuh"

namespace b200moe {
namespace {

constexpr int BM = 128;      // routes per token tile (MMA M)
constexpr int BNW = 256;     // weight rows per item (MMA N)
constexpr int BK = 64;       // K per MMA stage (one 128B swizzle atom of f16)
constexpr int kTokStages = 5;
constexpr int kWStages = 3;
constexpr int kRawStages = 2;
constexpr int kDequantWarps = 8;
constexpr int kEpiWarp0 = 2 + kDequantWarps;
constexpr int kThreads = (kEpiWarp0 + 4) * 32;
constexpr int kTokBytes = BM * BK * 2;   // 16 KB
constexpr int kWBytes = BNW * BK * 2;    // 32 KB
constexpr uint32_t kTmemCols = 2 * BNW;  // 512
constexpr int kUnits = BNW / 32;         // tile pairs per item

// FMT 0 / 1: NVFP4 / MXFP4 in the decode bank's units (tile pair x 128 K, eight
// per raw stage: 256 weight rows x 128 K).  FMT 2 / 3: NVFP4 / MXFP4 weight
// units of the block-scaled path's layout (two 128-row tiles x 256 K, codes
// swizzled, scales blocked), one per raw stage; fewer token and weight stages
// keep the larger raw stages inside shared memory.  MXFP4 scales are rebased
// on the fly by the projection's global (2^(emax - 140)), as the decode bank's
// prepack stores them.
template <int FMT>
struct TcFmt {
  static constexpr bool kWeightUnits = FMT >= 2;
  static constexpr int U = kWeightUnits ? 2 * (128 * 128 + 4 * 512) : fp4_unit_bytes(FMT);
  static constexpr int RAW = kWeightUnits ? U : kUnits * U;
  static constexpr int KB_PER_RAW = kWeightUnits ? 4 : 2;  // 64-wide K blocks per raw stage
  static constexpr int KT = kWeightUnits ? 256 : kFp4KTile;  // K per unit
  static constexpr int TOK_STAGES = kWeightUnits ? 3 : kTokStages;
  static constexpr int W_STAGES = kWeightUnits ? 3 : kWStages;
  static constexpr int RAW_STAGES = kRawStages;
};

template <int FMT>
constexpr size_t tc_smem() {
  using F = TcFmt<FMT>;
  return 1024 /*align*/ + size_t(F::TOK_STAGES) * kTokBytes + size_t(F::W_STAGES) * kWBytes +
         size_t(F::RAW_STAGES) * F::RAW + 256 /*barriers*/;
}

// ---- tcgen05 helpers
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  // K-major, 128B swizzle: rows of 128 B, 8-row atoms 1024 B apart (SBO), LBO unused (1)
  return uint64_t((smem_addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16, D f32, A and B f16, both K-major, N = BNW, M = BM
constexpr uint32_t kIdesc = (1u << 4) | (uint32_t(BNW >> 3) << 17) | (uint32_t(BM >> 4) << 24);
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ __half swiglu1(float g, float u, float limit) {
  g = g > limit ? limit : g;
  u = u > limit ? limit : u;
  u = u < -limit ? -limit : u;
  return __float2half_rn(__fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u));
}

}  // namespace

template <int FMT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const TcArgs a, const __grid_constant__ CUtensorMap tmap) {
  using F = TcFmt<FMT>;
  constexpr int kTokStages = F::TOK_STAGES, kWStages = F::W_STAGES, kRawStages = F::RAW_STAGES;
  static_assert(tc_smem<FMT>() <= 227 * 1024, "shared memory");
  extern __shared__ uint8_t smem_raw[];
  // 1024-aligned tiles (swizzle atoms)
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - smem_u32(smem_raw));
  uint8_t* tok = base;                                  // [kTokStages][16 KB]
  uint8_t* wt = tok + kTokStages * kTokBytes;           // [kWStages][32 KB]
  uint8_t* raw = wt + kWStages * kWBytes;               // [kRawStages][RAW]
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + kRawStages * F::RAW);
  uint64_t* tok_full = bars;                          // TMA tx
  uint64_t* tok_empty = tok_full + kTokStages;        // MMA commit
  uint64_t* w_full = tok_empty + kTokStages;          // dequant warps
  uint64_t* w_empty = w_full + kWStages;              // MMA commit
  uint64_t* raw_full = w_empty + kWStages;            // bulk tx
  uint64_t* raw_empty = raw_full + kRawStages;        // dequant warps
  uint64_t* acc_full = raw_empty + kRawStages;        // [2] MMA commit
  uint64_t* acc_empty = acc_full + 2;                 // [2] epilogue warps
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  volatile int* abort_ptr = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTokStages; ++s) {
      mbar_init(&tok_full[s], 1);
      mbar_init(&tok_empty[s], 1);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&w_full[s], kDequantWarps);
      mbar_init(&w_empty[s], 1);
    }
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kDequantWarps);
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  pdl_wait();  // the plan, gathered rows and (W2) SwiGLU rows of the launches before are complete

  const int n_kb = a.K / BK;
  const int n_kt = a.K / F::KT;
  const int n_items = a.n_chunks[a.bank] * a.n_rt;

  auto item_ok = [&](const Chunk& ch) {
    return ch.slot >= 0 && ch.slot < a.n_slots && ch.count >= 1 && ch.count <= BM && ch.begin >= 0 &&
           ch.begin + ch.count <= a.S;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t gt = 0, graw = 0;
      uint32_t issued_t = 0, par_t = 0, issued_r = 0, par_r = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const Chunk ch = a.chunks[item / a.n_rt];
        if (!item_ok(ch)) {
          set_error(a.err, kErrBounds);
          continue;
        }
        const int rt = item % a.n_rt;
        const uint8_t* wbase = a.region + int64_t(ch.slot) * a.slot_stride;
        for (int kb = 0; kb < n_kb; ++kb) {
          if (kb % F::KB_PER_RAW == 0) {
            const int r = graw % kRawStages;
            const uint32_t ph = (graw / kRawStages) & 1u;
            if (*abort_ptr || !mbar_wait(&raw_empty[r], ph ^ 1u, a.err)) {
              *abort_ptr = 1;
              break;
            }
            mbar_arrive_expect_tx(&raw_full[r], uint32_t(F::RAW));
            const int kt = kb / F::KB_PER_RAW;
            if (F::kWeightUnits) {  // the item's weight unit of this K tile: one copy
              bulk_g2s_hint(raw + r * F::RAW, wbase + (int64_t(rt) * n_kt + kt) * F::U, F::U, &raw_full[r], pol);
            } else {
              for (int u = 0; u < kUnits; ++u) {
                const int tp = rt * kUnits + u;
                bulk_g2s_hint(raw + r * F::RAW + u * F::U, wbase + (int64_t(tp) * n_kt + kt) * F::U, F::U,
                              &raw_full[r], pol);
              }
            }
            issued_r |= 1u << r;
            par_r = (par_r & ~(1u << r)) | (ph << r);
            ++graw;
          }
          const int s = gt % kTokStages;
          const uint32_t ph = (gt / kTokStages) & 1u;
          if (*abort_ptr || !mbar_wait(&tok_empty[s], ph ^ 1u, a.err)) {
            *abort_ptr = 1;
            break;
          }
          mbar_arrive_expect_tx(&tok_full[s], uint32_t(kTokBytes));
          tma_load_2d(tok + s * kTokBytes, &tmap, kb * BK, ch.begin, &tok_full[s]);
          issued_t |= 1u << s;
          par_t = (par_t & ~(1u << s)) | (ph << s);
          ++gt;
        }
        if (*abort_ptr) break;
      }
      // no copy may be in flight when the CTA exits
      for (int s = 0; s < kTokStages; ++s)
        if (issued_t & (1u << s)) mbar_wait(&tok_full[s], (par_t >> s) & 1u, a.err);
      for (int r = 0; r < kRawStages; ++r)
        if (issued_r & (1u << r)) mbar_wait(&raw_full[r], (par_r >> r) & 1u, a.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t gk = 0, acc_i = 0;
      bool committed = false;
      uint32_t last_b = 0, last_ph = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const Chunk ch = a.chunks[item / a.n_rt];
        if (!item_ok(ch)) continue;
        const uint32_t b = acc_i & 1u, bph = (acc_i >> 1) & 1u;
        if (*abort_ptr || !mbar_wait(&acc_empty[b], bph ^ 1u, a.err)) {
          *abort_ptr = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem_base + b * BNW;
        bool ok = true;
        for (int kb = 0; kb < n_kb; ++kb, ++gk) {
          const int st = gk % kTokStages, sw = gk % kWStages;
          const uint32_t pt = (gk / kTokStages) & 1u, pw = (gk / kWStages) & 1u;
          if (*abort_ptr || !mbar_wait(&tok_full[st], pt, a.err) || !mbar_wait(&w_full[sw], pw, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aaddr = smem_u32(tok + st * kTokBytes), baddr = smem_u32(wt + sw * kWBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(dcol, umma_desc_sw128(aaddr + k * 32), umma_desc_sw128(baddr + k * 32), (kb | k) != 0);
          umma_commit(&tok_empty[st]);
          umma_commit(&w_empty[sw]);
        }
        // commit even a partial item, so its MMAs can be waited for before exit
        umma_commit(&acc_full[b]);
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
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------ dequant
    // the 16 pieces of a block (8 tile pairs x 2 m16 row tiles) spread over the dequant warps
    const int dw = warp - 2;
    const int r = lane >> 2, q = lane & 3;
    uint32_t gk = 0, graw = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const Chunk ch = a.chunks[item / a.n_rt];
      if (!item_ok(ch)) continue;
      // MXFP4 weight units: the rebase exponent of this thread's projection, once per item (global =
      // 2^(gexp - 1)); a global load inside the K loop below stalled every block on its latency
      int gexp = 0;
      if (FMT == 3) frexpf(a.globals[ch.slot * 3 + (EPI == 0 ? ((dw * 32 + lane) >> 7) : 2)], &gexp);
      bool ok = true;
      for (int kb = 0; kb < n_kb && ok; ++kb, ++gk) {
        const int rs = graw % kRawStages;
        const uint32_t rph = (graw / kRawStages) & 1u;
        if (kb % F::KB_PER_RAW == 0) {
          ok = !*abort_ptr && mbar_wait(&raw_full[rs], rph, a.err);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
        }
        const int sw = gk % kWStages;
        const uint32_t pw = (gk / kWStages) & 1u;
        ok = !*abort_ptr && mbar_wait(&w_empty[sw], pw ^ 1u, a.err);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        uint8_t* dst = wt + sw * kWBytes;
        const int half = kb & 1;
        if (F::kWeightUnits) {
          // one weight row per thread: B row = its row in the unit (W13: gate tile then up tile; W2: the
          // 256 rows in order), the 64 K of this block = 16-byte chunks 2 q, 2 q + 1 of the swizzled row
          const int row = dw * 32 + lane, tile = row >> 7, rr = row & 127, q4 = kb & 3;
          const uint8_t* unit = raw + rs * F::RAW;
          const uint8_t* crow = unit + tile * (128 * 128) + rr * 128;
          const uint32_t sw4 =
              *reinterpret_cast<const uint32_t*>(unit + 2 * (128 * 128) + tile * 2048 + q4 * 512 + (rr & 31) * 16 +
                                                 (rr >> 5) * 4);
          uint32_t sc[4];
          if (FMT == 2) {  // four E4M3 scales, one per 16
            const uint32_t p01 = e4m3x2_to_f16x2(sw4 & 0xffffu), p23 = e4m3x2_to_f16x2(sw4 >> 16);
            sc[0] = lo_half2(p01);
            sc[1] = hi_half2(p01);
            sc[2] = lo_half2(p23);
            sc[3] = hi_half2(p23);
          } else {  // two E8M0 scales, one per 32, as f16 2^(e - 127 - rebase)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              int f = int((sw4 >> (8 * j)) & 255u) - 127 - (gexp - 1) + 15;
              f = f < 1 ? 1 : f > 30 ? 30 : f;  // out-of-range blocks are all-zero (checked at load)
              sc[2 * j] = sc[2 * j + 1] = (uint32_t(f) << 10) * 0x10001u;
            }
          }
          uint8_t* drow = dst + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int c = 2 * q4 + cc;
            const uint4 cw = *reinterpret_cast<const uint4*>(crow + ((c ^ (rr & 7)) << 4));
            const uint32_t wv[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {  // elements 32 cc + 8 w .. +7: 16-wide block 2 cc + w / 2
              uint32_t o[4];
              e2m1x8_scaled(wv[w], sc[2 * cc + (w >> 1)], o);
              *reinterpret_cast<uint4*>(drow + (((4 * cc + w) ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        } else {
#pragma unroll
        for (int pc = dw; pc < 2 * kUnits; pc += kDequantWarps) {
          const int u = pc >> 1, mt = pc & 1;
          const uint8_t* unit = raw + rs * F::RAW + u * F::U;
          const uint2 sc = FMT == 0 ? *reinterpret_cast<const uint2*>(unit + 2048 + mt * 128 + (r * 2 + (q >> 1)) * 8)
                                    : *reinterpret_cast<const uint2*>(unit + 2048 + mt * 64 + r * 8);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 cw = *reinterpret_cast<const uint4*>(unit + mt * 1024 + h * 512 + lane * 16);
            const uint32_t swd = h == 0 ? sc.x : sc.y;
            // this K half's two scales as broadcast f16x2 (bytes 2*half, 2*half + 1 of swd)
            uint32_t s2[2];
            if (FMT == 0) {
              const uint32_t pair = e4m3x2_to_f16x2(half ? (swd >> 16) : swd);
              s2[0] = lo_half2(pair);
              s2[1] = hi_half2(pair);
            } else {
              const uint32_t b0 = half ? (swd >> 16) & 255u : swd & 255u;
              const uint32_t b1 = half ? (swd >> 24) : (swd >> 8) & 255u;
              s2[0] = (b0 << 10) * 0x10001u;
              s2[1] = (b1 << 10) * 0x10001u;
            }
            // W13: B rows 0-127 = gate rows of the 8 pairs, 128-255 = their up rows
            // W2: B rows = the 256 rows of the 8 pairs in order
            const int row = EPI == 0 ? mt * 128 + u * 16 + r + 8 * h : u * 32 + mt * 16 + r + 8 * h;
            uint8_t* drow = dst + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              const uint32_t w = half ? (cc ? cw.w : cw.z) : (cc ? cw.y : cw.x);
              uint32_t o[4];
              e2m1x8_scaled(w, s2[cc], o);
              // elements 32cc + 8q .. +7 of this 64-wide K block, chunk 4cc + q (128B swizzle)
              *reinterpret_cast<uint4*>(drow + (((cc * 4 + q) ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        }
        }
        fence_proxy_async();
        __syncwarp();
        const bool raw_done = kb % F::KB_PER_RAW == F::KB_PER_RAW - 1;
        if (lane == 0) {
          mbar_arrive(&w_full[sw]);
          if (raw_done) mbar_arrive(&raw_empty[rs]);
        }
        if (raw_done) ++graw;
      }
      if (!ok) {
        *abort_ptr = 1;
        break;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;           // TMEM lanes 32*quarter ..
    const int n = quarter * 32 + lane;      // route of this thread in the token tile
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
      tc_fence_after();
      const float* gl = a.globals + ch.slot * 3;
      const bool mine = n < ch.count;
      const int p = ch.begin + n;
      const int route = mine ? a.perm[p] : 0;
      const uint32_t tcol = tmem_base + (uint32_t(quarter * 32) << 16) + b * BNW;
      if (EPI == 0) {
        const float g1 = gl[0], g3 = gl[1];
        __half* irow = static_cast<__half*>(a.inter) + int64_t(p) * a.inter_stride + rt * 128;
        for (int cc = 0; cc < 4; ++cc) {
          float gv[32], uv[32];
          tmem_ld32(tcol + cc * 32, gv);
          tmem_ld32(tcol + 128 + cc * 32, uv);
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            // fp16 y13 as the reference rounds it, then the limited SwiGLU
            const __half h0 = swiglu1(__half2float(__float2half_rn(gv[2 * i] * g1)),
                                      __half2float(__float2half_rn(uv[2 * i] * g3)), a.limit);
            const __half h1 = swiglu1(__half2float(__float2half_rn(gv[2 * i + 1] * g1)),
                                      __half2float(__float2half_rn(uv[2 * i + 1] * g3)), a.limit);
            o[i] = uint32_t(__half_as_ushort(h0)) | (uint32_t(__half_as_ushort(h1)) << 16);
          }
          if (mine) {
            uint4* dst = reinterpret_cast<uint4*>(irow + cc * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
          }
        }
      } else {
        const float g2 = gl[2];
        __half* yrow = static_cast<__half*>(a.y2) + int64_t(route) * a.H + rt * BNW;
        for (int cc = 0; cc < BNW / 32; ++cc) {
          float v[32];
          tmem_ld32(tcol + cc * 32, v);
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const __half2 h2 = __floats2half2_rn(v[2 * i] * g2, v[2 * i + 1] * g2);
            o[i] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          if (mine) {
            uint4* dst = reinterpret_cast<uint4*>(yrow + cc * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      ++acc_i;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
  }
  pdl_trigger();  // the next launch may take this SM (and its TMEM) now
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// fp16 [rows][cols] row-major, box [BM rows x BK cols], 128B swizzle.
int make_token_map(void* map_out, const void* base, int64_t rows, int64_t cols) {
  auto fn = encode_fn();
  if (!fn) return -1;
  CUtensorMap* m = static_cast<CUtensorMap*>(map_out);
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols * 2)};
  cuuint32_t box[2] = {cuuint32_t(BK), cuuint32_t(BM)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1;
}

size_t tc_map_bytes() { return sizeof(CUtensorMap); }

template <int FMT, int EPI>
static int launch_tc_one(cudaStream_t s, const TcArgs& a, const void* map, int grid) {
  const size_t smem = tc_smem<FMT>();
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << dev))) {
    if (cudaFuncSetAttribute(tc_gemm_kernel<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
        cudaSuccess)
      return -1;
    attr_dev_mask |= 1 << dev;
  }
  return launch_chain(tc_gemm_kernel<FMT, EPI>, dim3(grid), dim3(kThreads), smem, s, a,
                      *static_cast<const CUtensorMap*>(map)) == cudaSuccess
             ? 0
             : -1;
}

int make_u8_tile_map(void* map_out, const void* base, int64_t rows, int64_t row_bytes, int box_bytes, int box_rows) {
  auto fn = encode_fn();
  if (!fn || row_bytes % 16 || box_bytes > 128 || (reinterpret_cast<uintptr_t>(base) & 15)) return -1;
  CUtensorMap* m = static_cast<CUtensorMap*>(map_out);
  cuuint64_t dims[2] = {cuuint64_t(row_bytes), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(row_bytes)};
  cuuint32_t box[2] = {cuuint32_t(box_bytes), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1;
}

int launch_tc_gemm(cudaStream_t s, int fmt, int epi, const TcArgs& a, const void* map, int grid) {
  if (fmt == 0) return epi == 0 ? launch_tc_one<0, 0>(s, a, map, grid) : launch_tc_one<0, 1>(s, a, map, grid);
  if (fmt == 1) return epi == 0 ? launch_tc_one<1, 0>(s, a, map, grid) : launch_tc_one<1, 1>(s, a, map, grid);
  if (fmt == 2) return epi == 0 ? launch_tc_one<2, 0>(s, a, map, grid) : launch_tc_one<2, 1>(s, a, map, grid);
  if (fmt == 3) return epi == 0 ? launch_tc_one<3, 0>(s, a, map, grid) : launch_tc_one<3, 1>(s, a, map, grid);
  return -1;
}

// ---------------------------------------------------- permuted fp16 rows
// xperm[p] = fp16(x[perm[p] / k]) for p < S (x fp16 or bf16).  One warp per sorted row: the row's token is
// one load, then the lanes issue all of a 4 KB slice's 16-byte loads before the first store, so each warp keeps
// the slice in flight instead of one dependent perm -> x -> store chain per thread.
__device__ __forceinline__ uint4 row_to_f16(uint4 v, int bf16) {
  if (!bf16) return v;
  uint32_t in[4] = {v.x, v.y, v.z, v.w}, o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 h2 = __floats2half2_rn(__uint_as_float(in[j] << 16), __uint_as_float(in[j] & 0xffff0000u));
    o[j] = *reinterpret_cast<uint32_t*>(&h2);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

constexpr int kGatherThreads = 256;

__global__ void __launch_bounds__(kGatherThreads) gather_rows_kernel(const uint16_t* __restrict__ x, int bf16,
                                                                     const int32_t* __restrict__ perm, int S, int k,
                                                                     int H, uint16_t* __restrict__ xperm) {
  constexpr int kU = 8;  // 16-byte loads in flight per lane
  const int per_row = H / 8;
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (kGatherThreads / 32);
  pdl_wait();
  pdl_trigger();
  for (int p = blockIdx.x * (kGatherThreads / 32) + threadIdx.x / 32; p < S; p += warps) {
    const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(perm[p] / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(xperm + int64_t(p) * H);
    for (int c0 = 0; c0 < per_row; c0 += 32 * kU) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int c = c0 + 32 * u + lane;
        if (c < per_row) v[u] = src[c];
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int c = c0 + 32 * u + lane;
        if (c < per_row) dst[c] = row_to_f16(v[u], bf16);
      }
    }
  }
}

int launch_gather_rows(cudaStream_t s, const void* x, int bf16, const int32_t* perm, int S, int k, int H,
                       void* xperm) {
  const int rows_per_block = kGatherThreads / 32;
  const int blocks = std::min((S + rows_per_block - 1) / rows_per_block, 148 * 8);
  return launch_chain(gather_rows_kernel, dim3(blocks < 1 ? 1 : blocks), dim3(kGatherThreads), 0, s,
                      static_cast<const uint16_t*>(x), bf16, perm, S, k, H, static_cast<uint16_t*>(xperm)) ==
                 cudaSuccess
             ? 0
             : -1;
}

}  // namespace b200moe
