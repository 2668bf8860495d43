// Skinny grouped expert GEMM for decode (1..16 routes per expert chunk).
//
// Replaces the reference's grouped QPN launches (engine/.../experts/nvfp4_8r_native.py:929-944,
// external skinny_moe_qpn_sm70) plus its SwiGLU (nvfp4_8r_swiglu.py) and weighted
// reduce (_mtp_weighted_reduce, restated at nvfp4_8r_iq_tail.py:106-120).
//
// Persistent CTAs (two per SM for FP4, one for IQ2) walk work items (route chunk
// x row block).  Warp 8 is the producer: it streams each item's prepacked weight
// units and the chunk's activation rows into a shared-memory ring (4 stages FP4,
// 6 IQ2) with cp.async.bulk, completion counted on mbarriers.  Warps 0..7
// consume: each owns one tile pair (32 weight rows) of the item and one of ks K
// slices (ks = the split-K the route plan chose for this call, read at run
// time; a chunk holds 16 / ks routes); it dequantizes 4-bit codes to f16 in
// registers (cvt.e2m1x2, block scale exact in f16) and multiplies on the tensor
// cores (m16n8k16, f32 accumulate), routes as the N dimension.
//   EPI 0 (W13): y13 = acc * global, rounded to fp16 as the reference's y13 is,
//     then the limited SwiGLU in FP32 -> fp16 inter rows (by route position).
//   EPI 1 (W2): y2[route] = fp16(acc * global), the reference's fp16 y2 row;
//     the CTA that completes a (token, 32-row tile) -- counted with one atomic
//     per route -- forms sum over slots of f32(y2) * router weight in slot
//     order (the reference's weighted reduce) and writes out.  The sum is
//     always taken in slot order, so the result does not depend on timing.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "internal.h"
#include "layout.cuh"

namespace b200moe {

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kRouteSlots = kRouteSlotsPerChunk;  // activation row slots per stage (KS * route chunk)

// FP4: two CTAs per SM (18 warps) with a 4-stage ring each; IQ2: one CTA with 6.
template <int FMT>
struct Fmt {
  static constexpr int KT = FMT == 2 ? kIq2KTile : kFp4KTile;            // K per unit
  static constexpr int U = FMT == 2 ? kIq2UnitBytes : fp4_unit_bytes(FMT); // unit bytes
  static constexpr int XRS = 2 * KT + 64;                                // x row slot bytes
  static constexpr int STAGE = kConsumerWarps * U + kRouteSlots * XRS;
  static constexpr int CTAS = FMT == 2 ? 1 : 2;                          // CTAs per SM
  static constexpr int STAGES = CTAS == 2 ? 4 : 6;
};
constexpr int kMaxStages = 6;

constexpr int kRedBytes = kConsumerWarps * 32 * 16 * 4;
constexpr int kIq2TableWords = 256 * 4 + 128 * 4 + 16;  // grid f16, sign masks, (0.5 + s) f16x2
constexpr int kListInts = 1 + 2 * 128;

template <int FMT>
constexpr size_t smem_total() {
  return 128 + size_t(Fmt<FMT>::STAGES) * Fmt<FMT>::STAGE + kRedBytes + (FMT == 2 ? kIq2TableWords * 4 : 0) +
         kListInts * 4;
}

size_t gemv_smem_bytes(int fmt, int) {
  return fmt == 0 ? smem_total<0>() : fmt == 1 ? smem_total<1>() : smem_total<2>();
}

int gemv_ctas_per_sm(int fmt) { return fmt == 2 ? Fmt<2>::CTAS : Fmt<0>::CTAS; }

// ---------------------------------------------------------------- FP4 step
// acc[mt][nt][j]: one accumulator per k16 step parity, so each tile has two
// independent MMA chains; they are summed in the epilogue.
template <int FMT>
__device__ __forceinline__ void fp4_step(uint32_t wb, uint32_t xb, int ntiles, int lane,
                                         float (&acc)[2][2][2][4]) {
  constexpr int XRS = Fmt<FMT>::XRS;
  const int r = lane >> 2, q = lane & 3;
  uint4 cw[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) cw[mt][h] = lds128(wb + mt * 1024 + h * 512 + lane * 16);
  // block scales of this thread's rows (r, r + 8) for the 4 K chunks of the
  // stage, as f16x2 with the scale in both halves: sh[mt][row half][chunk]
  uint32_t sh[2][2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const uint2 sc = FMT == 0 ? lds64(wb + 2048 + mt * 128 + (r * 2 + (q >> 1)) * 8) : lds64(wb + 2048 + mt * 64 + r * 8);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t v = h == 0 ? sc.x : sc.y;  // bytes: chunks 0..3
      if (FMT == 0) {
        const uint32_t h01 = e4m3x2_to_f16x2(v), h23 = e4m3x2_to_f16x2(v >> 16);
        sh[mt][h][0] = lo_half2(h01);
        sh[mt][h][1] = hi_half2(h01);
        sh[mt][h][2] = lo_half2(h23);
        sh[mt][h][3] = hi_half2(h23);
      } else {
        // rebased E8M0 exponent b -> f16 2^(b - 15) in both halves: b << 10 | b << 26
#pragma unroll
        for (int c = 0; c < 4; ++c) sh[mt][h][c] = __byte_perm(v, 0, 0x0404u | (c << 12) | (c << 4)) << 2;
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 xv[2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
      if (nt < ntiles) xv[nt] = lds128(xb + (nt * 8 + r) * XRS + c * 64 + q * 16);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint32_t s0 = sh[mt][0][c], s1 = sh[mt][1][c];
      const uint32_t w0 = c == 0 ? cw[mt][0].x : c == 1 ? cw[mt][0].y : c == 2 ? cw[mt][0].z : cw[mt][0].w;
      const uint32_t w1 = c == 0 ? cw[mt][1].x : c == 1 ? cw[mt][1].y : c == 2 ? cw[mt][1].z : cw[mt][1].w;
      uint32_t o0[4], o1[4];
      e2m1x8_scaled(w0, s0, o0);  // row r: bytes 0,1 -> k16 step 0, bytes 2,3 -> step 1
      e2m1x8_scaled(w1, s1, o1);  // row r + 8
      uint32_t a[4] = {o0[0], o1[0], o0[1], o1[1]};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
        if (nt < ntiles) mma_16816(acc[mt][nt][0], a, xv[nt].x, xv[nt].y);
      uint32_t a2[4] = {o0[2], o1[2], o0[3], o1[3]};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
        if (nt < ntiles) mma_16816(acc[mt][nt][1], a2, xv[nt].z, xv[nt].w);
    }
  }
}

// ---------------------------------------------------------------- IQ2 step
// One 256-wide super-block.  A = grid * sign * (0.5 + s) is exact in f16; the
// super-block scale d * 0.25 is applied to a per-block partial in FP32.
__device__ __forceinline__ void iq2_step(uint32_t wb, uint32_t xb, uint32_t tbl, int ntiles, int lane,
                                         float (&acc)[2][2][2][4]) {
  constexpr int XRS = Fmt<2>::XRS;
  const int r = lane >> 2, q = lane & 3;
  float t[2][2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) t[mt][nt][i] = 0.f;
  const uint32_t tgrid = tbl, tsign = tbl + 256 * 16, tscale = tbl + 256 * 16 + 128 * 16;
#pragma unroll 1
  for (int ibp = 0; ibp < 4; ++ibp) {
    uint4 qw[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) qw[mt][h] = lds128(wb + mt * 1024 + h * 512 + r * 64 + ibp * 16);
#pragma unroll
    for (int i2 = 0; i2 < 2; ++i2) {
      const int ib = 2 * ibp + i2;
      uint4 xv[2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
        if (nt < ntiles) xv[nt] = lds128(xb + (nt * 8 + r) * XRS + ib * 64 + q * 16);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t v[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t a0 = i2 == 0 ? qw[mt][h].x : qw[mt][h].z;
          const uint32_t a1 = i2 == 0 ? qw[mt][h].y : qw[mt][h].w;
          const uint32_t gi = (a0 >> (8 * q)) & 255u;
          const uint32_t si = (a1 >> (7 * q)) & 127u;
          const uint32_t sc = lds32(tscale + (a1 >> 28) * 4);
          const uint4 g4 = lds128(tgrid + gi * 16);
          const uint4 m4 = lds128(tsign + si * 16);
          v[h][0] = hmul2(g4.x ^ m4.x, sc);
          v[h][1] = hmul2(g4.y ^ m4.y, sc);
          v[h][2] = hmul2(g4.z ^ m4.z, sc);
          v[h][3] = hmul2(g4.w ^ m4.w, sc);
        }
        uint32_t a[4] = {v[0][0], v[1][0], v[0][1], v[1][1]};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          if (nt < ntiles) mma_16816(t[mt][nt], a, xv[nt].x, xv[nt].y);
        uint32_t a2[4] = {v[0][2], v[1][2], v[0][3], v[1][3]};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          if (nt < ntiles) mma_16816(t[mt][nt], a2, xv[nt].z, xv[nt].w);
      }
    }
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const uint32_t dp = lds32(wb + 2048 + mt * 32 + r * 4);
    const __half2 d2 = *reinterpret_cast<const __half2*>(&dp);
    const float d0 = __low2float(d2) * 0.25f, d1 = __high2float(d2) * 0.25f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      acc[mt][nt][0][0] = fmaf(t[mt][nt][0], d0, acc[mt][nt][0][0]);
      acc[mt][nt][0][1] = fmaf(t[mt][nt][1], d0, acc[mt][nt][0][1]);
      acc[mt][nt][0][2] = fmaf(t[mt][nt][2], d1, acc[mt][nt][0][2]);
      acc[mt][nt][0][3] = fmaf(t[mt][nt][3], d1, acc[mt][nt][0][3]);
    }
  }
}

__device__ __forceinline__ bool chunk_ok(const Chunk& ch, int rc, const GemvArgs& a) {
  return ch.slot >= 0 && ch.slot < a.n_slots && ch.count >= 1 && ch.count <= rc && ch.begin >= 0 &&
         ch.begin + ch.count <= a.S;
}

// Limited SwiGLU of one (gate, up) pair, FP32 round-to-nearest ops on the
// fp16-rounded y13 values; NaN passes through the clamps.
__device__ __forceinline__ __half swiglu_one(float g, float u, float limit) {
  g = g > limit ? limit : g;
  u = u > limit ? limit : u;
  u = u < -limit ? -limit : u;
  const float act = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
  return __float2half_rn(__fmul_rn(act, u));
}

template <int FMT, int EPI, int KS>
__device__ __forceinline__ void gemv_body(const GemvArgs& a, uint8_t* smem) {
  using F = Fmt<FMT>;
  constexpr int kStages = F::STAGES;
  constexpr int TP = kConsumerWarps / KS;  // tile pairs per item
  constexpr int RC = kRouteSlots / KS;     // routes per chunk
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStages;
  uint8_t* stages = smem + 128;
  float* red = reinterpret_cast<float*>(stages + size_t(kStages) * F::STAGE);  // [warp][16][lane]
  uint32_t* tables = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(red) + kRedBytes);
  int* list = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(tables) + (FMT == 2 ? kIq2TableWords * 4 : 0));
  __shared__ int abort_flag;
  volatile int* abort_ptr = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
    abort_flag = 0;
    list[0] = 0;
  }
  if (FMT == 2)
    for (int i = threadIdx.x; i < kIq2TableWords; i += kGemvThreads) tables[i] = a.iq2_tables[i];
  __syncthreads();

  const int n_kt = a.K / F::KT;
  const int steps = n_kt / KS;
  const int n_rb = a.n_tp / TP;
  const int n_items = a.n_chunks[a.bank] * n_rb;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = policy_evict_first();
    uint32_t g = 0;
    uint32_t issued = 0, parity = 0;  // per stage: copies issued, parity of the last issue
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const Chunk ch = a.chunks[item / n_rb];
      if (!chunk_ok(ch, RC, a)) {
        if (lane == 0) set_error(a.err, kErrBounds);
        continue;
      }
      const int rb = item % n_rb;
      const uint8_t* wbase = a.region + int64_t(ch.slot) * a.slot_stride;
      // activation row of this lane's copy (lanes 8 .. 8 + KS*RC)
      const int xi = lane - 8;
      const int xks = xi / RC, xj = xi % RC;
      const bool xlane = xi >= 0 && xi < KS * RC && xj < ch.count;
      int64_t xrow = 0;
      if (xlane) {
        const int p = ch.begin + xj;
        xrow = a.x_by_token ? a.perm[p] / a.top_k : p;
        if (xrow < 0 || xrow >= a.n_x_rows) {
          set_error(a.err, kErrBounds);
          xrow = 0;
        }
      }
      const uint32_t tx = uint32_t(kConsumerWarps * F::U + KS * ch.count * 2 * F::KT);
      for (int st = 0; st < steps; ++st, ++g) {
        const int s = g % kStages;
        const uint32_t ph = (g / kStages) & 1u;
        bool ok = !*abort_ptr && mbar_wait(&empty[s], ph ^ 1u, a.err);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          *abort_ptr = 1;
          continue;
        }
        uint8_t* sb = stages + size_t(s) * F::STAGE;
        issued |= 1u << s;
        parity = (parity & ~(1u << s)) | (ph << s);
        if (lane == 0) mbar_arrive_expect_tx(&full[s], tx);
        __syncwarp();
        if (lane < kConsumerWarps) {
          const int tpl = lane / KS, ks = lane % KS;
          const int tp = rb * TP + tpl, kt = ks * steps + st;
          bulk_g2s_hint(sb + lane * F::U, wbase + (int64_t(tp) * n_kt + kt) * F::U, F::U, &full[s], pol);
        } else if (xlane) {
          const int kt = xks * steps + st;
          const uint8_t* src = static_cast<const uint8_t*>(a.xsrc) + (xrow * a.x_row_stride + int64_t(kt) * F::KT) * 2;
          bulk_g2s(sb + kConsumerWarps * F::U + xi * F::XRS, src, 2 * F::KT, &full[s]);
        }
      }
    }
    // No bulk copy may still be in flight when the CTA exits (after an abort the
    // consumers stop waiting): wait, bounded, for the last issue of every stage.
    if (lane == 0) {
      for (int s = 0; s < kStages; ++s)
        if (issued & (1u << s)) mbar_wait(&full[s], (parity >> s) & 1u, a.err);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int ks = warp % KS, tpl = warp / KS;
    const int r = lane >> 2, q = lane & 3;
    const uint32_t tbl = smem_u32(tables);
    uint32_t g = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const Chunk ch = a.chunks[item / n_rb];
      if (!chunk_ok(ch, RC, a)) continue;
      const int rb = item % n_rb;
      const int tp = rb * TP + tpl;
      const int ntiles = (ch.count + 7) >> 3;
      float acc2[2][2][2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc2[mt][nt][j][i] = 0.f;
      for (int st = 0; st < steps; ++st, ++g) {
        const int s = g % kStages;
        const uint32_t ph = (g / kStages) & 1u;
        bool ok = !*abort_ptr && mbar_wait(&full[s], ph, a.err);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          *abort_ptr = 1;
          continue;
        }
        const uint32_t sb = smem_u32(stages + size_t(s) * F::STAGE);
        const uint32_t wb = sb + warp * F::U;
        const uint32_t xb = sb + kConsumerWarps * F::U + ks * RC * F::XRS;
        if (FMT == 2) iq2_step(wb, xb, tbl, ntiles, lane, acc2);
        else fp4_step<FMT>(wb, xb, ntiles, lane, acc2);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      float acc[2][2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[mt][nt][i] = acc2[mt][nt][0][i] + acc2[mt][nt][1][i];
      // split-K partials: fixed order ks = 0, 1, ..
      if (KS > 1) {
        float* mine = red + warp * 32 * 16 + lane;
        if (ks != 0) {
#pragma unroll
          for (int i = 0; i < 16; ++i) mine[i * 32] = (&acc[0][0][0])[i];
        }
        named_bar(1, kConsumerWarps * 32);
        if (ks == 0) {
          for (int kk = 1; kk < KS; ++kk) {
            const float* other = red + (warp + kk) * 32 * 16 + lane;
#pragma unroll
            for (int i = 0; i < 16; ++i) (&acc[0][0][0])[i] += other[i * 32];
          }
        }
        named_bar(1, kConsumerWarps * 32);
      }
      const bool aborted = *abort_ptr != 0;
      if (ks == 0 && !aborted) {
        const float* gl = a.globals ? a.globals + ch.slot * 3 : nullptr;
        if (EPI == 0) {
          const float g1 = gl ? gl[0] : 1.f, g3 = gl ? gl[1] : 1.f;
          __half* inter = static_cast<__half*>(a.inter);
          __half* dbg = static_cast<__half*>(a.dbg_y13);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int n = nt * 8 + 2 * q + e;
              if (n >= ch.count) continue;
              const int p = ch.begin + n;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int j = 16 * tp + r + 8 * h;
                const __half gh = __float2half_rn(acc[0][nt][2 * h + e] * g1);
                const __half uh = __float2half_rn(acc[1][nt][2 * h + e] * g3);
                inter[int64_t(p) * a.inter_stride + j] = swiglu_one(__half2float(gh), __half2float(uh), a.limit);
                if (dbg) {
                  dbg[int64_t(p) * 2 * a.inter_stride + j] = gh;
                  dbg[int64_t(p) * 2 * a.inter_stride + a.inter_stride + j] = uh;
                }
              }
            }
        } else {
          const float g2 = gl ? gl[2] : 1.f;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int n = nt * 8 + 2 * q + e;
              if (n >= ch.count) continue;
              const int route = a.perm[ch.begin + n];
              __half* yrow = static_cast<__half*>(a.y2) + int64_t(route) * a.H;
#pragma unroll
              for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                  yrow[32 * tp + 16 * mt + r + 8 * h] = __float2half_rn(acc[mt][nt][2 * h + e] * g2);
            }
        }
      }
      if (EPI == 1) {
        // completion count per (token, 32-row tile); the last route sums in slot order
        __threadfence();
        named_bar(1, kConsumerWarps * 32);
        const int t = threadIdx.x;
        if (!aborted && t < ch.count * TP) {
          const int n = t / TP, tl = t % TP;
          const int route = a.perm[ch.begin + n];
          const int tok = route / a.top_k;
          const int tile = rb * TP + tl;
          int* cnt = a.counters + int64_t(tok) * (a.H / 32) + tile;
          const int old = atomicAdd(cnt, 1);
          if (old == a.top_k - 1) {
            const int pos = atomicAdd(&list[0], 1);
            list[1 + 2 * pos] = tok;
            list[2 + 2 * pos] = tile;
          }
        }
        named_bar(1, kConsumerWarps * 32);
        const int nl = list[0];
        for (int e = warp; e < nl; e += kConsumerWarps) {
          const int tok = list[1 + 2 * e], tile = list[2 + 2 * e];
          __threadfence();
          const int row = 32 * tile + lane;
          const unsigned short* y2 = static_cast<const unsigned short*>(a.y2);
          float sum = 0.f;
          for (int slot = 0; slot < a.top_k; ++slot) {
            const int route = tok * a.top_k + slot;
            const float y = __half2float(__ushort_as_half(__ldcg(y2 + int64_t(route) * a.H + row)));
            sum = __fmaf_rn(y, __ldcg(a.w_eff + route), sum);
          }
          a.out[int64_t(tok) * a.H + row] = sum;
          if (lane == 0) a.counters[int64_t(tok) * (a.H / 32) + tile] = 0;
        }
        named_bar(1, kConsumerWarps * 32);
        if (threadIdx.x == 0) list[0] = 0;
      }
    }
  }
  __syncthreads();
}

// One kernel per format and epilogue; the split-K is read from the device
// (chosen by the route plan from this call's chunk counts), so the choice
// follows the routing without a host round trip, also inside a CUDA graph.
template <int FMT, int EPI>
__global__ void __launch_bounds__(kGemvThreads, Fmt<FMT>::CTAS) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  switch (a.ks_sel[a.bank]) {
    case 1: gemv_body<FMT, EPI, 1>(a, smem); break;
    case 2: gemv_body<FMT, EPI, 2>(a, smem); break;
    case 4: gemv_body<FMT, EPI, 4>(a, smem); break;
    case 8: gemv_body<FMT, EPI, 8>(a, smem); break;
    default:
      if (threadIdx.x == 0) set_error(a.err, kErrRange);
  }
}

template <int FMT, int EPI>
static int launch_one(cudaStream_t s, const GemvArgs& a) {
  const size_t smem = smem_total<FMT>();
  static std::atomic<uint64_t> attr_set{0};  // devices whose attribute is set
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return -1;
  if (!(attr_set.load() >> dev & 1)) {
    if (cudaFuncSetAttribute(gemv_kernel<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
        cudaSuccess)
      return -1;
    attr_set.fetch_or(uint64_t(1) << dev);
  }
  gemv_kernel<FMT, EPI><<<a.grid, kGemvThreads, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_gemv(cudaStream_t s, const GemvArgs& a) {
  if (!a.ks_sel) return -1;
  if (a.fmt == 0) return a.epi == 0 ? launch_one<0, 0>(s, a) : launch_one<0, 1>(s, a);
  if (a.fmt == 1) return a.epi == 0 ? launch_one<1, 0>(s, a) : launch_one<1, 1>(s, a);
  if (a.fmt == 2) return a.epi == 0 ? launch_one<2, 0>(s, a) : launch_one<2, 1>(s, a);
  return -1;
}

}  // namespace b200moe
