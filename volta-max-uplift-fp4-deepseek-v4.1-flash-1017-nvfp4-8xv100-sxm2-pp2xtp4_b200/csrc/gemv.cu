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

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "internal.h"
#include "layout.cuh"

namespace b200moe {

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kRouteSlots = kRouteSlotsPerChunk;  // activation row slots per stage (KS * route chunk)

// FMT 0 / 1: NVFP4 / MXFP4; 2 / 3 / 4: the IQ bank's IQ2_XXS / IQ2_XS / IQ1_M.
// FP4: two CTAs per SM (18 warps) with a 4-stage ring each; IQ: one CTA with 6.
template <int FMT>
struct Fmt {
  static constexpr bool IQ = FMT >= 2;
  static constexpr int KT = IQ ? kIq2KTile : kFp4KTile;                  // K per unit
  static constexpr int U = IQ ? iq_unit_bytes(FMT) : fp4_unit_bytes(FMT); // unit bytes
  // activation bytes of one row per K tile (f16 for FP4; int8 + scale for IQ)
  static constexpr int XB = IQ ? kIq2XBlockBytes : 2 * KT;
  static constexpr int XRS = IQ ? 544 : 2 * KT + 64;                     // x row slot bytes
  static constexpr int STAGE = kConsumerWarps * U + kRouteSlots * XRS;
  static constexpr int CTAS = IQ ? 1 : 2;                                // CTAs per SM
  static constexpr int STAGES = CTAS == 2 ? 4 : 6;
  static constexpr int TWG = IQ ? iq_table_words(FMT) : 0;               // decode table words (global)
  // IQ2_XXS keeps 32 copies of its table in shared memory, word w of copy c at w * 32 + c: lane c reads
  // its own copy, so the random grid / sign lookups of a warp never share a bank
  static constexpr int TREP = FMT == 2 ? 32 : 1;
  static constexpr int TW = TWG * TREP;                                  // decode table words (shared)
};
constexpr int kMaxStages = 6;

constexpr int kRedBytes = kConsumerWarps * 32 * 16 * 4;
constexpr int kListInts = 1 + 2 * 128;

template <int FMT>
constexpr size_t smem_total() {
  return 128 + size_t(Fmt<FMT>::STAGES) * Fmt<FMT>::STAGE + kRedBytes + size_t(Fmt<FMT>::TW) * 4 + kListInts * 4;
}

size_t gemv_smem_bytes(int fmt, int) {
  return fmt == 0   ? smem_total<0>()
         : fmt == 1 ? smem_total<1>()
         : fmt == 2 ? smem_total<2>()
         : fmt == 3 ? smem_total<3>()
                    : smem_total<4>();
}

int gemv_ctas_per_sm(int fmt) { return fmt >= 2 ? Fmt<2>::CTAS : Fmt<0>::CTAS; }

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
// One 256-wide super-block on the int8 tensor path.  A weight is
// g * sign * (2s + 1) * d / 8 (ggml's IQ2_XXS: d * (0.5 + s) * 0.25 * g * sign)
// and an activation sx * (q1 + q2 / 254).  Per 32-wide sub-block the int8
// weights g * sign come from two 4-byte table reads and two byte permutes and
// meet both activation planes (two m16n8k32); each s32 partial is scaled by
// the integer 2s + 1 of its row, so the super-block sums stay exact in s32;
// (t1 + t2 / 254) * d / 8 * sx is applied once in FP32.
// Thread q owns elements 8q..8q+7 of each sub-block (grid entry q), which are
// the MMA's K positions 4q..4q+3 and 16+4q..16+4q+3, for weights and activations alike.
// Chunks of at most 4 routes (most decode chunks of the IQ bank) fill only
// half of an n8 MMA tile, so both activation planes share one MMA there
// ("packed"): column n holds route n & 3 of plane n >> 2.  Lanes q = 0, 1 then
// hold plane 1 of routes 2q, 2q + 1 and lanes q + 2 plane 2 of the same
// routes; iq_unpack_planes moves the plane-2 sums to the usual [plane] slots.
// The s32 sums are the same numbers, so both forms give the same bits.
__device__ __forceinline__ void iq_unpack_planes(int (&t)[2][2][2][4], int lane) {
  const bool low = (lane & 3) < 2;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = t[0][mt][0][i];
      const int o = __shfl_xor_sync(0xffffffffu, v, 2);
      t[0][mt][0][i] = low ? v : 0;
      t[1][mt][0][i] = low ? o : 0;
    }
}

template <bool PACK>
__device__ __forceinline__ void iq2_step(uint32_t wb, uint32_t xb, uint32_t tbl, int ntiles, int lane,
                                         float (&acc)[2][2][2][4]) {
  constexpr int XRS = Fmt<2>::XRS;
  constexpr uint32_t kPos = 0x002B1908u, kNeg = 0x00D5E7F8u;  // bytes 8, 25, 43, 0 and -8, -25, -43, 0
  const int r = lane >> 2, q = lane & 3;
  int t[2][2][2][4];  // [plane][mt][nt][i]
#pragma unroll
  for (int pl = 0; pl < 2; ++pl)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) t[pl][mt][nt][i] = 0;
  const uint32_t tl = tbl + lane * 4;  // this lane's copy of the tables (words 32 apart)
  const uint32_t tsign = tl + 256 * 128;
#pragma unroll 2
  for (int ibp = 0; ibp < 4; ++ibp) {
    uint4 qw[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) qw[mt][h] = lds128(wb + mt * 1024 + h * 512 + r * 64 + ibp * 16);
#pragma unroll
    for (int i2 = 0; i2 < 2; ++i2) {
      const int ib = 2 * ibp + i2;
      uint2 xv[2][2];  // [plane][nt]
      if (PACK) {
        xv[0][0] = lds64(xb + (r & 3) * XRS + (r >> 2) * 256 + ib * 32 + q * 8);
      } else {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          if (nt < ntiles) {
            xv[0][nt] = lds64(xb + (nt * 8 + r) * XRS + ib * 32 + q * 8);
            xv[1][nt] = lds64(xb + (nt * 8 + r) * XRS + 256 + ib * 32 + q * 8);
          }
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t sel[2];
        int c[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t a0 = i2 == 0 ? qw[mt][h].x : qw[mt][h].z;
          const uint32_t a1 = i2 == 0 ? qw[mt][h].y : qw[mt][h].w;
          const uint32_t gi = __byte_perm(a0, 0u, 0x4440u | uint32_t(q));  // byte q of a0
          const uint32_t si = (a1 >> (7 * q)) & 127u;
          sel[h] = lds32(tl + gi * 128) | lds32(tsign + si * 128);
          c[h] = int(((a1 >> 27) & 0x1Eu) | 1u);
        }
        const uint32_t a[4] = {__byte_perm(kPos, kNeg, sel[0]), __byte_perm(kPos, kNeg, sel[1]),
                               __byte_perm(kPos, kNeg, sel[0] >> 16), __byte_perm(kPos, kNeg, sel[1] >> 16)};
        if (PACK) {
          int d[4] = {0, 0, 0, 0};
          mma_16832_s8(d, a, xv[0][0].x, xv[0][0].y);
          t[0][mt][0][0] += d[0] * c[0];
          t[0][mt][0][1] += d[1] * c[0];
          t[0][mt][0][2] += d[2] * c[1];
          t[0][mt][0][3] += d[3] * c[1];
          continue;
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          if (nt < ntiles) {
#pragma unroll
            for (int pl = 0; pl < 2; ++pl) {
              int d[4] = {0, 0, 0, 0};
              mma_16832_s8(d, a, xv[pl][nt].x, xv[pl][nt].y);
              t[pl][mt][nt][0] += d[0] * c[0];
              t[pl][mt][nt][1] += d[1] * c[0];
              t[pl][mt][nt][2] += d[2] * c[1];
              t[pl][mt][nt][3] += d[3] * c[1];
            }
          }
        }
      }
    }
  }
  if (PACK) iq_unpack_planes(t, lane);
  constexpr float kPlane2 = 1.f / 254.f;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const uint32_t dp = lds32(wb + 2048 + mt * 32 + r * 4);
    const __half2 d2 = *reinterpret_cast<const __half2*>(&dp);
    const float d0 = __low2float(d2) * 0.125f, d1 = __high2float(d2) * 0.125f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      if (nt >= ntiles) continue;
      const float sx0 = __uint_as_float(lds32(xb + (nt * 8 + 2 * q) * XRS + 512));
      const float sx1 = __uint_as_float(lds32(xb + (nt * 8 + 2 * q + 1) * XRS + 512));
      const float sc[4] = {d0 * sx0, d0 * sx1, d1 * sx0, d1 * sx1};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        acc[mt][nt][0][i] = fmaf(fmaf(float(t[1][mt][nt][i]), kPlane2, float(t[0][mt][nt][i])), sc[i], acc[mt][nt][0][i]);
    }
  }
}

// ---------------------------------------------------------------- IQ2_XS / IQ1_M steps
// Both formats scale every 16 weights on their own, so each 32-wide sub-block
// takes two m16n8k16 MMAs, one per 16-weight group, each s32 partial scaled
// by its group's integer 2s + 1.  Thread q owns elements 4q..4q+3 of each
// group (half q & 1 of grid entry q >> 1, and of entry 2 + (q >> 1) in the
// second group): the k16 fragments' K positions, activations in natural order.
// The fp16 d / 8 and the activation scale apply once per super-block in FP32,
// as in iq2_step.
__device__ __forceinline__ void iq_finish(const int (&t)[2][2][2][4], const float (&dl)[2][2], uint32_t xb,
                                          int ntiles, int lane, float (&acc)[2][2][2][4]) {
  constexpr int XRS = Fmt<2>::XRS;
  constexpr float kPlane2 = 1.f / 254.f;
  const int q = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    if (nt >= ntiles) continue;
    const float sx0 = __uint_as_float(lds32(xb + (nt * 8 + 2 * q) * XRS + 512));
    const float sx1 = __uint_as_float(lds32(xb + (nt * 8 + 2 * q + 1) * XRS + 512));
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const float sc[4] = {dl[mt][0] * sx0, dl[mt][0] * sx1, dl[mt][1] * sx0, dl[mt][1] * sx1};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        acc[mt][nt][0][i] = fmaf(fmaf(float(t[1][mt][nt][i]), kPlane2, float(t[0][mt][nt][i])), sc[i], acc[mt][nt][0][i]);
    }
  }
}

// the activation fragments of one sub-block: [nt][plane][group] (packed: [0][0][group])
template <bool PACK>
__device__ __forceinline__ void iq_load_x(uint32_t xb, int ib, int ntiles, int lane, uint32_t (&xv)[2][2][2]) {
  constexpr int XRS = Fmt<2>::XRS;
  const int r = lane >> 2, q = lane & 3;
  if (PACK) {
#pragma unroll
    for (int grp = 0; grp < 2; ++grp)
      xv[0][0][grp] = lds32(xb + (r & 3) * XRS + (r >> 2) * 256 + ib * 32 + grp * 16 + 4 * q);
    return;
  }
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int pl = 0; pl < 2; ++pl)
#pragma unroll
      for (int grp = 0; grp < 2; ++grp)
        xv[nt][pl][grp] = nt < ntiles ? lds32(xb + (nt * 8 + r) * XRS + pl * 256 + ib * 32 + grp * 16 + 4 * q) : 0u;
}

// the two MMAs of one sub-block and tile, one per 16-weight group, for both planes
template <bool PACK>
__device__ __forceinline__ void iq_group_mmas(const uint32_t (&a)[2][2], const int (&c)[2][2],
                                              const uint32_t (&xv)[2][2][2], int ntiles, int (&t)[2][2][2][4],
                                              int mt) {
  if (PACK) {
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
      int d[4] = {0, 0, 0, 0};
      mma_16816_s8(d, a[grp][0], a[grp][1], xv[0][0][grp]);
      t[0][mt][0][0] += d[0] * c[grp][0];
      t[0][mt][0][1] += d[1] * c[grp][0];
      t[0][mt][0][2] += d[2] * c[grp][1];
      t[0][mt][0][3] += d[3] * c[grp][1];
    }
    return;
  }
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    if (nt >= ntiles) continue;
#pragma unroll
    for (int pl = 0; pl < 2; ++pl)
#pragma unroll
      for (int grp = 0; grp < 2; ++grp) {
        int d[4] = {0, 0, 0, 0};
        mma_16816_s8(d, a[grp][0], a[grp][1], xv[nt][pl][grp]);
        t[pl][mt][nt][0] += d[0] * c[grp][0];
        t[pl][mt][nt][1] += d[1] * c[grp][0];
        t[pl][mt][nt][2] += d[2] * c[grp][1];
        t[pl][mt][nt][3] += d[3] * c[grp][1];
      }
  }
}

// IQ2_XS (ggml's dequantize: d * (0.5 + s) * 0.25 * grid * sign, s the 4-bit
// scale of each 16 weights): a weight is g * sign (g in {8, 25, 43}) from the
// 9-bit grid index's magnitude codes and the 7-bit sign index's nibbles.
template <bool PACK>
__device__ __forceinline__ void iq2xs_step(uint32_t wb, uint32_t xb, uint32_t tbl, int ntiles, int lane,
                                           float (&acc)[2][2][2][4]) {
  constexpr uint32_t kPos = 0x002B1908u, kNeg = 0x00D5E7F8u;  // bytes 8, 25, 43, 0 and -8, -25, -43, 0
  const int r = lane >> 2, q = lane & 3;
  const uint32_t usel = (q >> 1) ? 0x4432u : 0x4410u;  // the u16 entry q >> 1 of a word, zero-extended
  int t[2][2][2][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) (&t[0][0][0][0])[i] = 0;
  const uint32_t tgrid = tbl + (q & 1) * (kIq2xsUpper * 4);  // this lane's half of every grid entry
  const uint32_t tsign = tbl + 512 * 4;  // sign nibbles from the unshifted copy: both lanes of an entry share a word
  const int h_sh = 16 * (q & 1);
  uint2 sc[2][2];  // [mt][h]: the row's 8 scale bytes
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) sc[mt][h] = lds64(wb + 2048 + mt * 128 + (h * 8 + r) * 8);
#pragma unroll 1
  for (int ibp = 0; ibp < 4; ++ibp) {
    uint4 qw[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) qw[mt][h] = lds128(wb + mt * 1024 + (h * 8 + r) * 64 + ibp * 16);
#pragma unroll
    for (int i2 = 0; i2 < 2; ++i2) {
      const int ib = 2 * ibp + i2;
      uint32_t xv[2][2][2];
      iq_load_x<PACK>(xb, ib, ntiles, lane, xv);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t a[2][2];
        int c[2][2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t w01 = i2 == 0 ? qw[mt][h].x : qw[mt][h].z;  // u16 entries 0, 1 of the sub-block
          const uint32_t w23 = i2 == 0 ? qw[mt][h].y : qw[mt][h].w;  // entries 2, 3
#pragma unroll
          for (int grp = 0; grp < 2; ++grp) {
            const uint32_t u = __byte_perm(grp ? w23 : w01, 0u, usel);
            const uint32_t sel = lds32(tgrid + (u & 511u) * 4) | (lds32(tsign + (u >> 9) * 4) >> h_sh);
            a[grp][h] = __byte_perm(kPos, kNeg, sel);
          }
          const uint32_t sb = ((ib < 4 ? sc[mt][h].x : sc[mt][h].y) >> (8 * (ib & 3))) & 255u;
          c[0][h] = int(2 * (sb & 15u) + 1);
          c[1][h] = int(2 * (sb >> 4) + 1);
        }
        iq_group_mmas<PACK>(a, c, xv, ntiles, t, mt);
      }
    }
  }
  float dl[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const uint32_t dp = lds32(wb + 2304 + mt * 32 + r * 4);
    const __half2 d2 = *reinterpret_cast<const __half2*>(&dp);
    dl[mt][0] = __low2float(d2) * 0.125f;
    dl[mt][1] = __high2float(d2) * 0.125f;
  }
  if (PACK) iq_unpack_planes(t, lane);
  iq_finish(t, dl, xb, ntiles, lane, acc);
}

// IQ1_M (ggml's dequantize: d * (2s + 1) * (grid + delta), grid in {-1, 0, 1},
// delta = +-1/8 per 8 weights, s the 3-bit scale of each 16 weights, d the
// fp16 in the scales' top nibbles): a weight is 8 * grid +- 1 in int8, times
// (2s + 1) on the s32 partial, times d / 8 in FP32.
template <bool PACK>
__device__ __forceinline__ void iq1m_step(uint32_t wb, uint32_t xb, uint32_t tbl, int ntiles, int lane,
                                          float (&acc)[2][2][2][4]) {
  constexpr uint32_t kPos = 0x000901F9u, kNeg = 0x0007FFF7u;  // bytes -7, 1, 9 (delta +) and -9, -1, 7 (delta -)
  const int r = lane >> 2, q = lane & 3;
  const int e0 = q >> 1;
  const uint32_t lsel[2] = {0x4440u | uint32_t(e0), 0x4440u | uint32_t(2 + e0)};  // qs byte of entry 2 grp + e0
  const uint32_t tgrid = tbl + (q & 1) * (kIq1mUpper * 4);  // this lane's half of every entry
  int t[2][2][2][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) (&t[0][0][0][0])[i] = 0;
  uint2 sc[2][2];  // [mt][h]: the row's four u16 scale words
  float dl[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      sc[mt][h] = lds64(wb + 1536 + mt * 128 + (h * 8 + r) * 8);
      const uint32_t lo = sc[mt][h].x, hi = sc[mt][h].y;
      const uint32_t dbits = ((lo >> 12) & 0x000Fu) | ((lo >> 24) & 0x00F0u) | ((hi >> 4) & 0x0F00u) | ((hi >> 16) & 0xF000u);
      dl[mt][h] = __half2float(__ushort_as_half(static_cast<unsigned short>(dbits))) * 0.125f;
    }
#pragma unroll 1
  for (int ibp = 0; ibp < 4; ++ibp) {
    uint2 qs[2][2];
    uint32_t qh[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        qs[mt][h] = lds64(wb + mt * 512 + (h * 8 + r) * 32 + ibp * 8);
        qh[mt][h] = lds32(wb + 1024 + mt * 256 + (h * 8 + r) * 16 + ibp * 4);
      }
#pragma unroll
    for (int i2 = 0; i2 < 2; ++i2) {
      const int ib = 2 * ibp + i2;
      uint32_t xv[2][2][2];
      iq_load_x<PACK>(xb, ib, ntiles, lane, xv);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t a[2][2];
        int c[2][2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t qsw = i2 == 0 ? qs[mt][h].x : qs[mt][h].y;  // qs bytes of entries 0..3
          const uint32_t sword = ibp < 2 ? (ibp == 0 ? sc[mt][h].x & 0xFFFFu : sc[mt][h].x >> 16)
                                         : (ibp == 2 ? sc[mt][h].y & 0xFFFFu : sc[mt][h].y >> 16);
#pragma unroll
          for (int grp = 0; grp < 2; ++grp) {
            const uint32_t nib = (qh[mt][h] >> (8 * (2 * i2 + grp) + 4 * e0)) & 15u;
            const uint32_t idx = __byte_perm(qsw, 0u, lsel[grp]) | ((nib & 7u) << 8);
            const uint32_t sel = lds32(tgrid + idx * 4) | ((nib & 8u) ? 0x44444444u : 0u);
            a[grp][h] = __byte_perm(kPos, kNeg, sel);
            c[grp][h] = int(2 * ((sword >> (3 * (2 * i2 + grp))) & 7u) + 1);
          }
        }
        iq_group_mmas<PACK>(a, c, xv, ntiles, t, mt);
      }
    }
  }
  if (PACK) iq_unpack_planes(t, lane);
  iq_finish(t, dl, xb, ntiles, lane, acc);
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
  int* list = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(tables) + F::TW * 4);
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
  if (F::IQ)
    for (int i = threadIdx.x; i < F::TW; i += kGemvThreads) tables[i] = a.iq2_tables[i / F::TREP];
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
      const uint32_t tx = uint32_t(kConsumerWarps * F::U + KS * ch.count * F::XB);
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
          // f16 rows (FP4) or int8 blocks of kIq2XBlockBytes per K tile (IQ2)
          const uint8_t* src = static_cast<const uint8_t*>(a.xsrc) +
                               (F::IQ ? (xrow * n_kt + kt) * F::XB : (xrow * a.x_row_stride + int64_t(kt) * F::KT) * 2);
          bulk_g2s(sb + kConsumerWarps * F::U + xi * F::XRS, src, F::XB, &full[s]);
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
        if constexpr (FMT == 2) {
          if (ch.count <= 4) iq2_step<true>(wb, xb, tbl, ntiles, lane, acc2);
          else iq2_step<false>(wb, xb, tbl, ntiles, lane, acc2);
        } else if constexpr (FMT == 3) {
          if (ch.count <= 4) iq2xs_step<true>(wb, xb, tbl, ntiles, lane, acc2);
          else iq2xs_step<false>(wb, xb, tbl, ntiles, lane, acc2);
        } else if constexpr (FMT == 4) {
          if (ch.count <= 4) iq1m_step<true>(wb, xb, tbl, ntiles, lane, acc2);
          else iq1m_step<false>(wb, xb, tbl, ntiles, lane, acc2);
        } else {
          fp4_step<FMT>(wb, xb, ntiles, lane, acc2);
        }
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
      if (EPI == 1 && a.counters) {  // (no counters: the caller combines the y2 rows itself)
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

// fp16 rows -> the IQ2 op's int8 activation blocks: per row and 256-wide K
// tile, q1 = rn(x * 127 / amax), q2 = rn((x - q1 * s) * 254 * 127 / amax)
// (both clamped to +-127), s = amax / 127 as f32 (0 for an all-zero block),
// kIq2XBlockBytes per block.  One warp per block.
// Rows [range[0], range[1]) when `range` is given (device: the IQ2 bank's
// sorted positions from the route plan), else [0, rows).
__global__ void quant_s8_kernel(const __half* __restrict__ src, int64_t src_stride, int K, int rows,
                                const int32_t* __restrict__ range, uint8_t* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int n_kt = K / kIq2KTile;
  pdl_wait();
  pdl_trigger();
  const int lo = range ? range[0] : 0, hi = range ? min(range[1], rows) : rows;
  const int64_t n_blocks = int64_t(max(hi - lo, 0)) * n_kt;
  for (int64_t blk = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) / 32; blk < n_blocks;
       blk += int64_t(gridDim.x) * blockDim.x / 32) {
    const int row = lo + int(blk / n_kt), kt = int(blk % n_kt);
    const uint4 v = *reinterpret_cast<const uint4*>(src + row * src_stride + int64_t(kt) * kIq2KTile + lane * 8);
    float f[8];
    const __half2* hv = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(hv[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? __fdiv_rn(127.f, amax) : 0.f;
    const float sx = amax / 127.f;
    uint32_t w1[2] = {0, 0}, w2[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q1 = max(-127, min(127, __float2int_rn(__fmul_rn(f[i], inv))));
      const float res = fmaf(-float(q1), sx, f[i]);
      const int q2 = max(-127, min(127, __float2int_rn(__fmul_rn(__fmul_rn(res, inv), 254.f))));
      w1[i >> 2] |= uint32_t(q1 & 255) << (8 * (i & 3));
      w2[i >> 2] |= uint32_t(q2 & 255) << (8 * (i & 3));
    }
    uint8_t* out = dst + (int64_t(row) * n_kt + kt) * kIq2XBlockBytes;
    *reinterpret_cast<uint2*>(out + lane * 8) = make_uint2(w1[0], w1[1]);
    *reinterpret_cast<uint2*>(out + 256 + lane * 8) = make_uint2(w2[0], w2[1]);
    if (lane < 4) reinterpret_cast<uint32_t*>(out + 512)[lane] = lane == 0 ? __float_as_uint(sx) : 0u;
  }
}

int launch_quant_s8(cudaStream_t s, const __half* src, int64_t src_stride, int K, int rows, const int32_t* range,
                    uint8_t* dst) {
  if (rows <= 0) return 0;
  const int64_t warps = int64_t(rows) * (K / kIq2KTile);
  const int64_t blocks = std::min<int64_t>((warps + 7) / 8, 148 * 16);
  return launch_chain(quant_s8_kernel, dim3(int(blocks)), dim3(256), 0, s, src, src_stride, K, rows, range, dst) ==
                 cudaSuccess
             ? 0
             : -1;
}

// One kernel per format and epilogue; the split-K is read from the device
// (chosen by the route plan from this call's chunk counts), so the choice
// follows the routing without a host round trip, also inside a CUDA graph.
template <int FMT, int EPI>
__global__ void __launch_bounds__(kGemvThreads, Fmt<FMT>::CTAS) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  switch (a.ks_sel[a.bank]) {
    case 1: gemv_body<FMT, EPI, 1>(a, smem); break;
    case 2: gemv_body<FMT, EPI, 2>(a, smem); break;
    case 4: gemv_body<FMT, EPI, 4>(a, smem); break;
    case 8: gemv_body<FMT, EPI, 8>(a, smem); break;
    default:
      if (threadIdx.x == 0) set_error(a.err, kErrRange);
  }
  pdl_trigger();
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
  return launch_chain(gemv_kernel<FMT, EPI>, dim3(a.grid), dim3(kGemvThreads), smem, s, a) == cudaSuccess ? 0 : -1;
}

int launch_gemv(cudaStream_t s, const GemvArgs& a) {
  if (!a.ks_sel) return -1;
  if (a.fmt == 0) return a.epi == 0 ? launch_one<0, 0>(s, a) : launch_one<0, 1>(s, a);
  if (a.fmt == 1) return a.epi == 0 ? launch_one<1, 0>(s, a) : launch_one<1, 1>(s, a);
  if (a.fmt == 2) return a.epi == 0 ? launch_one<2, 0>(s, a) : launch_one<2, 1>(s, a);
  if (a.fmt == 3) return a.epi == 0 ? launch_one<3, 0>(s, a) : launch_one<3, 1>(s, a);
  if (a.fmt == 4) return a.epi == 0 ? launch_one<4, 0>(s, a) : launch_one<4, 1>(s, a);
  return -1;
}

}  // namespace b200moe
