// HBM layout of the expert banks (the kernels' own "prepacked" format).
//
// FP4 bank (NVFP4 or MXFP4), per expert slot, two regions:
//   W13: units [tp < I/16][kt < H/128]; W2: units [tp < H/32][kt < I/128].
//   A unit is one "tile pair" (two m16 row tiles) over one 128-wide K tile:
//     [mt0 codes 1024 B][mt1 codes 1024 B][mt0 scales SB][mt1 scales SB]
//   W13 pairs gate rows 16tp.. (W1) with up rows 16tp.. (W3) so a warp holds
//   both halves of the SwiGLU in registers; W2's pair is rows 32tp..32tp+31.
//   Codes of one m16 tile: [h 2][lane 32][16 B].  Lane = 4r + q, row = r + 8h;
//   the 16 bytes are four 4-byte words, word c = natural bytes of elements
//   kt*128 + 32c + 8q .. +7 of that row (low nibble = even element).  With the
//   in-chunk K order "thread q owns elements 8q..8q+7 of every 32-chunk" the
//   mma.m16n8k16 A and B fragments of two k16 steps are exactly those bytes.
//   NVFP4 scales (SB = 128): [r 8][qb 2][h 2][c 4] = E4M3 byte of row r+8h,
//     16-block kt*8 + 2c + qb.
//   MXFP4 scales (SB = 64): [r 8][h 2][c 4] = biased f16 exponent of the block
//     scale after a per-projection rebase (value 2^(e-127) = 2^(s-15) * g).
// IQ2_XXS bank, per slot: W13 units [tp < I/16][kb < H/256], W2 units
//   [tp < H/32][kb < I/256]; a unit is [mt0 qs 1024][mt1 qs 1024][mt0 d 32][mt1 d 32]:
//   qs of one m16 tile = [h 2][r 8][64 B] (the block's 64 qs bytes, ggml order);
//   d = [r 8][h 2] fp16 super-block scales.
// IQ2_XS (74 B per 256 weights: d, 32 x u16 qs = 9-bit grid index | 7-bit
//   sign index, 8 scale bytes of two 4-bit scales per 32): units as IQ2_XXS,
//   [mt0 qs 1024][mt1 qs 1024][mt0 scales 128][mt1 scales 128][mt0 d 32][mt1 d 32];
//   qs = [h 2][r 8][64 B], scales = [h 2][r 8][8 B], d = [r 8][h 2].
// IQ1_M (56 B per 256 weights: 32 qs bytes, 16 qh bytes = per 8-weight group a
//   nibble of 3 high index bits and the delta sign, 4 x u16 scales = 3-bit
//   scale per 16 weights, the fp16 d in their top nibbles): units
//   [qs 2 x 512][qh 2 x 256][scales 2 x 128], each [mt][h 2][r 8][its bytes].
// IQ bank slots hold W13 units of the gate/up format then W2 units of the down
//   format (the two may differ, as GGUF layers mix them).
#pragma once

#include <stdint.h>

namespace b200moe {

constexpr int kFp4KTile = 128;   // K elements per FP4 unit
constexpr int kIq2KTile = 256;   // K elements per IQ2 unit
// The IQ2 op multiplies int8 weights by int8 activations on the tensor cores
// (the reference's IQ2 dot products are int8 too, ggml's with Q8_K blocks).
// One int8 plane per 256-wide block misses 1e-2 on SwiGLU rows (amax ~7x
// their RMS), so an activation block holds two planes: x ~ s * (q1 + q2/254),
// s = amax / 127, q2 the rounded residual (error <= amax / 64,516).  Layout
// per row and 256-wide K tile: q1 [256], q2 [256], s (f32), 12 bytes padding.
constexpr int kIq2XBlockBytes = 528;
// IQ2 decode tables (32-bit words): per grid entry the 2-bit magnitude codes
// of its 8 values in nibbles (8 -> 0, 25 -> 1, 43 -> 2), then per 7-bit sign
// index the 8 signs in bit 2 of each nibble; nibble j | sign j is a byte index
// into {8, 25, 43, -, -8, -25, -43, -}.
constexpr int kIq2TableWords = 256 + 128;
constexpr int kCodesPerTile = 1024;

__host__ __device__ constexpr int fp4_scale_bytes(int fmt) { return fmt == 0 ? 128 : 64; }
__host__ __device__ constexpr int fp4_unit_bytes(int fmt) { return 2 * kCodesPerTile + 2 * fp4_scale_bytes(fmt); }
constexpr int kIq2UnitBytes = 2 * 1024 + 2 * 32;

struct BankGeom {
  int64_t w13_bytes;   // per slot
  int64_t w2_bytes;    // per slot
  int64_t slot_bytes;  // w13 + w2
};

inline BankGeom fp4_geom(int fmt, int hidden, int inter) {
  const int64_t u = fp4_unit_bytes(fmt);
  BankGeom g;
  g.w13_bytes = int64_t(inter / 16) * (hidden / kFp4KTile) * u;
  g.w2_bytes = int64_t(hidden / 32) * (inter / kFp4KTile) * u;
  g.slot_bytes = g.w13_bytes + g.w2_bytes;
  return g;
}

// Codebook formats of the IQ bank, by kernel format id (2, 3, 4) and GGML type.
constexpr int kIq2xsUnitBytes = 2 * 1024 + 2 * 128 + 2 * 32;
constexpr int kIq1mUnitBytes = 2 * 512 + 2 * 256 + 2 * 128;
// IQ2_XS / IQ1_M grid words come twice: as built, then each shifted right by
// 16 (the selector nibbles of an entry's elements 4..7), so a lane that owns
// the upper half of its entries reads its byte-permute selectors directly
// (IQ2_XS sign nibbles are read from the first copy only, so the second holds
// the grid words alone).  The copy starts 16 words (half the banks) past the
// first: the two lanes that read the same entry then hit different banks
// instead of one bank twice.
constexpr int kIq2xsHalfWords = 512 + 128;   // grid magnitude codes [512], sign nibbles [128]
constexpr int kIq2xsGridWords = 512;
constexpr int kIq1mHalfWords = 2048;         // grid value codes [2048]
constexpr int kIqUpperPad = 16;
constexpr int kIq2xsUpper = kIq2xsHalfWords + kIqUpperPad;  // word offset of the shifted copy
constexpr int kIq1mUpper = kIq1mHalfWords + kIqUpperPad;
constexpr int kIq2xsTableWords = kIq2xsUpper + kIq2xsGridWords;
constexpr int kIq1mTableWords = kIq1mUpper + kIq1mHalfWords;
constexpr int kGgmlIq2xxs = 16, kGgmlIq2xs = 17, kGgmlIq1m = 29;

__host__ __device__ constexpr int iq_unit_bytes(int fmt) {
  return fmt == 2 ? kIq2UnitBytes : fmt == 3 ? kIq2xsUnitBytes : kIq1mUnitBytes;
}
__host__ __device__ constexpr int iq_table_words(int fmt) {
  return fmt == 2 ? kIq2TableWords : fmt == 3 ? kIq2xsTableWords : kIq1mTableWords;
}
__host__ __device__ constexpr int iq_block_bytes(int fmt) { return fmt == 2 ? 66 : fmt == 3 ? 74 : 56; }
// GGML type id -> kernel format id, -1 for a type the IQ bank does not hold
inline int iq_fmt_of_type(int ggml_type) {
  return ggml_type == kGgmlIq2xxs ? 2 : ggml_type == kGgmlIq2xs ? 3 : ggml_type == kGgmlIq1m ? 4 : -1;
}

inline BankGeom iq_geom(int fmt13, int fmt2, int hidden, int inter) {
  BankGeom g;
  g.w13_bytes = int64_t(inter / 16) * (hidden / kIq2KTile) * iq_unit_bytes(fmt13);
  g.w2_bytes = int64_t(hidden / 32) * (inter / kIq2KTile) * iq_unit_bytes(fmt2);
  g.slot_bytes = g.w13_bytes + g.w2_bytes;
  return g;
}

// ----------------------------------------------------- E4M3 / E2M1 helpers
// E4M3FN byte -> float (sign, bias 7, subnormal step 2^-9).
__host__ __device__ inline float e4m3_value(uint32_t b) {
  const int e = (b >> 3) & 15, m = b & 7;
  float v = e == 0 ? float(m) * 0.001953125f : ldexpf(1.f + float(m) * 0.125f, e - 7);
  return (b & 128) ? -v : v;
}

// Non-negative finite float -> E4M3FN byte, round to nearest even, saturating
// at 448.  The same steps as the oracle: quantum 2^(floor(log2 x) - 3) with the
// exponent floored at -6 (subnormal step 2^-9), rint (half-even), clamp, encode.
__device__ inline uint32_t e4m3_encode(float x) {
  if (!(x > 0.f)) return 0u;
  int ex;
  frexpf(x, &ex);
  int e = ex - 1;
  if (e < -6) e = -6;
  const float quantum = ldexpf(1.f, e - 3);
  float q = rintf(x / quantum) * quantum;  // exact: power-of-two quantum
  if (q > 448.f) q = 448.f;
  if (q == 0.f) return 0u;
  int qx;
  frexpf(q, &qx);
  const int qe = qx - 1;
  if (qe < -6) return uint32_t(rintf(ldexpf(q, 9)));
  const uint32_t man = uint32_t(rintf((ldexpf(q, -qe) - 1.f) * 8.f));
  return (uint32_t(qe + 7) << 3) | man;
}

// |t| -> E2M1 magnitude code, nearest with ties to the even code, saturating.
__device__ __forceinline__ uint32_t e2m1_code(float t) {
  return uint32_t(t > 0.25f) + uint32_t(t >= 0.75f) + uint32_t(t > 1.25f) + uint32_t(t >= 1.75f) +
         uint32_t(t > 2.5f) + uint32_t(t >= 3.5f) + uint32_t(t > 5.0f);
}

__device__ __forceinline__ float e2m1_mag(uint32_t c) {
  const float t[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  return t[c & 7];
}

// Smallest e with 6 * 2^e >= x (x > 0): the E8M0 exponent choice of the
// reference's exact fold, ceil(log2(x / 6)), in integer steps.
__device__ __forceinline__ int mx_exponent(float x) {
  int ex;
  const float m = frexpf(x, &ex);
  return m <= 0.75f ? ex - 3 : ex - 2;
}

}  // namespace b200moe
