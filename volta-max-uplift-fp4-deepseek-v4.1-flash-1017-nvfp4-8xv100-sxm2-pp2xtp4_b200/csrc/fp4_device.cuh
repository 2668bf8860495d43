// Device pieces shared by the block-scaled FP4 kernels (the expert GEMM of
// gemm_fp4.cu and the fused small-batch decode of decode.cu): stage layout of
// the weight units, UMMA descriptors, the kind::mxf4nvf4 MMA, TMEM loads, the
// limited SwiGLU, and the four-plane E2M1 quantization of activation rows.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"
#include "layout.cuh"

namespace b200moe {
namespace {

constexpr int kP = kFp4Planes;             // activation planes
constexpr int kATile = 128 * 128;          // weight tile: 128 rows x 256 FP4 = 16 KB
constexpr int kSFBytes = 4 * 512;          // the scale blocks of one 256-wide K tile
constexpr int kThreads = 7 * 32;           // producer, MMA, 4 epilogue warps, scale copier
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfCol = 256;           // scale columns start after the two accumulator buffers

// Stage layout by weight tiles per unit and routes per chunk (RC: the MMA's N
// is 4 planes x RC; small batches use small chunks, so the tensor pipe does not
// spend its time on empty columns).  Two tiles (W13: the gate and up tiles; W2:
// two adjacent 128-row tiles) make stages of 36 KB + the plane tile, 4 of them
// (5 where they fit measured slower on B200: configs[1] M = 64 639 -> 692 us);
// one tile 18 KB + the plane tile, 7 stages.  Each stage has its own TMEM scale
// columns: a scale copy never lands under an MMA still in flight.
template <int TILES, int RC, int MX = 0>
struct Fp4Stage {
  static constexpr int kRC = RC;         // routes per chunk
  static constexpr int kN = kP * RC;     // MMA N: 16, 32 or 64
  static constexpr int kBTile = kN * 128;  // activation tile: kN rows x 256 FP4
  // kind::mxf4nvf4: A and B E2M1 (1), K-major, N = kN, M = 128; scales UE4M3 per 16 (NVFP4) or, bit 23,
  // UE8M0 per 32 (MXFP4)
  static constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | (uint32_t(kN >> 3) << 17) | (uint32_t(MX) << 23) |
                                     (uint32_t(128 >> 4) << 24);
  static constexpr int kTiles = TILES;  // weight tiles per unit
  static constexpr int kUnit = kTiles * (kATile + kSFBytes);  // one weight unit, one bulk copy
  static constexpr int kOffAG = 0;
  static constexpr int kOffAU = kATile;  // W13 only
  static constexpr int kOffSFG = kTiles * kATile;
  static constexpr int kOffSFU = kOffSFG + kSFBytes;  // W13 only
  static constexpr int kOffB = kUnit;
  static constexpr int kOffSFB = kOffB + kBTile;
  static constexpr int kBytes = kOffSFB + kSFBytes;
  static constexpr int kStages = TILES == 2 ? 4 : 7;
  static constexpr uint32_t kSfCols = TILES == 2 ? 48 : 32;  // tile 0 (, tile 1), activations: 16 each
  static constexpr uint32_t kSfB = TILES == 2 ? 32 : 16;
  // accumulator columns of one item (TILES x N) and how many items' accumulators TMEM holds below the
  // scale columns: two (the epilogue of one item overlaps the next item's MMAs) up to N = 64, one at N = 128
  static constexpr uint32_t kAccCols = uint32_t(TILES * kN);
  static constexpr int kAccBufs = 2 * kAccCols <= kSfCol ? 2 : 1;
  static constexpr size_t kSmem = 1024 + size_t(kStages) * kBytes + 64 * 8;
  static_assert(kBytes % 1024 == 0, "128-byte swizzled tiles need 1024-byte aligned stages");
  static_assert(kAccBufs * kAccCols <= kSfCol, "accumulators below the scale columns");
  static_assert(kSfCol + kStages * kSfCols <= kTmemCols, "TMEM columns");
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

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

template <int MX>
__device__ __forceinline__ void mma_fp4(uint32_t d, uint64_t a, uint64_t b, uint32_t sfa, uint32_t sfb,
                                        uint32_t accumulate, uint32_t idesc) {
  if (MX)
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p; }" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb));
  else
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p; }" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb));
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

// ---------------------------------------------------------------- planes
// Nearest E2M1 value (ties to even) of v >= 0, and its 3-bit magnitude code:
// step 0.5 below 2, 1 below 4, 2 above, saturating at 6.
__device__ __forceinline__ float e2m1_round(float v) {
  const float q = v < 2.f ? rintf(v * 2.f) * 0.5f : v < 4.f ? rintf(v) : rintf(v * 0.5f) * 2.f;
  return fminf(q, 6.f);
}
__device__ __forceinline__ uint32_t e2m1_code_of(float q) {  // q on the E2M1 grid
  return q < 2.f ? uint32_t(q * 2.f) : q < 4.f ? uint32_t(q) + 2u : uint32_t(q * 0.5f) + 4u;
}
// Nearest E4M3 byte of x >= 0 (ties to even, saturating at 448) by the
// hardware conversion; both halves of the pair convert x.
__device__ __forceinline__ uint32_t e4m3_rn(float x) {
  uint16_t pair;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(pair) : "f"(x));
  return pair & 0xFFu;
}

// One half-block (8 consecutive elements, thread of lane = half-block index
// mod 32) of a row through the kP planes: per plane the E2M1 codes (w[p], 8
// nibbles) and, on lane 8j of a warp, the scale word of the 64-wide K step the
// lanes 8j .. 8j + 7 cover (word[p]).  g: the row's factor (its amax over
// 6 * 448 for NVFP4, 1 for MXFP4), inv_g its inverse; r: the elements, left
// holding the residual.  Every lane of the warp takes part (shuffles).
// The chain from one plane to the next is the scale: no division or rounded
// reciprocal on it (the E4M3 target is bm times a per-row constant; the
// reciprocal of the scale is the hardware approximation, or exact for MXFP4's
// powers of two): a code a rounding step off is absorbed by the next plane,
// which quantizes the residual taken with the exact scale.
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
template <int MX>
__device__ __forceinline__ void quantize_planes8(float (&r)[8], bool own, float g, float inv_g, uint32_t (&w)[kP],
                                                 uint32_t (&word)[kP]) {
  const float inv6g = inv_g * (1.f / 6.f);
#pragma unroll
  for (int p = 0; p < kP; ++p) {
    float bm = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) bm = fmaxf(bm, fabsf(r[e]));
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));  // the other half of the 16-block
    if (MX) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));  // the 32-block: four half-blocks
    uint32_t sc;
    float scale, rs;
    if (MX) {  // UE8M0: the smallest 2^e with 6 * 2^e >= bm
      const int e = bm > 0.f ? max(-126, min(127, mx_exponent(bm))) : -127;
      sc = own && bm > 0.f ? uint32_t(e + 127) : 0u;
      scale = sc ? __uint_as_float(sc << 23) : 0.f;  // 2^e, e >= -126: a normal float
      // 2^-e exactly: a normal float up to e = 126, 2^-127 (subnormal) at e = 127
      rs = sc == 0u ? 0.f : sc <= 253u ? __uint_as_float((254u - sc) << 23) : __uint_as_float(0x00200000u);
    } else {
      sc = own ? e4m3_rn(bm * inv6g) : 0u;
      // the E4M3 byte's value (sc < 0x80), built from its bits: 2^(e - 7) (1 + m / 8) or m 2^-9
      const uint32_t ex = sc >> 3, mn = sc & 7u;
      const float sv = ex ? __uint_as_float(((ex + 120u) << 23) | (mn << 20)) : float(mn) * 0.001953125f;
      scale = sv * g;
      rs = scale > 0.f ? rcp_approx(scale) : 0.f;
    }
    uint32_t cw = 0u;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = r[e] * rs;
      const float q = e2m1_round(fabsf(v));
      r[e] -= copysignf(q, v) * scale;
      cw |= (e2m1_code_of(q) | (v < 0.f ? 8u : 0u)) << (4 * e);
    }
    w[p] = cw;
    // the scale bytes of one 64-wide K step as one word from lane 8j: NVFP4 blocks 4j .. 4j + 3 (lanes
    // 8j, +2, +4, +6), MXFP4 blocks 2j, 2j + 1 (lanes 8j, 8j + 4)
    uint32_t wd = sc;
    if (MX) {
      wd |= __shfl_down_sync(0xffffffffu, sc, 4) << 8;
    } else {
      wd |= __shfl_down_sync(0xffffffffu, sc, 2) << 8;
      wd |= __shfl_down_sync(0xffffffffu, sc, 4) << 16;
      wd |= __shfl_down_sync(0xffffffffu, sc, 6) << 24;
    }
    word[p] = wd;
  }
}

// Store half-block hb's planes of sorted position pos (index n in its chunk,
// the chunk's scale blocks at sfb_chunk) into the plane rows and scale blocks.
__device__ __forceinline__ void store_planes8(const uint32_t (&w)[kP], const uint32_t (&word)[kP], int hb, int K,
                                              int pos, int n, uint8_t* planes, uint8_t* sfb_chunk) {
#pragma unroll
  for (int p = 0; p < kP; ++p) {
    *reinterpret_cast<uint32_t*>(planes + (int64_t(pos) * kP + p) * (K / 2) + hb * 4) = w[p];
    if ((hb & 7) == 0) {
      const int mr = n * kP + p;
      *reinterpret_cast<uint32_t*>(sfb_chunk + (hb >> 3) * 512 + (mr & 31) * 16 + (mr >> 5) * 4) = word[p];
    }
  }
}

// eight 16-bit values (f16, or bf16 when BF16) as floats
template <int BF16>
__device__ __forceinline__ void load8(const uint4& v, float (&r)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (BF16) {
      r[2 * e] = __uint_as_float(w[e] << 16);
      r[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
      r[2 * e] = f.x;
      r[2 * e + 1] = f.y;
    }
  }
}

// ---------------------------------------------------------------- plane rows
// The activation rows of the FP4 bank as kP E2M1 planes with their blocked
// scales in the chunk's SFB blocks (MMA row n * kP + p) and one FP32 factor g
// per row (its amax over 6 * 448: plane 0's block scales use E4M3's range and
// the later planes, each ~10x smaller, stay inside it).  With g fixed per row
// the planes are block-local: a CTA of kPlaneThreads takes a 1024-wide slice
// (blockIdx.y) of a row, a thread one half-block of 8 elements through all
// planes.
// BY_TOKEN (W13): token row ri of x, written to every FP4-bank route of the
// token (found through the plan's inverse permutation inv), so a token is
// quantized once for its top_k routes; the CTA finds the row amax itself and
// clears the W2 row maxima of those positions.  Otherwise (W2): the SwiGLU row
// of sorted position lo + ri, its amax taken by the W13 epilogue (rowmax).
// [lo, hi): the bank's sorted positions.  The whole CTA calls it.
constexpr int kPlaneThreads = 128;
constexpr int kSlice = kPlaneThreads * 8;
struct PlaneScratch {
  float red[kPlaneThreads / 32];
  int dst_pos[32], dst_sf[32], dst_n[32];
  int n_dst;
};
template <int BY_TOKEN, int BF16, int MX>
__device__ __forceinline__ void planes_row(PlaneScratch& sm, const uint16_t* src, int64_t src_stride, int K,
                                           const int32_t* inv, int top_k, const int32_t* chunk_of, int lo, int hi,
                                           int ri, uint32_t* rowmax, uint8_t* planes, uint8_t* sfb, float* gx) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nhb = K / 8, n_ks = K / 64;
  const int hb = blockIdx.y * kPlaneThreads + t;  // this thread's half-block
  const bool own = hb < nhb;
  __syncthreads();  // the previous row's destinations are read
  if (warp == 0) {
    int pos = -1;
    if (BY_TOKEN) {
      if (lane < top_k) {
        const int q = inv[int64_t(ri) * top_k + lane];
        if (q >= lo && q < hi) pos = q;
      }
    } else if (lane == 0) {
      pos = lo + ri;
    }
    const int cn = pos >= 0 ? chunk_of[pos] : 0;
    const unsigned have = __ballot_sync(0xffffffffu, pos >= 0);
    if (pos >= 0) {
      const int i = __popc(have & ((1u << lane) - 1u));
      sm.dst_pos[i] = pos;
      sm.dst_sf[i] = (cn >> 8) * n_ks * 512;
      sm.dst_n[i] = cn & 255;
    }
    if (lane == 0) sm.n_dst = __popc(have);
  }
  const uint16_t* row = src + (BY_TOKEN ? int64_t(ri) : int64_t(lo + ri)) * src_stride;
  float r[8];
  load8<BF16>(own ? *reinterpret_cast<const uint4*>(row + hb * 8) : make_uint4(0, 0, 0, 0), r);
  float amax = 0.f;
  if (BY_TOKEN) {  // the whole row's amax (every slice's CTA reads the row: it is L2-resident)
#pragma unroll 4
    for (int j = t; j < nhb; j += kPlaneThreads) {  // unrolled: the loads go out together
      float f[8];
      load8<BF16>(*reinterpret_cast<const uint4*>(row + j * 8), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) sm.red[warp] = amax;
  }
  __syncthreads();
  const int nd = sm.n_dst;
  if (nd == 0) return;
  if (BY_TOKEN) {
    amax = sm.red[0];
#pragma unroll
    for (int w = 1; w < kPlaneThreads / 32; ++w) amax = fmaxf(amax, sm.red[w]);
  } else {
    amax = __uint_as_float(rowmax[sm.dst_pos[0]]);
  }
  // MXFP4: power-of-two block scales cover any row, so no row factor (g = 1)
  const float g = MX ? 1.f : amax / (6.f * 448.f);
  const float inv_g = g > 0.f ? __frcp_rn(g) : 0.f;
  uint32_t w[kP], word[kP];
  quantize_planes8<MX>(r, own, g, inv_g, w, word);
  if (own)
    for (int d = 0; d < nd; ++d) store_planes8(w, word, hb, K, sm.dst_pos[d], sm.dst_n[d], planes, sfb + sm.dst_sf[d]);
  if (blockIdx.y == 0 && t < nd) {
    gx[sm.dst_pos[t]] = g;
    if (BY_TOKEN) rowmax[sm.dst_pos[t]] = 0u;  // the W13 epilogue takes the W2 row maxima afresh
  }
}

}  // namespace
}  // namespace b200moe
