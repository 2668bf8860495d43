// Packing kernels: NVFP4 / MXFP4 quantizers, the exact NVFP4 -> MXFP4 fold,
// and the prepack of natural-layout expert records into the banks' layout.
//
// The quantizers are this build's own definitions (the reference ships NVIDIA's
// packs); they follow the oracle's steps exactly, so the bytes are bit-equal.
// The fold follows the reference's offline fold
// (harness/benchmarks/nvfp4_8r/build_packs.py:120-151) step for step.
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"
#include "layout.cuh"

namespace b200moe {

// ------------------------------------------------------------ NVFP4 quantize
__global__ void amax_kernel(const float* __restrict__ w, int64_t n, uint32_t* __restrict__ out_bits) {
  float m = 0.f;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(w[i]));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));  // m >= 0: int order = float order
}

__device__ __forceinline__ float nvfp4_global_from_amax(float amax) {
  return amax > 0.f ? __fdiv_rn(amax, 2688.f) : 1.f;
}

// One thread per 16-element block.
__global__ void nvfp4_quant_kernel(const float* __restrict__ w, int64_t nblocks,
                                   const uint32_t* __restrict__ amax_bits, uint8_t* __restrict__ codes,
                                   uint8_t* __restrict__ scales) {
  const int64_t b = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (b >= nblocks) return;
  const float glob = nvfp4_global_from_amax(__uint_as_float(*amax_bits));
  const float denom = __fmul_rn(6.f, glob);
  float v[16];
  const float4* src = reinterpret_cast<const float4*>(w + b * 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 t = src[i];
    v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
  float bmax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
  const uint32_t sb = e4m3_encode(__fdiv_rn(bmax, denom));
  const float qs = __fmul_rn(e4m3_value(sb), glob);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t mag = qs > 0.f ? e2m1_code(__fdiv_rn(fabsf(v[i]), qs)) : 0u;
    uint32_t nib = mag | (v[i] < 0.f ? 8u : 0u);
    if (i < 8) lo |= nib << (4 * i);
    else hi |= nib << (4 * (i - 8));
  }
  reinterpret_cast<uint2*>(codes)[b] = make_uint2(lo, hi);
  scales[b] = uint8_t(sb);
}

__global__ void nvfp4_global_kernel(float* g) {
  *g = nvfp4_global_from_amax(__uint_as_float(*reinterpret_cast<uint32_t*>(g)));
}

// ------------------------------------------------------------ MXFP4 quantize
__global__ void mxfp4_quant_kernel(const float* __restrict__ w, int64_t nblocks, uint8_t* __restrict__ codes,
                                   uint8_t* __restrict__ e8m0, uint32_t* err) {
  const int64_t b = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (b >= nblocks) return;
  float v[32];
  const float4* src = reinterpret_cast<const float4*>(w + b * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 t = src[i];
    v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
  float bmax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
  int e = bmax > 0.f ? mx_exponent(bmax) : 0;
  if (e < -127 || e > 127) {
    set_error(err, kErrRange);
    e = e < -127 ? -127 : 127;
  }
  uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    uint32_t nib = e2m1_code(ldexpf(fabsf(v[i]), -e)) | (v[i] < 0.f ? 8u : 0u);
    words[i / 8] |= nib << (4 * (i % 8));
  }
  reinterpret_cast<uint4*>(codes)[b] = make_uint4(words[0], words[1], words[2], words[3]);
  e8m0[b] = uint8_t(e + 127);
}

// ------------------------------------------------------------------- fold
// One thread per 32-block (two NVFP4 16-blocks).
__global__ void fold_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                            const float* __restrict__ gptr, int64_t nblocks32, uint8_t* __restrict__ out_codes,
                            uint8_t* __restrict__ out_e8m0, uint32_t* err) {
  const int64_t b = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (b >= nblocks32) return;
  const float g = *gptr;
  const uint4 cw = reinterpret_cast<const uint4*>(codes)[b];
  const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
  const uint32_t sb[2] = {scales[2 * b], scales[2 * b + 1]};
  if ((sb[0] & 127) == 127 || (sb[1] & 127) == 127) set_error(err, kErrFormat);
  const float blk[2] = {e4m3_value(sb[0]), e4m3_value(sb[1])};
  float max32 = 0.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float mag = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) mag = fmaxf(mag, e2m1_mag((w[(16 * h + i) / 8] >> (4 * (i % 8))) & 7));
    max32 = fmaxf(max32, __fmul_rn(__fmul_rn(mag, blk[h]), g));
  }
  int e = max32 > 0.f ? mx_exponent(max32) : 0;
  if (e < -127 || e > 127) {
    set_error(err, kErrRange);
    e = 0;
  }
  uint32_t ow[4] = {0, 0, 0, 0};
  bool exact = true;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint32_t nib = (w[i / 8] >> (4 * (i % 8))) & 15;
    const float value = __fmul_rn(__fmul_rn(e2m1_mag(nib), blk[i / 16]), g);
    const float target = ldexpf(value, -e);
    // first E2M1 magnitude >= target (searchsorted left), clipped to 7
    uint32_t idx = uint32_t(target > 0.f) + uint32_t(target > 0.5f) + uint32_t(target > 1.f) +
                   uint32_t(target > 1.5f) + uint32_t(target > 2.f) + uint32_t(target > 3.f) +
                   uint32_t(target > 4.f);
    exact = exact && (ldexpf(e2m1_mag(idx), e) == value);
    ow[i / 8] |= (idx | (nib & 8)) << (4 * (i % 8));
  }
  if (!exact) set_error(err, kErrRange);
  reinterpret_cast<uint4*>(out_codes)[b] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  out_e8m0[b] = uint8_t(e + 127);
}

// ----------------------------------------------------------- FP4 prepack
// Natural arrays of one projection pair: row pointer function below.
struct Fp4Src {
  const uint8_t* codes;   // [rows][K/2]
  const uint8_t* scales;  // [rows][K/bs]
  int k;                  // K of this projection
};

// Per (slot, projection) exponent span of the MXFP4 blocks with a nonzero code:
// span[slot][proj][0] = min e8m0, [1] = max e8m0.
__global__ void mx_span_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ e8m0,
                               int rows_per_slot, int k, int rows_split, int n_slots,
                               int proj_base, int* __restrict__ span, uint32_t* err) {
  // one thread per 32-block of the [n_slots][rows_per_slot][k] array
  const int64_t nb = int64_t(n_slots) * rows_per_slot * (k / 32);
  for (int64_t b = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; b < nb; b += int64_t(gridDim.x) * blockDim.x) {
    const uint4 cw = reinterpret_cast<const uint4*>(codes)[b];
    // magnitude bits of all 32 nibbles: any nonzero?
    const uint32_t mag = (cw.x | cw.y | cw.z | cw.w) & 0x77777777u;
    const uint32_t s = e8m0[b];
    if (s == 255) set_error(err, kErrFormat);
    if (mag == 0) continue;
    const int64_t row = b / (k / 32);
    const int slot = int(row / rows_per_slot);
    const int r = int(row % rows_per_slot);
    const int proj = proj_base + (r >= rows_split ? 1 : 0);
    atomicMin(&span[(slot * 3 + proj) * 2 + 0], int(s));
    atomicMax(&span[(slot * 3 + proj) * 2 + 1], int(s));
  }
}

__global__ void span_init_kernel(int* span, int n) {
  for (int i = threadIdx.x + blockIdx.x * blockDim.x; i < n; i += gridDim.x * blockDim.x)
    span[i] = (i & 1) ? -1 : 1 << 20;
}

// Rebase of each MXFP4 projection: the largest nonzero block maps to f16
// exponent 28 (values up to 6 * 2^13); global = 2^(emax - 127 - 13).
__global__ void mx_globals_kernel(const int* __restrict__ span, int n_slots, float* __restrict__ globals) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_slots * 3) return;
  const int emax = span[2 * i + 1];
  globals[i] = emax < 0 ? 1.f : ldexpf(1.f, emax - 127 - 13);
}

// One CTA of 128 threads per unit (tile pair x K tile).  Threads 0..127 write
// the 2 x 1024 code bytes (16 each), then the 2 * SB scale bytes in a strided loop.
template <int FMT>
__global__ void fp4_prepack_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                   int rows_per_slot, int k, int n_tp, int pair_rows_second,
                                   int pair_stride_first, const float* __restrict__ globals,
                                   int proj_first, int proj_split_row, uint8_t* __restrict__ dst,
                                   int64_t dst_slot_stride, uint32_t* err) {
  constexpr int bs = FMT == 0 ? 16 : 32;
  constexpr int SB = fp4_scale_bytes(FMT);
  constexpr int U = fp4_unit_bytes(FMT);
  const int n_kt = k / kFp4KTile;
  const int slot = blockIdx.y;
  const int unit = blockIdx.x;  // tp * n_kt + kt
  const int tp = unit / n_kt, kt = unit % n_kt;
  const uint8_t* csrc = codes + int64_t(slot) * rows_per_slot * (k / 2);
  const uint8_t* ssrc = scales + int64_t(slot) * rows_per_slot * (k / bs);
  uint8_t* out = dst + int64_t(slot) * dst_slot_stride + int64_t(unit) * U;
  // natural row of (mt, row-in-tile): W13 pairs gate/up, W2 consecutive tiles
  auto nat_row = [&](int mt, int rr) {
    return mt == 0 ? tp * pair_stride_first + rr : pair_rows_second + tp * pair_stride_first + rr;
  };
  const int t = threadIdx.x;
  {
    const int mt = t / 64, h = (t / 32) & 1, lane = t & 31;
    const int r = lane >> 2, q = lane & 3;
    const int row = nat_row(mt, r + 8 * h);
    uint32_t wv[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int byte = kt * 64 + 16 * c + 4 * q;
      wv[c] = *reinterpret_cast<const uint32_t*>(csrc + int64_t(row) * (k / 2) + byte);
    }
    *reinterpret_cast<uint4*>(out + mt * kCodesPerTile + h * 512 + lane * 16) =
        make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
  for (int idx = t; idx < 2 * SB; idx += blockDim.x) {
    const int mt = idx / SB, i = idx % SB;
    uint32_t byte;
    if (FMT == 0) {  // [r 8][qb 2][h 2][c 4]
      const int r = i >> 4, qb = (i >> 3) & 1, h = (i >> 2) & 1, c = i & 3;
      const int row = nat_row(mt, r + 8 * h);
      byte = ssrc[int64_t(row) * (k / 16) + kt * 8 + 2 * c + qb];
      if ((byte & 127) == 127) set_error(err, kErrFormat);
    } else {  // [r 8][h 2][c 4], rebased f16 exponent
      const int r = i >> 3, h = (i >> 2) & 1, c = i & 3;
      const int row = nat_row(mt, r + 8 * h);
      const int e = ssrc[int64_t(row) * (k / 32) + kt * 4 + c];
      const int proj = proj_first + (row >= proj_split_row ? 1 : 0);
      int gexp;
      frexpf(globals[slot * 3 + proj], &gexp);  // global = 2^(gexp - 1)
      int s = e - 127 - (gexp - 1) + 15;
      // blocks whose 32 codes are all +-0 may take any scale
      const uint4 cw = *reinterpret_cast<const uint4*>(csrc + int64_t(row) * (k / 2) + (kt * 128 + 32 * c) / 2);
      const bool zero = ((cw.x | cw.y | cw.z | cw.w) & 0x77777777u) == 0;
      if (zero) s = 1;
      if (s < 1 || s > 30) {
        set_error(err, kErrRange);
        s = s < 1 ? 1 : 30;
      }
      byte = uint32_t(s);
    }
    out[2 * kCodesPerTile + mt * SB + i] = uint8_t(byte);
  }
}

// ----------------------------------------------------------- IQ2 prepack
// One CTA of 64 threads per unit: thread (mt, h, r) copies 64 qs bytes; the
// first 32 threads also write one d value each.
__global__ void iq2_prepack_kernel(const uint8_t* __restrict__ src_a, const uint8_t* __restrict__ src_b,
                                   int rows_per_slot_a, int rows_per_slot_b, int k, int pair_second,
                                   uint8_t* __restrict__ dst, int64_t dst_slot_stride) {
  const int n_kb = k / kIq2KTile;
  const int slot = blockIdx.y;
  const int unit = blockIdx.x;
  const int tp = unit / n_kb, kb = unit % n_kb;
  uint8_t* out = dst + int64_t(slot) * dst_slot_stride + int64_t(unit) * kIq2UnitBytes;
  const int t = threadIdx.x;
  const int mt = t >> 5, h = (t >> 4) & 1, r = (t >> 1) & 7, half = t & 1;
  // source row: W13 -> mt 0 from W1 (src_a) rows 16tp.., mt 1 from W3 (src_b);
  // W2 (pair_second == 0) -> both tiles from src_a rows 32tp + 16mt ..
  const uint8_t* src;
  int row;
  if (pair_second) {
    src = mt == 0 ? src_a + int64_t(slot) * rows_per_slot_a * n_kb * 66
                  : src_b + int64_t(slot) * rows_per_slot_b * n_kb * 66;
    row = 16 * tp + r + 8 * h;
  } else {
    src = src_a + int64_t(slot) * rows_per_slot_a * n_kb * 66;
    row = 32 * tp + 16 * mt + r + 8 * h;
  }
  const uint8_t* blk = src + (int64_t(row) * n_kb + kb) * 66;
  // 32 qs bytes per thread (half of 64), 16-bit aligned source -> byte copies
  uint8_t* qs_dst = out + mt * 1024 + h * 512 + r * 64 + half * 32;
#pragma unroll 8
  for (int i = 0; i < 32; ++i) qs_dst[i] = blk[2 + half * 32 + i];
  if (half == 0) {
    uint8_t* d_dst = out + 2048 + mt * 32 + (r * 2 + h) * 2;
    d_dst[0] = blk[0];
    d_dst[1] = blk[1];
  }
}

// ----------------------------------------------------- IQ2_XS / IQ1_M prepack
// One CTA of 32 threads per unit: thread (mt, h, r) copies the fields of its
// row's block into the unit (layout.cuh: IQ2_XS qs / scales / d, IQ1_M
// qs / qh / scales, each [mt][h][r] but IQ2_XS's d as [mt][r][h]).
template <int FMT>
__global__ void iq_prepack_kernel(const uint8_t* __restrict__ src_a, const uint8_t* __restrict__ src_b,
                                  int rows_per_slot_a, int rows_per_slot_b, int k, int pair_second,
                                  uint8_t* __restrict__ dst, int64_t dst_slot_stride) {
  constexpr int BB = iq_block_bytes(FMT);
  const int n_kb = k / kIq2KTile;
  const int slot = blockIdx.y, unit = blockIdx.x;
  const int tp = unit / n_kb, kb = unit % n_kb;
  uint8_t* out = dst + int64_t(slot) * dst_slot_stride + int64_t(unit) * iq_unit_bytes(FMT);
  const int t = threadIdx.x;
  const int mt = t >> 4, h = (t >> 3) & 1, r = t & 7, rr = h * 8 + r;
  const uint8_t* src;
  int row;
  if (pair_second) {  // W13: mt 0 = W1 rows 16tp.., mt 1 = W3 rows 16tp..
    src = mt == 0 ? src_a + int64_t(slot) * rows_per_slot_a * n_kb * BB
                  : src_b + int64_t(slot) * rows_per_slot_b * n_kb * BB;
    row = 16 * tp + rr;
  } else {  // W2: rows 32tp + 16mt ..
    src = src_a + int64_t(slot) * rows_per_slot_a * n_kb * BB;
    row = 32 * tp + 16 * mt + rr;
  }
  const uint8_t* blk = src + (int64_t(row) * n_kb + kb) * BB;
  if (FMT == 3) {  // d [0, 2), qs [2, 66), scales [66, 74)
    for (int i = 0; i < 64; ++i) out[mt * 1024 + rr * 64 + i] = blk[2 + i];
    for (int i = 0; i < 8; ++i) out[2048 + mt * 128 + rr * 8 + i] = blk[66 + i];
    out[2304 + mt * 32 + r * 4 + h * 2] = blk[0];
    out[2304 + mt * 32 + r * 4 + h * 2 + 1] = blk[1];
  } else {  // IQ1_M: qs [0, 32), qh [32, 48), scales [48, 56)
    for (int i = 0; i < 32; ++i) out[mt * 512 + rr * 32 + i] = blk[i];
    for (int i = 0; i < 16; ++i) out[1024 + mt * 256 + rr * 16 + i] = blk[32 + i];
    for (int i = 0; i < 8; ++i) out[1536 + mt * 128 + rr * 8 + i] = blk[48 + i];
  }
}

// ----------------------------------------------------------- host launchers
static inline int grid_for(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  return int(g < 1 ? 1 : (g > 1048576 ? 1048576 : g));
}

int launch_mx_rebase(cudaStream_t s, int hidden, int inter, int n, const uint8_t* w13c, const uint8_t* w13s,
                     const uint8_t* w2c, const uint8_t* w2s, float* slot_globals, int* span_scratch, uint32_t* err) {
  span_init_kernel<<<grid_for(int64_t(n) * 6, 256), 256, 0, s>>>(span_scratch, n * 6);
  mx_span_kernel<<<grid_for(int64_t(n) * 2 * inter * (hidden / 32), 256), 256, 0, s>>>(
      w13c, w13s, 2 * inter, hidden, inter, n, 0, span_scratch, err);
  mx_span_kernel<<<grid_for(int64_t(n) * hidden * (inter / 32), 256), 256, 0, s>>>(
      w2c, w2s, hidden, inter, hidden, n, 2, span_scratch, err);
  mx_globals_kernel<<<grid_for(n * 3, 128), 128, 0, s>>>(span_scratch, n, slot_globals);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_fp4_prepack(cudaStream_t s, int fmt, int hidden, int inter, int n,
                       const uint8_t* w13c, const uint8_t* w13s, const uint8_t* w2c, const uint8_t* w2s,
                       float* slot_globals, int* span_scratch, uint8_t* bank_slot0, int64_t slot_stride,
                       int64_t w13_bytes, uint32_t* err) {
  if (fmt == 1) {
    span_init_kernel<<<grid_for(int64_t(n) * 6, 256), 256, 0, s>>>(span_scratch, n * 6);
    mx_span_kernel<<<grid_for(int64_t(n) * 2 * inter * (hidden / 32), 256), 256, 0, s>>>(
        w13c, w13s, 2 * inter, hidden, inter, n, 0, span_scratch, err);
    mx_span_kernel<<<grid_for(int64_t(n) * hidden * (inter / 32), 256), 256, 0, s>>>(
        w2c, w2s, hidden, inter, hidden, n, 2, span_scratch, err);
    mx_globals_kernel<<<grid_for(n * 3, 128), 128, 0, s>>>(span_scratch, n, slot_globals);
  }
  // W13: tile pair tp = (W1 rows 16tp.., W3 rows I + 16tp..)
  dim3 g13((inter / 16) * (hidden / kFp4KTile), n);
  dim3 g2((hidden / 32) * (inter / kFp4KTile), n);
  if (fmt == 0) {
    fp4_prepack_kernel<0><<<g13, 128, 0, s>>>(w13c, w13s, 2 * inter, hidden, inter / 16, inter, 16,
                                               slot_globals, 0, inter, bank_slot0, slot_stride, err);
    fp4_prepack_kernel<0><<<g2, 128, 0, s>>>(w2c, w2s, hidden, inter, hidden / 32, 16, 32, slot_globals,
                                              2, 1 << 30, bank_slot0 + w13_bytes, slot_stride, err);
  } else {
    fp4_prepack_kernel<1><<<g13, 128, 0, s>>>(w13c, w13s, 2 * inter, hidden, inter / 16, inter, 16,
                                               slot_globals, 0, inter, bank_slot0, slot_stride, err);
    // W2: the second tile's rows 32tp + 16 + r are plain rows of the same projection
    fp4_prepack_kernel<1><<<g2, 128, 0, s>>>(w2c, w2s, hidden, inter, hidden / 32, 16, 32, slot_globals,
                                              2, 1 << 30, bank_slot0 + w13_bytes, slot_stride, err);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_iq2_prepack(cudaStream_t s, int fmt13, int fmt2, int hidden, int inter, int n, const uint8_t* w1,
                       const uint8_t* w3, const uint8_t* w2, uint8_t* bank_slot0, int64_t slot_stride,
                       int64_t w13_bytes) {
  dim3 g13((inter / 16) * (hidden / kIq2KTile), n);
  dim3 g2((hidden / 32) * (inter / kIq2KTile), n);
  uint8_t* w2dst = bank_slot0 + w13_bytes;
  switch (fmt13) {
    case 2: iq2_prepack_kernel<<<g13, 64, 0, s>>>(w1, w3, inter, inter, hidden, 1, bank_slot0, slot_stride); break;
    case 3: iq_prepack_kernel<3><<<g13, 32, 0, s>>>(w1, w3, inter, inter, hidden, 1, bank_slot0, slot_stride); break;
    case 4: iq_prepack_kernel<4><<<g13, 32, 0, s>>>(w1, w3, inter, inter, hidden, 1, bank_slot0, slot_stride); break;
    default: return -1;
  }
  switch (fmt2) {
    case 2: iq2_prepack_kernel<<<g2, 64, 0, s>>>(w2, nullptr, hidden, hidden, inter, 0, w2dst, slot_stride); break;
    case 3: iq_prepack_kernel<3><<<g2, 32, 0, s>>>(w2, nullptr, hidden, hidden, inter, 0, w2dst, slot_stride); break;
    case 4: iq_prepack_kernel<4><<<g2, 32, 0, s>>>(w2, nullptr, hidden, hidden, inter, 0, w2dst, slot_stride); break;
    default: return -1;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace b200moe

using namespace b200moe;

extern "C" int b200moe_quantize_nvfp4(void* stream, const float* w, int rows, int k, uint8_t* codes,
                                      uint8_t* scales, float* global_scale) {
  if (!w || !codes || !scales || !global_scale || rows < 1 || k < 16 || k % 16) return B200MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(codes) & 7)) return B200MOE_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = int64_t(rows) * k;
  if (cudaMemsetAsync(global_scale, 0, sizeof(float), s) != cudaSuccess) return B200MOE_ERR_CUDA;
  amax_kernel<<<grid_for(n, 256) > 4096 ? 4096 : grid_for(n, 256), 256, 0, s>>>(
      w, n, reinterpret_cast<uint32_t*>(global_scale));
  nvfp4_quant_kernel<<<grid_for(n / 16, 128), 128, 0, s>>>(
      w, n / 16, reinterpret_cast<const uint32_t*>(global_scale), codes, scales);
  nvfp4_global_kernel<<<1, 1, 0, s>>>(global_scale);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

extern "C" int b200moe_quantize_mxfp4(void* stream, const float* w, int rows, int k, uint8_t* codes,
                                      uint8_t* e8m0, uint32_t* err) {
  if (!w || !codes || !e8m0 || rows < 1 || k < 32 || k % 32) return B200MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(codes) & 15)) return B200MOE_ERR_ALIGN;
  const int64_t nb = int64_t(rows) * k / 32;
  mxfp4_quant_kernel<<<grid_for(nb, 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(w, nb, codes, e8m0, err);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}

extern "C" int b200moe_fold_nvfp4_to_mxfp4(void* stream, const uint8_t* codes, const uint8_t* scales,
                                           const float* global_scale, int rows, int k, uint8_t* out_codes,
                                           uint8_t* out_e8m0, uint32_t* err) {
  if (!codes || !scales || !global_scale || !out_codes || !out_e8m0 || rows < 1 || k < 32 || k % 32)
    return B200MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) || (reinterpret_cast<uintptr_t>(out_codes) & 15))
    return B200MOE_ERR_ALIGN;
  const int64_t nb = int64_t(rows) * k / 32;
  fold_kernel<<<grid_for(nb, 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(codes, scales, global_scale,
                                                                                 nb, out_codes, out_e8m0, err);
  return cudaGetLastError() == cudaSuccess ? B200MOE_OK : B200MOE_ERR_CUDA;
}
