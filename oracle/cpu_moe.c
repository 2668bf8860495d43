// CPU oracle / timed CPU baseline for the routed-expert MoE layer.
//
// TEST INFRASTRUCTURE ONLY: loaded by the tests and by bench.py's CPU legs,
// never by the product library.
//
// A C restatement, with every shape a parameter, of the reference's CPU expert
// kernel (harness/benchmarks/nvfp4_8r/cpu_mxfp4_moe.c:28-96, shapes fixed at
// 5120/576 there): per routed row, y13 = W13 x (W1 rows then W3 rows), the
// limited SwiGLU silu(min(g, L)) * clamp(u, -L, L) in FP32
// (engine/.../experts/nvfp4_8r_native.py:937-939), y2 = W2 inter, and
// out[row] += weight * y2.  Weights are read straight from the packed formats:
//   NVFP4  codes [R][K/2] (low nibble = even element), E4M3 scale per 16,
//          FP32 global per projection: value = (E2M1 * scale) * global
//          (harness/benchmarks/nvfp4_8r/accept_p1.py:53-84);
//   MXFP4  codes [R][K/2], E8M0 per 32: value = E2M1 * 2^(e-127)
//          (accept_p1.py:87-101).
// Accumulation is FP32; OpenMP splits the output rows of each projection.
//
// Two forms of the same expert:
//   oracle_expert       scalar, plain loops: the checker the tests compare with;
//   oracle_expert_avx2  the timed CPU baseline: AVX2 + FMA, as fast per weight
//                       byte as the reference's own AVX2 kernel (the tests time
//                       both on one shape), for NVFP4 and MXFP4 at any shape.
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static const float kE2M1[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                                -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

static float e4m3_value(uint8_t b) {
  int e = (b >> 3) & 15, m = b & 7;
  float v = e == 0 ? (float)m * 0.001953125f : ldexpf(1.f + (float)m / 8.f, e - 7);
  return (b & 128) ? -v : v;
}

static float e8m0_value(uint8_t s) { return ldexpf(1.f, (int)s - 127); }

// Block scale of one block (NVFP4: fmt 0, MXFP4: fmt 1).
static inline float block_scale(int fmt, uint8_t s) {
  return fmt == 0 ? e4m3_value(s) : e8m0_value(s);
}

// out[r * ldo] = sum_k W[n][k] x[r][k] for r < m, one weight row n.
static void row_dot(int fmt, const uint8_t *codes, const uint8_t *scales, int k,
                    const float *x, int ldx, int m, float *out, int ldo) {
  const int bs = fmt == 0 ? 16 : 32;
  float acc[64];
  for (int r = 0; r < m; r++) acc[r] = 0.f;
  float w[32];
  for (int b = 0; b < k / bs; b++) {
    const float s = block_scale(fmt, scales[b]);
    for (int j = 0; j < bs / 2; j++) {
      uint8_t c = codes[b * bs / 2 + j];
      w[2 * j] = kE2M1[c & 15] * s;
      w[2 * j + 1] = kE2M1[c >> 4] * s;
    }
    for (int r = 0; r < m; r++) {
      const float *xr = x + (size_t)r * ldx + (size_t)b * bs;
      float part = 0.f;
      for (int j = 0; j < bs; j++) part += w[j] * xr[j];
      acc[r] += part;
    }
  }
  for (int r = 0; r < m; r++) out[(size_t)r * ldo] = acc[r];
}

// One expert over m routed rows (m <= 64).
//   w13c [2I][H/2], w13s [2I][H/bs], w2c [H][I/2], w2s [H][I/bs]
//   g13: globals of W1 and W3 (NVFP4) or {1, 1} (MXFP4); g2: global of W2
//   x [*][H] fp32 token rows; rows[i]: token of route i; weight[i]: router weight
//   out [*][H] fp32, accumulated; scratch: >= m * (2I + I + H) floats
void oracle_expert(int fmt, int hidden, int inter, const uint8_t *w13c, const uint8_t *w13s,
                   const float *g13, const uint8_t *w2c, const uint8_t *w2s, float g2,
                   const float *x, const int *rows, const float *weight, int m, float limit,
                   float *out, float *scratch) {
  const int bs = fmt == 0 ? 16 : 32;
  float *xs = scratch;                                 // [m][H]
  float *gu = xs + (size_t)m * hidden;                 // [m][2I]
  float *act = gu + (size_t)m * 2 * inter;             // [m][I]
  float *y2 = act + (size_t)m * inter;                 // [m][H]
  for (int i = 0; i < m; i++) memcpy(xs + (size_t)i * hidden, x + (size_t)rows[i] * hidden, sizeof(float) * hidden);
#pragma omp parallel
  {
#pragma omp for schedule(static)
    for (int n = 0; n < 2 * inter; n++) {
      row_dot(fmt, w13c + (size_t)n * (hidden / 2), w13s + (size_t)n * (hidden / bs), hidden, xs,
              hidden, m, gu + n, 2 * inter);
      const float g = n < inter ? g13[0] : g13[1];
      for (int i = 0; i < m; i++) gu[(size_t)i * 2 * inter + n] *= g;
    }
#pragma omp for schedule(static)
    for (int t = 0; t < m * inter; t++) {
      int r = t / inter, j = t % inter;
      float g = gu[(size_t)r * 2 * inter + j], u = gu[(size_t)r * 2 * inter + inter + j];
      g = g > limit ? limit : g;
      u = u > limit ? limit : (u < -limit ? -limit : u);
      act[(size_t)r * inter + j] = g / (1.f + expf(-g)) * u;
    }
#pragma omp for schedule(static)
    for (int n = 0; n < hidden; n++) {
      row_dot(fmt, w2c + (size_t)n * (inter / 2), w2s + (size_t)n * (inter / bs), inter, act, inter,
              m, y2 + n, hidden);
    }
  }
  for (int i = 0; i < m; i++) {
    float *o = out + (size_t)rows[i] * hidden;
    const float *y = y2 + (size_t)i * hidden;
    for (int n = 0; n < hidden; n++) o[n] += weight[i] * (y[n] * g2);
  }
}

// Dequantize one projection to fp32 [R][K] (tests).
void oracle_dequant(int fmt, int rows, int k, const uint8_t *codes, const uint8_t *scales,
                    float global, float *out) {
  const int bs = fmt == 0 ? 16 : 32;
  for (int r = 0; r < rows; r++)
    for (int b = 0; b < k / bs; b++) {
      float s = block_scale(fmt, scales[(size_t)r * (k / bs) + b]);
      for (int j = 0; j < bs; j++) {
        uint8_t c = codes[(size_t)r * (k / 2) + (b * bs + j) / 2];
        float v = kE2M1[(j & 1) ? (c >> 4) : (c & 15)];
        out[(size_t)r * k + b * bs + j] = fmt == 0 ? (v * s) * global : v * s;
      }
    }
}

// ---------------------------------------------------------------------------
// AVX2 form.  A 32-element block is 16 code bytes: byte j holds element 2j in
// its low nibble and 2j+1 in its high nibble.  Instead of interleaving the
// decoded nibbles back into element order, the activation rows are split once
// per call into their even and odd elements per 32-block (xe, xo: 16 floats
// each), so the low nibbles dot with xe and the high nibbles with xo.  A nibble
// becomes twice its E2M1 value as an int8 by one byte shuffle (the values
// 0, 1, 2, 3, 4, 6, 8, 12 and their negatives are integers), then fp32; the
// block scale carries the factor 1/2.  Lanes 0-7 of each half-block vector are
// the block's first 16 elements (NVFP4 scale s0), lanes 8-15 its last 16 (s1).

// Block-scale values by byte, each times 1/2 (the int8 weights are 2 x E2M1).
static float kHalfE4M3[256], kHalfE8M0[256];

__attribute__((constructor)) static void init_scale_tables(void) {
  for (int b = 0; b < 256; b++) {
    kHalfE4M3[b] = 0.5f * e4m3_value((uint8_t)b);
    kHalfE8M0[b] = 0.5f * e8m0_value((uint8_t)b);
  }
}

void oracle_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

int oracle_threads(void) { return omp_get_max_threads(); }

// rows [m][k] -> [m][k]: per 32-block, 16 even elements then 16 odd elements
static void split_even_odd(const float *x, int ldx, int m, int k, float *out) {
  for (int r = 0; r < m; r++)
    for (int b = 0; b < k / 32; b++) {
      const float *src = x + (size_t)r * ldx + 32 * b;
      float *dst = out + (size_t)r * k + 32 * b;
      for (int j = 0; j < 16; j++) {
        dst[j] = src[2 * j];
        dst[16 + j] = src[2 * j + 1];
      }
    }
}

// out[r * ldo] = sum_k W[n][k] x[r][k], one weight row, x split by split_even_odd.
static void row_dot_avx2(int fmt, const uint8_t *codes, const uint8_t *scales, int k,
                         const float *xsplit, int m, float *out, int ldo) {
  const __m128i twice_e2m1 = _mm_setr_epi8(0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12);
  const __m128i nib = _mm_set1_epi8(0x0f);
  for (int r0 = 0; r0 < m; r0 += 8) {
    const int mr = m - r0 < 8 ? m - r0 : 8;
    __m256 acc[8];
    for (int r = 0; r < 8; r++) acc[r] = _mm256_setzero_ps();
    for (int b = 0; b < k / 32; b++) {
      const __m128i raw = _mm_loadu_si128((const __m128i *)(codes + 16 * b));
      const __m128i ev = _mm_shuffle_epi8(twice_e2m1, _mm_and_si128(raw, nib));
      const __m128i od = _mm_shuffle_epi8(twice_e2m1, _mm_and_si128(_mm_srli_epi16(raw, 4), nib));
      const __m256 we0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(ev));
      const __m256 we1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_unpackhi_epi64(ev, ev)));
      const __m256 wo0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(od));
      const __m256 wo1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_unpackhi_epi64(od, od)));
      float s0, s1;
      if (fmt == 0) {
        s0 = kHalfE4M3[scales[2 * b]];
        s1 = kHalfE4M3[scales[2 * b + 1]];
      } else {
        s0 = s1 = kHalfE8M0[scales[b]];
      }
      const __m256 vs0 = _mm256_set1_ps(s0), vs1 = _mm256_set1_ps(s1);
      if (fmt == 0) {  // a scale per 16: the two halves of the block apart
        for (int r = 0; r < mr; r++) {
          const float *xr = xsplit + (size_t)(r0 + r) * k + 32 * b;
          __m256 h0 = _mm256_mul_ps(we0, _mm256_loadu_ps(xr));
          h0 = _mm256_fmadd_ps(wo0, _mm256_loadu_ps(xr + 16), h0);
          __m256 h1 = _mm256_mul_ps(we1, _mm256_loadu_ps(xr + 8));
          h1 = _mm256_fmadd_ps(wo1, _mm256_loadu_ps(xr + 24), h1);
          acc[r] = _mm256_fmadd_ps(vs0, h0, acc[r]);
          acc[r] = _mm256_fmadd_ps(vs1, h1, acc[r]);
        }
      } else {  // one scale per 32
        for (int r = 0; r < mr; r++) {
          const float *xr = xsplit + (size_t)(r0 + r) * k + 32 * b;
          __m256 h = _mm256_mul_ps(we0, _mm256_loadu_ps(xr));
          h = _mm256_fmadd_ps(wo0, _mm256_loadu_ps(xr + 16), h);
          h = _mm256_fmadd_ps(we1, _mm256_loadu_ps(xr + 8), h);
          h = _mm256_fmadd_ps(wo1, _mm256_loadu_ps(xr + 24), h);
          acc[r] = _mm256_fmadd_ps(vs0, h, acc[r]);
        }
      }
    }
    for (int r = 0; r < mr; r++) {
      float lanes[8];
      _mm256_storeu_ps(lanes, acc[r]);
      out[(size_t)(r0 + r) * ldo] = ((lanes[0] + lanes[4]) + (lanes[1] + lanes[5])) +
                                    ((lanes[2] + lanes[6]) + (lanes[3] + lanes[7]));
    }
  }
}

// Same contract as oracle_expert; scratch >= m * (2H + 2I + I + H) floats.
void oracle_expert_avx2(int fmt, int hidden, int inter, const uint8_t *w13c, const uint8_t *w13s,
                        const float *g13, const uint8_t *w2c, const uint8_t *w2s, float g2,
                        const float *x, const int *rows, const float *weight, int m, float limit,
                        float *out, float *scratch) {
  const int bs = fmt == 0 ? 16 : 32;
  float *xs = scratch;                                 // [m][H] gathered rows
  float *xsp = xs + (size_t)m * hidden;                // [m][H] split
  float *gu = xsp + (size_t)m * hidden;                // [m][2I]
  float *act = gu + (size_t)m * 2 * inter;             // [m][I]
  float *actsp = act + (size_t)m * inter;              // [m][I] split
  float *y2 = actsp + (size_t)m * inter;               // [m][H]
  for (int i = 0; i < m; i++) memcpy(xs + (size_t)i * hidden, x + (size_t)rows[i] * hidden, sizeof(float) * hidden);
  split_even_odd(xs, hidden, m, hidden, xsp);
#pragma omp parallel
  {
#pragma omp for schedule(static)
    for (int n = 0; n < 2 * inter; n++) {
      row_dot_avx2(fmt, w13c + (size_t)n * (hidden / 2), w13s + (size_t)n * (hidden / bs), hidden, xsp, m,
                   gu + n, 2 * inter);
      const float g = n < inter ? g13[0] : g13[1];
      for (int i = 0; i < m; i++) gu[(size_t)i * 2 * inter + n] *= g;
    }
#pragma omp for schedule(static)
    for (int t = 0; t < m * inter; t++) {
      int r = t / inter, j = t % inter;
      float g = gu[(size_t)r * 2 * inter + j], u = gu[(size_t)r * 2 * inter + inter + j];
      g = g > limit ? limit : g;
      u = u > limit ? limit : (u < -limit ? -limit : u);
      act[(size_t)r * inter + j] = g / (1.f + expf(-g)) * u;
    }
#pragma omp single
    split_even_odd(act, inter, m, inter, actsp);
#pragma omp for schedule(static)
    for (int n = 0; n < hidden; n++)
      row_dot_avx2(fmt, w2c + (size_t)n * (inter / 2), w2s + (size_t)n * (inter / bs), inter, actsp, m,
                   y2 + n, hidden);
  }
  for (int i = 0; i < m; i++) {
    float *o = out + (size_t)rows[i] * hidden;
    const float *y = y2 + (size_t)i * hidden;
    for (int n = 0; n < hidden; n++) o[n] += weight[i] * (y[n] * g2);
  }
}
