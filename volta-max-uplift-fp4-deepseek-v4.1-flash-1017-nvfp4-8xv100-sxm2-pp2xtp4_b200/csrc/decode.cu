// Fused small-batch decode on the block-scaled FP4 tensor cores.
//
// A decode call of at most 64 routes on a layer whose experts all sit in the
// FP4 bank streams little per launch, so the chained path (route plan, x
// planes, W13, SwiGLU planes, W2, combine: six launches after gating) spends
// most of its time between launches.  Here the layer is two launches, W13 and
// W2 (replacing, like the chained path, the reference's QPN launches and its
// separate reduce: engine/.../experts/nvfp4_8r_native.py:929-960).
//
// Each CTA of either launch first plans the call itself: the stable order of
// the routes by expert slot and chunks of at most four routes per expert, the
// route plan's own order and chunking (route.cu plan_small), so sorted
// positions agree between the two launches and with the chained path.  It
// takes a contiguous range of items (chunk x weight unit row).  The producer
// warp streams the range's 36 KB weight units through a ring of stages from
// the start; four quantizer warps write the rows of the range's chunks (W13:
// the tokens' rows of x; W2: the SwiGLU rows W13 stored) as four E2M1 planes
// with their block scales straight into a shared-memory operand that holds
// the whole K, publishing it one 256-wide K tile at a time (warp w takes the
// tiles w, w + 4, ...), so the MMA warp's tcgen05.mma.kind::mxf4nvf4 on the
// first weight stage waits for one tile, not the row.  Four epilogue warps
// drain the TMEM accumulators: W13 stores the
// limited SwiGLU rows, W2 the fp16 y2 rows and then, through a completion
// count per (token, 256-column unit), the CTA that stores a unit's last route
// sums the token's routes in slot order into the output, the separate
// combine's arithmetic.  Planes, MMAs and sums are the chained path's, so the
// output is the same bits.
//
// Measured on B200 (configs[1], in-kernel %globaltimer stamps): the row
// quantization is the critical path.  One warp's call of the four-plane
// quantizer on a K tile takes ~5 us (a long dependent chain per half-block),
// so at M = 1 the first MMA starts ~9 us after the plan and the step takes
// 63.8 us against 57.6 us chained (M = 8: 264 against 170 us), where the
// plane launches spread the same work over many CTAs.  The layer therefore
// leaves this path off unless the caller turns it on
// (b200moe_set_decode_fusion).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "fp4_device.cuh"
#include "internal.h"

namespace b200moe {
namespace {

constexpr int kDecRC = 4;                     // routes per chunk: the MMA's N is 16
constexpr int kDecBTile = kP * kDecRC * 128;  // one 256-wide K tile of a chunk's plane rows (2 KB)
constexpr int kDecThreads = 320;              // producer, MMA, 4 epilogue warps, 4 quantizer warps
constexpr size_t kDecSmemLimit = 220 * 1024;  // dynamic part (the static plan arrays take the rest)

size_t decode_smem(int K, int stages) {
  const int n_kt = K / 256;
  return 1024 + size_t(stages) * Fp4Stage<2, kDecRC, 0>::kUnit + size_t(n_kt) * (kDecBTile + kSFBytes) +
         size_t(2 * stages + 5 + n_kt) * 8;
}

int decode_stages(int K) {
  if (K % 256 || K < 256) return 0;
  for (int st = 4; st >= 2; --st)
    if (decode_smem(K, st) <= kDecSmemLimit) return st;
  return 0;
}

// AND of pred over the `count` threads of named barrier `id` (every one of them calls it)
__device__ __forceinline__ bool named_bar_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; barrier.red.and.pred q, %2, %3, p; selp.u32 %0, 1, 0, q; }"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

template <int EPI, int MX, int BF16>
__global__ void __launch_bounds__(kDecThreads, 1) fp4_decode_kernel(const DecArgs a) {
  using St = Fp4Stage<2, kDecRC, MX>;
  constexpr int kN = St::kN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* stages = smem_raw + (base_u32 - smem_u32(smem_raw));
  const int n_st = a.stages, n_kt = a.K / 256, nhb = a.K / 8;
  uint8_t* btile = stages + size_t(n_st) * St::kUnit;  // [n_kt][16 rows x 128 B], 128-byte swizzled
  uint8_t* bsf = btile + n_kt * kDecBTile;             // [n_kt][4][512]: the planes' block scales
  uint64_t* full = reinterpret_cast<uint64_t*>(bsf + n_kt * kSFBytes);
  uint64_t* empty = full + n_st;
  uint64_t* acc_full = empty + n_st;  // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* b_empty = acc_empty + 2;   // the MMAs that read the operand are complete (MMA commit)
  uint64_t* bk_full = b_empty + 1;     // [n_kt] K tile kt of the chunk's planes is written (quantizer warp)
  __shared__ int s_key[kDecodeMaxRoutes];     // bank-0 slot of route i (n_keys: no expert)
  __shared__ int s_perm[kDecodeMaxRoutes];    // route at sorted position
  __shared__ int s_pkey[kDecodeMaxRoutes];    // slot at sorted position
  __shared__ int4 s_chunk[kDecodeMaxRoutes];  // (slot, first position, routes, 0)
  __shared__ int s_done[128];
  __shared__ float s_red[4][kDecRC];
  __shared__ float s_gx[kDecodeMaxRoutes][kDecRC];  // plane factor g of each chunk's routes
  __shared__ int s_nchunks, s_ndone;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  volatile int* abort_ptr = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < n_st; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(b_empty, 1);
    for (int kt = 0; kt < n_kt; ++kt) mbar_init(&bk_full[kt], 1);
    fence_barrier_init();
    abort_flag = 0;
  }
  // the plane operand starts as zeros: rows past a chunk's routes give zero columns
  for (int i = threadIdx.x; i < n_kt * (kDecBTile + kSFBytes) / 16; i += kDecThreads)
    reinterpret_cast<uint4*>(btile)[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base_sh;
  pdl_wait();  // ids and weights (gating) and, for W2, the SwiGLU rows of W13 are complete

  // ---------------------------------------------------------------- plan
  const int S = a.S;
  if (threadIdx.x < S) {
    const int e = a.ids[threadIdx.x];
    int key = a.n_keys;
    if (e < 0 || e >= a.num_experts) {
      set_error(a.err, kErrBounds);
    } else {
      const int k = a.key_of_expert[e];
      if (k < 0 || k >= a.n_keys) set_error(a.err, kErrBounds);
      else key = k;
    }
    s_key[threadIdx.x] = key;
  }
  __syncthreads();
  if (threadIdx.x < S) {  // stable rank by (slot, route)
    const int me = s_key[threadIdx.x] * kDecodeMaxRoutes + int(threadIdx.x);
    int rank = 0;
    for (int j = 0; j < S; ++j) rank += (s_key[j] * kDecodeMaxRoutes + j) < me;
    s_perm[rank] = threadIdx.x;
    s_pkey[rank] = s_key[threadIdx.x];
  }
  __syncthreads();
  if (warp == 0) {  // chunks of <= 4 routes per run of one slot, in position order (two positions a lane)
    int cnt[2], nch[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int p = 2 * lane + h;
      cnt[h] = 0;
      if (p < S) {
        const int k = s_pkey[p];
        if (k < a.n_keys && (p == 0 || s_pkey[p - 1] != k)) {
          int c = 1;
          while (p + c < S && s_pkey[p + c] == k) ++c;
          cnt[h] = c;
        }
      }
      nch[h] = (cnt[h] + kDecRC - 1) / kDecRC;
    }
    const int mine = nch[0] + nch[1];
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int ci = incl - mine;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int p = 2 * lane + h;
      for (int off = 0; off < cnt[h]; off += kDecRC)
        s_chunk[ci++] = make_int4(s_pkey[p], p + off, min(kDecRC, cnt[h] - off), 0);
    }
    if (lane == 31) s_nchunks = incl;
    if (EPI == 0 && blockIdx.x == 0 && a.perm_out)
      for (int p = lane; p < S; p += 32) a.perm_out[p] = s_perm[p];
  }
  __syncthreads();
  const int n_items = s_nchunks * a.n_rt;
  const int i0 = int(int64_t(blockIdx.x) * n_items / gridDim.x);
  const int i1 = int(int64_t(blockIdx.x + 1) * n_items / gridDim.x);
  auto item_ok = [&](const int4& ch) { return ch.x >= 0 && ch.x < a.n_slots && ch.z >= 1 && ch.z <= kDecRC; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer: weight units only
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t g = 0, issued = 0, parity = 0;
      for (int item = i0; item < i1 && !*abort_ptr; ++item) {
        const int4 ch = s_chunk[item / a.n_rt];
        if (!item_ok(ch)) {
          set_error(a.err, kErrBounds);
          continue;
        }
        const int rt = item % a.n_rt;
        const uint8_t* wu = a.wt + (int64_t(ch.x) * a.n_rt + rt) * n_kt * St::kUnit;
        for (int kt = 0; kt < n_kt; ++kt, ++g) {
          const int s = g % n_st;
          const uint32_t ph = (g / n_st) & 1u;
          if (*abort_ptr || !mbar_wait(&empty[s], ph ^ 1u, a.err)) {
            *abort_ptr = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[s], uint32_t(St::kUnit));
          bulk_g2s_hint(stages + s * St::kUnit, wu + int64_t(kt) * St::kUnit, St::kUnit, &full[s], pol);
          issued |= 1u << s;
          parity = (parity & ~(1u << s)) | (ph << s);
        }
      }
      // no copy may be in flight when the CTA exits
      for (int s = 0; s < n_st; ++s)
        if (issued & (1u << s)) mbar_wait(&full[s], (parity >> s) & 1u, a.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t g = 0, acc_i = 0, last_b = 0, last_ph = 0, nb = 0;
      bool committed = false;
      int cur = -1;
      for (int item = i0; item < i1; ++item) {
        const int ci = item / a.n_rt;
        const int4 ch = s_chunk[ci];
        if (!item_ok(ch)) continue;
        const bool first = ci != cur;  // the chunk's first item waits for each K tile of its planes
        if (first) {
          if (cur >= 0) commit_to(b_empty);  // the previous chunk's MMAs release the operand
          ++nb;
          cur = ci;
        }
        const uint32_t b = acc_i & 1u, bph = (acc_i >> 1) & 1u;
        if (*abort_ptr || !mbar_wait(&acc_empty[b], bph ^ 1u, a.err)) {
          *abort_ptr = 1;
          break;
        }
        fence_after();
        const uint32_t dg = tmem + b * St::kAccCols, du = dg + kN;
        bool ok = true;
        for (int kt = 0; kt < n_kt; ++kt, ++g) {
          const int s = g % n_st;
          const uint32_t ph = (g / n_st) & 1u;
          if (*abort_ptr || !mbar_wait(&full[s], ph, a.err) ||
              (first && !mbar_wait(&bk_full[kt], (nb - 1) & 1u, a.err))) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t st = smem_u32(stages + s * St::kUnit);
          const uint32_t bt = smem_u32(btile + kt * kDecBTile), bs = smem_u32(bsf + kt * kSFBytes);
          const uint32_t sfg = tmem + kSfCol + s * St::kSfCols, sfu = sfg + 16, sfb = sfg + St::kSfB;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sf_copy(sfg + 4 * j, st + St::kOffSFG + 512 * j);
            sf_copy(sfu + 4 * j, st + St::kOffSFU + 512 * j);
            sf_copy(sfb + 4 * j, bs + 512 * j);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t acc = (kt | j) != 0;
            const uint64_t bdesc = desc_sw128(bt + 32 * j);
            mma_fp4<MX>(dg, desc_sw128(st + St::kOffAG + 32 * j), bdesc, sfg + 4 * j, sfb + 4 * j, acc, St::kIdesc);
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
  } else if (warp >= 6) {
    // ------------------------------------------------------------ quantizer warps
    const int qq = threadIdx.x - 192;  // 0 .. 127
    const int qw = qq >> 5;
    const uint16_t* src = static_cast<const uint16_t*>(a.src);
    // source row of the route at sorted position pos: W13 its token's x row, W2 its SwiGLU row
    auto row_of = [&](int pos) {
      return EPI == 0 ? src + int64_t(s_perm[pos] / a.top_k) * a.src_stride : src + int64_t(pos) * a.src_stride;
    };
    uint32_t nq = 0;
    int cur = -1;
    for (int item = i0; item < i1; ++item) {
      const int ci = item / a.n_rt;
      const int4 ch = s_chunk[ci];
      if (!item_ok(ch) || ci == cur) continue;
      // a new chunk: its rows go into the operand once the MMAs of the previous chunk are done with it
      bool ok = true;
      if (qq == 0) ok = !*abort_ptr && mbar_wait(b_empty, (nq & 1u) ^ 1u, a.err);
      if (!named_bar_and(2, 128, ok)) {
        if (qq == 0) *abort_ptr = 1;
        break;
      }
      // the rows' amax (the plane factor g): four independent loads in flight per thread
#pragma unroll
      for (int n = 0; n < kDecRC; ++n) {
        if (n >= ch.z) break;
        const uint16_t* rp = row_of(ch.y + n);
        float am = 0.f;
#pragma unroll 4
        for (int hb = qq; hb < nhb; hb += 128) {
          float f[8];
          load8<BF16>(*reinterpret_cast<const uint4*>(rp + hb * 8), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(f[e]));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        if (lane == 0) s_red[qw][n] = am;
      }
      named_bar(2, 128);
      if (qq < ch.z) {
        const float m = fmaxf(fmaxf(s_red[0][qq], s_red[1][qq]), fmaxf(s_red[2][qq], s_red[3][qq]));
        // MXFP4: power-of-two block scales cover any row (g = 1); NVFP4: the row's amax over 6 * 448
        s_gx[ci][qq] = MX ? 1.f : m / (6.f * 448.f);
      }
      named_bar(2, 128);
      // K tile kt (32 half-blocks: one per lane) of every route of the chunk, then publish it
      for (int kt = qw; kt < n_kt; kt += 4) {
        const int hb = kt * 32 + lane;
        uint8_t* tb = btile + kt * kDecBTile;
        const int c16 = lane >> 2, sub = (lane & 3) * 4;
        for (int n = 0; n < ch.z; ++n) {
          const float g = s_gx[ci][n];
          const float inv_g = g > 0.f ? __frcp_rn(g) : 0.f;
          float r[8];
          load8<BF16>(*reinterpret_cast<const uint4*>(row_of(ch.y + n) + hb * 8), r);
          uint32_t w[kP], word[kP];
          quantize_planes8<MX>(r, true, g, inv_g, w, word);
          // 16-byte chunk lane / 4 of plane row n * 4 + p, 128-byte swizzled; the scale words from lanes 8j
#pragma unroll
          for (int p = 0; p < kP; ++p) {
            const int mr = n * kP + p;
            *reinterpret_cast<uint32_t*>(tb + mr * 128 + ((c16 ^ (mr & 7)) << 4) + sub) = w[p];
            if ((lane & 7) == 0)
              *reinterpret_cast<uint32_t*>(bsf + (hb >> 3) * 512 + (mr & 31) * 16 + (mr >> 5) * 4) = word[p];
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core's reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&bk_full[kt]);
      }
      ++nq;
      cur = ci;
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int q = threadIdx.x - 64;  // 0 .. 127
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter ..: the weight rows of this warp
    const int row = quarter * 32 + lane;
    const int units = a.H / 256;
    // out[tok][unit] = the slot-order sum of fma(f32(y2), w) over the token's routes (no expert: a zero row
    // with weight 0), then the unit's count starts again from zero; all 128 threads, two columns each
    auto combine_unit = [&](int tok, int unit) {
      __threadfence();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = unit * 256 + q + 128 * h;
        float sum = 0.f;
        for (int slot = 0; slot < a.top_k; ++slot) {
          const int r = tok * a.top_k + slot;
          const bool has = s_key[r] < a.n_keys;
          const float y = has ? __half2float(__ushort_as_half(
                                    __ldcg(reinterpret_cast<const unsigned short*>(a.y2) + int64_t(r) * a.H + col)))
                              : 0.f;
          sum = __fmaf_rn(y, has ? __ldg(a.w_in + r) : 0.f, sum);
        }
        a.out[int64_t(tok) * a.H + col] = sum;
      }
      if (q == 0) a.counters[int64_t(tok) * (a.H / 32) + unit * 8] = 0;
    };
    if (EPI == 1 && blockIdx.x == 0) {
      // routes without an expert arrive here, once per unit of their token, with nothing to store
      for (int r = 0; r < S; ++r) {
        if (s_key[r] < a.n_keys) continue;
        const int tok = r / a.top_k;
        if (q == 0) s_ndone = 0;
        named_bar(1, 128);
        for (int u = q; u < units; u += 128)
          if (atomicAdd(a.counters + int64_t(tok) * (a.H / 32) + u * 8, 1) == a.top_k - 1)
            s_done[atomicAdd(&s_ndone, 1)] = u;
        named_bar(1, 128);
        const int nd = s_ndone;
        for (int d = 0; d < nd; ++d) combine_unit(tok, s_done[d]);
        named_bar(1, 128);
      }
    }
    uint32_t acc_i = 0;
    for (int item = i0; item < i1; ++item) {
      const int ci = item / a.n_rt;
      const int4 ch = s_chunk[ci];
      if (!item_ok(ch)) continue;
      const int rt = item % a.n_rt;
      const float* gl = a.globals ? a.globals + ch.x * 3 : nullptr;
      const float gw0 = gl ? gl[EPI == 0 ? 0 : 2] : 1.f, gw1 = (gl && EPI == 0) ? gl[1] : 1.f;
      const uint32_t b = acc_i & 1u, bph = (acc_i >> 1) & 1u;
      const bool got = !*abort_ptr && mbar_wait(&acc_full[b], bph, a.err);
      if (!named_bar_and(1, 128, got)) {
        if (q == 0) *abort_ptr = 1;
        break;
      }
      fence_after();
      const uint32_t lanes = uint32_t(quarter * 32) << 16;
      float d0[kN], d1[kN];
      tmem_ld16(tmem + lanes + b * St::kAccCols, d0);
      tmem_ld16(tmem + lanes + b * St::kAccCols + kN, d1);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // the accumulator is in registers now
#pragma unroll
      for (int n = 0; n < kDecRC; ++n) {
        if (n >= ch.z) break;
        const int pos = ch.y + n;
        float v0 = 0.f, v1 = 0.f;
#pragma unroll
        for (int p = 0; p < kP; ++p) {
          v0 += d0[n * kP + p];
          v1 += d1[n * kP + p];
        }
        const float gx = s_gx[ci][n];  // written before the chunk's first K tile was published
        if (EPI == 0) {
          const float gh = __half2float(__float2half_rn(v0 * gx * gw0));
          const float uh = __half2float(__float2half_rn(v1 * gx * gw1));
          a.inter[int64_t(pos) * a.inter_stride + rt * 128 + row] = swiglu1(gh, uh, a.limit);
        } else {
          __half* yrow = a.y2 + int64_t(s_perm[pos]) * a.H + rt * 256 + row;
          yrow[0] = __float2half_rn(v0 * gx * gw0);
          yrow[128] = __float2half_rn(v1 * gx * gw0);
        }
      }
      ++acc_i;
      if (EPI == 1) {
        // count this unit's routes done; the CTA that completes a token's unit sums it
        if (q == 0) s_ndone = 0;
        __threadfence();
        named_bar(1, 128);
        if (q < ch.z) {
          const int tok = s_perm[ch.y + q] / a.top_k;
          if (atomicAdd(a.counters + int64_t(tok) * (a.H / 32) + rt * 8, 1) == a.top_k - 1)
            s_done[atomicAdd(&s_ndone, 1)] = tok;
        }
        named_bar(1, 128);
        const int nd = s_ndone;
        for (int d = 0; d < nd; ++d) combine_unit(s_done[d], rt);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  pdl_trigger();  // the next launch may take this SM (and its TMEM) now
}

template <int EPI, int MX, int BF16>
int launch_decode_one(cudaStream_t s, const DecArgs& a, int grid) {
  const size_t smem = decode_smem(a.K, a.stages);
  static std::atomic<uint64_t> attr_set{0};  // devices whose attribute is set
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return -1;
  if (!(attr_set.load() >> dev & 1)) {
    if (cudaFuncSetAttribute(fp4_decode_kernel<EPI, MX, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(kDecSmemLimit)) != cudaSuccess)
      return -1;
    attr_set.fetch_or(uint64_t(1) << dev);
  }
  return launch_chain(fp4_decode_kernel<EPI, MX, BF16>, dim3(grid), dim3(kDecThreads), smem, s, a) == cudaSuccess
             ? 0
             : -1;
}

}  // namespace

bool fp4_decode_fits(int K) { return decode_stages(K) >= 2; }

int launch_fp4_decode(cudaStream_t s, int epi, bool mx, bool bf16, const DecArgs& a_in, int grid) {
  DecArgs a = a_in;
  a.stages = decode_stages(a.K);
  if (a.stages < 2 || a.S < 1 || a.S > kDecodeMaxRoutes || a.H % 256 || a.H / 256 > 128 || a.n_keys != a.n_slots)
    return -1;
  if (epi == 1 && bf16) return -1;  // SwiGLU rows are fp16
  if (epi == 0) {
    if (mx) return bf16 ? launch_decode_one<0, 1, 1>(s, a, grid) : launch_decode_one<0, 1, 0>(s, a, grid);
    return bf16 ? launch_decode_one<0, 0, 1>(s, a, grid) : launch_decode_one<0, 0, 0>(s, a, grid);
  }
  return mx ? launch_decode_one<1, 1, 0>(s, a, grid) : launch_decode_one<1, 0, 0>(s, a, grid);
}

}  // namespace b200moe
