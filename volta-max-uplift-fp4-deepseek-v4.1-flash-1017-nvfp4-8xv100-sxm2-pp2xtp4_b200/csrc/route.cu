// Routing kernels: softmax top-k gating, the stable token -> expert permute
// with its group tables, and the bf16 -> f16 activation copy.
//
// The permute is a stable counting sort by key in one CTA (1024 threads):
// each warp owns a contiguous run of routes, counts its keys with a ballot split,
// the per-warp counts become per-warp offsets, and a second pass scatters each
// route to start[key] + (earlier warps' count) + (rank among equal keys in its
// batch).  That is exactly the stable argsort of the reference chain
// (engine/.../experts/nvfp4_8r_native.py:806-822) and the rank definition of
// the reference's one-launch plan (engine/.../experts/nvfp4_8r_group_plan.py:13-24),
// for any number of routes, not just the reference's 96.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <float.h>

#include "common.cuh"
#include "fp4_device.cuh"
#include "internal.h"

namespace b200moe {

constexpr int kPlanThreads = 1024;

// In-place exclusive scan of arr[0..len) in shared memory by the whole CTA;
// returns the total.  Every thread of the CTA must call it.
__device__ int block_exclusive_scan(int* arr, int len, int* wsum) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seg = (len + kPlanThreads - 1) / kPlanThreads;
  const int lo = tid * seg, hi = min(len, lo + seg);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += arr[i];
  int inc = local;
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int v = wsum[lane];
    int s = v;
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += u;
    }
    wsum[lane] = s - v;   // exclusive warp base
    if (lane == 31) wsum[32] = s;
  }
  __syncthreads();
  int run = wsum[warp] + inc - local;
  for (int i = lo; i < hi; ++i) {
    int v = arr[i];
    arr[i] = run;
    run += v;
  }
  const int total = wsum[32];
  __syncthreads();
  return total;
}

// The table entry a route's expert id reads first: its key, or its hot slot.
__device__ __forceinline__ int plan_entry(const PlanArgs& a, int e) {
  if (e < 0 || e >= a.num_experts) return 0;
  return (a.key_of_expert ? a.key_of_expert : a.hot_slot)[e];
}

// A route's key from its expert id e and that id's first table entry (plan_entry); kErrors = false only
// counts (the route's own CTA reports it).
template <bool kErrors = true>
__device__ __forceinline__ int plan_key_of(const PlanArgs& a, int e, int entry, int sentinel) {
  if (e < 0 || e >= a.num_experts) {
    if (kErrors) set_error(a.err, kErrBounds);
    return sentinel;
  }
  if (a.key_of_expert) {
    const int k = entry;
    if (k < 0 || k >= a.n_keys) {
      if (kErrors) set_error(a.err, kErrBounds);
      return sentinel;
    }
    return k;
  }
  const int hot = entry;
  if (!a.split) {
    if (hot < 0 || hot >= a.n_hot) {
      if (kErrors) set_error(a.err, kErrBounds);
      return sentinel;
    }
    return hot;
  }
  if (hot >= 0) return hot;
  const int sec = a.second_slot[e];
  return sec >= 0 ? a.n_hot + sec : a.n_hot + a.n_second;
}

__device__ __forceinline__ int plan_key(const PlanArgs& a, int i, int sentinel) {
  const int e = a.ids[i];
  return plan_key_of(a, e, plan_entry(a, e), sentinel);
}

// The lanes of this warp whose key equals this lane's (keys in [0, 2^bits), or -1 for no route): the bit-by-bit
// ballot split of a radix multisplit, a vote per key bit instead of one match.any, which serialises over the
// distinct keys (measured on B200, one CTA planning 32,768 routes over 385 keys: 76 against 95 us).
__device__ __forceinline__ unsigned warp_match_key(int key, int bits) {
  const unsigned valid = __ballot_sync(0xffffffffu, key >= 0);
  unsigned m = key >= 0 ? valid : ~valid;
  for (int b = 0; b < bits; ++b) {
    const bool one = (key >> b) & 1;
    const unsigned v = __ballot_sync(0xffffffffu, one);
    m &= one ? v : ~v;
  }
  return m;
}

// The keys of routes base0 + stride * u + lane, u < kBatch (-1 at or past hi): every id is loaded, then every
// table entry, before the first check can store an error flag, so the loads of the batches overlap.
template <int kBatch, bool kErrors = true>
__device__ __forceinline__ void plan_keys(const PlanArgs& a, int base0, int stride, int hi, int lane, int sentinel,
                                          int (&keys)[kBatch]) {
  int e[kBatch], entry[kBatch];
#pragma unroll
  for (int u = 0; u < kBatch; ++u) {
    const int i = base0 + stride * u + lane;
    e[u] = i < hi ? a.ids[i] : -1;
  }
#pragma unroll
  for (int u = 0; u < kBatch; ++u) entry[u] = plan_entry(a, e[u]);
#pragma unroll
  for (int u = 0; u < kBatch; ++u)
    keys[u] = base0 + stride * u + lane < hi ? plan_key_of<kErrors>(a, e[u], entry[u], sentinel) : -1;
}

// Routes per chunk for the split-K with the least modelled time, given the
// bank's chunk counts at 16, 8, 4 and 2 routes per chunk.
// Modelled time of split-K ks = 2^j for a bank with `chunks_j` chunks at 16 >> j routes per chunk.
__device__ __forceinline__ float model_t(const KsModel& m, int j, int chunks_j) {
  const int ks = 1 << j;
  const float chunks = fmaxf(1.f, float(chunks_j));
  float t = 0.f;
  for (int p = 0; p < 2; ++p) {
    const float items = chunks * m.tiles[p] / (8.f / ks);
    const float bytes = (8.f / ks) * m.kdim[p] * m.bpe;
    const float waves = ceilf(items / m.slots);
    t += waves * (fmaxf(bytes / m.bw_cta, fminf(items, m.slots) * bytes / m.bw_hbm) + m.per_wave);
  }
  return t;
}

// Called by a whole warp: lanes j = lane & 3 model the four split-Ks side by side (the divisions of one
// thread's four models in a row were a microsecond on the plan's critical path), then every lane picks the
// first allowed one with the least time.
__device__ __forceinline__ int model_rc_warp(const KsModel& m, int c0, int c1, int c2, int c3) {
  const int jm = threadIdx.x & 3;
  const float tm = model_t(m, jm, jm == 0 ? c0 : jm == 1 ? c1 : jm == 2 ? c2 : c3);
  int best = 1;
  float best_t = 3.0e38f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float t = __shfl_sync(0xffffffffu, tm, j);
    if (!(m.allowed >> j & 1)) continue;
    if (t < best_t * 0.999999f) {
      best_t = t;
      best = 1 << j;
    }
  }
  return kRouteSlotsPerChunk / best;
}

// Product plan of at most 32 routes by one warp (decode at M <= 4 for top-8):
// the same outputs as the block-wide path below -- stable order by key,
// chunk lists, split-K, bank ranges, key counts, routes without an expert --
// from a 32-wide bitonic sort of (key, route) and warp scans.
__device__ void plan_small(const PlanArgs& a, int n, int sentinel) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int key = lane < n ? plan_key(a, lane, sentinel) : 0x7fff;
  if (lane < n && a.w_eff) a.w_eff[lane] = key < a.n_keys ? a.w_in[lane] : 0.f;
  int c = (key << 5) | lane;  // stable: ties in key keep the route order
  for (int k = 2; k <= 32; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int o = __shfl_xor_sync(full, c, j);
      const bool take_min = ((lane & j) == 0) == ((lane & k) == 0);
      c = take_min ? min(c, o) : max(c, o);
    }
  const int pkey = lane < n ? (c >> 5) : 0x7fff, route = c & 31;
  if (lane < n) a.perm[lane] = route;
  if (lane < n && a.inv) a.inv[route] = lane;
  const int prev = __shfl_up_sync(full, pkey, 1);
  const bool starts = lane < n && (lane == 0 || prev != pkey);
  const unsigned smask = __ballot_sync(full, starts);
  const unsigned later = smask & ~((2u << lane) - 1u);  // (2u << 31) == 0: no later start for lane 31
  const int count = starts ? (later ? __ffs(later) - 1 : n) - lane : 0;
  if (a.key_counts) {
    for (int kk = lane; kk < a.n_keys; kk += 32) a.key_counts[kk] = 0;
    __syncwarp();
    if (starts && pkey < a.n_keys) a.key_counts[pkey] = count;
  }
  // routes without an expert (sorted last): zero y2 rows, count them done
  const int n_bad = __popc(__ballot_sync(full, lane < n && pkey == a.n_keys));
  if (n_bad > 0 && a.y2 && a.counters) {
    const int first = n - n_bad;
    for (int64_t idx = lane; idx < int64_t(n_bad) * a.H; idx += 32) {
      const int r = a.perm[first + int(idx / a.H)];
      static_cast<__half*>(a.y2)[int64_t(r) * a.H + idx % a.H] = __float2half_rn(0.f);
    }
    __threadfence();
    __syncwarp();
    const int tiles = a.H / 32;
    for (int idx = lane; idx < n_bad * tiles; idx += 32) {
      const int r = a.perm[first + idx / tiles], tile = idx % tiles;
      const int tok = r / a.top_k;
      int* cp = a.counters + int64_t(tok) * tiles + tile;
      if (atomicAdd(cp, 1) == a.top_k - 1) {
        for (int q = 0; q < 32; ++q) a.out[int64_t(tok) * a.H + 32 * tile + q] = 0.f;
        *cp = 0;
      }
    }
  }
  for (int b = 0; b < a.n_banks; ++b) {
    const bool mine = starts && pkey >= a.key_lo[b] && pkey < a.key_hi[b];
    int at[4];
    for (int j = 0; j < 4; ++j) {
      int v = mine ? (count + (16 >> j) - 1) / (16 >> j) : 0;
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(full, v, o);
      at[j] = v;
    }
    int rc = a.rc[b];
    if (rc == 0) rc = model_rc_warp(a.ks_model[b], at[0], at[1], at[2], at[3]);
    if (lane == 0 && a.ks_sel) a.ks_sel[b] = max(1, kRouteSlotsPerChunk / rc);
    const int lo = __popc(__ballot_sync(full, lane < n && pkey < a.key_lo[b]));
    const int hi = __popc(__ballot_sync(full, lane < n && pkey < a.key_hi[b]));
    if (a.bank_range && lane == 0) {
      a.bank_range[2 * b] = lo;
      a.bank_range[2 * b + 1] = hi;
    }
    // chunks: ceil(count / rc) per run of this bank, in key order
    const int nch = mine ? (count + rc - 1) / rc : 0;
    int incl = nch;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(full, incl, o);
      if (lane >= o) incl += v;
    }
    const int total = __shfl_sync(full, incl, 31);
    int ci = incl - nch;
    for (int off = 0; off < count && mine; off += rc, ++ci) {
      if (ci < a.max_chunks[b]) {
        Chunk ch;
        ch.slot = pkey - a.key_lo[b];
        ch.begin = lane + off;
        ch.count = min(rc, count - off);
        ch.pad = 0;
        a.chunks[b][ci] = ch;
        if (a.chunk_of && b == 0)
          for (int j = 0; j < ch.count; ++j) a.chunk_of[ch.begin + j] = (ci << 8) | j;
      }
    }
    if (lane == 0) {
      if (total > a.max_chunks[b]) set_error(a.err, kErrRange);
      a.n_chunks[b] = min(total, a.max_chunks[b]);
    }
  }
}

// Keys: product mode [0, n_keys) plus one sentinel bucket n_keys for a route
// without an expert; reference mode [0, n_hot) (resident) or
// [0, n_hot + n_second] (split, the last key being the WARM sentinel).
__global__ void __launch_bounds__(kPlanThreads, 1) plan_kernel(PlanArgs a) {
  extern __shared__ int smem[];
  __shared__ int wsum[33];
  __shared__ int misc[8];
  const bool product = a.key_of_expert != nullptr;
  const int nk = product ? a.n_keys + 1 : (a.split ? a.n_hot + a.n_second + 1 : a.n_hot + 1);
  const int sentinel = product ? a.n_keys : nk - 1;
  int* hist = smem;             // [32][nk]
  int* start = hist + 32 * nk;  // [nk]
  int* aux = start + nk;        // [nk]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ int s_recv;
  pdl_wait();
  pdl_trigger();
  if (a.recv.flags) {
    // expert-parallel receive: every source rank's rows are in once its data
    // flag reaches this step's epoch; the rows received are the reservation
    // counter of that epoch, then both counters start again from zero (no rank
    // reserves rows of the next step before this step's return reached it)
    if (tid == 0) {
      const int e = *a.recv.epoch;
      int n_in = 0;
      if (wait_flags(a.recv.flags, a.recv.n_flags, e, a.err)) {
        n_in = atomicExch(a.recv.resv + (e & 1), 0);
        atomicExch(a.recv.resv + ((e + 1) & 1), 0);
        if (n_in > a.n) {
          set_error(a.err, kErrRange);
          n_in = a.n;
        }
      }
      a.recv.out[0] = n_in;
      a.recv.out[1] = 0;
      a.recv.out[2] = n_in;
      s_recv = n_in;
    }
    __syncthreads();
  }
  // a.n_valid (device) bounds the routes of this call below the launch's a.n
  const int n = a.recv.flags ? s_recv : a.n_valid ? min(a.n, max(0, *a.n_valid)) : a.n;
  // routes past this call's count have no position (a stale one would send their rows' planes into a live
  // route's place)
  if (a.inv)
    for (int i = n + tid; i < a.n; i += blockDim.x) a.inv[i] = -1;
  if (product && n <= 32) {  // decode-sized plans: one warp, no block-wide phases
    if (warp == 0) plan_small(a, n, sentinel);
    return;
  }
  // A wide plan (gridDim.x > 1, product keys of a host-sized call without a fused combine) splits the routes
  // over gridDim.x - 1 CTAs: each counts every route's key (totals, and the routes before its own run) and
  // scatters its own run; the last CTA builds the chunk tables from the totals.  One CTA does it all otherwise.
  const bool wide = gridDim.x > 1;
  const bool tables = !wide || blockIdx.x == gridDim.x - 1;
  const int n_runs = wide ? gridDim.x - 1 : 1;
  const int per_run = (n + n_runs - 1) / n_runs;
  const int r_lo = tables && wide ? n : min(n, int(blockIdx.x) * per_run);
  const int r_hi = tables && wide ? n : min(n, r_lo + per_run);
  int* before = aux + nk;  // [nk] (wide only): routes of each key before this CTA's run
  for (int i = tid; i < 32 * nk; i += kPlanThreads) hist[i] = 0;
  if (wide)
    for (int key = tid; key < nk; key += kPlanThreads) aux[key] = before[key] = 0;
  __syncthreads();
  constexpr int kBatch = 8;
  if (wide) {  // every route's key, counted without its error (the route's own CTA reports that)
    for (int base0 = 0; base0 < n; base0 += kPlanThreads * kBatch) {
      int keys[kBatch];
      plan_keys<kBatch, false>(a, base0, kPlanThreads, n, tid, sentinel, keys);
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (keys[u] >= 0) {
          atomicAdd(&aux[keys[u]], 1);
          if (!tables && base0 + kPlanThreads * u + tid < r_lo) atomicAdd(&before[keys[u]], 1);
        }
    }
  }
  const int key_bits = 32 - __clz(nk - 1);  // keys are below nk
  const int len = r_hi - r_lo;
  const int per_warp = ((len + 31) / 32 + 31) / 32 * 32;
  const int wlo = r_lo + min(len, warp * per_warp), whi = min(r_hi, wlo + per_warp);
  // a warp with at most kBatch batches keeps their keys and weights in registers from pass 1 to pass 2
  const bool cached = per_warp <= 32 * kBatch;
  int keys[kBatch];
  float wv[kBatch];  // the routes' weights, loaded before the scatter's stores
  auto load_weights = [&](int base0) {
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      wv[u] = product && a.w_eff && keys[u] >= 0 && keys[u] < a.n_keys ? a.w_in[base0 + 32 * u + lane] : 0.f;
  };
  // pass 1: per-warp key counts, eight 32-route batches at a time (plan_keys)
  for (int base0 = wlo; base0 < whi; base0 += 32 * kBatch) {
    plan_keys<kBatch>(a, base0, 32, whi, lane, sentinel, keys);
    if (cached) load_weights(base0);
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (base0 + 32 * u >= whi) break;  // warp-uniform
      const int key = keys[u];
      const unsigned mask = warp_match_key(key, key_bits);
      if (key >= 0 && lane == __ffs(mask) - 1) hist[warp * nk + key] += __popc(mask);
      __syncwarp();
    }
  }
  __syncthreads();
  // per-key totals and per-warp offsets (a wide plan's totals are the counts of every route)
  for (int key = tid; key < nk; key += kPlanThreads) {
    int run = wide ? before[key] : 0;
    for (int w = 0; w < 32; ++w) {
      const int c = hist[w * nk + key];
      hist[w * nk + key] = run;
      run += c;
    }
    if (!wide) aux[key] = run;
    start[key] = aux[key];
  }
  __syncthreads();
  block_exclusive_scan(start, nk, wsum);
  // pass 2: stable scatter (the same batches, keys looked up ahead)
  for (int base0 = wlo; base0 < whi; base0 += 32 * kBatch) {
    if (!cached) {
      plan_keys<kBatch>(a, base0, 32, whi, lane, sentinel, keys);
      load_weights(base0);
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (base0 + 32 * u >= whi) break;  // warp-uniform
      const int i = base0 + 32 * u + lane;
      const int key = keys[u];
      const unsigned mask = warp_match_key(key, key_bits);
      if (key >= 0) {
        const int rank = __popc(mask & ((1u << lane) - 1u));
        const int pos = start[key] + hist[warp * nk + key] + rank;
        a.perm[pos] = i;
        if (a.inv) a.inv[i] = pos;
        if (product && a.w_eff) a.w_eff[i] = wv[u];
        if (a.iq_out) a.iq_out[i] = a.iq_slot[a.ids[i]];
      }
      __syncwarp();
      if (key >= 0 && lane == __ffs(mask) - 1) hist[warp * nk + key] += __popc(mask);
      __syncwarp();
    }
  }
  __syncthreads();

  if (product && aux[nk - 1] > 0 && a.y2 && a.counters) {
    // routes without an expert (sorted last): zero their rows, count them done
    const int first = start[nk - 1], cnt = aux[nk - 1];
    const int tiles = a.H / 32;
    for (int64_t idx = tid; idx < int64_t(cnt) * a.H; idx += kPlanThreads) {
      const int route = a.perm[first + int(idx / a.H)];
      static_cast<__half*>(a.y2)[int64_t(route) * a.H + idx % a.H] = __float2half_rn(0.f);
    }
    __threadfence();
    __syncthreads();
    for (int idx = tid; idx < cnt * tiles; idx += kPlanThreads) {
      const int route = a.perm[first + idx / tiles], tile = idx % tiles;
      const int tok = route / a.top_k;
      int* c = a.counters + int64_t(tok) * tiles + tile;
      if (atomicAdd(c, 1) == a.top_k - 1) {  // every route of this token lacked an expert
        for (int r = 0; r < 32; ++r) a.out[int64_t(tok) * a.H + 32 * tile + r] = 0.f;
        *c = 0;
      }
    }
    __syncthreads();
  }

  if (!tables) return;
  if (product && a.key_counts)
    for (int key = tid; key < a.n_keys; key += kPlanThreads) a.key_counts[key] = aux[key];

  __shared__ int rc_sel[2];
  if (product) {
    // chunk counts of every bank at 16, 8, 4 and 2 routes per chunk
    __shared__ int st[2][4];
    if (tid < 8) st[tid / 4][tid % 4] = 0;
    __syncthreads();
    for (int b = 0; b < a.n_banks; ++b)
      for (int base = a.key_lo[b]; base < a.key_hi[b]; base += kPlanThreads) {  // block-uniform trips
        const int key = base + tid;
        const int c = key < a.key_hi[b] ? aux[key] : 0;
        const int c16 = __reduce_add_sync(0xffffffffu, (c + 15) / 16);
        const int c8 = __reduce_add_sync(0xffffffffu, (c + 7) / 8);
        const int c4 = __reduce_add_sync(0xffffffffu, (c + 3) / 4);
        const int c2 = __reduce_add_sync(0xffffffffu, (c + 1) / 2);
        if (lane == 0 && c2 > 0) {  // one add per warp, not per key
          atomicAdd(&st[b][0], c16);
          atomicAdd(&st[b][1], c8);
          atomicAdd(&st[b][2], c4);
          atomicAdd(&st[b][3], c2);
        }
      }
    __syncthreads();
    if (warp == 0)
      for (int b = 0; b < a.n_banks; ++b) {
        int rc = a.rc[b];
        if (rc == 0) rc = model_rc_warp(a.ks_model[b], st[b][0], st[b][1], st[b][2], st[b][3]);  // split-K of
        if (lane == 0) {                                                                          // this bank
          rc_sel[b] = rc;
          if (a.ks_sel) a.ks_sel[b] = max(1, kRouteSlotsPerChunk / rc);
          if (a.bank_range) {
            a.bank_range[2 * b] = start[a.key_lo[b]];
            a.bank_range[2 * b + 1] = start[a.key_hi[b]];
          }
        }
      }
    __syncthreads();
  }

  if (product) {
    // route chunks of every bank: ceil(count / rc) chunks per non-empty key
    for (int b = 0; b < a.n_banks; ++b) {
      const int lo = a.key_lo[b], hi = a.key_hi[b], rc = rc_sel[b];
      if (hi <= lo) {  // a bank without keys has no chunks
        if (tid == 0) a.n_chunks[b] = 0;
        continue;
      }
      int* nch = hist;  // hist is free now: reuse as [nk]
      for (int key = tid; key < nk; key += kPlanThreads)
        nch[key] = (key >= lo && key < hi) ? (aux[key] + rc - 1) / rc : 0;
      __syncthreads();
      const int total = block_exclusive_scan(nch, nk, wsum);
      for (int key = lo + tid; key < hi; key += kPlanThreads) {
        const int cnt = aux[key];
        int c = nch[key];
        for (int off = 0; off < cnt; off += rc, ++c) {
          if (c < a.max_chunks[b]) {
            Chunk ch;
            ch.slot = key - lo;
            ch.begin = start[key] + off;
            ch.count = min(rc, cnt - off);
            ch.pad = 0;
            a.chunks[b][c] = ch;
            if (a.chunk_of && b == 0)
              for (int j = 0; j < ch.count; ++j) a.chunk_of[ch.begin + j] = (c << 8) | j;
          }
        }
      }
      if (tid == 0) {
        if (total > a.max_chunks[b]) set_error(a.err, kErrRange);
        a.n_chunks[b] = min(total, a.max_chunks[b]);
      }
      __syncthreads();
    }
    return;
  }

  // reference-parity tables (EXP/nvfp4_8r_group_plan.py:13-24)
  if (tid == 0) {
    int count_hot = 0, count_native = 0, groups_hot = 0, n_groups = 0, last = -1;
    for (int key = 0; key < nk; ++key) {
      const int c = aux[key];
      if (c == 0) continue;
      ++n_groups;
      last = key;
      if (key < a.n_hot) { count_hot += c; ++groups_hot; }
      if (key < a.n_hot + a.n_second) count_native += c;
    }
    misc[0] = count_hot; misc[1] = count_native; misc[2] = groups_hot; misc[3] = n_groups; misc[4] = last;
  }
  int* gidx = hist;  // reuse: group index of each key
  for (int key = tid; key < nk; key += kPlanThreads) gidx[key] = aux[key] > 0 ? 1 : 0;
  __syncthreads();
  block_exclusive_scan(gidx, nk, wsum);
  const int count_hot = misc[0], count_native = misc[1], groups_hot = misc[2], n_groups = misc[3], last = misc[4];
  for (int key = tid; key < nk; key += kPlanThreads) {
    if (aux[key] == 0) continue;
    const int g = gidx[key];
    a.goff_hot[g] = min(start[key], count_hot);
    a.gids_hot[g] = key < a.n_hot ? key : 0;
    if (a.host) {
      const int t = g - groups_hot;
      if (t >= 0) {
        a.goff_host[t] = min(start[key], count_native);
        a.gids_host[t] = min(max(key - a.n_hot, 0), a.n_second - 1);
      }
    }
  }
  for (int g = n_groups + tid; g <= n; g += kPlanThreads) {
    a.goff_hot[g] = count_hot;
    if (g < n) a.gids_hot[g] = 0;
  }
  if (a.host) {
    const int fill = n_groups == n ? min(max(last - a.n_hot, 0), a.n_second - 1) : 0;
    for (int t = n_groups - groups_hot + tid; t <= n; t += kPlanThreads) {
      a.goff_host[t] = count_native;
      if (t < n) a.gids_host[t] = fill;
    }
  }
}

size_t plan_smem_bytes(int n_keys_total) { return size_t(34) * n_keys_total * sizeof(int); }

// Routes per scatter CTA of a wide plan, and the calls that take one: a single 1024-thread CTA spends about
// 2.3 ns per route at 32,768 routes (B200), where each of 33 CTAs counts all routes' keys and scatters 1,024.
constexpr int kPlanWideRoutes = 1024;
constexpr int kPlanWideMin = 4096;

int launch_plan(cudaStream_t s, const PlanArgs& a) {
  const bool product = a.key_of_expert != nullptr;
  const int nk = product ? a.n_keys + 1 : (a.split ? a.n_hot + a.n_second + 1 : a.n_hot + 1);
  const size_t smem = plan_smem_bytes(nk);
  if (smem > 200 * 1024) return -1;
  if (product && a.n <= 32) {  // the one-warp path needs neither the block nor the shared histograms
    return launch_chain(plan_kernel, dim3(1), dim3(32), 0, s, a) == cudaSuccess ? 0 : -1;
  }
  static std::atomic<uint64_t> attr_set{0};  // devices whose attribute is set
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return -1;
  if (!(attr_set.load() >> dev & 1)) {
    if (cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
      return -1;
    attr_set.fetch_or(uint64_t(1) << dev);
  }
  const bool wide = product && !a.recv.flags && !a.n_valid && !a.counters && a.n >= kPlanWideMin &&
                    smem + nk * sizeof(int) <= 200 * 1024;
  if (wide) {
    const int runs = (a.n + kPlanWideRoutes - 1) / kPlanWideRoutes;
    return launch_chain(plan_kernel, dim3(runs + 1), dim3(kPlanThreads), smem + nk * sizeof(int), s, a) ==
                   cudaSuccess ? 0 : -1;
  }
  return launch_chain(plan_kernel, dim3(1), dim3(kPlanThreads), smem, s, a) == cudaSuccess ? 0 : -1;
}

// Route plan and the token rows' FP4 planes in one launch, for decode calls of
// at most 32 routes on the block-scaled path: every CTA of the plane grid
// (token row x 1024-wide slice) runs the one-warp plan itself -- CTA (0, 0)
// into the layer's plan buffers, the others into shared memory, the same
// values -- and then quantizes its slice, which needs the token's sorted
// positions the plan just made.  Saves the plan's own launch.
template <int BF16, int MX>
__global__ void __launch_bounds__(kPlaneThreads) plan_planes_kernel(PlanArgs a, const uint16_t* __restrict__ src,
                                                                   int64_t src_stride, int K, int n_tokens,
                                                                   uint32_t* rowmax, uint8_t* planes, uint8_t* sfb,
                                                                   float* gx) {
  __shared__ PlaneScratch sm;
  __shared__ int s_perm[32], s_inv[32], s_chunk_of[32], s_nch[2], s_range[4];
  __shared__ Chunk s_chunks[2][32];
  pdl_wait();
  pdl_trigger();
  PlanArgs p = a;
  if (blockIdx.x != 0 || blockIdx.y != 0) {  // a private copy of the plan: only CTA (0, 0) writes the layer's
    p.perm = s_perm;
    p.inv = s_inv;
    p.chunk_of = s_chunk_of;
    p.chunks[0] = s_chunks[0];
    p.chunks[1] = s_chunks[1];
    p.n_chunks = s_nch;
    p.bank_range = s_range;
    p.w_eff = nullptr;
    p.key_counts = nullptr;
    p.ks_sel = nullptr;
    p.y2 = nullptr;
    p.counters = nullptr;
  }
  if (threadIdx.x < 32) plan_small(p, a.n, a.n_keys);
  __syncthreads();
  const int lo = p.bank_range[0], hi = p.bank_range[1];
  for (int ri = blockIdx.x; ri < n_tokens; ri += gridDim.x)
    planes_row<1, BF16, MX>(sm, src, src_stride, K, p.inv, a.top_k, p.chunk_of, lo, hi, ri, rowmax, planes, sfb, gx);
}

int launch_plan_planes(cudaStream_t s, const PlanArgs& a, bool bf16, bool mx, const void* x, int64_t src_stride,
                       int K, int n_tokens, uint32_t* rowmax, uint8_t* planes, uint8_t* sfb, float* gx) {
  // the one-warp plan's shape (product keys, <= 32 routes, the layer's own routing) and the x planes' (bank 0)
  if (!a.key_of_expert || a.n < 1 || a.n > 32 || a.recv.flags || a.n_valid || !a.inv || !a.chunk_of ||
      !a.bank_range || a.top_k > 32 || K % 256 || n_tokens < 1)
    return -1;
  for (int b = 0; b < a.n_banks; ++b)
    if (a.max_chunks[b] < a.n) return -1;  // the private copies hold up to 32 chunks per bank
  const dim3 grid(std::min(n_tokens, 148 * 8), (K + kSlice - 1) / kSlice);
  auto kernel = bf16 ? (mx ? plan_planes_kernel<1, 1> : plan_planes_kernel<1, 0>)
                     : (mx ? plan_planes_kernel<0, 1> : plan_planes_kernel<0, 0>);
  return launch_chain(kernel, grid, dim3(kPlaneThreads), 0, s, a, static_cast<const uint16_t*>(x), src_stride, K,
                      n_tokens, rowmax, planes, sfb, gx) == cudaSuccess
             ? 0
             : -1;
}

// ------------------------------------------------------------------ gating
// One warp per token.  ids: the k largest logits, larger first, ties to the
// smaller id.  weights: exp(l - l_max) in double for the k chosen, summed in
// rank order, divided, rounded once to float.
//
// Each lane keeps the best of its own logits (ids lane + 32 j); a round takes
// the warp's largest by one integer max reduction over order-preserving keys
// of the lanes' bests, then the smallest id among the lanes holding that value
// by one min reduction, and only the winner's lane rescans its logits.  Zeros
// are keyed as +0, so -0 and +0 tie and the smaller id wins, as in a compare.
__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u >> 31) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k >> 31) ? (k & 0x7fffffffu) : ~k);
}

template <int MAXV>
__global__ void gating_kernel(const float* __restrict__ logits, int T, int E, int k, int32_t* __restrict__ ids,
                              float* __restrict__ w, uint32_t* err) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  pdl_wait();
  pdl_trigger();
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < T; t += warps) {
    const float* row = logits + int64_t(t) * E;
    float v[MAXV];
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int idx = lane + 32 * j;
      v[j] = idx < E ? __ldg(row + idx) : -INFINITY;
      if (idx < E && !isfinite(v[j])) {
        set_error(err, kErrFormat);
        v[j] = -FLT_MAX;
      }
    }
    // this lane's best: the first (smallest id) of its largest logits
    auto lane_best = [&](int& bj) {
      float b = v[0];
      bj = 0;
#pragma unroll
      for (int j = 1; j < MAXV; ++j)
        if (v[j] > b) {
          b = v[j];
          bj = j;
        }
      return b;
    };
    int bj;
    float bv = lane_best(bj);
    float my_v = 0.f;
    int my_i = 0;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      if (r >= k) break;
      const uint32_t key = order_key(bv);
      const uint32_t kmax = __reduce_max_sync(full, key);
      const uint32_t cand = key == kmax ? uint32_t(lane + 32 * bj) : 0xffffffffu;
      const uint32_t imin = __reduce_min_sync(full, cand);
      if (lane == r) {
        my_v = key_value(kmax);
        my_i = int(imin);
      }
      if (int(imin & 31u) == lane) {  // the winner leaves; only its lane looks again
        const int wj = int(imin >> 5);
#pragma unroll
        for (int j = 0; j < MAXV; ++j)
          if (j == wj) v[j] = -INFINITY;
        bv = lane_best(bj);
      }
    }
    // weights: exp(l - l_max) in double, summed in rank order, divided, rounded once
    const float vmax = __shfl_sync(full, my_v, 0);
    const double ex = lane < k ? exp(double(my_v) - double(vmax)) : 0.0;
    double total = 0.0;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      if (r >= k) break;
      total = total + __shfl_sync(full, ex, r);
    }
    if (lane < k) {
      ids[int64_t(t) * k + lane] = my_i;
      w[int64_t(t) * k + lane] = float(ex / total);
    }
  }
}

int launch_gating(cudaStream_t s, const float* logits, int T, int E, int k, int32_t* ids, float* w,
                  uint32_t* err) {
  const int threads = 256;
  int blocks = (T + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  auto kernel = E <= 128 ? gating_kernel<4> : E <= 256 ? gating_kernel<8> : E <= 512 ? gating_kernel<16>
                                                                                    : gating_kernel<32>;
  return launch_chain(kernel, dim3(blocks), dim3(threads), 0, s, logits, T, E, k, ids, w, err) == cudaSuccess ? 0
                                                                                                               : -1;
}

// ------------------------------------------------------- bf16 -> f16 copy
__global__ void convert_bf16_kernel(const uint4* __restrict__ x, int64_t n8, uint4* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    uint4 v = x[i];
    uint32_t in[4] = {v.x, v.y, v.z, v.w}, out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __uint_as_float(in[j] << 16), hi = __uint_as_float(in[j] & 0xffff0000u);
      __half2 h = __floats2half2_rn(lo, hi);
      out[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    y[i] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

int launch_convert_bf16(cudaStream_t s, const void* x, int64_t n, void* x16) {
  const int64_t n8 = n / 8;
  int blocks = int((n8 + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  return launch_chain(convert_bf16_kernel, dim3(blocks), dim3(256), 0, s, static_cast<const uint4*>(x), n8,
                      static_cast<uint4*>(x16)) == cudaSuccess
             ? 0
             : -1;
}

}  // namespace b200moe
