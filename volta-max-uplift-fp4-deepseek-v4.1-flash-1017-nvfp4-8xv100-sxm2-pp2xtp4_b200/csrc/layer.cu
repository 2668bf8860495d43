// The layer object and the C ABI of include/b200moe.h.
//
// A layer owns its expert banks (prepacked HBM layout, see layout.cuh), the
// slot maps, and a workspace sized at create for max_tokens (decode) and
// max_prefill_tokens; forward never allocates and never waits for the host.
// The forward is: [bf16 -> f16 copy] -> route plan (one CTA) -> per bank
// W13 (+ SwiGLU) -> per bank W2 (+ slot-order combine into `out`).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "layout.cuh"

using namespace b200moe;

struct b200moe_layer {
  b200moe_config cfg;
  int device = 0;
  int grid = 148;
  // banks: 0 = FP4 (NVFP4 / MXFP4), 1 = IQ codebook experts (IQ2_XXS / IQ2_XS / IQ1_M per projection)
  uint8_t* bank[2] = {nullptr, nullptr};
  BankGeom geom[2] = {};
  float* globals = nullptr;        // [n_fp4][3]
  int* span = nullptr;             // [n_fp4][3][2] MXFP4 load scratch
  int iq_fmt[2] = {2, 2};          // kernel format of the IQ bank's W13 and W2 (2 / 3 / 4)
  uint32_t* iq_tables[2] = {nullptr, nullptr};  // decode tables of those formats
  bool iq_tables_set[2] = {false, false};
  int32_t* key_of_expert = nullptr;
  bool maps_set = false, tables_set = false;  // tables_set: both projections' tables
  int ks_fixed[2] = {0, 0};  // split-K per bank set by the caller (0: chosen per launch)
  int fuse_max_routes = 0;  // decode calls of at most this many routes take the fused launches (0: off)

  // workspace
  int s_max = 0, t_max = 0;
  int32_t* perm = nullptr;
  float* w_eff = nullptr;
  Chunk* chunks[2] = {nullptr, nullptr};
  int max_chunks = 0;
  int32_t* n_chunks = nullptr;
  int32_t* ks_sel = nullptr;  // [2] split-K per bank, written by the route plan
  int32_t* bank_range = nullptr;  // [2][2] sorted positions of each bank's routes, written by the route plan
  __half* x16 = nullptr;
  uint8_t* xq = nullptr;      // IQ2 int8 activation blocks of the token rows
  uint8_t* interq = nullptr;  // IQ2 int8 activation blocks of the SwiGLU rows (by sorted position)
  __half* inter = nullptr;
  __half* y2 = nullptr;
  int32_t* counters = nullptr;
  uint32_t* err = nullptr;
  void* dbg_y13 = nullptr;
  // FP4 bank on the block-scaled tensor path (prefill_gemm = 2): natural NVFP4 codes and
  // blocked scales per projection, the activation planes, their blocked scales and factors
  uint8_t* f4_units[2] = {nullptr, nullptr};  // weight units [n][K/256 tiles of 128 rows]: W13, W2
  uint8_t* f4_planes[2] = {nullptr, nullptr}; // [plane_rows][P][K/2]
  uint8_t* f4_sfb[2] = {nullptr, nullptr};    // [f4_max_chunks][K/64][512]
  float* f4_gx[2] = {nullptr, nullptr};       // [P][plane_rows]
  int32_t* route_pos = nullptr;                // [s_max]: sorted position of each route (the plan's inverse)
  int32_t* f4_chunk_of = nullptr;              // [s_max]: (chunk << 8) | index in chunk of an FP4-bank position
  uint32_t* f4_rowmax = nullptr;               // [plane_rows]: amax bits of each SwiGLU row (W2 planes)
  int f4_plane_rows = 0, f4_max_chunks = 0;
  alignas(128) unsigned char f4_map_x[2][4][128] = {};  // [W13, W2][4, 8, 16, 32 routes per chunk]
  // prefill on tcgen05: permuted fp16 token rows and the TMA maps of the two B operands
  __half* xperm = nullptr;
  alignas(128) unsigned char map_x[128] = {};
  alignas(128) unsigned char map_inter[128] = {};
  // optional timing: events[0] at forward start, events[j + 1] after launch j
  cudaEvent_t events[16] = {};
  int n_events = 0;
};

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

template <typename T>
int dalloc(T** p, size_t count) {
  if (count == 0) {
    *p = nullptr;
    return B200MOE_OK;
  }
  if (cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return B200MOE_ERR_NOMEM;
  }
  return B200MOE_OK;
}

void free_layer(b200moe_layer* L) {
  void* ptrs[] = {L->bank[0], L->bank[1], L->globals, L->span, L->iq_tables[0], L->iq_tables[1], L->key_of_expert, L->perm,
                  L->w_eff, L->chunks[0], L->chunks[1], L->n_chunks, L->x16, L->inter, L->y2,
                  L->counters, L->err, L->xperm, L->ks_sel, L->bank_range, L->xq, L->interq,
                  L->f4_units[0], L->f4_units[1], L->f4_planes[0], L->f4_planes[1],
                  L->f4_sfb[0], L->f4_sfb[1], L->f4_gx[0], L->f4_gx[1], L->route_pos,
                  L->f4_chunk_of, L->f4_rowmax};
  for (void* p : ptrs)
    if (p) cudaFree(p);
}

bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Split-K of a bank's skinny GEMV: fixed by the caller (rc = 16 / ks), or 0 =
// chosen by the route plan on the device from this call's chunk counts with
// the model below.  ks warps share the K of a tile pair and a chunk holds
// 16 / ks routes, so a larger ks gives more chunks (each re-reads its expert's
// weights) and more, smaller items.  The constants were fitted on B200 sweeps
// (M = 1..64, one and two banks, both formats): one FP4 CTA streams about
// 18.4 GB/s (two per SM) and one IQ2 CTA about 6 GB/s (ALU-bound decode); all
// busy CTAs share about 4.8 TB/s (FP4) or 2 TB/s (IQ2); 2 us fixed per wave.
int fixed_rc(const b200moe_layer* L, int bank) {
  return L->ks_fixed[bank] ? kRouteSlotsPerChunk / L->ks_fixed[bank] : 0;
}

KsModel ks_model(const b200moe_layer* L, int bank) {
  const auto& c = L->cfg;
  const bool iq2 = bank == 1;
  const int kt = iq2 ? kIq2KTile : kFp4KTile;
  KsModel m{};
  for (int j = 0; j < 4; ++j) {
    const int ks = 1 << j;
    if ((c.hidden / kt) % ks == 0 && (c.inter / kt) % ks == 0) m.allowed |= 1 << j;
  }
  m.slots = float(L->grid * gemv_ctas_per_sm(iq2 ? 2 : c.fp4_format));
  m.bpe = iq2 ? 32.f * float(iq_block_bytes(L->iq_fmt[0])) / 256.f : (c.fp4_format == B200MOE_NVFP4 ? 18.f : 17.f);
  m.bw_cta = iq2 ? 6e9f : 18.4e9f;
  m.bw_hbm = iq2 ? 2.0e12f : 4.8e12f;
  m.per_wave = 2e-6f;
  m.tiles[0] = float(c.inter / 16);
  m.tiles[1] = float(c.hidden / 32);
  m.kdim[0] = float(c.hidden);
  m.kdim[1] = float(c.inter);
  return m;
}

// Per-call intermediates of a forward: the layer's own (allocated at create)
// or the library's static array (b200moe_forward_static).
struct Workspace {
  int32_t* perm;
  float* w_eff;
  Chunk* chunks[2];
  int max_chunks;
  int32_t* n_chunks;
  int32_t* ks_sel;
  int32_t* bank_range;
  __half* x16;
  __half* inter;
  __half* y2;
  int32_t* counters;
  uint8_t* xq;
  uint8_t* interq;
  void* dbg_y13;
  bool own = false;  // the layer's own workspace (not the static array)
};

Workspace layer_workspace(b200moe_layer* L) {
  Workspace w{};
  w.perm = L->perm;
  w.w_eff = L->w_eff;
  w.chunks[0] = L->chunks[0];
  w.chunks[1] = L->chunks[1];
  w.max_chunks = L->max_chunks;
  w.n_chunks = L->n_chunks;
  w.ks_sel = L->ks_sel;
  w.bank_range = L->bank_range;
  w.x16 = L->x16;
  w.inter = L->inter;
  w.y2 = L->y2;
  w.counters = L->counters;
  w.xq = L->xq;
  w.interq = L->interq;
  w.dbg_y13 = L->dbg_y13;
  w.own = true;
  return w;
}

// Rows mode (b200moe_forward_rows): every row is one route of a top-1 layer,
// the number of rows of this call is on the device, and the fp16 y2 rows are
// the output (no weighted combine).
struct RowsMode {
  const int32_t* n_valid;    // device: rows of this call
  const int32_t* row_range;  // device [2]: {0, rows of this call}
  __half* y2;                // fp16 [max rows][H]
};

struct Marks {
  const b200moe_layer* L;
  cudaStream_t s;
  int next = 0;
  void mark() {
    if (next < L->n_events) cudaEventRecord(L->events[next], s);
    ++next;
  }
};

int run_forward(b200moe_layer* L, const Workspace& ws_in, cudaStream_t s, const void* x, int x_dtype,
                const int32_t* ids, const float* w, float* out, int m, bool prefill = false,
                const RowsMode* rows = nullptr, const EpRecvWait* recv = nullptr,
                const EpReturn* ep_ret = nullptr) {
  const auto& c = L->cfg;
  Marks marks{L, s};
  if (!L->maps_set) return B200MOE_ERR_STATE;
  if (c.n_iq2 > 0 && !L->tables_set) return B200MOE_ERR_STATE;
  if (!x || !ids || (!rows && (!w || !out))) return B200MOE_ERR_INVALID_ARG;
  if (x_dtype != B200MOE_F16 && x_dtype != B200MOE_BF16) return B200MOE_ERR_DTYPE;
  if (!aligned(x, 16) || (out && !aligned(out, 16))) return B200MOE_ERR_ALIGN;
  Workspace ws = ws_in;
  if (rows) {
    ws.y2 = rows->y2;
    ws.counters = nullptr;
    ws.w_eff = nullptr;
    out = nullptr;
  }
  const int S = m * c.top_k;
  const __half* xsrc = static_cast<const __half*>(x);
  // the fused small-batch decode (decode.cu, off unless set: measured slower): an FP4-only layer on the
  // block-scaled path, at most fuse_max_routes routes, the layer's own routing (not expert-parallel rows),
  // no y13 capture
  const bool fused = !rows && c.prefill_gemm >= 2 && c.n_fp4 > 0 && c.n_iq2 == 0 && S <= L->fuse_max_routes &&
                     S <= kDecodeMaxRoutes && !ws.dbg_y13 && ws_in.counters && fp4_decode_fits(c.hidden) &&
                     fp4_decode_fits(c.inter);
  // bf16 x feeds the block-scaled path's planes directly; only the GEMV banks (and the tcgen05 row gather,
  // which converts itself) want it in fp16
  const bool x_bf16_direct =
      x_dtype == B200MOE_BF16 && c.prefill_gemm >= 2 && c.n_fp4 > 0 && c.n_iq2 == 0 && (ws.own || fused);
  marks.mark();
  if (x_dtype == B200MOE_BF16 && !x_bf16_direct) {
    if (launch_convert_bf16(s, x, int64_t(m) * c.hidden, ws.x16)) return B200MOE_ERR_CUDA;
    xsrc = ws.x16;
  }
  marks.mark();  // after the bf16 conversion (or none): the event layout does not depend on x's dtype
  if (fused) {
    DecArgs d{};
    d.n_slots = c.n_fp4;
    d.ids = ids;
    d.w_in = w;
    d.S = S;
    d.top_k = c.top_k;
    d.num_experts = c.num_experts;
    d.key_of_expert = L->key_of_expert;
    d.n_keys = c.n_fp4 + c.n_iq2;
    d.globals = c.fp4_format == B200MOE_NVFP4 ? L->globals : nullptr;
    d.H = c.hidden;
    d.err = L->err;
    const bool mx = c.fp4_format == B200MOE_MXFP4;
    // W13 (+ SwiGLU): the token rows of x planed in each CTA
    d.wt = L->f4_units[0];
    d.K = c.hidden;
    d.n_rt = c.inter / 128;
    d.src = x_bf16_direct ? x : static_cast<const void*>(xsrc);
    d.src_stride = c.hidden;
    d.inter = ws.inter;
    d.inter_stride = c.inter;
    d.limit = c.swiglu_limit;
    d.perm_out = ws.perm;
    if (launch_fp4_decode(s, 0, mx, x_bf16_direct, d, L->grid)) return B200MOE_ERR_CUDA;
    marks.mark();
    // W2 (+ combine): the SwiGLU rows planed in each CTA, the token rows summed by the CTA that completes them
    d.wt = L->f4_units[1];
    d.K = c.inter;
    d.n_rt = c.hidden / 256;
    d.src = ws.inter;
    d.src_stride = c.inter;
    d.y2 = ws.y2;
    d.counters = ws_in.counters;
    d.out = out;
    d.perm_out = nullptr;
    if (launch_fp4_decode(s, 1, mx, false, d, L->grid)) return B200MOE_ERR_CUDA;
    marks.mark();
    return B200MOE_OK;
  }
  // int8 blocks of the token rows for the IQ2 bank's W13 (in rows mode after the plan, which may be the
  // launch that learns how many rows this call has)
  auto quant_rows = [&]() {
    if (launch_quant_s8(s, xsrc, c.hidden, c.hidden, m, rows ? rows->row_range : nullptr, ws.xq)) return false;
    marks.mark();
    return true;
  };
  if (c.n_iq2 > 0 && !rows && !quant_rows()) return B200MOE_ERR_CUDA;
  // prefill with the tcgen05 GEMM: the FP4 bank's chunks are 128-route token tiles
  // (NVFP4 weight units of the block-scaled layout feed the tcgen05 GEMM too: long prefills run there)
  // prefill_gemm 2: prefills of >= kTcUnitsMinRoutes on the f16 GEMM over the weight units (measured faster
  // than the block-scaled kernel with 32-route chunks: c3 T = 4,096 W13 1.84 against 2.47 ms); 3: every call
  // on the block-scaled kernel
  const bool tc_units = c.prefill_gemm == 2 && S >= kTcUnitsMinRoutes;
  const bool tc = !rows && prefill && (c.prefill_gemm == 1 || tc_units) && c.n_fp4 > 0 && L->xperm;
  const bool f4 = c.prefill_gemm >= 2 && c.n_fp4 > 0 && !tc;
  // the block-scaled path's plane buffers are the layer's own (sized at create), also under the static array
  if (f4 && S > L->s_max) return B200MOE_ERR_RANGE;
  // W2 writes y2 rows only and one launch after it does the slot-order combine: fused into the W2
  // epilogue the combine's fences, atomics and re-reads stall the pipeline (measured on B200: the
  // decode GEMV at M = 64 0.849 against 0.877 ms, the tcgen05 prefill W2 1.10 against 2.12 ms).
  // Small decode calls keep the fused form, where it saves a launch: the block-scaled W2 up to
  // kFusedCombineRoutes routes, the GEMV up to 32 (and in the allocation-free decode); a layer with
  // both banks fuses in both W2 launches or in neither (they share the completion counts).
  const bool sep_combine = !rows && (tc || (f4 && S > kFusedCombineRoutes) || (!f4 && ws.own && S > 32));
  if (sep_combine) ws.counters = nullptr;
  PlanArgs p{};
  p.ids = ids;
  p.n = S;
  p.n_valid = rows ? rows->n_valid : nullptr;
  if (recv) p.recv = *recv;
  p.num_experts = c.num_experts;
  p.key_of_expert = L->key_of_expert;
  p.n_keys = c.n_fp4 + c.n_iq2;
  p.perm = ws.perm;
  p.inv = (f4 || sep_combine) ? L->route_pos : nullptr;
  p.chunk_of = f4 ? L->f4_chunk_of : nullptr;
  p.n_banks = 2;
  p.key_lo[0] = 0;
  p.key_hi[0] = c.n_fp4;
  p.key_lo[1] = c.n_fp4;
  p.key_hi[1] = c.n_fp4 + c.n_iq2;
  for (int b = 0; b < 2; ++b) {
    p.rc[b] = (tc && b == 0) ? kTcTokenTile : (f4 && b == 0) ? fp4_routes_per_chunk(S) : fixed_rc(L, b);
    p.ks_model[b] = ks_model(L, b);
    p.max_chunks[b] = (f4 && b == 0) ? std::min(ws.max_chunks, L->f4_max_chunks) : ws.max_chunks;
    p.chunks[b] = ws.chunks[b];
  }
  p.n_chunks = ws.n_chunks;
  p.w_in = w;
  p.w_eff = ws.w_eff;
  p.y2 = ws.y2;
  p.counters = ws.counters;
  p.out = out;
  p.H = c.hidden;
  p.top_k = c.top_k;
  p.ks_sel = ws.ks_sel;
  p.bank_range = ws.bank_range;
  p.err = L->err;
  // decode of <= 32 routes on the block-scaled path: the plan and the token rows' planes are one launch
  const bool plan_with_planes = f4 && !rows && !recv && S <= 32;
  if (plan_with_planes) {
    if (launch_plan_planes(s, p, x_bf16_direct, c.fp4_format == B200MOE_MXFP4,
                           x_bf16_direct ? x : static_cast<const void*>(xsrc), c.hidden, c.hidden, m, L->f4_rowmax,
                           L->f4_planes[0], L->f4_sfb[0], L->f4_gx[0]))
      return B200MOE_ERR_CUDA;
  } else if (launch_plan(s, p)) {
    return B200MOE_ERR_CUDA;
  }
  marks.mark();
  if (c.n_iq2 > 0 && rows && !quant_rows()) return B200MOE_ERR_CUDA;
  if (tc) {
    if (launch_gather_rows(s, x, x_dtype == B200MOE_BF16, ws.perm, S, c.top_k, c.hidden, L->xperm))
      return B200MOE_ERR_CUDA;
    marks.mark();
  }
  for (int epi = 0; epi < 2; ++epi) {
    if (f4 && epi == 0 && plan_with_planes) marks.mark();  // made with the plan: an empty interval
    if (f4 && !(epi == 0 && plan_with_planes)) {  // the FP4 bank's activation rows as E2M1 planes
      if (launch_fp4_planes(s, epi == 0, epi == 0 && x_bf16_direct, c.fp4_format == B200MOE_MXFP4,
                            epi == 0 ? (x_bf16_direct ? x : static_cast<const void*>(xsrc)) : ws.inter,
                            epi == 0 ? c.hidden : c.inter,
                            epi == 0 ? c.hidden : c.inter, L->route_pos, c.top_k, L->f4_chunk_of, 0,
                            ws.bank_range, epi == 0 ? m : S, L->f4_rowmax, L->f4_planes[epi], L->f4_plane_rows,
                            L->f4_sfb[epi], L->f4_gx[epi]))
        return B200MOE_ERR_CUDA;
      marks.mark();
    }
    if (epi == 1 && c.n_iq2 > 0) {  // int8 blocks of the IQ2 routes' SwiGLU rows for the IQ2 bank's W2
      if (launch_quant_s8(s, ws.inter, c.inter, c.inter, S, ws.bank_range + 2, ws.interq)) return B200MOE_ERR_CUDA;
      marks.mark();
    }
    for (int b = 0; b < 2; ++b) {
      const int n_slots = b == 0 ? c.n_fp4 : c.n_iq2;
      if (n_slots == 0) continue;
      if (f4 && b == 0) {
        Fp4Args f{};
        f.wt = L->f4_units[epi];
        f.globals = c.fp4_format == B200MOE_NVFP4 ? L->globals : nullptr;  // MXFP4 has no FP32 global scale
        f.K = epi == 0 ? c.hidden : c.inter;
        f.n_rt = epi == 0 ? c.inter / 128 : c.hidden / 256;  // items of two 128-row tiles
        f.sfb = L->f4_sfb[epi];
        f.gx = L->f4_gx[epi];
        f.rowmax = L->f4_rowmax;
        f.plane_rows = L->f4_plane_rows;
        f.chunks = ws.chunks[0];
        f.n_chunks = ws.n_chunks;
        f.bank = 0;
        f.n_slots = n_slots;
        f.perm = ws.perm;
        f.S = S;
        f.top_k = c.top_k;
        f.inter = ws.inter;
        f.inter_stride = c.inter;
        f.limit = c.swiglu_limit;
        f.w_eff = ws.w_eff;
        f.y2 = ws.y2;
        f.counters = ws.counters;
        f.out = out;
        f.H = c.hidden;
        f.err = L->err;
        if (epi == 1 && ep_ret) f.ep = *ep_ret;  // y2 rows straight to their home ranks
        const int rc = fp4_routes_per_chunk(S);
        if (launch_fp4_gemm(s, epi, rc, c.fp4_format == B200MOE_MXFP4, f, L->f4_map_x[epi][fp4_rc_index(rc)],
                            L->grid))
          return B200MOE_ERR_CUDA;
        marks.mark();
        continue;
      }
      if (tc && b == 0) {
        TcArgs t{};
        if (c.prefill_gemm >= 2) {  // weight units: [slot][rt][kt] of 36 KB
          t.region = L->f4_units[epi];
          t.slot_stride = epi == 0 ? int64_t(2) * c.inter * (c.hidden / 2 + c.hidden / 16)
                                   : int64_t(c.hidden) * (c.inter / 2 + c.inter / 16);
        } else {
          t.region = L->bank[0] + (epi == 0 ? 0 : L->geom[0].w13_bytes);
          t.slot_stride = L->geom[0].slot_bytes;
        }
        t.n_slots = n_slots;
        t.globals = L->globals;
        t.K = epi == 0 ? c.hidden : c.inter;
        t.n_rt = epi == 0 ? c.inter / 128 : c.hidden / 256;
        t.chunks = ws.chunks[0];
        t.n_chunks = ws.n_chunks;
        t.bank = 0;
        t.perm = ws.perm;
        t.S = S;
        t.top_k = c.top_k;
        t.inter = ws.inter;
        t.inter_stride = c.inter;
        t.limit = c.swiglu_limit;
        t.y2 = ws.y2;
        t.H = c.hidden;
        t.err = L->err;
        const int tfmt = c.prefill_gemm >= 2 ? (c.fp4_format == B200MOE_NVFP4 ? 2 : 3) : c.fp4_format;
        if (launch_tc_gemm(s, tfmt, epi, t, epi == 0 ? L->map_x : L->map_inter, L->grid))
          return B200MOE_ERR_CUDA;
        marks.mark();
        continue;
      }
      GemvArgs g{};
      g.fmt = b == 0 ? c.fp4_format : L->iq_fmt[epi];
      g.epi = epi;
      g.ks_sel = ws.ks_sel;
      g.region = L->bank[b] + (epi == 0 ? 0 : L->geom[b].w13_bytes);
      g.slot_stride = L->geom[b].slot_bytes;
      g.n_slots = n_slots;
      g.globals = b == 0 ? L->globals : nullptr;
      g.K = epi == 0 ? c.hidden : c.inter;
      g.n_tp = epi == 0 ? c.inter / 16 : c.hidden / 32;
      g.chunks = ws.chunks[b];
      g.n_chunks = ws.n_chunks;
      g.bank = b;
      g.perm = ws.perm;
      g.S = S;
      g.top_k = c.top_k;
      if (b == 0) g.xsrc = epi == 0 ? static_cast<const void*>(xsrc) : static_cast<const void*>(ws.inter);
      else g.xsrc = epi == 0 ? static_cast<const void*>(ws.xq) : static_cast<const void*>(ws.interq);
      g.x_by_token = epi == 0;
      g.x_row_stride = epi == 0 ? c.hidden : c.inter;
      g.n_x_rows = epi == 0 ? m : S;
      g.inter = ws.inter;
      g.inter_stride = c.inter;
      g.dbg_y13 = ws.dbg_y13;
      g.limit = c.swiglu_limit;
      g.w_eff = ws.w_eff;
      g.y2 = ws.y2;
      g.counters = ws.counters;
      g.out = out;
      g.H = c.hidden;
      g.iq2_tables = b == 1 ? L->iq_tables[epi] : nullptr;
      g.err = L->err;
      g.grid = L->grid * gemv_ctas_per_sm(g.fmt);
      if (launch_gemv(s, g)) return B200MOE_ERR_CUDA;
      marks.mark();
    }
  }
  if (sep_combine) {
    if (launch_route_combine(s, static_cast<const __half*>(ws.y2), L->route_pos, ws.bank_range, 2, ws.w_eff, m,
                             c.top_k, c.hidden, out))
      return B200MOE_ERR_CUDA;
    marks.mark();
  }
  return B200MOE_OK;
}

}  // namespace

extern "C" {

const char* b200moe_status_name(int status) {
  switch (status) {
    case B200MOE_OK: return "B200MOE_OK";
    case B200MOE_ERR_INVALID_ARG: return "B200MOE_ERR_INVALID_ARG";
    case B200MOE_ERR_DTYPE: return "B200MOE_ERR_DTYPE";
    case B200MOE_ERR_ALIGN: return "B200MOE_ERR_ALIGN";
    case B200MOE_ERR_CUDA: return "B200MOE_ERR_CUDA";
    case B200MOE_ERR_BOUNDS: return "B200MOE_ERR_BOUNDS";
    case B200MOE_ERR_TIMEOUT: return "B200MOE_ERR_TIMEOUT";
    case B200MOE_ERR_FORMAT: return "B200MOE_ERR_FORMAT";
    case B200MOE_ERR_RANGE: return "B200MOE_ERR_RANGE";
    case B200MOE_ERR_NOMEM: return "B200MOE_ERR_NOMEM";
    case B200MOE_ERR_STATE: return "B200MOE_ERR_STATE";
    default: return "B200MOE_ERR_UNKNOWN";
  }
}

const char* b200moe_version(void) { return "b200moe 0.1 sm_100a"; }

}  // extern "C"

// Device address of the allocation-free decode's scratch array (defined with
// b200moe_forward_static below); layer creation looks it up on its device.
int static_scratch(int device, uint8_t** out);

extern "C" {

int b200moe_layer_create(const b200moe_config* cfg, int device, b200moe_layer** out) {
  if (!cfg || !out) return B200MOE_ERR_INVALID_ARG;
  *out = nullptr;
  const b200moe_config c = *cfg;
  if (c.hidden < 256 || c.hidden % 256 || c.inter < 128 || c.inter % 128 || c.num_experts < 1 ||
      c.num_experts > 1024 || c.top_k < 1 || c.top_k > 16 || c.top_k > c.num_experts || c.max_tokens < 1 ||
      c.max_tokens > 64 || c.max_prefill_tokens < 0 || c.n_fp4 < 0 || c.n_iq2 < 0 ||
      c.n_fp4 + c.n_iq2 < 1 || c.n_fp4 + c.n_iq2 > c.num_experts || !(c.swiglu_limit > 0.f))
    return B200MOE_ERR_INVALID_ARG;
  if (c.fp4_format != B200MOE_NVFP4 && c.fp4_format != B200MOE_MXFP4) return B200MOE_ERR_INVALID_ARG;
  if (c.n_iq2 > 0 && c.inter % 256) return B200MOE_ERR_INVALID_ARG;
  for (int t : {c.iq_type13, c.iq_type2})
    if (t != 0 && iq_fmt_of_type(t) < 0) return B200MOE_ERR_INVALID_ARG;
  if (c.prefill_gemm < 0 || c.prefill_gemm > 3) return B200MOE_ERR_INVALID_ARG;
  // the block-scaled FP4 path: NVFP4 (E4M3 scales per 16), K tiles of 256 on both projections
  if (c.prefill_gemm >= 2 && (c.hidden % 256 || c.inter % 256))
    return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(device);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return B200MOE_ERR_CUDA;
  if (prop.major != 10) return B200MOE_ERR_CUDA;  // built for sm_100a only
  auto* L = new b200moe_layer();
  L->cfg = c;
  L->device = device;
  L->grid = prop.multiProcessorCount;
  L->geom[0] = fp4_geom(c.fp4_format, c.hidden, c.inter);
  L->iq_fmt[0] = iq_fmt_of_type(c.iq_type13 ? c.iq_type13 : kGgmlIq2xxs);
  L->iq_fmt[1] = iq_fmt_of_type(c.iq_type2 ? c.iq_type2 : kGgmlIq2xxs);
  L->geom[1] = iq_geom(L->iq_fmt[0], L->iq_fmt[1], c.hidden, c.inter);
  L->t_max = std::max(c.max_tokens, c.max_prefill_tokens);
  L->s_max = L->t_max * c.top_k;
  L->max_chunks = L->s_max + c.num_experts;
  int st = B200MOE_OK;
  auto take = [&](int r) {
    if (st == B200MOE_OK) st = r;
  };
  const bool f4 = c.prefill_gemm >= 2;
  take(dalloc(&L->bank[0], f4 ? size_t(0) : size_t(c.n_fp4) * L->geom[0].slot_bytes));
  if (f4 && c.n_fp4 > 0) {
    const size_t H = c.hidden, I = c.inter, n = c.n_fp4;
    take(dalloc(&L->f4_units[0], n * 2 * I * (H / 2 + H / 16)));
    take(dalloc(&L->f4_units[1], n * H * (I / 2 + I / 16)));
  }
  take(dalloc(&L->bank[1], size_t(c.n_iq2) * L->geom[1].slot_bytes));
  take(dalloc(&L->globals, size_t(std::max(c.n_fp4, 1)) * 3));
  take(dalloc(&L->span, size_t(std::max(c.n_fp4, 1)) * 6));
  take(dalloc(&L->iq_tables[0], size_t(iq_table_words(L->iq_fmt[0]))));
  take(dalloc(&L->iq_tables[1], size_t(iq_table_words(L->iq_fmt[1]))));
  take(dalloc(&L->key_of_expert, size_t(c.num_experts)));
  take(dalloc(&L->perm, size_t(L->s_max)));
  take(dalloc(&L->route_pos, size_t(L->s_max)));
  take(dalloc(&L->w_eff, size_t(L->s_max)));
  take(dalloc(&L->chunks[0], size_t(L->max_chunks)));
  take(dalloc(&L->chunks[1], size_t(L->max_chunks)));
  take(dalloc(&L->n_chunks, 2));
  take(dalloc(&L->x16, size_t(L->t_max) * c.hidden));
  take(dalloc(&L->inter, size_t(L->s_max) * c.inter));
  take(dalloc(&L->y2, size_t(L->s_max) * c.hidden));
  take(dalloc(&L->counters, size_t(L->t_max) * (c.hidden / 32)));
  take(dalloc(&L->err, 1));
  take(dalloc(&L->ks_sel, 2));
  take(dalloc(&L->bank_range, 4));
  if (c.n_iq2 > 0) {
    take(dalloc(&L->xq, size_t(L->t_max) * (c.hidden / kIq2KTile) * kIq2XBlockBytes));
    take(dalloc(&L->interq, size_t(L->s_max) * (c.inter / kIq2KTile) * kIq2XBlockBytes));
  }
  if (f4 && c.n_fp4 > 0) {
    L->f4_plane_rows = L->s_max + kFp4TcRoutes;
    // chunks of <= 4, 8 or 16 routes (calls of <= 64, <= 1024 or more routes)
    L->f4_max_chunks = std::max(std::max(64 / 4, 1024 / 8), (L->s_max + 15) / 16) + c.n_fp4;
    const size_t P = kFp4Planes, R = L->f4_plane_rows, H = c.hidden, I = c.inter;
    take(dalloc(&L->f4_planes[0], P * R * H / 2));
    take(dalloc(&L->f4_planes[1], P * R * I / 2));
    take(dalloc(&L->f4_sfb[0], size_t(L->f4_max_chunks) * (H / 64) * 512));
    take(dalloc(&L->f4_sfb[1], size_t(L->f4_max_chunks) * (I / 64) * 512));
    take(dalloc(&L->f4_gx[0], R));
    take(dalloc(&L->f4_gx[1], R));
    take(dalloc(&L->f4_chunk_of, size_t(L->s_max)));
    take(dalloc(&L->f4_rowmax, R));
    if (st == B200MOE_OK &&
        (make_u8_tile_map(L->f4_map_x[0][0], L->f4_planes[0], int64_t(P * R), H / 2, 128, 4 * kFp4Planes) ||
         make_u8_tile_map(L->f4_map_x[0][1], L->f4_planes[0], int64_t(P * R), H / 2, 128, 8 * kFp4Planes) ||
         make_u8_tile_map(L->f4_map_x[0][2], L->f4_planes[0], int64_t(P * R), H / 2, 128, 16 * kFp4Planes) ||
         make_u8_tile_map(L->f4_map_x[0][3], L->f4_planes[0], int64_t(P * R), H / 2, 128, 32 * kFp4Planes) ||
         make_u8_tile_map(L->f4_map_x[1][0], L->f4_planes[1], int64_t(P * R), I / 2, 128, 4 * kFp4Planes) ||
         make_u8_tile_map(L->f4_map_x[1][1], L->f4_planes[1], int64_t(P * R), I / 2, 128, 8 * kFp4Planes) ||
         make_u8_tile_map(L->f4_map_x[1][2], L->f4_planes[1], int64_t(P * R), I / 2, 128, 16 * kFp4Planes) ||
         make_u8_tile_map(L->f4_map_x[1][3], L->f4_planes[1], int64_t(P * R), I / 2, 128, 32 * kFp4Planes)))
      st = B200MOE_ERR_CUDA;
  }
  if (c.prefill_gemm >= 1 && c.max_prefill_tokens > 0 && c.n_fp4 > 0) {
    take(dalloc(&L->xperm, size_t(L->s_max) * c.hidden));
    if (st == B200MOE_OK && (make_token_map(L->map_x, L->xperm, L->s_max, c.hidden) ||
                             make_token_map(L->map_inter, L->inter, L->s_max, c.inter)))
      st = B200MOE_ERR_CUDA;
  }
  if (st == B200MOE_OK) {
    if (cudaMemset(L->counters, 0, size_t(L->t_max) * (c.hidden / 32) * 4) != cudaSuccess ||
        cudaMemset(L->err, 0, 4) != cudaSuccess || cudaMemset(L->n_chunks, 0, 8) != cudaSuccess ||
        cudaMemset(L->inter, 0, size_t(L->s_max) * c.inter * 2) != cudaSuccess ||
        cudaMemset(L->globals, 0, size_t(std::max(c.n_fp4, 1)) * 12) != cudaSuccess ||
        (L->f4_sfb[0] && cudaMemset(L->f4_sfb[0], 0, size_t(L->f4_max_chunks) * (c.hidden / 64) * 512) != cudaSuccess) ||
        (L->f4_sfb[1] && cudaMemset(L->f4_sfb[1], 0, size_t(L->f4_max_chunks) * (c.inter / 64) * 512) != cudaSuccess) ||
        cudaDeviceSynchronize() != cudaSuccess)
      st = B200MOE_ERR_CUDA;
  }
  if (st == B200MOE_OK) {
    // Look up the allocation-free decode's scratch address on this device now,
    // outside any stream capture (the lookup may load the module), so that the
    // first b200moe_forward_static call does no set-up of its own.
    uint8_t* scratch = nullptr;
    st = static_scratch(device, &scratch);
  }
  if (st != B200MOE_OK) {
    free_layer(L);
    delete L;
    return st;
  }
  *out = L;
  return B200MOE_OK;
}

int b200moe_layer_destroy(b200moe_layer* L) {
  if (!L) return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(L->device);
  cudaDeviceSynchronize();
  free_layer(L);
  delete L;
  return B200MOE_OK;
}

int b200moe_set_slot_maps(b200moe_layer* L, const int32_t* fp4_slot, const int32_t* iq2_slot) {
  if (!L || !fp4_slot) return B200MOE_ERR_INVALID_ARG;
  const auto& c = L->cfg;
  std::vector<int32_t> key(c.num_experts, -1);
  std::vector<int> seen0(c.n_fp4, 0), seen1(c.n_iq2, 0);
  for (int e = 0; e < c.num_experts; ++e) {
    const int a = fp4_slot[e], b = iq2_slot ? iq2_slot[e] : -1;
    if (a >= c.n_fp4 || b >= c.n_iq2 || a < -1 || b < -1) return B200MOE_ERR_INVALID_ARG;
    if (a >= 0 && b >= 0) return B200MOE_ERR_INVALID_ARG;  // one bank per expert
    if (a >= 0) {
      if (seen0[a]++) return B200MOE_ERR_INVALID_ARG;
      key[e] = a;
    } else if (b >= 0) {
      if (seen1[b]++) return B200MOE_ERR_INVALID_ARG;
      key[e] = c.n_fp4 + b;
    }
  }
  for (int v : seen0)
    if (v != 1) return B200MOE_ERR_INVALID_ARG;
  for (int v : seen1)
    if (v != 1) return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(L->device);
  if (cudaMemcpy(L->key_of_expert, key.data(), key.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return B200MOE_ERR_CUDA;
  L->maps_set = true;
  return B200MOE_OK;
}

// Decode tables of one IQ format (layout.cuh): per grid entry its 8 values as
// nibble codes (IQ2: magnitudes 8, 25, 43 -> 0, 1, 2; IQ1_M: -1, 0, 1 -> 0, 1, 2),
// then for the IQ2 formats per 7-bit sign index its 8 signs in bit 2 of each
// nibble.  Written to the projections whose format it is.
static int set_iq_tables(b200moe_layer* L, int fmt, const int8_t* grid, int n_entries, const uint8_t* ksigns) {
  const int want = fmt == 2 ? 256 : fmt == 3 ? 512 : 2048;
  if (!L || !grid || n_entries != want || (fmt != 4 && !ksigns)) return B200MOE_ERR_INVALID_ARG;
  if (L->iq_fmt[0] != fmt && L->iq_fmt[1] != fmt) return B200MOE_ERR_INVALID_ARG;
  std::vector<uint32_t> t(iq_table_words(fmt), 0u);
  for (int e = 0; e < n_entries; ++e)
    for (int j = 0; j < 8; ++j) {
      const int8_t g = grid[e * 8 + j];
      const int code = fmt == 4 ? (g == -1 ? 0 : g == 0 ? 1 : g == 1 ? 2 : -1)
                                : (g == 8 ? 0 : g == 25 ? 1 : g == 43 ? 2 : -1);
      if (code < 0) return B200MOE_ERR_INVALID_ARG;
      t[e] |= uint32_t(code) << (4 * j);
    }
  if (fmt != 4)
    for (int si = 0; si < 128; ++si)
      for (int j = 0; j < 8; ++j) t[n_entries + si] |= ((uint32_t(ksigns[si]) >> j) & 1u) << (4 * j + 2);
  if (fmt != 2) {  // the upper-half copy (layout.cuh)
    const int half = fmt == 3 ? kIq2xsGridWords : kIq1mHalfWords;  // grid words only
    const int upper = fmt == 3 ? kIq2xsUpper : kIq1mUpper;
    for (int i = 0; i < half; ++i) t[upper + i] = t[i] >> 16;
  }
  DeviceGuard guard(L->device);
  for (int p = 0; p < 2; ++p)
    if (L->iq_fmt[p] == fmt) {
      if (cudaMemcpy(L->iq_tables[p], t.data(), t.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return B200MOE_ERR_CUDA;
      L->iq_tables_set[p] = true;
    }
  L->tables_set = L->iq_tables_set[0] && L->iq_tables_set[1];
  return B200MOE_OK;
}

int b200moe_set_iq2_tables(b200moe_layer* L, const int8_t* grid, const uint8_t* ksigns) {
  return set_iq_tables(L, 2, grid, 256, ksigns);
}

int b200moe_set_iq_grid(b200moe_layer* L, int ggml_type, const int8_t* grid, int n_entries, const uint8_t* ksigns) {
  const int fmt = iq_fmt_of_type(ggml_type);
  if (fmt < 0) return B200MOE_ERR_INVALID_ARG;
  return set_iq_tables(L, fmt, grid, n_entries, ksigns);
}

int b200moe_load_fp4(b200moe_layer* L, void* stream, int slot_begin, int n, const uint8_t* w13c,
                     const uint8_t* w13s, const uint8_t* w2c, const uint8_t* w2s, const float* globals) {
  if (!L || !w13c || !w13s || !w2c || !w2s || n < 1 || slot_begin < 0 || slot_begin + n > L->cfg.n_fp4)
    return B200MOE_ERR_INVALID_ARG;
  const auto& c = L->cfg;
  if (c.fp4_format == B200MOE_NVFP4 && !globals) return B200MOE_ERR_INVALID_ARG;
  if (!aligned(w13c, 16) || !aligned(w2c, 16) || !aligned(w13s, 4) || !aligned(w2s, 4)) return B200MOE_ERR_ALIGN;
  DeviceGuard guard(L->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* gdst = L->globals + size_t(slot_begin) * 3;
  if (c.fp4_format == B200MOE_NVFP4 &&
      cudaMemcpyAsync(gdst, globals, size_t(n) * 12, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return B200MOE_ERR_CUDA;
  if (c.prefill_gemm >= 2) {  // weight units for the block-scaled tensor path (and the tcgen05 prefill)
    const size_t H = c.hidden, I = c.inter, b = size_t(slot_begin);
    const bool mx = c.fp4_format == B200MOE_MXFP4;
    if (mx && launch_mx_rebase(s, c.hidden, c.inter, n, w13c, w13s, w2c, w2s, gdst, L->span, L->err))
      return B200MOE_ERR_CUDA;
    const float* g = mx ? gdst : nullptr;
    if (launch_fp4_tile(s, mx, w13c, w13s, n, int(2 * I), int(H), true, g, L->err,
                        L->f4_units[0] + b * 2 * I * (H / 2 + H / 16)) ||
        launch_fp4_tile(s, mx, w2c, w2s, n, int(H), int(I), false, g, L->err,
                        L->f4_units[1] + b * H * (I / 2 + I / 16)))
      return B200MOE_ERR_CUDA;
    return B200MOE_OK;
  }
  uint8_t* dst = L->bank[0] + size_t(slot_begin) * L->geom[0].slot_bytes;
  if (launch_fp4_prepack(s, c.fp4_format, c.hidden, c.inter, n, w13c, w13s, w2c, w2s, gdst, L->span, dst,
                         L->geom[0].slot_bytes, L->geom[0].w13_bytes, L->err))
    return B200MOE_ERR_CUDA;
  return B200MOE_OK;
}

int b200moe_load_iq2(b200moe_layer* L, void* stream, int slot_begin, int n, const uint8_t* w1,
                     const uint8_t* w3, const uint8_t* w2) {
  if (!L || !w1 || !w3 || !w2 || n < 1 || slot_begin < 0 || slot_begin + n > L->cfg.n_iq2)
    return B200MOE_ERR_INVALID_ARG;
  const auto& c = L->cfg;
  DeviceGuard guard(L->device);
  uint8_t* dst = L->bank[1] + size_t(slot_begin) * L->geom[1].slot_bytes;
  if (launch_iq2_prepack(static_cast<cudaStream_t>(stream), L->iq_fmt[0], L->iq_fmt[1], c.hidden, c.inter, n, w1,
                         w3, w2, dst, L->geom[1].slot_bytes, L->geom[1].w13_bytes))
    return B200MOE_ERR_CUDA;
  return B200MOE_OK;
}

int b200moe_route(b200moe_layer* L, void* stream, const float* logits, int32_t* ids, float* w, int T) {
  if (!L || !logits || !ids || !w || T < 1) return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(L->device);
  if (launch_gating(static_cast<cudaStream_t>(stream), logits, T, L->cfg.num_experts, L->cfg.top_k, ids, w, L->err))
    return B200MOE_ERR_CUDA;
  return B200MOE_OK;
}

int b200moe_forward(b200moe_layer* L, void* stream, const void* x, int x_dtype, const int32_t* ids,
                    const float* w, float* out, int M) {
  if (!L || M < 1 || M > L->cfg.max_tokens) return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(L->device);
  return run_forward(L, layer_workspace(L), static_cast<cudaStream_t>(stream), x, x_dtype, ids, w, out, M);
}

int b200moe_forward_prefill(b200moe_layer* L, void* stream, const void* x, int x_dtype, const int32_t* ids,
                            const float* w, float* out, int T) {
  if (!L || T < 1 || T > L->t_max) return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(L->device);
  return run_forward(L, layer_workspace(L), static_cast<cudaStream_t>(stream), x, x_dtype, ids, w, out, T, true);
}

int b200moe_forward_rows(b200moe_layer* L, void* stream, const void* rows, const int32_t* expert_ids,
                         const int32_t* n_valid, const int32_t* row_range, int max_rows, void* y2) {
  if (!L || !rows || !expert_ids || !n_valid || !row_range || !y2 || max_rows < 1 || max_rows > L->t_max)
    return B200MOE_ERR_INVALID_ARG;
  if (L->cfg.top_k != 1) return B200MOE_ERR_INVALID_ARG;
  if (!aligned(y2, 16)) return B200MOE_ERR_ALIGN;
  DeviceGuard guard(L->device);
  RowsMode rm{n_valid, row_range, static_cast<__half*>(y2)};
  return run_forward(L, layer_workspace(L), static_cast<cudaStream_t>(stream), rows, B200MOE_F16, expert_ids,
                     nullptr, nullptr, max_rows, true, &rm);
}

int b200moe_ep_forward(b200moe_ep* ep, b200moe_layer* L, void* stream, int fuse_return) {
  if (!ep || !L) return B200MOE_ERR_INVALID_ARG;
  EpRecvWait w{};
  if (int st = ep_recv_wait(ep, &w)) return st;
  if (w.device != L->device || L->cfg.top_k != 1 || w.max_rows > L->t_max) return B200MOE_ERR_INVALID_ARG;
  EpReturn r{};
  if (fuse_return) {  // only a block-scaled FP4-only layer writes every y2 row in one epilogue
    if (L->cfg.prefill_gemm < 2 || L->cfg.n_iq2 > 0 || L->cfg.n_fp4 < 1) return B200MOE_ERR_INVALID_ARG;
    if (int st = ep_return_targets(ep, &r)) return st;
  }
  DeviceGuard guard(L->device);
  RowsMode rm{w.out, w.out + 1, static_cast<__half*>(w.y2)};
  return run_forward(L, layer_workspace(L), static_cast<cudaStream_t>(stream), w.rows, B200MOE_F16, w.expert_ids,
                     nullptr, nullptr, w.max_rows, true, &rm, &w, fuse_return ? &r : nullptr);
}

int b200moe_check_errors(b200moe_layer* L, void* stream, uint32_t* bits) {
  if (!L) return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(L->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return B200MOE_ERR_CUDA;
  uint32_t e = 0;
  if (cudaMemcpy(&e, L->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return B200MOE_ERR_CUDA;
  if (cudaMemset(L->err, 0, 4) != cudaSuccess) return B200MOE_ERR_CUDA;
  if (bits) *bits = e;
  // after an error the combine counters may hold partial counts: start clean
  if (e && cudaMemset(L->counters, 0, size_t(L->t_max) * (L->cfg.hidden / 32) * 4) != cudaSuccess)
    return B200MOE_ERR_CUDA;
  if (e & kErrBounds) return B200MOE_ERR_BOUNDS;
  if (e & kErrTimeout) return B200MOE_ERR_TIMEOUT;
  if (e & kErrFormat) return B200MOE_ERR_FORMAT;
  if (e & kErrRange) return B200MOE_ERR_RANGE;
  return B200MOE_OK;
}

int b200moe_set_debug_y13(b200moe_layer* L, void* y13) {
  if (!L) return B200MOE_ERR_INVALID_ARG;
  L->dbg_y13 = y13;
  return B200MOE_OK;
}

int b200moe_debug_perm(const b200moe_layer* L, void* stream, int32_t* dst, int n) {
  if (!L || !dst || n < 1 || n > L->s_max) return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(L->device);
  if (cudaMemcpyAsync(dst, L->perm, size_t(n) * 4, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return B200MOE_ERR_CUDA;
  return B200MOE_OK;
}

int b200moe_set_timing_events(b200moe_layer* L, void* const* events, int n) {
  if (!L || n < 0 || n > 16 || (n > 0 && !events)) return B200MOE_ERR_INVALID_ARG;
  for (int i = 0; i < n; ++i) L->events[i] = static_cast<cudaEvent_t>(events[i]);
  L->n_events = n;
  return B200MOE_OK;
}

int b200moe_set_decode_fusion(b200moe_layer* L, int max_routes) {
  if (!L || max_routes < 0) return B200MOE_ERR_INVALID_ARG;
  L->fuse_max_routes = std::min(max_routes, kDecodeMaxRoutes);
  return B200MOE_OK;
}

int b200moe_set_split_k(b200moe_layer* L, int ks_fp4, int ks_iq2) {
  if (!L) return B200MOE_ERR_INVALID_ARG;
  const auto& c = L->cfg;
  const int ks[2] = {ks_fp4, ks_iq2};
  for (int b = 0; b < 2; ++b) {
    const int kt = b == 0 ? kFp4KTile : kIq2KTile;
    if (ks[b] != 0 && ks[b] != 1 && ks[b] != 2 && ks[b] != 4 && ks[b] != 8) return B200MOE_ERR_INVALID_ARG;
    if (ks[b] && ((c.hidden / kt) % ks[b] || (c.inter / kt) % ks[b])) return B200MOE_ERR_INVALID_ARG;
  }
  L->ks_fixed[0] = ks_fp4;
  L->ks_fixed[1] = ks_iq2;
  return B200MOE_OK;
}

int b200moe_debug_inter(const b200moe_layer* L, void* stream, void* dst, int rows) {
  if (!L || !dst || rows < 1 || rows > L->s_max) return B200MOE_ERR_INVALID_ARG;
  DeviceGuard guard(L->device);
  if (cudaMemcpyAsync(dst, L->inter, size_t(rows) * L->cfg.inter * 2, cudaMemcpyDeviceToDevice,
                      static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return B200MOE_ERR_CUDA;
  return B200MOE_OK;
}

int b200moe_route_plan(void* stream, const int32_t* ids, int n, int num_experts, const int32_t* hot_slot,
                       const int32_t* second_slot, int n_hot, int n_second, int split, int host,
                       const int32_t* iq_slot, int32_t* perm, int32_t* gids_hot, int32_t* goff_hot,
                       int32_t* gids_host, int32_t* goff_host, int32_t* iq_out, uint32_t* err) {
  if (!ids || n < 1 || n > 4096 || !hot_slot || !perm || !gids_hot || !goff_hot || num_experts < 1 || n_hot < 1)
    return B200MOE_ERR_INVALID_ARG;
  if (split && (!second_slot || n_second < 1)) return B200MOE_ERR_INVALID_ARG;
  if (host && (!split || !gids_host || !goff_host)) return B200MOE_ERR_INVALID_ARG;
  if ((iq_slot == nullptr) != (iq_out == nullptr)) return B200MOE_ERR_INVALID_ARG;
  if (n_hot + (split ? n_second : 0) + 1 > 4096) return B200MOE_ERR_INVALID_ARG;
  PlanArgs p{};
  p.ids = ids;
  p.n = n;
  p.num_experts = num_experts;
  p.hot_slot = hot_slot;
  p.second_slot = second_slot;
  p.n_hot = n_hot;
  p.n_second = split ? n_second : 1;
  p.split = split;
  p.host = host;
  p.iq_slot = iq_slot;
  p.perm = perm;
  p.gids_hot = gids_hot;
  p.goff_hot = goff_hot;
  p.gids_host = gids_host;
  p.goff_host = goff_host;
  p.iq_out = iq_out;
  p.err = err;
  if (launch_plan(static_cast<cudaStream_t>(stream), p)) return B200MOE_ERR_CUDA;
  return B200MOE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode forward with a fixed, library-owned workspace (no allocation).
//
// b200moe_forward keeps its per-call intermediates (route permutation, route
// chunks, fp16 activations, SwiGLU rows, W2 route rows, combine
// counters) in a workspace that b200moe_layer_create allocates for each layer.
// Some callers cannot allocate device memory at the time they need a decode
// forward: an engine that hands all free HBM to its KV cache after start-up
// and forbids later cudaMalloc calls, or code that must run where its own
// allocator may not be entered.  b200moe_forward_static runs the same kernels
// with that workspace taken from one array compiled into this library, so
// the call allocates nothing.  The array lives on every GPU that loads the
// library until the process exits, it is shared by all layers and all calls,
// and calls that overlap on the GPU race on it.
namespace {

constexpr int kStaticMaxTokens = 16;
constexpr int kStaticMaxTopK = 8;
constexpr int kStaticMaxHidden = 4096;
constexpr int kStaticMaxInter = 2048;
constexpr int kStaticMaxSlots = 512;  // experts held by one layer on this GPU
constexpr int kStaticRoutes = kStaticMaxTokens * kStaticMaxTopK;
constexpr size_t kStaticMaxChunks = kStaticRoutes + kStaticMaxSlots;

constexpr size_t align256(size_t v) { return (v + 255) / 256 * 256; }
constexpr size_t kOffPerm = 0;
constexpr size_t kOffWeff = kOffPerm + align256(kStaticRoutes * 4);
constexpr size_t kOffChunks0 = kOffWeff + align256(kStaticRoutes * 4);
constexpr size_t kOffChunks1 = kOffChunks0 + align256(kStaticMaxChunks * sizeof(Chunk));
constexpr size_t kOffNChunks = kOffChunks1 + align256(kStaticMaxChunks * sizeof(Chunk));
constexpr size_t kOffKsSel = kOffNChunks + 64;
constexpr size_t kOffBankRange = kOffNChunks + 128;
constexpr size_t kOffX16 = kOffNChunks + 256;
constexpr size_t kOffInter = kOffX16 + align256(size_t(kStaticMaxTokens) * kStaticMaxHidden * 2);
constexpr size_t kOffYw = kOffInter + align256(size_t(kStaticRoutes) * kStaticMaxInter * 2);
constexpr size_t kOffCounters = kOffYw + align256(size_t(kStaticRoutes) * kStaticMaxHidden * 2);
constexpr size_t kOffXq = kOffCounters + align256(size_t(kStaticMaxTokens) * (kStaticMaxHidden / 32) * 4);
constexpr size_t kOffInterq =
    kOffXq + align256(size_t(kStaticMaxTokens) * (kStaticMaxHidden / kIq2KTile) * kIq2XBlockBytes);
constexpr size_t kStaticScratchBytes =
    kOffInterq + align256(size_t(kStaticRoutes) * (kStaticMaxInter / kIq2KTile) * kIq2XBlockBytes);

// 2,409,728 bytes per GPU at the limits above.
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch per device (the host-side name of the
// array is not a device address), looked up by b200moe_layer_create on the
// layer's device with that device current.
constexpr int kMaxDevices = 64;
uint8_t* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

}  // namespace

int static_scratch(int device, uint8_t** out) {
  if (device < 0 || device >= kMaxDevices) return B200MOE_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return B200MOE_ERR_CUDA;
    }
    g_scratch_addr[device] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch_addr[device];
  return B200MOE_OK;
}

extern "C" int b200moe_forward_static(b200moe_layer* L, void* stream, const void* x, int x_dtype,
                                      const int32_t* ids, const float* w, float* out, int M) {
  if (!L || M < 1 || M > L->cfg.max_tokens) return B200MOE_ERR_INVALID_ARG;
  const auto& c = L->cfg;
  if (M > kStaticMaxTokens || c.top_k > kStaticMaxTopK || c.hidden > kStaticMaxHidden ||
      c.inter > kStaticMaxInter || c.n_fp4 + c.n_iq2 > kStaticMaxSlots)
    return B200MOE_ERR_RANGE;
  if (!L->maps_set) return B200MOE_ERR_STATE;
  if (c.n_iq2 > 0 && !L->tables_set) return B200MOE_ERR_STATE;
  if (!x || !ids || !w || !out) return B200MOE_ERR_INVALID_ARG;
  if (x_dtype != B200MOE_F16 && x_dtype != B200MOE_BF16) return B200MOE_ERR_DTYPE;
  if (!aligned(x, 16) || !aligned(out, 16)) return B200MOE_ERR_ALIGN;
  DeviceGuard guard(L->device);
  uint8_t* ws = nullptr;
  if (int st = static_scratch(L->device, &ws)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Workspace w_{};
  w_.perm = reinterpret_cast<int32_t*>(ws + kOffPerm);
  w_.w_eff = reinterpret_cast<float*>(ws + kOffWeff);
  w_.chunks[0] = reinterpret_cast<Chunk*>(ws + kOffChunks0);
  w_.chunks[1] = reinterpret_cast<Chunk*>(ws + kOffChunks1);
  w_.max_chunks = int(kStaticMaxChunks);
  w_.n_chunks = reinterpret_cast<int32_t*>(ws + kOffNChunks);
  w_.ks_sel = reinterpret_cast<int32_t*>(ws + kOffKsSel);
  w_.bank_range = reinterpret_cast<int32_t*>(ws + kOffBankRange);
  w_.x16 = reinterpret_cast<__half*>(ws + kOffX16);
  w_.inter = reinterpret_cast<__half*>(ws + kOffInter);
  w_.y2 = reinterpret_cast<__half*>(ws + kOffYw);
  w_.counters = reinterpret_cast<int32_t*>(ws + kOffCounters);
  w_.xq = ws + kOffXq;
  w_.interq = ws + kOffInterq;
  w_.dbg_y13 = nullptr;
  // The array keeps the previous call's contents: the combine counters must
  // start at zero (the SwiGLU rows and int8 blocks are rewritten before use).
  if (cudaMemsetAsync(w_.counters, 0, size_t(M) * (c.hidden / 32) * 4, s) != cudaSuccess) return B200MOE_ERR_CUDA;
  return run_forward(L, w_, s, x, x_dtype, ids, w, out, M);
}
