// Internal launchers shared between the library's translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct b200moe_ep;  // the expert-parallel exchange object of the C ABI (ep_p2p.cu)

namespace b200moe {

// Activation rows staged per GEMV stage: a chunk holds 16 / ks routes.
constexpr int kRouteSlotsPerChunk = 16;

// Block-scaled FP4 tensor path: activation planes and routes per chunk.
constexpr int kFp4Planes = 4;
constexpr int kFp4TcRoutes = 32;  // largest routes per chunk of the block-scaled FP4 path

// ---- packing (pack.cu)
// MXFP4: per (slot, projection) global 2^(emax - 140) so the largest nonzero block maps to f16 exponent 28
int launch_mx_rebase(cudaStream_t s, int hidden, int inter, int n, const uint8_t* w13c, const uint8_t* w13s,
                     const uint8_t* w2c, const uint8_t* w2s, float* slot_globals, int* span_scratch, uint32_t* err);
int launch_fp4_prepack(cudaStream_t s, int fmt, int hidden, int inter, int n, const uint8_t* w13c,
                       const uint8_t* w13s, const uint8_t* w2c, const uint8_t* w2s, float* slot_globals,
                       int* span_scratch, uint8_t* bank_slot0, int64_t slot_stride, int64_t w13_bytes,
                       uint32_t* err);
// IQ bank: W13 units in format fmt13, W2 units in fmt2 (2 IQ2_XXS, 3 IQ2_XS, 4 IQ1_M) from ggml blocks
int launch_iq2_prepack(cudaStream_t s, int fmt13, int fmt2, int hidden, int inter, int n, const uint8_t* w1,
                       const uint8_t* w3, const uint8_t* w2, uint8_t* bank_slot0, int64_t slot_stride,
                       int64_t w13_bytes);

// ---- routing (route.cu)
struct Chunk {  // one route chunk of one expert group: routes perm[begin .. begin+count)
  int32_t slot;
  int32_t begin;
  int32_t count;
  int32_t pad;
};

// Time model of one bank's skinny GEMV (W13 + W2) for the split-K choice:
// waves of items over the persistent CTA slots, a wave taking the longer of
// one CTA streaming its item and all busy CTAs sharing HBM, plus a fixed cost.
struct KsModel {
  int allowed;        // bit j set: ks = 1 << j divides both projections' K tiles
  float slots;        // persistent CTA slots (SMs x CTAs per SM)
  float bpe;          // weight bytes per K element of a 32-row tile pair
  float bw_cta, bw_hbm, per_wave;  // bytes/s of one CTA, of HBM; seconds per wave
  float tiles[2], kdim[2];         // tile pairs and K of W13 and W2
};

// Expert-parallel receive of one step (ep_p2p.cu): the route plan of the
// owner's forward waits until every rank's data flag reaches *epoch, takes the
// rows received from the reservation counter of that epoch and resets both.
struct EpRecvWait {
  const int* flags;  // [n_flags] data flags of the source ranks
  int n_flags;
  const int* epoch;  // the step in flight
  int* resv;         // [2] reservation counters (by epoch parity)
  int32_t* out;      // [3]: rows received, then {0, rows}
  const void* rows;  // fp16 [max_rows][H] received rows
  const int32_t* expert_ids;
  void* y2;          // fp16 [max_rows][H] local y2 rows
  int max_rows;
  int device;
};

// Expert-parallel return fused into the W2 epilogue of an owner's FP4 bank:
// each route's y2 row goes straight into its home rank's y2home buffer
// (home[row] = (rank << 24) | route index at home), and the kernel's last CTA
// raises this rank's return flag on every rank (mbox word world + rank).
constexpr int kEpMaxPeers = 16;
struct EpReturn {
  const int32_t* home;           // null: no fused return
  uint8_t* peer[kEpMaxPeers];    // every rank's shared exchange allocation
  int64_t off_y2home, off_mbox;  // offsets in it
  int world, rank;
  const int* epoch;              // the step in flight
  int* done;                     // CTAs finished (reset by the last)
};

struct PlanArgs {
  const int32_t* ids;  // [n] expert id per route (flat t*k + slot)
  int n;
  const int32_t* n_valid;  // optional (device): routes of this call, <= n
  EpRecvWait recv;         // optional (recv.flags set): wait for an expert-parallel receive first
  int num_experts;
  // product keys: key_of_expert[e] in [0, n_keys) or -1 (not on this GPU / invalid)
  const int32_t* key_of_expert;
  int n_keys;
  // reference-parity keys (used when key_of_expert == nullptr)
  const int32_t* hot_slot;
  const int32_t* second_slot;
  int n_hot, n_second, split, host;
  const int32_t* iq_slot;
  // outputs
  int32_t* perm;        // [n]
  int32_t* inv;         // optional [n]: sorted position of each route (perm's inverse)
  int32_t* chunk_of;    // optional [n]: (chunk << 8) | index in chunk, for bank 0's positions
  // product: chunk lists of up to two banks (bank b = keys [key_lo[b], key_hi[b]))
  int n_banks;
  int key_lo[2], key_hi[2], rc[2], max_chunks[2];
  Chunk* chunks[2];
  int32_t* n_chunks;    // [2]
  int32_t* key_counts;  // optional [n_keys]: routes per key (product mode)
  // product: a bank with rc[b] == 0 gets its split-K chosen here from this
  // plan's exact chunk counts (ks_model[b]); ks_sel[b] receives the split-K the
  // GEMV of bank b runs with (16 / rc for a fixed rc)
  KsModel ks_model[2];
  int32_t* ks_sel;
  int32_t* bank_range;  // optional [2][2]: sorted positions [begin, end) of each bank's routes
  const float* w_in;    // [n] router weights (product)
  float* w_eff;         // [n] weight used by the combine (0 for a route without an expert)
  // product: a route without an expert gets a zero y2 row and its completion
  // counts (so the fused combine still sees k arrivals per token and tile)
  void* y2;             // fp16 [n][H] W2 rows by route index
  int32_t* counters;    // [tokens][H/32]
  float* out;           // [tokens][H]
  int H;
  int top_k;
  // reference-parity tables
  int32_t* gids_hot;
  int32_t* goff_hot;
  int32_t* gids_host;
  int32_t* goff_host;
  int32_t* iq_out;
  uint32_t* err;
};

// Block-scaled FP4 GEMM (tcgen05.mma.kind::mxf4nvf4) of the FP4 bank.
struct Fp4Args {
  const uint8_t* wt;      // weight units [slot][n_rt][K/256] (codes in the swizzled order + blocked scales)
  const float* globals;   // [slot][3] FP32 global scales (NVFP4)
  int K;
  int n_rt;               // items per chunk: W13 I/128 (gate + up tiles), W2 H/256 (two row tiles)
  const uint8_t* sfb;     // activation plane scales blocked: [chunk][K/64][512]
  const float* gx;        // [plane_rows] per-row plane factor g
  uint32_t* rowmax;       // W13: [plane_rows] amax (float bits) of each SwiGLU row, for the W2 planes
  int plane_rows;
  const Chunk* chunks;
  const int32_t* n_chunks;
  int bank;
  int n_slots;
  const int32_t* perm;
  int S;
  int top_k;
  __half* inter;
  int inter_stride;
  float limit;
  const float* w_eff;
  void* y2;
  int32_t* counters;
  float* out;
  int H;
  uint32_t* err;
  EpReturn ep;  // W2 only, optional
};
int launch_fp4_gemm(cudaStream_t s, int epi, int rc, bool mx, const Fp4Args& a, const void* map_x, int grid);

// Fused small-batch decode of an FP4-only layer (decode.cu): two launches, W13
// and W2, each planning the call's routes itself, quantizing its chunks'
// activation rows into shared memory and (W2) combining the token rows.
constexpr int kDecodeMaxRoutes = 64;
// decode calls of at most this many routes combine in the block-scaled W2 epilogue (no combine launch)
constexpr int kFusedCombineRoutes = 64;
struct DecArgs {
  const uint8_t* wt;          // weight units of this projection [slot][n_rt][K/256]
  const float* globals;       // NVFP4 [slot][3] FP32 global scales, null for MXFP4
  int K;                      // H (W13) or I (W2)
  int n_rt;                   // items per chunk: W13 I/128, W2 H/256
  int n_slots;
  const void* src;            // W13: token rows x [M][H] (f16 or bf16); W2: the SwiGLU rows [S][inter] (f16)
  int64_t src_stride;         // elements
  const int32_t* ids;         // [S] expert ids (route = token * top_k + slot)
  const float* w_in;          // [S] routing weights
  int S;
  int top_k;
  int num_experts;
  const int32_t* key_of_expert;  // expert -> bank-0 slot (n_keys: none)
  int n_keys;
  __half* inter;              // W13 out: SwiGLU rows at sorted positions, stride inter_stride
  int inter_stride;
  float limit;
  __half* y2;                 // W2: fp16 rows by route [S][H]
  int32_t* counters;          // W2: [M][H/32] completion counts (zero between calls)
  float* out;                 // W2: [M][H]
  int H;
  int32_t* perm_out;          // W13: the sorted order, written by CTA 0
  uint32_t* err;
  int stages;                 // weight stages in shared memory
};
// 0 when the fused decode launches, -1 when the shape does not fit it (the caller takes the chained path)
int launch_fp4_decode(cudaStream_t s, int epi, bool mx, bool bf16, const DecArgs& a, int grid);
bool fp4_decode_fits(int K);
// routes per chunk of the block-scaled FP4 path for a call of S routes (the MMA's N is 4 x this)
inline int fp4_routes_per_chunk(int S) { return S <= 64 ? 4 : S <= 1024 ? 8 : S < 4096 ? 16 : 32; }
inline int fp4_rc_index(int rc) { return rc == 4 ? 0 : rc == 8 ? 1 : rc == 16 ? 2 : 3; }
int launch_fp4_planes(cudaStream_t s, bool by_token, bool bf16, bool mx, const void* src, int64_t src_stride, int K,
                      const int32_t* inv, int top_k, const int32_t* chunk_of, int bank,
                      const int32_t* bank_range, int max_rows, uint32_t* rowmax, uint8_t* planes, int plane_rows,
                      uint8_t* sfb, float* gx);
int launch_route_combine(cudaStream_t s, const __half* y2, const int32_t* inv, const int32_t* bank_range,
                         int n_banks, const float* w, int T, int k, int H, float* out);
int launch_fp4_tile(cudaStream_t s, bool mx, const uint8_t* codes, const uint8_t* scales, int n_slots,
                    int rows_per_slot, int K, bool gate_up, const float* globals, uint32_t* err, uint8_t* out);
// 2D uint8 TMA map with 128-byte swizzle: rows x row_bytes, box box_bytes x box_rows, zero fill out of range
int make_u8_tile_map(void* map_out, const void* base, int64_t rows, int64_t row_bytes, int box_bytes, int box_rows);

size_t plan_smem_bytes(int n_keys);
// the receive of this rank's expert-parallel exchange object (the C ABI's b200moe_ep)
int ep_recv_wait(const ::b200moe_ep* E, EpRecvWait* w);
// the fused return's targets (ep_p2p.cu)
int ep_return_targets(const ::b200moe_ep* E, EpReturn* r);
// fp16 rows -> int8 blocks of kIq2XBlockBytes per 256-wide K tile (IQ2 activations)
int launch_quant_s8(cudaStream_t s, const __half* src, int64_t src_stride, int K, int rows, const int32_t* range,
                    uint8_t* dst);
int launch_plan(cudaStream_t s, const PlanArgs& a);
// the plan of <= 32 routes and the FP4 planes of the token rows in one launch (x: f16, or bf16 when bf16)
int launch_plan_planes(cudaStream_t s, const PlanArgs& a, bool bf16, bool mx, const void* x, int64_t src_stride,
                       int K, int n_tokens, uint32_t* rowmax, uint8_t* planes, uint8_t* sfb, float* gx);
int launch_gating(cudaStream_t s, const float* logits, int T, int E, int k, int32_t* ids, float* w,
                  uint32_t* err);
int launch_convert_bf16(cudaStream_t s, const void* x, int64_t n, void* x16);

// ---- decode / skinny grouped GEMV (gemv.cu)
struct GemvArgs {
  int fmt;                    // 0 NVFP4, 1 MXFP4, 2 IQ2_XXS
  int epi;                    // 0: W13 -> SwiGLU -> inter; 1: W2 -> weighted combine
  const int32_t* ks_sel;      // device [2]: K splits per item (1, 2, 4, 8) of each bank, set by the plan
  const uint8_t* region;      // slot 0 of this projection region
  int64_t slot_stride;        // bytes between slots
  int n_slots;
  const float* globals;       // [slots][3] or nullptr
  int K;                      // reduction length
  int n_tp;                   // tile pairs per expert in this region
  const Chunk* chunks;
  const int32_t* n_chunks;    // device count of this bank's chunks
  int bank;                   // index into n_chunks
  const int32_t* perm;        // [S]
  int S;
  int top_k;
  const void* xsrc;           // f16 rows
  int x_by_token;             // 1: row perm[p] / k; 0: row p
  int64_t x_row_stride;       // elements
  int n_x_rows;               // rows available in xsrc (bounds check)
  void* inter;                // W13 output f16 [S][inter_stride]
  int inter_stride;
  void* dbg_y13;              // optional f16 [S][2 * inter_stride]
  float limit;
  const float* w_eff;         // [S] by route index
  void* y2;                   // fp16 [S][H] W2 rows (x global, unweighted) by route index
  int32_t* counters;          // [tokens][H/32]
  float* out;                 // [tokens][H]
  int H;
  const uint32_t* iq2_tables; // the IQ format's decode tables (iq_table_words(fmt) words)
  uint32_t* err;
  int grid;                   // persistent CTAs
};

// ---- prefill grouped GEMM on tcgen05 (gemm_tc.cu)
struct TcArgs;
int make_token_map(void* map_out, const void* base, int64_t rows, int64_t cols);
size_t tc_map_bytes();
int launch_gather_rows(cudaStream_t s, const void* x, int bf16, const int32_t* perm, int S, int k, int H,
                       void* xperm);
constexpr int kTcTokenTile = 128;
// prefill calls of at least this many routes run a block-scaled-layout bank on the tcgen05 f16 GEMM
constexpr int kTcUnitsMinRoutes = 4096;

size_t gemv_smem_bytes(int fmt, int ks);
int gemv_ctas_per_sm(int fmt);
int launch_gemv(cudaStream_t s, const GemvArgs& a);

struct TcArgs {
  const uint8_t* region;   // slot 0 of the W13 or W2 region (decode bank layout)
  int64_t slot_stride;
  int n_slots;
  const float* globals;    // [slots][3]
  int K;                   // H (W13) or I (W2)
  int n_rt;                // row tiles of 256 weight rows: I/128 (W13) or H/256 (W2)
  const Chunk* chunks;     // token tiles (<= 128 routes each) of this bank
  const int32_t* n_chunks;
  int bank;
  const int32_t* perm;
  int S;
  int top_k;
  void* inter;             // W13 output f16 [S][I] by sorted position
  int inter_stride;
  float limit;
  void* y2;                // fp16 [S][H] W2 rows by route index (combined by the launch after W2)
  int H;
  uint32_t* err;
};
int launch_tc_gemm(cudaStream_t s, int fmt, int epi, const TcArgs& a, const void* map, int grid);

}  // namespace b200moe
