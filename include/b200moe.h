/*
 * b200moe.h -- C ABI of the B200 (sm_100a) routed-expert MoE layer.
 *
 * This is the drop-in boundary for the reference build's routed-expert
 * FusedMoE quant-method plugin.  Reference interfaces replaced (paths relative
 * to the reference project; EXP = engine/src/vllm/model_executor/layers/fused_moe/experts):
 *
 *   b200moe_layer_create / _destroy   NativeV41Moe.__init__ / three_tier
 *                                     (EXP/nvfp4_8r_native.py:645-745, 770-808):
 *                                     fixed buffers sized for max_tokens, all
 *                                     kernels ready before any graph capture.
 *   b200moe_set_slot_maps             tiers.slot_maps -> slot_of_expert maps
 *                                     (EXP/nvfp4_8r_tiers.py:169-179;
 *                                     EXP/nvfp4_8r_native.py:687-717).
 *   b200moe_load_fp4 / _load_iq2      NativeExpertSet.from_raw / IqWarmBank
 *                                     (EXP/nvfp4_8r_native.py:275-323, 522-570):
 *                                     records into HBM in the kernels' layout.
 *   b200moe_route                     the engine router that produces
 *                                     (topk_ids, topk_weights) ahead of
 *                                     engine/patches/gguf_moe.patch:53.
 *   b200moe_forward                   NativeV41Moe.forward
 *                                     (EXP/nvfp4_8r_native.py:913-961): decode,
 *                                     1 <= M <= max_tokens, no host sync, no
 *                                     allocation, CUDA-graph capturable.
 *   b200moe_forward_prefill           NativeV41Moe.forward_prefill
 *                                     (EXP/nvfp4_8r_native.py:970-1094): any
 *                                     T <= max_prefill_tokens.
 *   b200moe_route_plan                GroupPlanner.plan / the _compact chain
 *                                     (EXP/nvfp4_8r_group_plan.py:163-332;
 *                                     EXP/nvfp4_8r_native.py:806-889): the
 *                                     reference's perm / gids / goff / iq tables.
 *   b200moe_quantize_nvfp4 / _mxfp4   offline packing (the reference's packs were
 *   b200moe_fold_nvfp4_to_mxfp4       made by NVIDIA and folded by
 *                                     harness/benchmarks/nvfp4_8r/build_packs.py:120-151).
 *
 * Conventions: every function returns an int status (b200moe_status).  Device
 * pointers are plain CUDA device addresses on the layer's device; `stream` is a
 * cudaStream_t passed as void*.  Nothing here allocates after create, and
 * nothing in forward / forward_prefill / route synchronizes with the host.
 */
#ifndef B200MOE_H_
#define B200MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  B200MOE_OK = 0,
  B200MOE_ERR_INVALID_ARG = 1, /* shape, count, pointer or config refused on the host */
  B200MOE_ERR_DTYPE = 2,       /* unsupported dtype code */
  B200MOE_ERR_ALIGN = 3,       /* a pointer without the alignment the layout needs */
  B200MOE_ERR_CUDA = 4,        /* a CUDA runtime call failed */
  B200MOE_ERR_BOUNDS = 5,      /* a kernel found an id, slot or offset out of range */
  B200MOE_ERR_TIMEOUT = 6,     /* a bounded device wait ran out */
  B200MOE_ERR_FORMAT = 7,      /* a packed value the format forbids (E4M3 NaN, E8M0 255) */
  B200MOE_ERR_RANGE = 8,       /* a value the kernel layout cannot hold */
  B200MOE_ERR_NOMEM = 9,       /* device allocation failed at create */
  B200MOE_ERR_STATE = 10       /* call out of order (weights or maps not set) */
} b200moe_status;

typedef enum { B200MOE_F16 = 0, B200MOE_BF16 = 1, B200MOE_F32 = 2 } b200moe_dtype;

typedef enum { B200MOE_NVFP4 = 0, B200MOE_MXFP4 = 1, B200MOE_IQ2XXS = 2 } b200moe_format;

/* Shape and residency of one layer on one GPU.  Bank 0 holds FP4 experts
 * (NVFP4 or MXFP4), bank 1 IQ codebook experts (IQ2_XXS, IQ2_XS or IQ1_M per
 * projection); the slot maps say which expert id sits in which slot of which
 * bank. */
typedef struct {
  int32_t hidden;             /* H: multiple of 256 */
  int32_t inter;              /* I: multiple of 128 (256 when bank 1 is used) */
  int32_t num_experts;        /* E: global expert ids 0..E-1, E <= 1024 */
  int32_t top_k;              /* k: 1..16 */
  int32_t max_tokens;         /* decode M limit of b200moe_forward, 1..64 */
  int32_t max_prefill_tokens; /* T limit of forward_prefill (0: no prefill workspace) */
  int32_t fp4_format;         /* B200MOE_NVFP4 or B200MOE_MXFP4 */
  int32_t n_fp4;              /* slots in bank 0 */
  int32_t n_iq2;              /* slots in bank 1 (IQ codebook experts) */
  float swiglu_limit;         /* limited SwiGLU bound (reference: 10.0) */
  int32_t prefill_gemm;       /* FP4 bank kernels: 0 = the skinny decode kernels for every call,
                                 1 = forward_prefill on the tcgen05 grouped GEMM (f16 dequantized
                                 weight tiles, route tiles of 128), decode on the skinny kernels,
                                 2 = hidden and inter multiples of 256: decode and prefills below
                                 4096 routes on the block-scaled FP4 tensor cores
                                 (tcgen05.mma.kind::mxf4nvf4 with the format's block scales in
                                 TMEM: E4M3 per 16 or E8M0 per 32; activations as four E2M1
                                 planes, ~1e-4 relative), longer prefills on the tcgen05 f16
                                 GEMM; both read the bank as swizzled weight units; the fastest
                                 layout for decode and prefill,
                                 3 = the layout of 2 with every call on the block-scaled kernel
                                 (32-route chunks from 4096 routes; slower for long prefills) */
  int32_t iq_type13;          /* GGML type of bank 1's gate/up (W1, W3): 16 IQ2_XXS (0 = 16),
                                 17 IQ2_XS, 29 IQ1_M -- the routed-expert types GGUF layers mix,
                                 engine/.../experts/nvfp4_8r_tiers.py:35 */
  int32_t iq_type2;           /* GGML type of bank 1's down projection (W2), same codes */
} b200moe_config;

typedef struct b200moe_layer b200moe_layer;

const char* b200moe_status_name(int status);
/* Library version string and the CUDA architecture it was built for. */
const char* b200moe_version(void);

int b200moe_layer_create(const b200moe_config* cfg, int device, b200moe_layer** out);
int b200moe_layer_destroy(b200moe_layer* layer);

/* Host int32 [E] maps: slot of each expert in bank 0 / bank 1, -1 where absent.
 * Every expert must sit in exactly one bank, and each bank's slots must be
 * covered exactly once. */
int b200moe_set_slot_maps(b200moe_layer* layer, const int32_t* fp4_slot, const int32_t* iq2_slot);

/* IQ2_XXS codebook: grid int8 [256][8] and ksigns uint8 [128] (host). */
int b200moe_set_iq2_tables(b200moe_layer* layer, const int8_t* grid, const uint8_t* ksigns);

/* Codebook of one IQ format by GGML type (host arrays, ggml's data): 16
 * IQ2_XXS grid int8 [256][8] of 8/25/43 + ksigns [128]; 17 IQ2_XS grid
 * [512][8] of 8/25/43 + ksigns [128]; 29 IQ1_M grid [2048][8] of -1/0/1, no
 * ksigns (NULL).  n_entries = the grid's rows.  Every format the layer's IQ
 * bank uses (config iq_type13 / iq_type2) needs its codebook before a forward. */
int b200moe_set_iq_grid(b200moe_layer* layer, int ggml_type, const int8_t* grid, int n_entries,
                        const uint8_t* ksigns);

/* Load n consecutive bank-0 slots from natural-layout device arrays:
 *   w13_codes [n][2I][H/2] (W1 rows then W3 rows, low nibble = even element),
 *   w13_scales [n][2I][H/bs], w2_codes [n][H][I/2], w2_scales [n][H][I/bs],
 *   bs = 16 (E4M3, NVFP4) or 32 (E8M0, MXFP4);
 *   globals: device float [n][3] = (W1, W3, W2) FP32 global scales for NVFP4;
 *   ignored (may be NULL) for MXFP4. */
int b200moe_load_fp4(b200moe_layer* layer, void* stream, int slot_begin, int n,
                     const uint8_t* w13_codes, const uint8_t* w13_scales, const uint8_t* w2_codes,
                     const uint8_t* w2_scales, const float* globals);

/* Load n consecutive bank-1 slots from ggml blocks of the configured IQ types
 * (B bytes per 256 weights: IQ2_XXS 66, IQ2_XS 74, IQ1_M 56): w1, w3
 * [n][I][H/256][B of iq_type13], w2 [n][H][I/256][B of iq_type2] (device). */
int b200moe_load_iq2(b200moe_layer* layer, void* stream, int slot_begin, int n, const uint8_t* w1,
                     const uint8_t* w3, const uint8_t* w2);

/* Router: logits fp32 [T][E] -> topk_ids int32 [T][k], topk_weights fp32 [T][k]:
 * softmax top-k with renormalised weights (ties to the smaller id). */
int b200moe_route(b200moe_layer* layer, void* stream, const float* logits, int32_t* topk_ids,
                  float* topk_weights, int T);

/* Decode forward: x [M][H] (f16 or bf16), ids int32 [M][k], weights fp32 [M][k]
 * -> out fp32 [M][H] = sum over slots (slot order) of w * expert(x). */
int b200moe_forward(b200moe_layer* layer, void* stream, const void* x, int x_dtype,
                    const int32_t* topk_ids, const float* topk_weights, float* out, int M);

/* Prefill forward: same contract for any 1 <= T <= max_prefill_tokens. */
int b200moe_forward_prefill(b200moe_layer* layer, void* stream, const void* x, int x_dtype,
                            const int32_t* topk_ids, const float* topk_weights, float* out, int T);

/* Decode forward that allocates nothing.  No counterpart in the reference:
 * the reference's decode buffers are allocated with the layer.
 *
 * Same contract and kernels as b200moe_forward, but the per-call scratch
 * (route permutation, route chunks, fp16 activations, SwiGLU rows, W2 route
 * rows, combine counters) sits in one fixed array inside this library
 * instead of the layer's workspace.  It is for callers that cannot allocate
 * device memory when they run a decode step, e.g. an engine that gives all
 * free HBM to its KV cache after start-up and allows no cudaMalloc later.
 * Limits: M <= 16 (and, as for b200moe_forward, M <= the layer's max_tokens,
 * else B200MOE_ERR_INVALID_ARG), top_k <= 8, hidden <= 4096, inter <= 2048,
 * and at most 512 experts held by the layer; larger sizes return
 * B200MOE_ERR_RANGE.  The array (about 2.4 MB) is held on every GPU that loads
 * the library until exit.  b200moe_layer_create looks up the array's device
 * address on the layer's device, so this call itself does no set-up.  Every
 * call shares the array and zeroes its combine counters on `stream` first;
 * calls that overlap on the GPU race. */
int b200moe_forward_static(b200moe_layer* layer, void* stream, const void* x, int x_dtype,
                           const int32_t* topk_ids, const float* topk_weights, float* out, int M);

/* Wait for `stream`, then read and clear the layer's kernel error word.
 * Returns the status the bits map to (B200MOE_OK when none); *bits gets them. */
int b200moe_check_errors(b200moe_layer* layer, void* stream, uint32_t* bits);

/* Debug taps.  set_debug_y13 (device pointer or NULL): the W13 launch also
 * writes y13 fp16 [rows][2I] by route position.  debug_perm copies the route
 * permutation of the last forward (route index at each sorted position) into
 * dst (device int32 [n]) on `stream`. */
int b200moe_set_debug_y13(b200moe_layer* layer, void* y13);
int b200moe_debug_perm(const b200moe_layer* layer, void* stream, int32_t* dst, int n);
/* Copy the SwiGLU output rows (fp16 [rows][I], by sorted route position) of the
 * last forward into dst (device). */
int b200moe_debug_inter(const b200moe_layer* layer, void* stream, void* dst, int rows);

/* Split-K of the skinny GEMV per bank (ks in {1, 2, 4, 8}; K tiles of hidden
 * and inter divisible by ks; 0 = the default: the route plan chooses it on
 * the device for every call from that call's routing, so a captured graph
 * adapts at replay and equal inputs always give equal bits).  A route's output bits depend only on ks, so two layers with the
 * same fixed ks give bit-equal y2 rows whatever else they route (the
 * expert-parallel owner and the single-GPU layer).  No reference counterpart:
 * the reference's QPN grid rule (test_p3_split_groups.py:33-41) fixes its
 * K split from the shape alone. */
int b200moe_set_split_k(b200moe_layer* layer, int ks_fp4, int ks_iq2);

/* Fused small-batch decode.  On a layer whose experts all sit in the FP4 bank
 * (n_iq2 = 0) with prefill_gemm 2 or 3, a forward of at most max_routes routes
 * (M * top_k; at most 64) runs as two launches, W13 and W2, instead of the
 * chained ones (route plan with the x planes, W13, SwiGLU planes, W2 with the
 * combine): each CTA plans the call itself, quantizes its chunk's rows into
 * shared memory and the W2 launch combines each token's rows once their last
 * route is stored.  Same output bits as the chained path.  The default is 0
 * (off): on B200 the fused form is slower (configs[1] M = 1: 63.8 against
 * 57.6 us; M = 8: 264 against 170 us), because every CTA quantizes its
 * chunk's whole rows before its first MMA, a chain the chained path spreads
 * over many CTAs.  No reference counterpart (the reference's decode is
 * the QPN launch chain of engine/.../experts/nvfp4_8r_native.py:929-960). */
int b200moe_set_decode_fusion(b200moe_layer* layer, int max_routes);

/* Timing hook: with n > 0 cudaEvent_t handles, forward / forward_prefill
 * record events[0] on the stream before their first launch and events[j + 1]
 * after launch j (bf16 copy, recorded also when x is fp16 and nothing is
 * copied; plan; [prefill with tcgen05: row gather]; W13 per bank; W2 per bank).  n = 0 turns
 * it off.  The events stay owned by the caller. */
int b200moe_set_timing_events(b200moe_layer* layer, void* const* events, int n);

/* Reference route plan (GroupPlanner.plan semantics), one launch:
 *   key = hot_slot[id] if >= 0, else (split) n_hot + second_slot[id] if >= 0,
 *   else n_hot + n_second; perm = stable sort of keys; gids_hot/goff_hot the
 *   HBM launch tables; with `host` the rotated second-launch tables; with
 *   iq_slot non-NULL the IQ slot of every route.  n <= 4096 routes. */
int b200moe_route_plan(void* stream, const int32_t* ids, int n, int num_experts,
                       const int32_t* hot_slot, const int32_t* second_slot, int n_hot, int n_second,
                       int split, int host, const int32_t* iq_slot, int32_t* perm,
                       int32_t* gids_hot, int32_t* goff_hot, int32_t* gids_host, int32_t* goff_host,
                       int32_t* iq_out, uint32_t* err);

/* ---- Expert parallelism (no counterpart in the reference, which refuses EP:
 * engine/patches/gguf_moe.patch:57-58).  Expert e lives on rank
 * owner_of_expert[e]; the exchange is NCCL all-to-all issued by the host. */

/* Decode route counters of one layer, updated on the device (one launch, so a
 * captured graph counts at every replay).  Replaces RouteStats.count,
 * engine/src/vllm/model_executor/layers/fused_moe/experts/nvfp4_8r_stats.py:81-98.
 * topk_ids: n route ids of one call; is_host / is_warm: uint8 [num_experts]
 * tier masks; stat int64 [5] (calls, routes, HOST routes, distinct HOST experts
 * per call summed, WARM routes), gap_hist int64 [7] (HOST routes by rounds
 * since their expert's last HOST use: <=1, 2, <=4, <=16, <=64, <=256, more or
 * never), routes int64 [num_experts], last_round int32 [num_experts + 1]
 * (-2^30 = never; entry num_experts takes the non-HOST routes' writes).  The
 * round of a call is stat[0] before it.  An id outside [0, num_experts) is
 * skipped and sets the bounds bit in *err. */
int b200moe_route_stats(void* stream, const int32_t* topk_ids, int n, int num_experts, const uint8_t* is_host,
                        const uint8_t* is_warm, int64_t* stat, int64_t* gap_hist, int64_t* routes,
                        int32_t* last_round, uint32_t* err);

/* Softmax top-k gating without a layer (same rule as b200moe_route). */
int b200moe_gate(void* stream, const float* logits, int T, int num_experts, int top_k, int32_t* topk_ids,
                 float* topk_weights, uint32_t* err);

/* Bytes of device workspace b200moe_ep_dispatch needs for max_routes = T * k. */
size_t b200moe_ep_workspace_bytes(int max_routes, int world);

/* Sort this GPU's T * k routes by owner rank (stable), count them per rank
 * (send_counts, device int32 [world]) and gather, in that order, each route's
 * fp16 activation row (send_rows [T*k][H]) and expert id (send_experts);
 * route_pos[route] = its position in that order. */
int b200moe_ep_dispatch(void* stream, const void* x, int x_dtype, const int32_t* topk_ids, int T, int k,
                        int num_experts, int world, const int32_t* owner_of_expert, int H, void* send_rows,
                        int32_t* send_experts, int32_t* route_pos, int32_t* send_counts, void* workspace,
                        size_t workspace_bytes, uint32_t* err);

/* out[t] = residual[t] (if non-NULL) + sum over slots, in slot order, of
 * fma(f32(y2[route_pos[t*k + s]]), w[t*k + s]) for y2 fp16 [T*k][H] returned
 * by the owners in dispatch order -- the single-GPU combine's arithmetic. */
int b200moe_ep_combine(void* stream, const void* y2, const int32_t* route_pos, const float* topk_weights, int T,
                       int k, int H, const float* residual, float* out);

/* Expert-parallel exchange over NVLink peer memory (no NCCL, no host sync:
 * the whole step can be captured in one CUDA graph).  Each rank creates one
 * exchange object whose shared buffers all ranks map through CUDA IPC:
 * create -> ipc_handle (64 bytes) -> exchange the handles among the ranks on
 * the host -> connect (world x 64 bytes, rank order).  A step, on every rank
 * in the same order: ep_push (each of this rank's T*k routes reserves a row in
 * its owner's buffer and stores its fp16 row and expert id there; no rank
 * waits for another), ep_forward (the local top-1 layer on the rows received:
 * its first launch waits for every rank's push), ep_return (y2 rows back to
 * their home ranks; fused into ep_forward's W2 for FP4-only layers),
 * ep_combine_p2p (slot-order combine + residual).
 * Waits are bounded (B200MOE_ERR_TIMEOUT through ep_check_errors).  All ranks
 * must be alive at destroy (call it after a host barrier).  No reference
 * counterpart: the reference refuses expert parallelism
 * (engine/patches/gguf_moe.patch:57-58). */
typedef struct b200moe_ep b200moe_ep;
int b200moe_ep_create(int device, int world, int rank, int hidden, int max_routes, b200moe_ep** out);
int b200moe_ep_ipc_handle(b200moe_ep* ep, void* handle);
int b200moe_ep_connect(b200moe_ep* ep, const void* handles);
int b200moe_ep_destroy(b200moe_ep* ep);
int b200moe_ep_recv_buffers(b200moe_ep* ep, void** rows, int32_t** expert_ids, int32_t** n_valid,
                            int32_t** row_range, void** y2, int* max_rows);
int b200moe_ep_push(b200moe_ep* ep, void* stream, const void* x, int x_dtype, const int32_t* topk_ids, int T,
                    int k, int num_experts, const int32_t* owner_of_expert);
/* The local experts of a top-1 layer (its owner map = this rank's experts) on
 * the rows this step brought in: waits (bounded) for every rank's push, then
 * b200moe_forward_rows on the receive buffers.  fuse_return = 0: the y2 rows
 * stay local for ep_return.  fuse_return = 1 (a prefill_gemm >= 2 layer whose
 * experts are all FP4): the W2 epilogue stores each y2 row straight into its
 * home rank's buffer and raises this rank's return flag, so no ep_return call
 * follows; other layers return B200MOE_ERR_INVALID_ARG. */
int b200moe_ep_forward(b200moe_ep* ep, b200moe_layer* layer, void* stream, int fuse_return);
int b200moe_ep_return(b200moe_ep* ep, void* stream);
int b200moe_ep_combine_p2p(b200moe_ep* ep, void* stream, const int32_t* topk_ids, const float* topk_weights,
                           int T, int k, int num_experts, const int32_t* owner_of_expert, const float* residual,
                           float* out);
int b200moe_ep_check_errors(b200moe_ep* ep, void* stream, uint32_t* bits);
/* Synchronize; the routes received in the last step and up to max of their
 * expert ids (host memory). */
int b200moe_ep_received(b200moe_ep* ep, void* stream, int32_t* n, int32_t* expert_ids, int max);

/* Top-1 layer forward on rows that are routes (expert parallel owners): the
 * device int *n_valid (<= max_rows) says how many rows this call has,
 * row_range = {0, *n_valid}; writes the fp16 y2 row of every route (the
 * reference's y2, before any weighting) into y2 [max_rows][H].  No host sync. */
int b200moe_forward_rows(b200moe_layer* layer, void* stream, const void* rows, const int32_t* expert_ids,
                         const int32_t* n_valid, const int32_t* row_range, int max_rows, void* y2);

/* Dense tensor-core throughput of `device`, measured.  No counterpart in the
 * reference (its tensor path is V100 mma.sync): the roofline denominators of
 * this build's kernels.  kind 0 tcgen05.mma kind::f16 (N 256), 1 kind::f8f6f4
 * E4M3 (N 256), 2 kind::mxf4nvf4 block16 UE4M3 (N 128), 3 kind::mxf4nvf4
 * block32 UE8M0 (N 128), 4 kind::f16 (N 128); M 128, one CTA per SM issuing
 * `iters` x 4 MMAs on shared-memory operands.  *tflops = dense FLOP/s / 1e12,
 * *ms = the timed launch. */
int b200moe_mma_peak(int device, int kind, int iters, float* tflops, float* ms);

/* fp32 -> fp16 copy of n values (n % 4 == 0), round to nearest. */
int b200moe_f32_to_f16(void* stream, const float* x, int64_t n, void* y);

/* Packing (device arrays): fp32 W [rows][k] -> NVFP4 codes [rows][k/2],
 * E4M3 scales [rows][k/16], global (device float, one) / MXFP4 codes and E8M0
 * [rows][k/32].  Same rounding as the oracle: RNE, ties to even, saturating. */
int b200moe_quantize_nvfp4(void* stream, const float* w, int rows, int k, uint8_t* codes,
                           uint8_t* scales, float* global_scale);
int b200moe_quantize_mxfp4(void* stream, const float* w, int rows, int k, uint8_t* codes,
                           uint8_t* e8m0, uint32_t* err);
/* Exact NVFP4 -> MXFP4 fold; a block that cannot fold sets kErrRange in *err. */
int b200moe_fold_nvfp4_to_mxfp4(void* stream, const uint8_t* codes, const uint8_t* scales,
                                const float* global_scale, int rows, int k, uint8_t* out_codes,
                                uint8_t* out_e8m0, uint32_t* err);

#ifdef __cplusplus
}
#endif

#endif /* B200MOE_H_ */
