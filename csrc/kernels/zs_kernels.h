// C ABI of the zstep_b200 sm_100a kernel library.
//
// Every entry point takes raw device pointers plus a cudaStream_t and returns 0 on
// success or a negative code for a rejected argument / launch failure.  The torch
// binding layer (bindings.cpp) and any non-torch host (the C++ master's own tests,
// ctypes) call these directly.  Kernels report device-side failures (bounded waits
// that ran out, bad shapes seen on device) through the `err` word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// ----------------------------------------------------------------------------------
// MXFP8 GEMM (tcgen05 block-scaled): out[tokens, features] = act[tokens, K] . W[features, K]^T
// ----------------------------------------------------------------------------------
enum GemmEpilogue {
  kEpiStoreBf16 = 0,      // out bf16 [rows, ldo], column = feature
  kEpiStoreF32 = 1,       // out f32  [rows, ldo]
  kEpiSiluQuant = 2,      // gate/up tile pairs -> silu(g)*u -> MXFP8 out (e4m3 [rows, ldo]) + out_sf atoms
  kEpiScatterScaled = 3,  // out bf16 [row_dst[row], ldo] = acc * row_scale[row]
  kEpiArgmaxPartial = 4,  // out u64 [rows, ldo = Npad/128]: per-tile packed argmax key
  kEpiPushLL = 5,         // row-parallel partials pushed to the fused all-reduce (push_* fields)
};

typedef struct GemmMxf8Args {
  const uint8_t* a;        // weights e4m3 [groups * n_pad, k]
  const uint8_t* sfa;      // weight scale atoms [groups, n_pad/128, k/128, 512]
  const uint8_t* b;        // activations e4m3 [b_rows, k]
  const uint8_t* sfb;      // activation scale atoms [b_rows/128, k/128, 512]
  int k;
  int n_pad;               // padded features per group (multiple of 128)
  int n_valid;             // real features per group (stores skip the padding)
  int groups;
  int b_rows;              // rows of the activation buffer (multiple of 128)
  int m_rows;              // dense mode: number of token rows
  const int* group_count;  // grouped mode: [groups] tokens per group (device)
  const int* group_offset; // grouped mode: [groups] first row of each group's segment
  const int* chunk_prefix; // grouped mode: [groups+1] prefix of ceil(count/chunk_rows); NULL = dense
  int chunk_rows;          // grouped mode: rows per chunk the prefix was built for (== block_n)
  int max_items;           // grouped mode: optional cap on CTAs (0 = one per SM)
  int last_m0, last_mt;    // grouped mode: the last group computes only 128-row tiles [last_m0, last_m0 +
                           // last_mt) (last_mt 0 = all tiles; a tensor-parallel rank's slice of the shared expert)
  int block_n;             // tokens per work item: 32 (decode) or 128
  int k_splits;            // dense mode, kEpiStoreF32 only: split K into this many partials
  long long split_stride;  // elements between split partials in out
  int a_tiled;             // 1: weights pre-tiled as [groups*n_pad/128][k/128][128 rows][128 B]
  int a_fp4;               // 1: weights are packed e2m1 (MXFP4), pre-tiled [..][k/128][128 rows][64 B];
                           //    widened to e4m3 in shared memory (scales unchanged)
                           //    (each TMA box one contiguous 16 KiB block); 0: row-major
  int epi_mode;
  void* out;
  int ldo;                 // leading dimension of out in elements
  uint8_t* out_sf;         // kEpiSiluQuant: scale atoms of the quantized output
  const int* row_dst;      // kEpiScatterScaled
  const float* row_scale;  // kEpiScatterScaled
  int* err;                // device error word (may be NULL)
  // In-kernel split-K (any epilogue, dense or grouped): each output tile's K range is
  // split over fix_splits CTAs; each writes an fp32 partial to ws, and the last to
  // arrive (tile_sem counter) sums all partials in split order and runs the epilogue.
  int fix_splits;          // 1 = off; must divide k/128
  float* ws;               // >= tiles * fix_splits * 128 * block_n floats
  int* tile_sem;           // >= tiles ints, zero before the first call (kept zero after)
  int max_tiles;           // capacity of ws / tile_sem in tiles (the kernel checks)
  // kEpiArgmaxPartial sampling (optional): rows with row_temp > 0 take the argmax of
  // logit / temp + Gumbel(seed, pos, id_offset + feature), i.e. a sample from
  // softmax(logit / temp); rows with temp <= 0 stay greedy.
  const float* row_temp;
  const long long* row_seed;
  const int* row_pos;
  int id_offset;           // global id of feature 0 (vocab shard offset)
  const float* sample_any; // optional scalar: <= 0 means no row samples (skips the per-row loads)
  // kEpiPushLL: the GEMM is the producer of a tensor-parallel all-reduce (row-parallel
  // projection).  Each output value leaves the epilogue as bf16 inside an LL line (4
  // features of one token + the all-reduce call's epoch) stored straight into the receive
  // slots of zs_fused_allreduce_norm over NVLink: the row's owner (FAR_TWOSHOT) or every
  // rank (FAR_ONESHOT).  The all-reduce then runs with `pushed` set.  No fp32 partials
  // touch HBM.  Whole K per item (no split-K); n_valid = hidden, a multiple of 4.
  void* push_part[8];      // the protocol's symmetric receive buffers of every rank
  const uint32_t* push_epoch;  // that protocol's epoch counter (read, not advanced)
  int push_world, push_rank, push_rows, push_mode;
} GemmMxf8Args;

int zs_gemm_mxf8(const GemmMxf8Args* args, cudaStream_t stream);

// ----------------------------------------------------------------------------------
// MXFP8 quantization and fused norms
// ----------------------------------------------------------------------------------
// Quantize bf16 rows [rows, k] into e4m3 [rows, k] + scale atoms [ceil(rows/128), k/128, 512].
int zs_quant_mxf8(const void* x_bf16, int rows, int k, int ld_x, uint8_t* q, uint8_t* sf,
                  cudaStream_t stream);

// residual[r] = bf16(residual[r] + sum_t delta[r, t]) (if delta != NULL), then
// y = rmsnorm(residual[r]) * (w + w_offset); y written as bf16 (normed, optional) and/or
// MXFP8 (q + sf, optional).  Reduction in fp32, hidden % 2048 == 0.  Delta terms are
// bf16, or f32 when delta_f32 != 0 (split-K partials); terms are summed in index order.
// Gathered terms (optional, [rows, n_terms]): with term_index, term t of row r is row
// term_index[r*n_terms+t] of delta (negative: skipped; term_stride unused), times
// term_scale[r*n_terms+t] when term_scale is given.
int zs_add_rmsnorm_quant(void* residual, const void* delta, int n_terms, long long delta_row_stride,
                         long long delta_term_stride, int delta_f32, const int* term_index,
                         const float* term_scale, const void* weight, float w_offset,
                         float eps, int rows, int hidden, void* normed, uint8_t* q, uint8_t* sf,
                         cudaStream_t stream);

// hidden[r] = embed[ids[r]]; then as zs_add_rmsnorm_quant without delta.
int zs_embed_rmsnorm_quant(const int* ids, const void* embed, void* hidden, const void* weight,
                           float w_offset, float eps, int rows, int hidden_size, void* normed,
                           uint8_t* q, uint8_t* sf, cudaStream_t stream);

// Reduce per-tile argmax keys [rows, tiles] to a token id and its logit per row.
int zs_argmax_reduce(const unsigned long long* keys, int rows, int tiles, int* out_ids,
                     float* out_vals, unsigned long long* out_keys, cudaStream_t stream);

// ----------------------------------------------------------------------------------
// GatedDeltaNet (Qwen3.5 linear attention)
// ----------------------------------------------------------------------------------
typedef struct GdnArgs {
  const void* proj;        // bf16 [rows, ld_proj]: [q | k | v | z | b | a] per the layout below
  int ld_proj;
  int num_k_heads;         // local q/k heads
  int num_v_heads;         // local v heads (multiple of num_k_heads)
  int head_k;              // 128
  int head_v;              // 128
  const void* conv_w;      // bf16 [conv_dim, 4]; conv_dim = 2*Hk*dk + Hv*dv
  void* conv_state;        // bf16 [slots, 2, conv_dim, 3] (double-buffered by position parity)
  float* ssm_state;        // f32  [slots, Hv, dv, dk]  (row v holds the dk coefficients)
  const float* a_log;      // [Hv]
  const float* dt_bias;    // [Hv]
  const void* norm_w;      // bf16 [dv] gated RMSNorm weight
  float eps;
  const int* slots;        // [rows] state slot of each row
  const int* positions;    // [rows] position of the row's token (0 => fresh state)
  int rows;
  void* out_bf16;          // optional bf16 [rows, Hv*dv]
  uint8_t* out_q;          // optional MXFP8 [rows_pad, Hv*dv]
  uint8_t* out_sf;         //   + scale atoms
  // Prefill (varlen) extension: rows grouped into sequences.
  const int* seq_start;    // [num_seqs+1] row ranges (prefill only)
  int num_seqs;
  const int* ckpt_rows;    // prefill: [num_seqs * max_ckpt] row index after which to snapshot (-1 none)
  const int* ckpt_slots;   // prefill: matching checkpoint slot ids
  int max_ckpt;
  int* err;
  const int* out_slots;    // prefill: optional [num_seqs] slot receiving the final state (and
                           // conv window) instead of the input slot, which stays untouched
  int impl;                // prefill: 0 = by length (chunked for >= 16 rows per sequence on
                           // average), 1 = token-sequential, 2 = chunked
  int max_seq_rows;        // prefill: rows per sequence are at most this (0: unknown).  With
                           // impl 0, 1..ZS_GDN_ROWS_MAX and no checkpoints the rows run on the
                           // streaming decode kernel (speculative verify and replay)
} GdnArgs;

#define ZS_GDN_ROWS_MAX 4

int zs_gdn_decode(const GdnArgs* args, cudaStream_t stream);
int zs_gdn_decode_rows(const GdnArgs* args, cudaStream_t stream);
int zs_gdn_prefill(const GdnArgs* args, cudaStream_t stream);

// ----------------------------------------------------------------------------------
// Gated GQA attention (Qwen3.5 full-attention layers), paged KV, 16-token pages
// ----------------------------------------------------------------------------------
typedef struct AttnArgs {
  const void* qkv;         // bf16 [rows, ld_qkv]: per q head [q(256) | gate(256)], then K heads, V heads
  int ld_qkv;
  int num_q_heads;         // local
  int num_kv_heads;        // local
  int head_dim;            // 256
  int rotary_dim;          // 64 (partial rope on the first rotary_dim dims)
  float rope_theta;
  const void* q_norm_w;    // bf16 [head_dim] (zero-centered: scale = 1 + w)
  const void* k_norm_w;
  float eps;
  void* k_cache;           // bf16 [pages, kv_heads, 16 x 256] pre-swizzled blocks (attention.cu)
  void* v_cache;
  int page_size;
  const int* page_table;   // [slots, max_pages]
  int max_pages;
  const int* slots;        // [rows]
  const int* positions;    // [rows]
  int rows;
  void* q_out;             // bf16 [rows, Hq, head_dim] (normed + roped)
  void* gate_out;          // bf16 [rows, Hq, head_dim]
  // decode
  const int* seq_lens;     // [rows] context length including the current token
  float* partial;          // split-K scratch
  int num_splits;
  float sm_scale;
  void* out_bf16;          // [rows, Hq*head_dim] gated attention output
  uint8_t* out_q;          // optional MXFP8 output
  uint8_t* out_sf;
  // prefill varlen
  const int* seq_start;    // [num_seqs+1]
  int num_seqs;
  int* err;
  int impl;                // 0: tensor cores for GQA groups of 4..16 heads, else SIMT; 1: SIMT; 2: tensor cores
} AttnArgs;

int zs_attn_prologue(const AttnArgs* args, cudaStream_t stream);
int zs_attn_decode(const AttnArgs* args, cudaStream_t stream);
int zs_attn_prefill(const AttnArgs* args, cudaStream_t stream);

// Allocation-free variant of zs_attn_decode (no counterpart in the reference): same inputs
// and outputs, `partial` is ignored and the split-KV records go to a fixed device array of
// ZS_ATTN_NOALLOC_SCRATCH_FLOATS floats inside this library, for callers that cannot
// allocate device memory when they call.  Returns 0 on success, -3 when
// rows * num_q_heads * num_splits * 260 exceeds that size (nothing is launched), -4 when the
// array's address cannot be looked up, and zs_attn_decode's codes otherwise.  All calls on
// a device share the array: calls that overlap in time race.  The first call on a device
// does a one-time address lookup; make it before any stream capture.
#define ZS_ATTN_NOALLOC_SCRATCH_FLOATS (2 * 1024 * 1024)
int zs_attn_decode_noalloc(const AttnArgs* args, cudaStream_t stream);

// ----------------------------------------------------------------------------------
// MoE routing
// ----------------------------------------------------------------------------------
typedef struct MoeRouteArgs {
  const float* logits;     // f32 [rows, ld_logits]: router logits (num_experts) then shared-gate logit
  int ld_logits;
  int logit_splits;        // split-K partials of the router GEMM (summed in order); <= 1: one
  long long logit_split_stride;
  int chunk_rows;          // chunk size of the consuming grouped GEMM (32 or 128)
  int rows;
  int num_experts;         // routed experts (global)
  int top_k;
  int norm_topk;           // renormalise the top-k weights to sum 1
  int scoring;             // 0 = softmax, 1 = sigmoid, 2 = sqrt(softplus) (1, 2: + bias, grouped)
  const float* bias;       // sigmoid scoring: per-expert correction bias (may be NULL)
  int n_group, topk_group; // grouped routing (sigmoid scoring)
  float routed_scale;
  int shared_gate_col;     // column of the shared-expert gate logit (-1: shared weight 1)
  int expert_begin;        // experts [expert_begin, expert_end) are local (EP); others dropped
  int expert_end;
  int has_shared;          // local group `expert_end - expert_begin` is the shared expert
  // outputs
  int* topk_ids;           // [rows, top_k] global expert ids
  float* topk_w;           // [rows, top_k]
  int* group_count;        // [G] G = local experts (+1 if shared)
  int* group_offset;       // [G]
  int* chunk_prefix;       // [G+1]
  int* pair_slot;          // [rows, top_k + 1] row in the grouped buffer (-1 if not local)
  int* row_dst;            // [grouped rows] destination pair row (token * (top_k+1) + j)
  float* row_scale;        // [grouped rows] routing weight
  int max_grouped_rows;
  // activation scatter
  const uint8_t* x_q;      // [rows, hidden] e4m3
  const uint8_t* x_sf;     // scale atoms of x
  int hidden;
  uint8_t* xg_q;           // [max_grouped_rows, hidden]
  uint8_t* xg_sf;          // atoms
  int* err;
  int* pair_src;           // optional [rows, top_k+1]: grouped row of each (token, pair), -1 = none
  float* pair_w;           // optional [rows, top_k+1]: routing weight of each pair
} MoeRouteArgs;

int zs_moe_route(const MoeRouteArgs* args, cudaStream_t stream);

// ----------------------------------------------------------------------------------
// Fused tensor-parallel collectives over NVLink peer memory (symmetric buffers)
// ----------------------------------------------------------------------------------
#define FAR_CTAS 128  // grid of the two-shot all-reduces (co-resident; CTA c pairs with CTA c of every rank)

// Protocols of zs_fused_allreduce_norm (the host picks one per call from the row count):
//   FAR_ONESHOT  : every rank pushes its rows to every rank as 16-byte LL lines (two bf16
//                  pairs + the call's epoch twice); one NVLink hop, parity-double-buffered.
//   FAR_TWOSHOT  : LL lines to the row's owner, owner reduces and pushes the result to all.
//   FAR_PLAIN    : two-shot with plain bf16 rows (no flag words: full link bandwidth); per
//                  (source, CTA) flags published with a system-scope release after the
//                  data, for prefill-sized reductions.
//   FAR_NVLS     : NVLink SHARP through an NVSwitch multicast object: every rank stores its
//                  local sums into its own multicast-bound buffer; each rank reduces its
//                  column slice of every row with multimem.ld_reduce (the switch adds the
//                  ranks' copies) and broadcasts the result with multimem.st.  Two
//                  multicast-counter barriers per call.
#define FAR_ONESHOT 0
#define FAR_TWOSHOT 1
#define FAR_PLAIN 2
#define FAR_NVLS 3
#define FAR_ONESHOT_ROWS 64  // capacity (rows) of the one-shot buffers

typedef struct FusedArArgs {
  int rank, world;
  int protocol;              // FAR_ONESHOT / FAR_TWOSHOT / FAR_PLAIN / FAR_NVLS
  const void* delta;         // local partial terms: delta[row*row_stride + t*term_stride + col]
  int n_terms;
  const int* term_index;     // optional gathered terms (as in zs_add_rmsnorm_quant)
  const float* term_scale;
  long long row_stride, term_stride;
  int delta_f32;             // terms are f32 (split-K partials) or bf16 (MoE pair rows)
  // Symmetric buffers (per rank, this protocol's area):
  //   ONESHOT: part = LL lines [2 parities][world][FAR_ONESHOT_ROWS][hidden/4]
  //   TWOSHOT: part = LL lines [world][ceil(rows/world)][hidden/4], out = LL lines [rows][hidden/4]
  //   PLAIN  : part = bf16 [world][ceil(rows/world)][hidden],       out = bf16 [rows][hidden]
  //   NVLS   : part = bf16 [rows][hidden], out = bf16 [rows][hidden], flags = u32 [2][FAR_CTAS];
  //            only this rank's entries are used, the peers' copies are reached through
  //            the multicast addresses below
  void* part[8];
  void* out[8];
  uint32_t* flags[8];        // PLAIN: u32 [2][world][FAR_CTAS] per rank (phase, source, CTA)
  void* mc_part;             // NVLS: multicast addresses of the part / out / flags areas
  void* mc_out;
  uint32_t* mc_flags;
  uint32_t* epoch;           // local device counter of this protocol (same sequence on every rank)
  uint32_t* grid_counter;    // local device counter: the last CTA of a call advances the epoch
  void* residual;            // bf16 [rows, hidden], replicated residual stream (in/out)
  const void* weight;        // RMSNorm weight
  float w_offset, eps;
  int rows, hidden;
  int pushed;                // 1: a kEpiPushLL GEMM already delivered this rank's lines (ONESHOT / TWOSHOT)
  void* normed;              // optional bf16 output
  uint8_t* q;                // optional MXFP8 output + scale atoms
  uint8_t* sf;
  int* err;
  unsigned int timeout_ms;   // bound on every cross-rank wait (0: 5000 ms)
} FusedArArgs;

int zs_fused_allreduce_norm(const FusedArArgs* args, cudaStream_t stream);

// In-place fp32 sum over ranks of data[rows, cols] (one-shot push over NVLink, summed in
// rank order so every rank gets the same bits).  buf: symmetric LL lines (two floats +
// epoch twice, 16 bytes) [2 parities][world][max_rows * cols / 2] per rank.
typedef struct SumArArgs {
  int rank, world;
  float* data;
  int rows, cols, max_rows;
  void* buf[8];
  uint32_t* epoch;
  uint32_t* grid_counter;
  int* err;
  unsigned int timeout_ms;
  // Plain two-shot (rows above the one-shot capacity; set plain = 1): fp32 rows through
  // part [world][ceil(rows/world)][cols] and out [rows][cols] per rank, with per-(source,
  // CTA) release/acquire flags [2][8][FAR_CTAS] (the FAR_PLAIN scheme).
  int plain;
  void* part[8];
  void* out[8];
  uint32_t* flags[8];
} SumArArgs;

#define SUM_CTAS 148  // grid of zs_allreduce_sum_f32

int zs_allreduce_sum_f32(const SumArArgs* args, cudaStream_t stream);

// Global greedy / sampled token over vocab shards in one kernel: each row's per-tile keys
// of this rank's shard are max-reduced, rebased to global ids, pushed to every rank as one
// LL line ([2 parities][world][max_rows] lines of 16 bytes per rank) and max-reduced over
// the ranks.  Every rank ends with the same ids.
typedef struct ArgmaxArArgs {
  int rank, world, rows, max_rows;
  const unsigned long long* tile_keys;  // this rank's [rows, tiles] packed keys (local ids)
  int tiles;
  int id_offset;             // global id of this rank's first vocab entry
  void* lines[8];            // symmetric LL line buffers
  uint32_t* epoch;           // its own counter
  uint32_t* grid_counter;
  int* out_ids;
  float* out_vals;
  int* err;
  unsigned int timeout_ms;   // bound on every cross-rank wait (0: 5000 ms)
} ArgmaxArArgs;

int zs_allreduce_argmax(const ArgmaxArArgs* args, cudaStream_t stream);

// ----------------------------------------------------------------------------------
// Expert-parallel MoE all-to-all over NVLink peer memory (ep.cu)
// ----------------------------------------------------------------------------------
// Rank r owns the routed experts [r * E / W, (r + 1) * E / W).  Every rank's symmetric
// block holds (byte offsets below, identical on every rank):
//   flags  u32 [64]                    arrival words: [0, 8) dispatch, [8, 16) combine (by source)
//   counts uint2 [W][E]                (pair count, epoch) of every source for every expert
//   q      e4m3 [recv_cap][hidden]     received rows, grouped by local expert (128-row aligned)
//   sf     scale atoms of q            tcgen05 block-scale layout of the grouped GEMM
//   meta   int2 [recv_cap]             (source << 24 | token * top_k + k, weight bits); -1 = padding
//   comb   bf16 [max_tokens * top_k][hidden]  expert outputs returned to their source
#define EP_MAX_WORLD 8
#define EP_MAX_EXPERTS 1024

typedef struct EpArgs {
  int rank, world;
  int tokens;                  // local tokens of this call (<= max_tokens, may be 0)
  int max_tokens;              // per-rank capacity (same on every rank)
  int hidden;                  // multiple of 512
  int top_k;                   // <= 16
  int num_experts;             // global routed experts, a multiple of world, <= EP_MAX_EXPERTS
  int recv_cap;                // rows of q / meta (multiple of 128)
  int chunk_rows;              // 32 or 128: work chunk of the consuming grouped GEMM
  const int* topk_ids;         // [tokens, top_k] global expert ids (-1: no expert)
  const float* topk_w;         // [tokens, top_k]
  const void* x;               // bf16 [tokens, hidden]: quantized to MXFP8 on the way out
  char* sym[EP_MAX_WORLD];     // every rank's symmetric block
  long long off_flags, off_counts, off_q, off_sf, off_meta, off_comb;
  // rank-local scratch (zeroed once at allocation; the kernels keep it consistent)
  int* cnt;                    // [num_experts]
  int* pair_slot;              // [max_tokens * top_k]
  unsigned long long* bar;     // grid-barrier counter
  uint32_t* epoch;             // [2]: dispatch, combine (advanced by the kernels)
  // dispatch outputs for the local grouped GEMM (the format of zs_moe_route)
  int* group_count;            // [E / W]
  int* group_offset;           // [E / W]
  int* chunk_prefix;           // [E / W + 1]
  int* recv_rows;              // [1]: padded rows of the grouped buffer
  // combine
  const void* y;               // bf16 [y_rows, ldy]: expert outputs in receive order
  long long ldy;
  int y_rows;                  // rows of y (a combine with more received rows reports kErrBadShape)
  const void* residual;        // optional bf16 [tokens, hidden] added to the weighted sum
  void* out;                   // bf16 [tokens, hidden]
  int* err;
  unsigned int timeout_ms;     // bound on every cross-rank wait (0: 5 s)
} EpArgs;

// Dispatch: MXFP8-quantize each token row once and store it over NVLink into the grouped
// receive buffer of every rank that owns one of its top-k experts; counts travel first
// so every sender knows every receiver's segment layout.  Returns when this rank's
// receive buffer is complete.  One cooperative launch.
int zs_ep_dispatch(const EpArgs* args, cudaStream_t stream);
// Combine: return every received row's expert output to its source, then each source
// sums its tokens' top-k outputs in k order with their routing weights (+ residual).
int zs_ep_combine(const EpArgs* args, cudaStream_t stream);

// ----------------------------------------------------------------------------------
// DeepSeek-style layers: mHC, MLA, DSA indexer, MoE combine (deepseek.cu)
// ----------------------------------------------------------------------------------
typedef struct MhcPartialArgs {
  float* x;                   // fp32 [rows, 4, hidden] residual streams (read; written in modes 1, 2)
  int rows, hidden;
  int m;                      // mixing logits of the site: 24 (pre|post|res) or 4 (final collapse)
  const float* fn;            // fp32 [m, 4 * hidden]
  int mode;                   // 0: X as is; 1: apply the previous site's update; 2: X = embed[ids]
  const float* y;             // mode 1: fp32 [rows, hidden] sublayer output (bf16-rounded on use)
  const float* mix_prev;      // mode 1: [rows, 4 + 16] post | res of the previous site
  const int* ids;             // mode 2
  const __nv_bfloat16* embed; // mode 2: [vocab, hidden]
  float* partial;             // [rows, slices, m + 1]
} MhcPartialArgs;

typedef struct MhcFinalizeArgs {
  const float* x;             // [rows, 4, hidden]
  int rows, hidden, m, slices;
  const float* partial;       // [rows, slices, m + 1]
  const float* base;          // [m]
  const float* scale;         // [3] (or [1] for the final collapse)
  float eps;
  int sinkhorn_iters;
  float* mix_out;             // m == 24: [rows, 4 + 16] post | res
  const __nv_bfloat16* weight;  // RMSNorm scale [hidden] (plain, no offset)
  uint8_t* q;                 // MXFP8 [rows, hidden] of rmsnorm(pre @ X)
  uint8_t* sf;
} MhcFinalizeArgs;

int zs_mhc_partial(const MhcPartialArgs* args, cudaStream_t stream);
int zs_mhc_slices(int hidden);
int zs_mhc_finalize(const MhcFinalizeArgs* args, cudaStream_t stream);

// RMSNorm (plain scale) of a strided bf16 slice of `width` columns, then MXFP8.
int zs_rms_quant(const void* x, int ld_x, int width, const void* w, float eps, int rows, uint8_t* q, uint8_t* sf,
                 cudaStream_t stream);

typedef struct MlaPrologueArgs {
  const __nv_bfloat16* proj;  // [rows, ld_proj]: q_a | kv_a (kv_lora + rope) | index k | index weights
  int ld_proj, off_kva, off_ik, off_iw;
  const __nv_bfloat16* qi;    // [rows, ld_qi]: local heads x (nope | rope) then index queries
  int ld_qi, off_iq;
  int rows, heads, qk_dim, nope, rope, kv_lora, index_heads, index_dim;
  const __nv_bfloat16* kv_norm;   // [kv_lora]
  const __nv_bfloat16* ik_norm;   // [index_dim]
  float eps, theta, iw_scale;
  const int* slot;
  const int* pos;
  const int* page_table;
  int max_pages, page_size;
  __nv_bfloat16* ckv_cache;   // [pages, page_size, kv_lora + rope]
  __nv_bfloat16* ik_cache;    // [pages, page_size, index_dim]
  __nv_bfloat16* q_pe;        // [rows, heads, rope]
  __nv_bfloat16* iq;          // [rows, index_heads, index_dim]
  float* iw;                  // [rows, index_heads]
} MlaPrologueArgs;

int zs_mla_prologue(const MlaPrologueArgs* args, cudaStream_t stream);
int zs_mla_absorb_q(const void* qi, int ld_qi, int qk_dim, int nope, const void* w_uk, int kv_lora, int heads,
                    int rows, void* q_lat, cudaStream_t stream);

typedef struct MlaAttnArgs {
  const __nv_bfloat16* q_lat;  // [rows, heads, kv_lora]
  const __nv_bfloat16* q_pe;   // [rows, heads, rope]
  const __nv_bfloat16* ckv_cache;
  const int* page_table;
  int max_pages, page_size;
  const int* slot;
  const int* sel;              // [rows, ld_sel] selected positions (ascending)
  int ld_sel;
  const int* n_sel;            // [rows]
  int rows, heads, kv_lora, rope, splits;
  float sm_scale;
  float* partial;              // [rows, heads, splits, kv_lora + 4]
  int impl;                    // 0 / 1: SIMT kernel; 2: tensor cores (tcgen05)
  int* err;                    // optional error word (bounded mbarrier waits of impl 2)
} MlaAttnArgs;

size_t zs_mla_attn_smem(int heads);
int zs_mla_attn(const MlaAttnArgs* args, cudaStream_t stream);

typedef struct MlaUpArgs {
  const float* partial;        // from zs_mla_attn
  int rows, heads, splits, v_dim;
  const __nv_bfloat16* w_uv_t; // [heads, kv_lora, v]
  uint8_t* q;                  // MXFP8 [rows, heads * v]
  uint8_t* sf;
} MlaUpArgs;

int zs_mla_up(const MlaUpArgs* args, cudaStream_t stream);

typedef struct DsaScoresArgs {
  const __nv_bfloat16* iq;     // [rows, index_heads, 128]
  const float* iw;             // [rows, index_heads]
  const __nv_bfloat16* ik_cache;
  const int* page_table;
  int max_pages, page_size;
  const int* slot;
  const int* ctx_len;          // [rows] keys visible to each row (position + 1)
  int rows, index_heads, topk;
  float scale;
  float* scores;               // [rows, ld_scores]
  int ld_scores;
  int* err;                    // bounded-wait failures
} DsaScoresArgs;

typedef struct DsaTopkArgs {
  const float* scores;
  int ld_scores;
  const int* ctx_len;
  int rows, topk;
  int* sel;                    // [rows, ld_sel]
  int ld_sel;
  int* n_sel;
} DsaTopkArgs;

int zs_dsa_scores(const DsaScoresArgs* args, int max_ctx, cudaStream_t stream);
int zs_dsa_topk(const DsaTopkArgs* args, cudaStream_t stream);

// y[t] = sum_j w[t, j] * rows_in[src[t, j]] (fp32; src -1 skipped; fixed order).
int zs_gather_sum(const void* rows_in, const int* src, const float* w, int k1, int hidden, int rows, float* y,
                  cudaStream_t stream);

// ----------------------------------------------------------------------------------
// Full-distribution sampling (sampling.cu)
// ----------------------------------------------------------------------------------
typedef struct SampleArgs {
  float* logits;               // fp32 [rows, ld], whole vocabulary (penalties are applied in place)
  int ld, vocab, rows;
  const float* temperature;    // [rows]; <= 0: greedy
  const int* top_k;            // [rows]; 0: off (may be NULL)
  const float* top_p;          // [rows]; 1: off (may be NULL)
  const float* presence;       // [rows] (may be NULL)
  const float* frequency;      // [rows] (may be NULL)
  const float* repetition;     // [rows] (may be NULL; 1 = off)
  const unsigned long long* seed;  // [rows] draw seed
  const int* hist;             // [rows, hist_ld] generated-token history (may be NULL)
  int hist_ld;
  const int* hist_len;         // [rows]
  int want_logprobs;           // 1: chosen-token logprob and top_n logprobs of the raw logits
  int top_n;                   // <= 5
  int* out_token;              // [rows]
  float* out_logprob;          // [rows]
  int* out_top_ids;            // [rows, 5]
  float* out_top_lp;           // [rows, 5]
} SampleArgs;

int zs_sample(const SampleArgs* args, cudaStream_t stream);

// On-device greedy verify of a speculative step (n sequences x (k+1) rows); see sampling.cu.
typedef struct SpecVerifyArgs {
  int n, k, dummy_slot;
  const int* ids;       // [n*(k+1)] row tokens: last accepted token, then k drafts
  const int* targets;   // [n*(k+1)] target greedy token after each row
  const int* pos;       // [n*(k+1)] row positions
  const int* slot;      // [n*(k+1)] row slots
  int* record;          // [n, k+2] out: acc_len, then k+1 accepted tokens (-1 padded)
  int* rep_start;       // [n+1] out: replay row ranges (compacted)
  long long* rep_idx;   // [n*(k+1)] out: source row of each replay row
  int* rep_slot;        // [n*(k+1)] out
  int* rep_pos;         // [n*(k+1)] out
  int* mtp_ids;         // [n*(k+1)] out: draft-head catch-up rows (padding rows -> dummy slot)
  int* mtp_pos;
  int* mtp_slot;
  int* mtp_len;
  long long* last_row;  // [n] out: catch-up row of each sequence's newest token
} SpecVerifyArgs;

int zs_spec_verify(const SpecVerifyArgs* args, cudaStream_t stream);

// Programmatic dependent launch of the compute kernels (on by default).
void zs_set_pdl(int on);
int zs_pdl_enabled();

int zs_symm_alloc(size_t bytes, void** ptr);
int zs_symm_free(void* ptr);
int zs_ipc_handle(void* ptr, void* handle_out);
int zs_ipc_open(const void* handle, void** ptr);
int zs_ipc_close(void* ptr);

#ifdef __cplusplus
}
#endif
