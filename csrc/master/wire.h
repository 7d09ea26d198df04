// Shared-memory ABI between the zstep master and its GPU worker processes.
//
// One POSIX shared-memory segment holds:
//   [0, 4096)                superblock (magic, version, geometry, layout hash, abort word)
//   [4096, 8192)             kMaxWorkers worker status records (64 bytes each)
//   plan slots  x kPlanSlots  StepHeader + 256-byte aligned arrays (tokens, positions, ...)
//   result slots x kResultSlots StepResultHeader + per-sequence SeqStepOutput records
// Plan/result slots are double-buffered so the master can stage step N+1 while the
// workers execute step N.  A slot is published by a release store of its step_id after
// every other field is written; readers acquire-load step_id first.
//
// Workers refuse a segment whose magic, version or layout hash differ from their own,
// so master and worker builds can never disagree silently about offsets.  The Python
// mirror (zstep_b200/runtime/wire.py) computes the same layout and hash; a golden test
// checks both against each other.
//
// Reference parity: crates/zs-wire/src/lib.rs (superblock, worker slot state, step
// header/plan layout, decode buckets, flags, opcodes, FNV-1a layout hash).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <cstring>

namespace zs {
namespace wire {

constexpr uint64_t kMagic = 0x3030324253545A5AULL;  // "ZZTSB200" little-endian
constexpr uint32_t kVersion = 1;
constexpr int kMaxWorkers = 8;
constexpr int kPlanSlots = 2;
constexpr int kResultSlots = 2;
constexpr int kMaxSpecTokens = 8;   // verify width / accepted tokens per sequence per step
constexpr int kMaxTopLogprobs = 5;
constexpr size_t kSuperblockBytes = 4096;
constexpr size_t kWorkerRegionBytes = 4096;
constexpr size_t kWorkerStateBytes = 64;
constexpr size_t kAbortOffset = 128;
constexpr size_t kAlign = 256;

// Step header flags.
constexpr uint32_t kFlagDecodeOnly = 1u << 0;      // every row is a single decode token
constexpr uint32_t kFlagDeviceTokens = 1u << 1;    // inputs = last tokens kept on device
constexpr uint32_t kFlagNextPublished = 1u << 2;   // step N+1 is published before N is read
constexpr uint32_t kFlagSampling = 1u << 3;        // some sequence samples stochastically
constexpr uint32_t kFlagPenalty = 1u << 4;         // some sequence uses presence/frequency penalty
constexpr uint32_t kFlagSpecVerify = 1u << 5;      // rows carry [last token, drafts...] per sequence
constexpr uint32_t kFlagLogprobs = 1u << 6;        // some sequence wants logprobs

enum Opcode : uint32_t {
  kOpNormal = 0,
  kOpWarmup = 1,
  kOpReload = 2,
  kOpKvTransfer = 3,
  kOpShutdown = 4,
};

enum WorkerStatus : uint32_t {
  kWorkerStarting = 0,
  kWorkerReady = 1,
  kWorkerRunning = 2,
  kWorkerExited = 3,
  kWorkerError = 99,
};

// Decode CUDA-graph batch buckets (padded batch sizes the workers capture).
constexpr std::array<uint32_t, 19> kDecodeBuckets = {1,   2,   4,   8,   16,  24,  32,  48,  64, 96,
                                                     128, 160, 192, 224, 256, 320, 384, 448, 512};

inline uint32_t select_bucket(uint32_t n) {
  for (uint32_t b : kDecodeBuckets)
    if (b >= n) return b;
  return 0;  // larger than every bucket: run eagerly
}

struct alignas(64) Superblock {
  uint64_t magic;
  uint32_t version;
  uint32_t layout_hash;
  uint32_t world_size;
  uint32_t max_seqs;
  uint32_t max_step_tokens;
  uint32_t max_pages_per_seq;
  uint32_t page_size;
  uint32_t vocab_size;
  uint64_t plan_offset;
  uint64_t plan_slot_bytes;
  uint64_t result_offset;
  uint64_t result_slot_bytes;
  uint64_t total_bytes;
  uint32_t master_pid;
  uint32_t reserved0;
  uint8_t pad[kAbortOffset - 88];
  uint32_t abort_word;  // at kAbortOffset: nonzero => every worker stops
};
static_assert(offsetof(Superblock, abort_word) == kAbortOffset, "abort word offset");
static_assert(sizeof(Superblock) <= kSuperblockBytes, "superblock size");

struct alignas(64) WorkerState {
  uint32_t status;
  uint32_t error_code;
  uint64_t ready_step;     // last step id whose execution finished
  uint64_t heartbeat_ns;   // CLOCK_MONOTONIC, refreshed by the worker's watchdog thread
  uint32_t pid;
  uint32_t rank;
  uint64_t gpu_exec_us;    // device time of the last step
  uint8_t pad[kWorkerStateBytes - 40];
};
static_assert(sizeof(WorkerState) == kWorkerStateBytes, "worker state size");

struct alignas(64) StepHeader {
  uint64_t step_id;        // published last (release); 0 = never published
  uint32_t opcode;
  uint32_t flags;
  uint32_t num_rows;       // token rows in this step
  uint32_t num_seqs;       // sequences (query_start has num_seqs + 1 entries)
  uint32_t num_dirty_rows; // page-table rows updated by this step
  uint32_t bucket;         // decode graph bucket (0 = eager)
  uint32_t num_ckpt;       // recurrent-state checkpoint saves requested
  uint32_t num_kv_ops;     // KvTransfer ops
  uint64_t master_ns;      // master clock at publish
  uint8_t pad[64 - 48];
};
static_assert(sizeof(StepHeader) == 64, "step header size");

// Sampling parameters of one sequence (indexed by its row in seq arrays).
struct SamplingParams {
  float temperature;   // 0 => greedy
  float top_p;
  int32_t top_k;       // 0 => disabled
  float presence_penalty;
  float frequency_penalty;
  float repetition_penalty;
  uint64_t seed;
  int32_t logprobs;    // number of top logprobs requested (0..kMaxTopLogprobs), -1 none
  int32_t pad;
};
static_assert(sizeof(SamplingParams) == 40, "sampling params size");

struct alignas(64) StepResultHeader {
  uint64_t step_id;     // published last (release) by rank 0
  uint32_t status;      // 0 ok
  uint32_t num_seqs;
  uint64_t gpu_exec_us;
  uint8_t pad[64 - 24];
};
static_assert(sizeof(StepResultHeader) == 64, "result header size");

struct SeqStepOutput {
  int32_t req_slot;
  int32_t num_tokens;                   // accepted tokens this step (>= 1 when sampling)
  int32_t tokens[kMaxSpecTokens];
  float logprobs[kMaxSpecTokens];
  int32_t top_ids[kMaxTopLogprobs];
  float top_logprobs[kMaxTopLogprobs];
  int32_t next_drafts[kMaxSpecTokens];  // drafts proposed for the next verify step
  int32_t num_drafts;
  int32_t pad;
};
static_assert(sizeof(SeqStepOutput) == 4 * (4 + 3 * kMaxSpecTokens + 2 * kMaxTopLogprobs), "output size");

// Offsets (from the slot base) of the arrays in one plan slot.
struct PlanLayout {
  size_t header = 0;
  size_t token_ids = 0;      // i32 [max_step_tokens]
  size_t positions = 0;      // i32 [max_step_tokens]
  size_t row_slot = 0;       // i32 [max_step_tokens] request slot of each row
  size_t query_start = 0;    // i32 [max_seqs + 1]   row range of each sequence
  size_t seq_slot = 0;       // i32 [max_seqs]       request slot of each sequence
  size_t seq_len = 0;        // i32 [max_seqs]       context length after this step
  size_t sample_row = 0;     // i32 [max_seqs]       row whose logits are sampled (-1: none)
  size_t sampling = 0;       // SamplingParams [max_seqs]
  size_t dirty_rows = 0;     // i32 [max_seqs]       page-table rows (request slots) updated
  size_t dirty_pages = 0;    // i32 [max_seqs * max_pages_per_seq]
  size_t ckpt_row = 0;       // i32 [max_ckpt]       rows after which state is snapshotted
  size_t ckpt_slot = 0;      // i32 [max_ckpt]       checkpoint slot of each snapshot
  size_t restore_slot = 0;   // i32 [max_seqs]       checkpoint slot to restore before the seq (-1)
  size_t spec_width = 0;     // i32 [max_seqs]       verify rows of the seq (0 = not a verify seq)
  size_t kv_ops = 0;         // i32 [max_kv_ops * 3] (direction, device page, host slot)
  size_t bytes = 0;
  uint32_t max_ckpt = 0;
  uint32_t max_kv_ops = 0;
};

struct ResultLayout {
  size_t header = 0;
  size_t outputs = 0;  // SeqStepOutput [max_seqs]
  size_t bytes = 0;
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline PlanLayout plan_layout(uint32_t max_seqs, uint32_t max_step_tokens, uint32_t max_pages_per_seq) {
  PlanLayout l;
  size_t o = 0;
  auto put = [&](size_t& field, size_t bytes) {
    o = align_up(o, kAlign);
    field = o;
    o += bytes;
  };
  l.max_ckpt = max_step_tokens < 4096 ? max_step_tokens : 4096;
  l.max_kv_ops = 1024;
  put(l.header, sizeof(StepHeader));
  put(l.token_ids, 4ull * max_step_tokens);
  put(l.positions, 4ull * max_step_tokens);
  put(l.row_slot, 4ull * max_step_tokens);
  put(l.query_start, 4ull * (max_seqs + 1));
  put(l.seq_slot, 4ull * max_seqs);
  put(l.seq_len, 4ull * max_seqs);
  put(l.sample_row, 4ull * max_seqs);
  put(l.sampling, sizeof(SamplingParams) * max_seqs);
  put(l.dirty_rows, 4ull * max_seqs);
  put(l.dirty_pages, 4ull * max_seqs * max_pages_per_seq);
  put(l.ckpt_row, 4ull * l.max_ckpt);
  put(l.ckpt_slot, 4ull * l.max_ckpt);
  put(l.restore_slot, 4ull * max_seqs);
  put(l.spec_width, 4ull * max_seqs);
  put(l.kv_ops, 12ull * l.max_kv_ops);
  l.bytes = align_up(o, 4096);
  return l;
}

inline ResultLayout result_layout(uint32_t max_seqs) {
  ResultLayout l;
  l.header = 0;
  l.outputs = kAlign;
  l.bytes = align_up(kAlign + sizeof(SeqStepOutput) * max_seqs, 4096);
  return l;
}

struct Geometry {
  uint32_t world_size = 1;
  uint32_t max_seqs = 256;
  uint32_t max_step_tokens = 8192;
  uint32_t max_pages_per_seq = 256;
  uint32_t page_size = 16;
  uint32_t vocab_size = 0;
};

struct SegmentLayout {
  Geometry geo;
  PlanLayout plan;
  ResultLayout result;
  size_t plan_offset = 0;
  size_t result_offset = 0;
  size_t total_bytes = 0;
};

inline SegmentLayout segment_layout(const Geometry& g) {
  SegmentLayout s;
  s.geo = g;
  s.plan = plan_layout(g.max_seqs, g.max_step_tokens, g.max_pages_per_seq);
  s.result = result_layout(g.max_seqs);
  s.plan_offset = kSuperblockBytes + kWorkerRegionBytes;
  s.result_offset = s.plan_offset + kPlanSlots * s.plan.bytes;
  s.total_bytes = s.result_offset + kResultSlots * s.result.bytes;
  return s;
}

// FNV-1a (32-bit) over the little-endian u64 encoding of every layout number, in a
// fixed order.  The Python mirror hashes the same sequence.
inline uint32_t fnv1a_u64s(const uint64_t* v, size_t n) {
  uint32_t h = 2166136261u;
  for (size_t i = 0; i < n; ++i)
    for (int b = 0; b < 8; ++b) {
      h ^= static_cast<uint8_t>(v[i] >> (8 * b));
      h *= 16777619u;
    }
  return h;
}

inline uint32_t layout_hash(const SegmentLayout& s) {
  const PlanLayout& p = s.plan;
  const uint64_t v[] = {kVersion,
                        sizeof(Superblock),
                        sizeof(WorkerState),
                        sizeof(StepHeader),
                        sizeof(SamplingParams),
                        sizeof(StepResultHeader),
                        sizeof(SeqStepOutput),
                        kAbortOffset,
                        s.geo.world_size,
                        s.geo.max_seqs,
                        s.geo.max_step_tokens,
                        s.geo.max_pages_per_seq,
                        s.geo.page_size,
                        p.token_ids,
                        p.positions,
                        p.row_slot,
                        p.query_start,
                        p.seq_slot,
                        p.seq_len,
                        p.sample_row,
                        p.sampling,
                        p.dirty_rows,
                        p.dirty_pages,
                        p.ckpt_row,
                        p.ckpt_slot,
                        p.restore_slot,
                        p.spec_width,
                        p.kv_ops,
                        p.bytes,
                        s.result.outputs,
                        s.result.bytes,
                        s.plan_offset,
                        s.result_offset,
                        s.total_bytes};
  return fnv1a_u64s(v, sizeof(v) / sizeof(v[0]));
}

// Release/acquire helpers on 64-bit words living in shared memory.
inline void store_release_u64(uint64_t* p, uint64_t v) {
  __atomic_store_n(p, v, __ATOMIC_RELEASE);
}
inline uint64_t load_acquire_u64(const uint64_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void store_release_u32(uint32_t* p, uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }
inline uint32_t load_acquire_u32(const uint32_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }

}  // namespace wire
}  // namespace zs
