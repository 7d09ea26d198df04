// Continuous-batching serving engine of the master.
//
// Owns the request slots, the paged-KV pools and the prefix tree, decides every step
// which tokens run (decode rows of running sequences, piggybacked with chunks of
// pending prefills up to the step token budget), stages the step plan, executes it on
// a Backend (the shared-memory worker coordinator, or a scripted mock) and turns the
// step results into per-request token events.
//
// Key policies (reference parity in brackets, crates/zs-scheduler/src/serving.rs):
//  * whole-request KV reservation at admission (prompt + max_tokens), LRU eviction of
//    unpinned prefix nodes when the pool runs short          [kv_demand_fits :833]
//  * FIFO or SRPT prefill admission with a starvation cap     [PrefillSchedulingPolicy :221]
//  * chunked prefill (max_prefill_chunk, step token budget)    [stage_prefill_row :2848]
//  * mixed decode + prefill steps                              [stage_mixed_step :2489]
//  * decode-only steps padded to a graph bucket                [stage_decode_step :3077]
//  * automatic prefix caching with recurrent-state checkpoints: nodes are promoted
//    after the prefill step that completed them, with a checkpoint slot snapshotted
//    at the node's last row; a prefix hit restores the leaf's checkpoint
//                                                              [admit_request_into_sequence :604]
//  * n-gram speculative decoding with greedy verify            [ngram_draft_tokens :483]
#pragma once

#include <stdint.h>

#include <chrono>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <optional>
#include <string>
#include <vector>

#include "dram_tier.h"
#include "kv.h"
#include "wire.h"

namespace zs {
namespace engine {

struct Sampling {
  float temperature = 0.f;
  float top_p = 1.f;
  int32_t top_k = 0;
  float presence_penalty = 0.f;
  float frequency_penalty = 0.f;
  float repetition_penalty = 1.f;
  uint64_t seed = 0;
  int32_t logprobs = -1;
};

struct Request {
  uint64_t id = 0;
  std::vector<int32_t> prompt;
  Sampling sampling;
  uint32_t max_tokens = 16;
  bool ignore_eos = false;
  std::vector<int32_t> eos_ids;
};

enum class Finish : int { kNone = 0, kStop = 1, kLength = 2, kCancelled = 3, kError = 4 };

struct TokenEvent {
  uint64_t request_id = 0;
  std::vector<int32_t> tokens;
  std::vector<float> logprobs;
  std::vector<std::vector<std::pair<int32_t, float>>> top_logprobs;
  Finish finish = Finish::kNone;
  uint32_t prompt_tokens = 0;
  uint32_t completion_tokens = 0;
  uint32_t cached_tokens = 0;
  bool first = false;  // first generated token of the request (TTFT)
};

struct Config {
  uint32_t max_seqs = 256;
  uint32_t max_step_tokens = 8192;
  uint32_t max_prefill_chunk = 2048;
  uint32_t page_size = 16;
  uint32_t num_pages = 32768;          // device pages (page 0 is reserved as the dummy page)
  uint32_t max_model_len = 32768;
  bool prefix_caching = false;
  uint32_t pages_per_node = 1;         // APC node = pages_per_node pages
  bool recurrent_state = false;        // model keeps per-slot recurrent state (GDN)
  uint32_t num_ckpt_slots = 0;         // recurrent checkpoint slots (after the live slots)
  std::string prefill_policy = "fifo"; // "fifo" | "srpt"
  // SRPT starvation cap: the oldest waiting request is admitted next (and holds back shorter
  // ones until it fits) once it has waited this many engine steps or this many ms (0: off).
  uint32_t starvation_steps = 64;
  uint32_t starvation_ms = 60000;
  // Mixed steps (decode rows + prefill chunks): at most max(max_mixed_step_tokens, decodes + 1)
  // rows (0: off, max_step_tokens).  With dynamic_prefill_budget the cap ramps linearly to
  // max_step_tokens as the prefill backlog (uncomputed prompt tokens of running and waiting
  // requests) grows from backlog_low_tokens to backlog_high_tokens.
  uint32_t max_mixed_step_tokens = 0;
  bool dynamic_prefill_budget = false;
  uint32_t backlog_low_tokens = 2048;
  uint32_t backlog_high_tokens = 16384;
  uint32_t max_waiting = 4096;
  std::string spec_method = "none";    // "none" | "ngram" | "mtp" | "dspark" (last two: drafts from the worker)
  uint32_t num_spec_tokens = 0;
  // n-gram drafts: the longest suffix of ngram_max..ngram_min tokens that occurred earlier
  // proposes the tokens that followed its most recent earlier occurrence.
  uint32_t ngram_min = 2;
  uint32_t ngram_max = 5;
  std::string kv_hash_seed = "42";
  uint32_t dram_blocks = 0;            // host DRAM tier blocks (0: off); needs APC, 1 page per node,
                                       // and a model without recurrent state
  double dram_loading_area = 0.10;     // share of HBM pages kept free for DRAM reloads
  uint32_t in_flight_depth = 0;        // 1: publish the next decode step before processing this one
};

// Host-side staged step (the coordinator copies it into a shared-memory plan slot).
struct StepPlan {
  uint32_t opcode = wire::kOpNormal;
  uint32_t flags = 0;
  uint32_t bucket = 0;
  std::vector<int32_t> token_ids, positions, row_slot;
  std::vector<int32_t> query_start, seq_slot, seq_len, sample_row;
  std::vector<wire::SamplingParams> sampling;
  std::vector<int32_t> dirty_rows;
  std::vector<std::vector<int32_t>> dirty_pages;
  std::vector<int32_t> ckpt_row, ckpt_slot, restore_slot;
  std::vector<int32_t> spec_width;  // per sequence: verify rows (0 = normal)
};

struct StepResult {
  uint32_t status = 0;
  uint64_t gpu_exec_us = 0;
  std::vector<wire::SeqStepOutput> outputs;  // one per sequence of the plan (plan order)
};

class Backend {
 public:
  virtual ~Backend() = default;
  virtual bool execute(const StepPlan& plan, StepResult* result) = 0;
  virtual std::string error() const { return {}; }
  // Asynchronous pair for in-flight pipelining: publish a step now, collect its result
  // later (in submission order).  The default runs the step at submit time.
  virtual bool submit(const StepPlan& plan) {
    pending_.emplace_back();
    return execute(plan, &pending_.back());
  }
  virtual bool collect(StepResult* result) {
    if (pending_.empty()) return false;
    *result = std::move(pending_.front());
    pending_.pop_front();
    return true;
  }
  // True when submit() returns before the step ran (the engine then runs ahead).
  virtual bool async_capable() const { return async_; }
  void set_async(bool on) { async_ = on; }

 protected:
  std::deque<StepResult> pending_;
  bool async_ = false;
};

struct EngineStats {
  uint32_t waiting = 0, running = 0;
  double kv_usage = 0.0;
  uint64_t steps = 0, decode_steps = 0, prefill_tokens = 0, decode_tokens = 0, preemptions = 0;
  uint64_t prefix_queries = 0, prefix_query_tokens = 0, prefix_hit_tokens = 0, prefix_evictions = 0;
  uint64_t spec_drafts = 0, spec_accepted = 0, spec_verify_rows = 0;
  uint64_t spec_verify_steps = 0;  // sequence-level verify steps (one per sequence per step)
  uint64_t last_gpu_us = 0;
  // Host DRAM tier of the prefix cache (zero when off).
  uint64_t dram_capacity = 0, dram_occupied = 0, dram_offloads = 0, dram_reloads = 0, dram_evictions = 0;
  uint64_t dram_hit_tokens = 0;
  uint64_t run_ahead_steps = 0;  // decode steps published before the previous one was processed
};

class Engine {
 public:
  Engine(Config cfg, std::shared_ptr<Backend> backend);
  ~Engine();
  // Returns false when the waiting queue is full (overload).
  bool submit(Request r);
  bool cancel(uint64_t id);
  // One scheduling iteration; executes at most one step.  Returns the token events.
  std::vector<TokenEvent> step();
  bool has_work() const;
  bool poisoned() const { return poisoned_; }
  std::string error() const { return error_; }
  EngineStats stats() const;
  const Config& config() const { return cfg_; }
  // Prefill chunk size for the steps staged from now on (the parity check's unchunked and
  // chunked passes run on one engine).
  void set_max_prefill_chunk(uint32_t n) { cfg_.max_prefill_chunk = n ? n : 1; }
  kv::PrefixTree* prefix_tree() { return tree_.get(); }
  size_t free_pages() const { return pages_.available(); }
  size_t free_ckpt_slots() const { return ckpt_slots_.available(); }
  size_t free_slots() const { return free_slots_.size(); }
  // The last staged plan (tests and the micro-step benchmark inspect it).
  const StepPlan& last_plan() const { return plan_; }
  void set_event_sink(kv::KvEventSink sink);

 private:
  struct Seq;
  bool admit_one();
  std::unique_ptr<Seq> make_seq(Request&& r);
  void stage(StepPlan& p, std::vector<Seq*>& order);
  void finish(Seq* s, Finish why, std::vector<TokenEvent>* out);
  void retire(Seq* s);
  std::vector<int32_t> ngram_drafts(const Seq& s) const;
  struct Inflight {
    StepPlan plan;
    std::vector<Seq*> order;
  };
  void process(std::vector<Seq*>& order, const StepResult& res, std::vector<TokenEvent>* events, bool defer);
  void fail_all(std::vector<TokenEvent>* events);
  bool can_run_ahead(const Inflight& cur) const;
  // Drafts come from the worker's model head (MTP for Qwen, DSpark for DeepSeek).
  bool model_drafts() const { return cfg_.spec_method == "mtp" || cfg_.spec_method == "dspark"; }
  std::vector<TokenEvent> step_async();
  // Evict LRU prefix leaves until n pages were freed, demoting them to the DRAM tier.
  void evict_pages(size_t n);
  // Run page copies between HBM and the DRAM tier as KvTransfer steps.
  bool transfer(const std::vector<kv::KvTransferOp>& ops);
  // Extend `lease` (the HBM match of `key`) with DRAM-resident continuation blocks.
  void reload_from_dram(const std::vector<int32_t>& key, kv::PrefixLease& lease);

  Config cfg_;
  std::shared_ptr<Backend> backend_;
  kv::BlockPool pages_;
  kv::BlockPool ckpt_slots_;
  std::unique_ptr<kv::PrefixTree> tree_;
  std::unique_ptr<kv::DramTier> dram_;
  std::deque<Request> waiting_;
  std::map<uint64_t, uint64_t> waiting_since_;  // request id -> step when queued
  std::map<uint64_t, std::chrono::steady_clock::time_point> waiting_at_;  // request id -> time queued
  uint32_t mixed_step_budget(uint32_t decode_rows) const;
  std::vector<int32_t> free_slots_;
  std::map<int32_t, std::unique_ptr<Seq>> running_;  // by request slot
  std::deque<Inflight> inflight_;                     // published, not yet processed steps
  std::vector<std::unique_ptr<Seq>> zombies_;         // finished, still covered by an in-flight step
  StepPlan plan_;
  EngineStats stats_;
  bool poisoned_ = false;
  std::string error_;
};

// Deterministic SplitMix64 random prompts (bench tiers): token ids in [low, high).
std::vector<std::vector<int32_t>> random_prompts(uint64_t seed, size_t count, size_t len, int32_t low, int32_t high);
uint64_t splitmix64(uint64_t& state);

}  // namespace engine
}  // namespace zs
