#include "engine.h"

#include <algorithm>
#include <cmath>
#include <stdexcept>

namespace zs {
namespace engine {

struct Engine::Seq {
  Request req;
  int32_t slot = -1;
  std::vector<int32_t> tokens;  // prompt + generated
  uint32_t prompt_len = 0;
  uint32_t computed = 0;        // tokens whose KV / recurrent state is in cache
  uint32_t generated = 0;
  uint32_t cached_tokens = 0;   // prompt tokens served from the prefix cache
  kv::PrefixLease prefix;       // pinned cached / promoted nodes
  kv::BlockLease own;           // own pages not promoted yet (front = next node)
  kv::BlockLease held;          // own pages that lost a promotion race (still in use)
  std::vector<int32_t> page_table;
  bool table_dirty = true;
  int32_t restore_slot = -1;    // checkpoint restored before the first prefill chunk
  uint64_t last_node = 0;       // deepest node of this sequence's prefix in the tree
  uint32_t promoted_nodes = 0;
  std::vector<int32_t> drafts;
  // Staged in the current step:
  uint32_t rows = 0;            // rows of this sequence in the step
  bool sampled = false;
  std::vector<std::pair<uint32_t, kv::BlockLease>> promote;  // (node index, checkpoint lease)
  bool first_emitted = false;
  bool finished = false;        // finished while a later in-flight step still covers it
};

uint64_t splitmix64(uint64_t& state) {
  uint64_t z = (state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

std::vector<std::vector<int32_t>> random_prompts(uint64_t seed, size_t count, size_t len, int32_t low, int32_t high) {
  std::vector<std::vector<int32_t>> out(count, std::vector<int32_t>(len));
  uint64_t st = seed;
  const uint64_t span = uint64_t(std::max(1, high - low));
  for (auto& p : out)
    for (auto& t : p) t = low + int32_t(splitmix64(st) % span);
  return out;
}

Engine::Engine(Config cfg, std::shared_ptr<Backend> backend)
    : cfg_(std::move(cfg)),
      backend_(std::move(backend)),
      pages_(int32_t(cfg_.num_pages) - 1, 1),  // page 0 = dummy page for padding rows
      ckpt_slots_(int32_t(cfg_.num_ckpt_slots), int32_t(cfg_.max_seqs)) {
  if (cfg_.prefix_caching)
    tree_ = std::make_unique<kv::PrefixTree>(cfg_.page_size, cfg_.pages_per_node, cfg_.kv_hash_seed);
  // The DRAM tier keeps one page per block and no recurrent checkpoint, so it needs
  // APC nodes of one page and a model whose whole state is in the paged KV.
  if (cfg_.dram_blocks > 0 && tree_ && cfg_.pages_per_node == 1 && !cfg_.recurrent_state)
    dram_ = std::make_unique<kv::DramTier>(cfg_.dram_blocks, cfg_.page_size, cfg_.num_pages - 1,
                                           cfg_.dram_loading_area);
  for (int32_t s = int32_t(cfg_.max_seqs) - 1; s >= 0; --s) free_slots_.push_back(s);
}

void Engine::evict_pages(size_t n) {
  if (!tree_ || n == 0) return;
  auto victims = tree_->evict_lru(n);
  if (!dram_ || victims.empty()) return;
  // The victims' pages are back in the pool but nothing has been allocated since, so
  // their contents are intact until the copies below run.
  std::vector<kv::KvTransferOp> ops;
  std::vector<kv::Hash> keys;
  for (const auto& v : victims) {
    if (v.pages.size() != 1) continue;
    if (auto op = dram_->admit(v.hash, v.pages[0])) {
      ops.push_back(*op);
      keys.push_back(v.hash);
    }
  }
  if (!ops.empty() && !transfer(ops))
    for (const auto& k : keys) dram_->rollback(k);
}

bool Engine::transfer(const std::vector<kv::KvTransferOp>& ops) {
  const size_t per = std::max<size_t>(1, cfg_.max_step_tokens);
  for (size_t i = 0; i < ops.size(); i += per) {
    StepPlan p;
    p.opcode = wire::kOpKvTransfer;
    p.query_start = {0};
    for (size_t j = i; j < std::min(ops.size(), i + per); ++j) {
      p.token_ids.push_back(ops[j].hbm_page);
      p.positions.push_back(ops[j].dram_slot);
      p.row_slot.push_back(ops[j].h2d ? 1 : 0);
    }
    StepResult r;
    if (!backend_->execute(p, &r) || r.status != 0) {
      error_ = "KV transfer failed: " + backend_->error();
      return false;
    }
  }
  return true;
}

void Engine::reload_from_dram(const std::vector<int32_t>& key, kv::PrefixLease& lease) {
  if (!dram_ || !tree_) return;
  const uint32_t ps = cfg_.page_size;
  const size_t first = lease.matched_nodes();
  if ((first + 1) * ps > key.size()) return;
  const auto hashes = kv::compute_block_hashes(key, ps, cfg_.kv_hash_seed);
  size_t n = std::min(dram_->continuation(hashes, first), pages_.available());
  if (n == 0) return;
  auto got = pages_.allocate(n);
  if (!got) return;
  const auto slots = dram_->take(hashes, first, n);
  std::vector<kv::KvTransferOp> ops;
  for (size_t j = 0; j < slots.size(); ++j) ops.push_back(kv::KvTransferOp{got->ids()[j], slots[j], true});
  const bool ok = transfer(ops);
  dram_->release(slots);
  if (!ok) return;  // the pages return to the pool; the blocks are recomputed instead
  uint64_t parent = lease.leaf_node();
  for (size_t j = 0; j < slots.size(); ++j) {
    kv::BlockLease page = got->take_front(1);
    kv::BlockLease aux;
    const uint64_t id = tree_->insert(parent, key.data() + (first + j) * ps, page, aux);
    if (id == 0) break;
    parent = id;
  }
  lease.release();
  lease = tree_->match(key);
}

Engine::~Engine() = default;

void Engine::set_event_sink(kv::KvEventSink sink) {
  if (tree_) tree_->set_event_sink(std::move(sink));
}

bool Engine::submit(Request r) {
  if (waiting_.size() >= cfg_.max_waiting) return false;
  waiting_since_[r.id] = stats_.steps;
  waiting_at_[r.id] = std::chrono::steady_clock::now();
  waiting_.push_back(std::move(r));
  return true;
}

bool Engine::cancel(uint64_t id) {
  for (auto it = waiting_.begin(); it != waiting_.end(); ++it) {
    if (it->id == id) {
      waiting_since_.erase(id);
      waiting_at_.erase(id);
      waiting_.erase(it);
      return true;
    }
  }
  for (auto& kvp : running_) {
    if (kvp.second->req.id == id) {
      if (!inflight_.empty()) {  // an in-flight step still covers it: retire once that completes
        kvp.second->finished = true;
        zombies_.push_back(std::move(kvp.second));
      } else {
        retire(kvp.second.get());
      }
      running_.erase(kvp.first);
      return true;
    }
  }
  return false;
}

bool Engine::has_work() const { return !waiting_.empty() || !running_.empty() || !inflight_.empty(); }

EngineStats Engine::stats() const {
  EngineStats s = stats_;
  s.waiting = uint32_t(waiting_.size());
  s.running = uint32_t(running_.size());
  const size_t total = cfg_.num_pages - 1;
  s.kv_usage = total ? 1.0 - double(pages_.available()) / double(total) : 0.0;
  if (tree_) {
    const auto t = tree_->stats();
    s.prefix_queries = t.queries;
    s.prefix_query_tokens = t.query_tokens;
    s.prefix_hit_tokens = t.hit_tokens;
    s.prefix_evictions = t.evictions;
  }
  if (dram_) {
    const auto d = dram_->stats();
    s.dram_capacity = d.capacity_blocks;
    s.dram_occupied = d.occupied_blocks;
    s.dram_offloads = d.offloads;
    s.dram_reloads = d.reloads;
    s.dram_evictions = d.evictions;
    s.dram_hit_tokens = d.hit_tokens;
  }
  return s;
}

// ---------------------------------------------------------------------------- admission
bool Engine::admit_one() {
  if (waiting_.empty() || free_slots_.empty()) return false;
  // Pick the candidate: FIFO, or shortest prompt first (SRPT) unless some request
  // has waited longer than the starvation cap.
  size_t pick = 0;
  if (cfg_.prefill_policy == "srpt") {
    size_t oldest = 0;
    for (size_t i = 1; i < waiting_.size(); ++i)
      if (waiting_since_[waiting_[i].id] < waiting_since_[waiting_[oldest].id]) oldest = i;
    const uint64_t oid = waiting_[oldest].id;
    const auto waited_ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                               std::chrono::steady_clock::now() - waiting_at_[oid]).count();
    if (stats_.steps - waiting_since_[oid] >= cfg_.starvation_steps ||
        (cfg_.starvation_ms > 0 && waited_ms >= (long long)cfg_.starvation_ms)) {
      pick = oldest;
    } else {
      for (size_t i = 1; i < waiting_.size(); ++i)
        if (waiting_[i].prompt.size() < waiting_[pick].prompt.size()) pick = i;
    }
  }
  Request& r = waiting_[pick];
  const uint32_t ps = cfg_.page_size;
  const uint64_t want = std::min<uint64_t>(uint64_t(r.prompt.size()) + r.max_tokens, cfg_.max_model_len);
  const uint32_t total_pages = uint32_t((want + ps - 1) / ps);
  if (r.prompt.empty() || r.prompt.size() >= cfg_.max_model_len || total_pages > cfg_.num_pages - 1) {
    // Can never fit: fail this request (the caller reports it).
    auto s = make_seq(std::move(r));
    waiting_since_.erase(s->req.id);
    waiting_at_.erase(s->req.id);
    waiting_.erase(waiting_.begin() + pick);
    s->slot = -1;
    error_ = "request " + std::to_string(s->req.id) + " exceeds the model length or KV capacity";
    return false;
  }
  // Prefix match over prompt[:-1] (the last token must be computed to sample).
  kv::PrefixLease lease;
  if (tree_) {
    std::vector<int32_t> key(r.prompt.begin(), r.prompt.end() - 1);
    lease = tree_->match(key);
    if (cfg_.recurrent_state && lease.matched_nodes() > 0 && lease.leaf_aux() < 0) lease.release();
    if (dram_) reload_from_dram(key, lease);
  }
  const uint32_t matched_pages = uint32_t(lease.pages().size());
  const uint32_t own_needed = total_pages > matched_pages ? total_pages - matched_pages : 0;
  // With the DRAM tier, keep its loading area free (unless nothing else could run).
  const size_t reserve = dram_ && !running_.empty() ? dram_->loading_area_pages() : 0;
  if (pages_.available() < own_needed + reserve && tree_) evict_pages(own_needed + reserve - pages_.available());
  if (pages_.available() < own_needed + reserve) return false;  // wait for running requests to finish
  auto own = pages_.allocate(own_needed);
  auto seq = make_seq(std::move(r));
  waiting_since_.erase(seq->req.id);
  waiting_at_.erase(seq->req.id);
  waiting_.erase(waiting_.begin() + pick);
  seq->slot = free_slots_.back();
  free_slots_.pop_back();
  seq->page_table = lease.pages();
  seq->page_table.insert(seq->page_table.end(), own->ids().begin(), own->ids().end());
  seq->own = std::move(*own);
  seq->computed = lease.matched_tokens();
  seq->cached_tokens = lease.matched_tokens();
  seq->restore_slot = cfg_.recurrent_state ? lease.leaf_aux() : -1;
  seq->last_node = lease.leaf_node();
  seq->promoted_nodes = uint32_t(lease.matched_nodes());
  seq->prefix = std::move(lease);
  running_[seq->slot] = std::move(seq);
  return true;
}

std::unique_ptr<Engine::Seq> Engine::make_seq(Request&& r) {
  auto s = std::make_unique<Seq>();
  s->tokens = r.prompt;
  s->prompt_len = uint32_t(r.prompt.size());
  s->req = std::move(r);
  return s;
}

// ---------------------------------------------------------------------------- drafting
std::vector<int32_t> Engine::ngram_drafts(const Seq& s) const {
  // Longest suffix first (ngram_max down to ngram_min tokens): its most recent earlier
  // occurrence proposes the up to k tokens that followed it.
  const auto& t = s.tokens;
  const size_t k = cfg_.num_spec_tokens, lo = std::max<uint32_t>(1, cfg_.ngram_min);
  if (t.size() < 2 || k == 0) return {};
  const size_t hi = std::min<size_t>(cfg_.ngram_max, t.size() - 1);
  for (size_t n = hi; n >= lo; --n) {
    for (size_t start = t.size() - n; start-- > 0;) {
      if (std::equal(t.begin() + start, t.begin() + start + n, t.end() - n)) {
        const size_t b = start + n, e = std::min(b + k, t.size());
        return std::vector<int32_t>(t.begin() + b, t.begin() + e);
      }
    }
  }
  return {};
}

uint32_t Engine::mixed_step_budget(uint32_t decode_rows) const {
  const uint32_t top = cfg_.max_step_tokens;
  if (cfg_.max_mixed_step_tokens == 0 || decode_rows == 0) return top;
  const uint32_t base = std::min(std::max(cfg_.max_mixed_step_tokens, decode_rows + 1), top);
  if (!cfg_.dynamic_prefill_budget || base >= top) return base;
  const uint64_t lo = cfg_.backlog_low_tokens, hi = std::max(cfg_.backlog_high_tokens, cfg_.backlog_low_tokens);
  uint64_t backlog = 0;
  for (const auto& kvp : running_) backlog += kvp.second->prompt_len - std::min(kvp.second->computed, kvp.second->prompt_len);
  for (const auto& r : waiting_) {
    if (backlog >= hi) break;
    backlog += r.prompt.size();
  }
  if (backlog <= lo) return base;
  if (backlog >= hi || hi == lo) return top;
  return uint32_t(std::min<uint64_t>(top, base + (uint64_t)(top - base) * (backlog - lo) / (hi - lo)));
}

// ---------------------------------------------------------------------------- staging
void Engine::stage(StepPlan& p, std::vector<Seq*>& order) {
  p = StepPlan();
  p.query_start.push_back(0);
  uint32_t budget = cfg_.max_step_tokens;
  bool any_prefill = false, any_spec = false, any_sampling = false, any_penalty = false, any_logprobs = false;
  const uint32_t nt = tree_ ? tree_->node_tokens() : 0;

  auto add_seq = [&](Seq* s, uint32_t rows, const int32_t* toks, uint32_t pos0, bool sample, uint32_t spec_w) {
    const int32_t row0 = int32_t(p.token_ids.size());
    for (uint32_t i = 0; i < rows; ++i) {
      p.token_ids.push_back(toks[i]);
      p.positions.push_back(int32_t(pos0 + i));
      p.row_slot.push_back(s->slot);
    }
    p.query_start.push_back(int32_t(p.token_ids.size()));
    p.seq_slot.push_back(s->slot);
    p.seq_len.push_back(int32_t(pos0 + rows));
    p.sample_row.push_back(sample ? int32_t(p.token_ids.size()) - 1 : -1);
    p.spec_width.push_back(int32_t(spec_w));
    wire::SamplingParams sp{};
    sp.temperature = s->req.sampling.temperature;
    sp.top_p = s->req.sampling.top_p;
    sp.top_k = s->req.sampling.top_k;
    sp.presence_penalty = s->req.sampling.presence_penalty;
    sp.frequency_penalty = s->req.sampling.frequency_penalty;
    sp.repetition_penalty = s->req.sampling.repetition_penalty;
    sp.seed = s->req.sampling.seed + s->generated;
    sp.logprobs = s->req.sampling.logprobs;
    p.sampling.push_back(sp);
    any_sampling |= sp.temperature > 0.f;
    any_penalty |= sp.presence_penalty != 0.f || sp.frequency_penalty != 0.f || sp.repetition_penalty != 1.f;
    any_logprobs |= sp.logprobs >= 0;
    p.restore_slot.push_back(s->restore_slot);
    s->restore_slot = -1;
    s->rows = rows;
    s->sampled = sample;
    order.push_back(s);
    (void)row0;
  };

  // 1. Decode rows (all sequences past their prompt), optionally with draft tokens.
  for (auto& kvp : running_) {
    Seq* s = kvp.second.get();
    if (s->computed < s->prompt_len) continue;
    const uint32_t pos = s->computed;  // feed tokens[computed]
    std::vector<int32_t> rows{s->tokens[pos]};
    uint32_t spec_w = 0;
    if (cfg_.spec_method == "ngram" && cfg_.num_spec_tokens > 0) {
      s->drafts = ngram_drafts(*s);
      const uint32_t room = uint32_t(cfg_.max_model_len) - pos - 1;
      while (s->drafts.size() > room) s->drafts.pop_back();
      const uint32_t left = s->req.max_tokens - s->generated;
      while (!s->drafts.empty() && s->drafts.size() + 1 > left) s->drafts.pop_back();
    } else if (model_drafts()) {
      // drafts were proposed by the worker (MTP or DSpark head) in the previous step's result
    } else {
      s->drafts.clear();
    }
    if (!s->drafts.empty()) {
      rows.insert(rows.end(), s->drafts.begin(), s->drafts.end());
      spec_w = uint32_t(rows.size());
      any_spec = true;
      stats_.spec_drafts += s->drafts.size();
    }
    if (rows.size() > budget) continue;
    budget -= uint32_t(rows.size());
    add_seq(s, uint32_t(rows.size()), rows.data(), pos, true, spec_w);
  }
  // 2. Prefill chunks, in admission (slot) order, within the mixed-step budget when the
  // step also carries decode rows (speculative steps keep the full step budget).
  if (cfg_.spec_method == "none" && !order.empty()) {
    const uint32_t used = cfg_.max_step_tokens - budget;
    const uint32_t cap = mixed_step_budget(uint32_t(order.size()));
    budget = cap > used ? std::min(budget, cap - used) : 0;
  }
  for (auto& kvp : running_) {
    Seq* s = kvp.second.get();
    if (s->computed >= s->prompt_len || budget == 0) continue;
    const uint32_t chunk = std::min({s->prompt_len - s->computed, cfg_.max_prefill_chunk, budget});
    const uint32_t c0 = s->computed, c1 = c0 + chunk;
    const int32_t row_base = int32_t(p.token_ids.size());
    add_seq(s, chunk, s->tokens.data() + c0, c0, c1 == s->prompt_len, 0);
    budget -= chunk;
    any_prefill = true;
    // APC: checkpoint + promote the nodes this chunk completes.
    if (tree_) {
      for (uint32_t node = s->promoted_nodes + uint32_t(s->promote.size()); (node + 1) * nt <= c1; ++node) {
        if ((node + 1) * nt <= c0) continue;
        kv::BlockLease aux;
        if (cfg_.recurrent_state) {
          auto a = ckpt_slots_.allocate(1);
          if (!a) {
            evict_pages(1);
            a = ckpt_slots_.allocate(1);
          }
          if (!a) break;  // no checkpoint slot: stop promoting this sequence
          p.ckpt_row.push_back(row_base + int32_t((node + 1) * nt - 1 - c0));
          p.ckpt_slot.push_back(a->ids()[0]);
          aux = std::move(*a);
        }
        s->promote.emplace_back(node, std::move(aux));
      }
    }
  }
  // 3. Page-table rows of newly admitted sequences.
  for (Seq* s : order) {
    if (s->table_dirty) {
      p.dirty_rows.push_back(s->slot);
      p.dirty_pages.push_back(s->page_table);
      s->table_dirty = false;
    }
  }
  if (!any_prefill && !any_spec && !order.empty()) {
    p.flags |= wire::kFlagDecodeOnly;
    p.bucket = wire::select_bucket(uint32_t(order.size()));
  }
  if (any_spec) p.flags |= wire::kFlagSpecVerify;
  if (any_sampling) p.flags |= wire::kFlagSampling;
  if (any_penalty) p.flags |= wire::kFlagPenalty | wire::kFlagSampling;
  if (any_logprobs) p.flags |= wire::kFlagLogprobs;
}

// ---------------------------------------------------------------------------- step
std::vector<TokenEvent> Engine::step() {
  if (cfg_.in_flight_depth > 0 && backend_->async_capable()) return step_async();
  std::vector<TokenEvent> events;
  if (poisoned_) return events;
  while (admit_one()) {
  }
  if (!error_.empty() && running_.empty() && waiting_.empty()) {
    // An unfittable request was dropped by admit_one.
  }
  if (running_.empty()) return events;
  std::vector<Seq*> order;
  stage(plan_, order);
  if (order.empty()) return events;
  ++stats_.steps;
  if (plan_.flags & wire::kFlagDecodeOnly) ++stats_.decode_steps;
  StepResult res;
  if (!backend_->execute(plan_, &res) || res.status != 0 || res.outputs.size() < order.size()) {
    fail_all(&events);
    return events;
  }
  process(order, res, &events, false);
  return events;
}

void Engine::fail_all(std::vector<TokenEvent>* events) {
  poisoned_ = true;
  error_ = backend_->error().empty() ? "worker step failed" : backend_->error();
  for (auto& kvp : running_) {
    TokenEvent ev;
    ev.request_id = kvp.second->req.id;
    ev.finish = Finish::kError;
    events->push_back(ev);
    retire(kvp.second.get());
  }
  running_.clear();
  for (auto& z : zombies_) retire(z.get());
  zombies_.clear();
  inflight_.clear();
}

void Engine::process(std::vector<Seq*>& order, const StepResult& res, std::vector<TokenEvent>* events_out,
                     bool defer) {
  std::vector<TokenEvent>& events = *events_out;
  stats_.last_gpu_us = res.gpu_exec_us;
  std::vector<int32_t> done;
  for (size_t i = 0; i < order.size(); ++i) {
    Seq* s = order[i];
    if (s->finished) continue;  // output of a run-ahead step past the sequence's end
    const wire::SeqStepOutput& out = res.outputs[i];
    // Promote the prefix nodes completed by this step.
    for (auto& pr : s->promote) {
      const uint32_t node = pr.first;
      kv::BlockLease pages = s->own.take_front(cfg_.pages_per_node);
      bool created = false;
      const uint64_t id = tree_->insert(s->last_node, s->tokens.data() + size_t(node) * tree_->node_tokens(), pages,
                                        pr.second, &created);
      if (!created) s->held.absorb(std::move(pages));  // lost a race: keep using our copy
      if (id == 0) break;
      s->last_node = id;
      s->prefix = tree_->pin_chain(id);
      ++s->promoted_nodes;
    }
    s->promote.clear();
    if (!s->sampled) {
      s->computed += s->rows;
      stats_.prefill_tokens += s->rows;
      continue;
    }
    const bool was_prefill = s->computed < s->prompt_len;
    if (was_prefill) stats_.prefill_tokens += s->rows; else stats_.decode_tokens += 1;
    // Accepted tokens: for a verify step, drafts that matched plus the bonus token.
    const int32_t n_tok = std::max(1, std::min<int32_t>(out.num_tokens, wire::kMaxSpecTokens));
    if (s->rows > 1 && !was_prefill) {
      stats_.spec_verify_rows += s->rows;
      stats_.spec_verify_steps += 1;
      stats_.spec_accepted += uint32_t(n_tok - 1);
      s->computed += uint32_t(n_tok);  // fed row 0 + accepted drafts
    } else {
      s->computed += s->rows;
    }
    TokenEvent ev;
    ev.request_id = s->req.id;
    ev.prompt_tokens = s->prompt_len;
    ev.cached_tokens = s->cached_tokens;
    ev.first = !s->first_emitted;
    s->first_emitted = true;
    Finish fin = Finish::kNone;
    for (int32_t j = 0; j < n_tok; ++j) {
      const int32_t tok = out.tokens[j];
      s->tokens.push_back(tok);
      ++s->generated;
      ev.tokens.push_back(tok);
      ev.logprobs.push_back(out.logprobs[j]);
      if (s->req.sampling.logprobs > 0 && j == 0) {
        std::vector<std::pair<int32_t, float>> top;
        for (int32_t q = 0; q < std::min<int32_t>(s->req.sampling.logprobs, wire::kMaxTopLogprobs); ++q)
          top.emplace_back(out.top_ids[q], out.top_logprobs[q]);
        ev.top_logprobs.push_back(std::move(top));
      }
      const bool eos = !s->req.ignore_eos &&
                       std::find(s->req.eos_ids.begin(), s->req.eos_ids.end(), tok) != s->req.eos_ids.end();
      if (eos) {
        fin = Finish::kStop;
        break;
      }
      if (s->generated >= s->req.max_tokens || s->tokens.size() >= cfg_.max_model_len) {
        fin = Finish::kLength;
        break;
      }
    }
    if (model_drafts()) {
      s->drafts.assign(out.next_drafts, out.next_drafts + std::max(0, std::min<int32_t>(out.num_drafts, wire::kMaxSpecTokens)));
    }
    ev.completion_tokens = s->generated;
    ev.finish = fin;
    events.push_back(std::move(ev));
    if (fin != Finish::kNone) done.push_back(s->slot);
  }
  for (int32_t slot : done) {
    auto it = running_.find(slot);
    if (defer) {  // a later in-flight step still reads this slot and its pages
      it->second->finished = true;
      zombies_.push_back(std::move(it->second));
    } else {
      retire(it->second.get());
    }
    running_.erase(it);
  }
}


// ---------------------------------------------------------------------------- in-flight depth 1
// While the running set is a stable pure-decode batch, the step after the one in flight
// is published before the in-flight step's results are processed: its inputs are the
// tokens the workers just sampled (kept per slot on the worker side, flag DEVICE_TOKENS),
// so result processing and plan staging here overlap the GPU.  A sequence that finishes
// in the processed step still appears in the step already published; it is kept (slot
// and pages reserved) until that step completes and its extra output is dropped.
bool Engine::can_run_ahead(const Inflight& cur) const {
  if (!(cur.plan.flags & wire::kFlagDecodeOnly) || !waiting_.empty() || !zombies_.empty()) return false;
  if (cur.order.size() != running_.size()) return false;
  for (size_t i = 0; i < cur.order.size(); ++i) {
    const Seq* s = cur.order[i];
    if (s->finished || s->rows != 1 || !s->sampled || !s->drafts.empty()) return false;
    // The step in flight produces token generated + 1; the ahead step token generated + 2.
    if (s->generated + 2 > s->req.max_tokens || s->tokens.size() + 2 >= cfg_.max_model_len) return false;
  }
  return true;
}

std::vector<TokenEvent> Engine::step_async() {
  std::vector<TokenEvent> events;
  if (poisoned_) return events;
  if (inflight_.empty()) {
    while (admit_one()) {
    }
    if (running_.empty()) return events;
    std::vector<Seq*> order;
    stage(plan_, order);
    if (order.empty()) return events;
    ++stats_.steps;
    if (plan_.flags & wire::kFlagDecodeOnly) ++stats_.decode_steps;
    if (!backend_->submit(plan_)) {
      fail_all(&events);
      return events;
    }
    inflight_.push_back(Inflight{plan_, order});
  }
  if (inflight_.size() == 1 && can_run_ahead(inflight_.front())) {
    Inflight next{inflight_.front().plan, inflight_.front().order};
    StepPlan& p = next.plan;
    p.flags |= wire::kFlagDeviceTokens;
    for (auto& t : p.token_ids) t = -1;
    for (auto& x : p.positions) ++x;
    for (auto& x : p.seq_len) ++x;
    for (auto& sp : p.sampling) ++sp.seed;  // seed = request seed + generated index
    p.dirty_rows.clear();
    p.dirty_pages.clear();
    p.ckpt_row.clear();
    p.ckpt_slot.clear();
    for (auto& r : p.restore_slot) r = -1;
    ++stats_.steps;
    ++stats_.decode_steps;
    ++stats_.run_ahead_steps;
    if (!backend_->submit(p)) {
      fail_all(&events);
      return events;
    }
    inflight_.push_back(std::move(next));
  }
  StepResult res;
  Inflight cur = std::move(inflight_.front());
  inflight_.pop_front();
  if (!backend_->collect(&res) || res.status != 0 || res.outputs.size() < cur.order.size()) {
    fail_all(&events);
    return events;
  }
  process(cur.order, res, &events, !inflight_.empty());
  if (inflight_.empty()) {
    for (auto& z : zombies_) retire(z.get());
    zombies_.clear();
  }
  return events;
}

void Engine::retire(Seq* s) {
  s->promote.clear();  // returns unused checkpoint slots
  s->prefix.release();
  s->own.release();
  s->held.release();
  if (s->slot >= 0) free_slots_.push_back(s->slot);
  s->slot = -1;
}

void Engine::finish(Seq* s, Finish why, std::vector<TokenEvent>* out) {
  TokenEvent ev;
  ev.request_id = s->req.id;
  ev.finish = why;
  ev.completion_tokens = s->generated;
  out->push_back(ev);
}

}  // namespace engine
}  // namespace zs
