#include "serve_loop.h"

#include <chrono>

#include "shm.h"

namespace zs {
namespace serve {

namespace {
double now_s() { return (double)monotonic_ns() * 1e-9; }

std::vector<double> latency_bounds() {
  return {0.001, 0.0025, 0.005, 0.01, 0.02, 0.04, 0.06, 0.08, 0.1, 0.25, 0.5, 0.75,
          1.0,   2.5,    5.0,   7.5,  10.0, 20.0, 40.0, 80.0, 160.0, 640.0, 2560.0};
}
std::vector<double> tpot_bounds() {
  return {0.001, 0.0025, 0.005, 0.0075, 0.01, 0.015, 0.02, 0.025, 0.03, 0.04, 0.05, 0.075,
          0.1,   0.15,   0.2,   0.3,    0.4,  0.5,   0.75,  1.0,   2.5,  5.0,  7.5,  10.0, 20.0, 40.0, 80.0};
}
}  // namespace

const char* state_name(EngineState s) {
  switch (s) {
    case EngineState::kStarting: return "starting";
    case EngineState::kReady: return "ready";
    case EngineState::kDraining: return "draining";
    case EngineState::kFaulted: return "faulted";
  }
  return "unknown";
}

// ------------------------------------------------------------------ histogram
Histogram::Histogram(std::vector<double> bounds)
    : bounds_(std::move(bounds)), buckets_(new std::atomic<uint64_t>[bounds_.size() + 1]) {
  for (size_t i = 0; i <= bounds_.size(); ++i) buckets_[i].store(0);
}

void Histogram::observe(double v) {
  size_t i = 0;
  while (i < bounds_.size() && v > bounds_[i]) ++i;
  buckets_[i].fetch_add(1);
  count_.fetch_add(1);
  sum_us_.fetch_add((uint64_t)(v * 1e6 + 0.5));
}

std::vector<uint64_t> Histogram::counts() const {
  std::vector<uint64_t> c(bounds_.size() + 1);
  for (size_t i = 0; i <= bounds_.size(); ++i) c[i] = buckets_[i].load();
  return c;
}

double Histogram::sum() const { return (double)sum_us_.load() * 1e-6; }

OnlineMetrics::OnlineMetrics() : ttft(latency_bounds()), tpot(tpot_bounds()), e2e(latency_bounds()) {}

// ------------------------------------------------------------------ stream
bool RequestStream::pop(StreamEvent* ev, int timeout_ms) {
  std::unique_lock<std::mutex> lk(mu_);
  if (!cv_.wait_for(lk, std::chrono::milliseconds(timeout_ms), [&] { return !q_.empty(); })) return false;
  *ev = std::move(q_.front());
  q_.pop_front();
  return true;
}

void RequestStream::push(StreamEvent ev) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    if (ev.finish != engine::Finish::kNone) closed_.store(true);
    q_.push_back(std::move(ev));
  }
  cv_.notify_all();
}

// ------------------------------------------------------------------ loop
ServeLoop::ServeLoop(std::shared_ptr<engine::Engine> engine, std::shared_ptr<void> keepalive, size_t max_waiting)
    : engine_(std::move(engine)), keepalive_(std::move(keepalive)), max_waiting_(max_waiting) {}

ServeLoop::~ServeLoop() { shutdown(); }

void ServeLoop::start() {
  if (thread_.joinable()) return;
  set_state(EngineState::kReady);
  thread_ = std::thread([this] { run(); });
}

SubmitError ServeLoop::submit(engine::Request r, std::shared_ptr<RequestStream>* out) {
  const EngineState st = state();
  if (st == EngineState::kStarting) return SubmitError::kStarting;
  if (st == EngineState::kDraining) return SubmitError::kDraining;
  if (st == EngineState::kFaulted) return SubmitError::kFaulted;
  std::lock_guard<std::mutex> lk(mu_);
  if (in_system_.load() >= max_waiting_ + engine_->config().max_seqs) {
    metrics_.requests_rejected.fetch_add(1);
    return SubmitError::kOverloaded;
  }
  auto s = std::make_shared<RequestStream>(r.id);
  Track t;
  t.stream = s;
  t.t_submit = now_s();
  live_[r.id] = t;
  submits_.push_back(std::move(r));
  in_system_.fetch_add(1);
  *out = s;
  cv_.notify_all();
  return SubmitError::kOk;
}

void ServeLoop::cancel(uint64_t id) {
  std::lock_guard<std::mutex> lk(mu_);
  cancels_.push_back(id);
  cv_.notify_all();
}

void ServeLoop::drain() {
  if (state() != EngineState::kFaulted) set_state(EngineState::kDraining);
  cv_.notify_all();
}

bool ServeLoop::idle() const { return in_system_.load() == 0; }

engine::EngineStats ServeLoop::stats() const {
  std::lock_guard<std::mutex> lk(mu_);
  return stats_;
}

std::string ServeLoop::error() const {
  std::lock_guard<std::mutex> lk(mu_);
  return error_;
}

void ServeLoop::shutdown() {
  stop_.store(true);
  cv_.notify_all();
  if (thread_.joinable()) thread_.join();
}

void ServeLoop::fail_all(const std::string& why) {
  std::lock_guard<std::mutex> lk(mu_);
  error_ = why;
  for (auto& kv : live_) {
    StreamEvent ev;
    ev.finish = engine::Finish::kError;
    ev.error = why;
    kv.second.stream->push(std::move(ev));
    metrics_.requests_error.fetch_add(1);
  }
  live_.clear();
  submits_.clear();
  in_system_.store(0);
}

void ServeLoop::run() {
  while (!stop_.load()) {
    std::deque<engine::Request> subs;
    std::vector<uint64_t> cancels;
    {
      std::unique_lock<std::mutex> lk(mu_);
      if (submits_.empty() && cancels_.empty() && !engine_->has_work())
        cv_.wait_for(lk, std::chrono::milliseconds(20));
      subs.swap(submits_);
      cancels.swap(cancels_);
    }
    for (auto& r : subs) {
      const uint64_t id = r.id;
      if (!engine_->submit(std::move(r))) {
        std::lock_guard<std::mutex> lk(mu_);
        auto it = live_.find(id);
        if (it != live_.end()) {
          StreamEvent ev;
          ev.finish = engine::Finish::kError;
          ev.error = "overloaded";
          it->second.stream->push(std::move(ev));
          live_.erase(it);
          in_system_.fetch_sub(1);
          metrics_.requests_rejected.fetch_add(1);
        }
      }
    }
    for (uint64_t id : cancels) {
      engine_->cancel(id);
      std::lock_guard<std::mutex> lk(mu_);
      auto it = live_.find(id);
      if (it != live_.end()) {
        StreamEvent ev;
        ev.finish = engine::Finish::kCancelled;
        ev.completion_tokens = it->second.generated;
        it->second.stream->push(std::move(ev));
        live_.erase(it);
        in_system_.fetch_sub(1);
        metrics_.requests_cancelled.fetch_add(1);
      }
    }
    if (!engine_->has_work()) continue;
    std::vector<engine::TokenEvent> events = engine_->step();
    if (engine_->poisoned()) {
      set_state(EngineState::kFaulted);
      fail_all(engine_->error());
      continue;
    }
    const double t = now_s();
    std::lock_guard<std::mutex> lk(mu_);
    stats_ = engine_->stats();
    for (auto& e : events) {
      auto it = live_.find(e.request_id);
      if (it == live_.end()) continue;  // cancelled meanwhile
      Track& tr = it->second;
      if (!e.tokens.empty()) {
        if (tr.generated == 0) {
          tr.t_first = t;
          metrics_.ttft.observe(t - tr.t_submit);
        } else {
          const double dt = (t - tr.t_last) / (double)e.tokens.size();
          for (size_t k = 0; k < e.tokens.size(); ++k) metrics_.tpot.observe(dt);
        }
        tr.t_last = t;
        tr.generated += (uint32_t)e.tokens.size();
        metrics_.generation_tokens.fetch_add(e.tokens.size());
      }
      StreamEvent ev;
      ev.tokens = std::move(e.tokens);
      ev.logprobs = std::move(e.logprobs);
      ev.top_logprobs = std::move(e.top_logprobs);
      ev.finish = e.finish;
      ev.prompt_tokens = e.prompt_tokens;
      ev.completion_tokens = e.completion_tokens;
      ev.cached_tokens = e.cached_tokens;
      const bool done = ev.finish != engine::Finish::kNone;
      if (done) {
        metrics_.prompt_tokens.fetch_add(ev.prompt_tokens);
        metrics_.cached_prompt_tokens.fetch_add(ev.cached_tokens);
        metrics_.e2e.observe(t - tr.t_submit);
        if (ev.finish == engine::Finish::kLength) metrics_.requests_length.fetch_add(1);
        else if (ev.finish == engine::Finish::kError) metrics_.requests_error.fetch_add(1);
        else metrics_.requests_ok.fetch_add(1);
      }
      tr.stream->push(std::move(ev));
      if (done) {
        live_.erase(it);
        in_system_.fetch_sub(1);
      }
    }
  }
}

// ------------------------------------------------------------------ mock backend
int32_t mock_next_token(int32_t last, int32_t pos, int32_t low, int32_t high) {
  uint64_t h = (uint64_t)(uint32_t)last * 0x9E3779B97F4A7C15ull ^ ((uint64_t)(uint32_t)pos + 0x632BE59BD9B4E019ull);
  h ^= h >> 29;
  h *= 0xBF58476D1CE4E5B9ull;
  h ^= h >> 32;
  return low + (int32_t)(h % (uint64_t)(high - low));
}

namespace {
class MockBackend : public engine::Backend {
 public:
  MockBackend(int32_t low, int32_t high, int32_t eos, int32_t every) : low_(low), high_(high), eos_(eos), every_(every) {}
  int32_t f(int32_t tok, int32_t pos) const {
    if (eos_ >= 0 && every_ > 0 && (pos + 1) % every_ == 0) return eos_;
    return mock_next_token(tok, pos, low_, high_);
  }
  bool execute(const engine::StepPlan& p, engine::StepResult* r) override {
    const size_t n = p.seq_slot.size();
    r->status = 0;
    r->outputs.assign(n, wire::SeqStepOutput{});
    for (size_t i = 0; i < n; ++i) {
      wire::SeqStepOutput& o = r->outputs[i];
      o.req_slot = p.seq_slot[i];
      o.num_tokens = 0;
      if (p.sample_row[i] < 0) continue;
      const int r0 = p.query_start[i], r1 = p.query_start[i + 1];
      const int width = i < p.spec_width.size() ? p.spec_width[i] : 0;
      if (width > 0) {
        int acc = 0;
        for (int row = r0; row < r1 && acc < wire::kMaxSpecTokens; ++row) {
          const int32_t target = f(p.token_ids[row], p.positions[row]);
          o.tokens[acc] = target;
          o.logprobs[acc] = -0.5f;
          ++acc;
          if (row + 1 >= r1 || p.token_ids[row + 1] != target) break;
        }
        o.num_tokens = acc;
      } else {
        const int row = r1 - 1;
        o.tokens[0] = f(p.token_ids[row], p.positions[row]);
        o.logprobs[0] = -0.5f;
        o.num_tokens = 1;
      }
      for (int k = 0; k < wire::kMaxTopLogprobs; ++k) {
        o.top_ids[k] = low_ + k;
        o.top_logprobs[k] = -1.0f - k;
      }
    }
    return true;
  }

 private:
  int32_t low_, high_, eos_, every_;
};
}  // namespace

std::shared_ptr<engine::Backend> make_mock_backend(int32_t low, int32_t high, int32_t eos_id, int32_t eos_every) {
  return std::make_shared<MockBackend>(low, high, eos_id, eos_every);
}

}  // namespace serve
}  // namespace zs
