// Online serving loop: one thread owns the Engine and drives it step by step; request
// handlers talk to it through a bounded command queue and read their tokens from a
// per-request stream.
//
//  * submit -> Overloaded (waiting queue full, HTTP 429), Draining / Faulted (503)
//  * cancel -> the request leaves at the next step boundary; its pages return to the
//    pool (the engine's leases), no KV leaks
//  * drain  -> stop admitting; in-flight requests finish; state Draining
//  * a poisoned engine (worker died, kernel error) turns the state to Faulted and fails
//    every open stream
// Lock-free counters and fixed-bucket histograms back the Prometheus endpoint.
//
// Reference parity: crates/zs-scheduler/src/serve_loop.rs (LoopEvent :124, SubmitError
// :152, EngineState :164, OnlineMetrics :184, run_loop :479, spawn_mock :1358).
#pragma once

#include <stdint.h>

#include <atomic>
#include <condition_variable>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "engine.h"

namespace zs {
namespace serve {

enum class EngineState : int { kStarting = 0, kReady = 1, kDraining = 2, kFaulted = 3 };
const char* state_name(EngineState s);

enum class SubmitError : int { kOk = 0, kOverloaded, kDraining, kFaulted, kStarting };

// Cumulative histogram with fixed upper bounds (seconds).
class Histogram {
 public:
  explicit Histogram(std::vector<double> bounds);
  void observe(double v);
  const std::vector<double>& bounds() const { return bounds_; }
  std::vector<uint64_t> counts() const;  // per bucket (not cumulative), last = +Inf
  double sum() const;
  uint64_t count() const { return count_.load(); }

 private:
  std::vector<double> bounds_;
  std::unique_ptr<std::atomic<uint64_t>[]> buckets_;
  std::atomic<uint64_t> count_{0};
  std::atomic<uint64_t> sum_us_{0};
};

struct OnlineMetrics {
  OnlineMetrics();
  std::atomic<uint64_t> requests_ok{0}, requests_length{0}, requests_cancelled{0}, requests_error{0},
      requests_rejected{0}, prompt_tokens{0}, generation_tokens{0}, cached_prompt_tokens{0};
  Histogram ttft, tpot, e2e;
};

// One event delivered to a request's consumer.
struct StreamEvent {
  std::vector<int32_t> tokens;
  std::vector<float> logprobs;
  std::vector<std::vector<std::pair<int32_t, float>>> top_logprobs;
  engine::Finish finish = engine::Finish::kNone;
  uint32_t prompt_tokens = 0, completion_tokens = 0, cached_tokens = 0;
  std::string error;
};

class RequestStream {
 public:
  explicit RequestStream(uint64_t id) : id_(id) {}
  uint64_t id() const { return id_; }
  // Waits up to timeout_ms; returns false on timeout.
  bool pop(StreamEvent* ev, int timeout_ms);
  void push(StreamEvent ev);
  bool closed() const { return closed_.load(); }

 private:
  friend class ServeLoop;
  uint64_t id_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<StreamEvent> q_;
  std::atomic<bool> closed_{false};
};

class ServeLoop {
 public:
  // `keepalive` holds the backend owner (e.g. the coordinator) for the loop's lifetime.
  ServeLoop(std::shared_ptr<engine::Engine> engine, std::shared_ptr<void> keepalive = nullptr,
            size_t max_waiting = 1024);
  ~ServeLoop();
  void start();  // spawns the engine thread; state Ready
  SubmitError submit(engine::Request r, std::shared_ptr<RequestStream>* out);
  void cancel(uint64_t id);
  void drain();
  void shutdown();
  bool idle() const;  // no waiting or running requests
  EngineState state() const { return (EngineState)state_.load(); }
  void set_state(EngineState s) { state_.store((int)s); }
  OnlineMetrics& metrics() { return metrics_; }
  engine::EngineStats stats() const;
  std::string error() const;
  uint64_t next_request_id() { return next_id_.fetch_add(1) + 1; }

 private:
  struct Track {
    std::shared_ptr<RequestStream> stream;
    double t_submit = 0, t_first = 0, t_last = 0;
    uint32_t generated = 0;
  };
  void run();
  void fail_all(const std::string& why);

  std::shared_ptr<engine::Engine> engine_;
  std::shared_ptr<void> keepalive_;
  size_t max_waiting_;
  std::thread thread_;
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::deque<engine::Request> submits_;
  std::vector<uint64_t> cancels_;
  std::map<uint64_t, Track> live_;
  std::atomic<int> state_{(int)EngineState::kStarting};
  std::atomic<bool> stop_{false};
  std::atomic<uint64_t> next_id_{0};
  std::atomic<size_t> in_system_{0};
  engine::EngineStats stats_;
  std::string error_;
  OnlineMetrics metrics_;
};

// Deterministic scripted backend (no GPU, no workers): each sampled row's next token is
// a hash of its last input token and position, mapped into [low, high); `eos_every`
// > 0 makes position multiples of it emit `eos_id`.  Verify rows accept a draft when it
// equals that function, so speculative paths are exercised too.
std::shared_ptr<engine::Backend> make_mock_backend(int32_t low, int32_t high, int32_t eos_id = -1,
                                                   int32_t eos_every = 0);
int32_t mock_next_token(int32_t last, int32_t pos, int32_t low, int32_t high);

}  // namespace serve
}  // namespace zs
