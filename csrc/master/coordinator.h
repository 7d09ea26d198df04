// Master side of the shared-memory transport: spawns the worker processes, publishes
// step plans into double-buffered plan slots, wakes the workers through per-rank
// eventfds and waits for their completion eventfds in short slices, checking child
// liveness, worker status words and heartbeats between slices.  Any failure sets the
// segment's abort word so every worker stops, and surfaces as an engine error.
//
// Reference parity: crates/zs-scheduler/src/coordinator.rs (launch :343,
// spawn_workers :733 with PR_SET_PDEATHSIG, publish_prepared :619, wait_all :630,
// check_peer_states_and_heartbeats :911, Drop :717).
#pragma once

#include <sys/types.h>

#include <map>
#include <deque>
#include <string>
#include <vector>

#include "engine.h"
#include "shm.h"
#include "wire.h"

namespace zs {

struct CoordinatorConfig {
  wire::Geometry geo;
  std::vector<std::string> worker_argv;      // command; per-rank fd/rank flags are appended
  std::map<std::string, std::string> env;    // extra environment for the workers
  int ready_timeout_ms = 600000;
  int step_timeout_ms = 120000;
  int heartbeat_timeout_ms = 5000;
  int slice_ms = 200;
  std::string shm_name;                      // POSIX shared-memory object name (empty: unique per run)
};

class Coordinator : public engine::Backend {
 public:
  explicit Coordinator(CoordinatorConfig cfg);
  ~Coordinator() override;
  // Create the segment, spawn the workers and wait until all report READY.
  void launch();
  bool execute(const engine::StepPlan& plan, engine::StepResult* result) override;
  // Publish a step and return; collect() waits for the oldest published step's result.
  bool submit(const engine::StepPlan& plan) override;
  bool collect(engine::StepResult* result) override;
  bool async_capable() const override { return true; }
  std::string error() const override { return error_; }
  void shutdown();
  // Check every worker (alive, no error status, fresh heartbeat while busy).
  bool healthy(std::string* why);
  const wire::SegmentLayout& layout() const { return layout_; }
  uint8_t* segment() const { return arena_.base(); }
  std::vector<pid_t> pids() const { return pids_; }
  uint64_t last_step() const { return step_id_; }
  // Metrics
  uint64_t publish_ns_total = 0, wait_ns_total = 0, steps = 0;

 private:
  void write_plan(const engine::StepPlan& plan, uint8_t* slot, uint64_t step_id);
  bool wait_all(uint64_t step_id, int timeout_ms);
  void set_abort(const std::string& why);

  CoordinatorConfig cfg_;
  wire::SegmentLayout layout_;
  ShmArena arena_;
  std::vector<EventFd> plan_efd_, done_efd_;
  std::vector<pid_t> pids_;
  uint64_t step_id_ = 0;
  std::deque<uint64_t> inflight_;  // published step ids, oldest first
  std::string error_;
  bool launched_ = false;
};

// Write a staged plan into a plan slot (shared by the coordinator and tests).
void write_plan_slot(const wire::SegmentLayout& l, const engine::StepPlan& plan, uint8_t* slot, uint64_t step_id);

}  // namespace zs
