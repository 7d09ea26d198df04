#include "coordinator.h"

#include <errno.h>
#include <fcntl.h>
#include <signal.h>
#include <sys/prctl.h>
#include <sys/wait.h>
#include <unistd.h>

#include <atomic>
#include <cstring>
#include <stdexcept>

namespace zs {

namespace {
std::atomic<uint64_t> g_segment_counter{0};

void clear_cloexec(int fd) {
  const int flags = fcntl(fd, F_GETFD);
  if (flags >= 0) fcntl(fd, F_SETFD, flags & ~FD_CLOEXEC);
}
}  // namespace

void write_plan_slot(const wire::SegmentLayout& l, const engine::StepPlan& p, uint8_t* slot, uint64_t step_id) {
  const wire::PlanLayout& pl = l.plan;
  auto h = reinterpret_cast<wire::StepHeader*>(slot + pl.header);
  const uint32_t rows = uint32_t(p.token_ids.size());
  const uint32_t seqs = uint32_t(p.seq_slot.size());
  if (rows > l.geo.max_step_tokens || seqs > l.geo.max_seqs) throw std::runtime_error("plan exceeds geometry");
  auto put = [&](size_t off, const std::vector<int32_t>& v) {
    if (!v.empty()) std::memcpy(slot + off, v.data(), v.size() * 4);
  };
  put(pl.token_ids, p.token_ids);
  put(pl.positions, p.positions);
  put(pl.row_slot, p.row_slot);
  put(pl.query_start, p.query_start);
  put(pl.seq_slot, p.seq_slot);
  put(pl.seq_len, p.seq_len);
  put(pl.sample_row, p.sample_row);
  if (!p.sampling.empty()) std::memcpy(slot + pl.sampling, p.sampling.data(), p.sampling.size() * sizeof(wire::SamplingParams));
  put(pl.dirty_rows, p.dirty_rows);
  for (size_t i = 0; i < p.dirty_pages.size(); ++i) {
    const auto& row = p.dirty_pages[i];
    const size_t n = std::min<size_t>(row.size(), l.geo.max_pages_per_seq);
    int32_t* dst = reinterpret_cast<int32_t*>(slot + pl.dirty_pages) + i * l.geo.max_pages_per_seq;
    std::memcpy(dst, row.data(), n * 4);
    for (size_t j = n; j < l.geo.max_pages_per_seq; ++j) dst[j] = 0;
  }
  if (p.ckpt_row.size() > pl.max_ckpt) throw std::runtime_error("too many checkpoints in one step");
  put(pl.ckpt_row, p.ckpt_row);
  put(pl.ckpt_slot, p.ckpt_slot);
  put(pl.restore_slot, p.restore_slot);
  put(pl.spec_width, p.spec_width);
  h->opcode = p.opcode;
  h->flags = p.flags;
  h->num_rows = rows;
  h->num_seqs = seqs;
  h->num_dirty_rows = uint32_t(p.dirty_rows.size());
  h->bucket = p.bucket;
  h->num_ckpt = uint32_t(p.ckpt_row.size());
  h->num_kv_ops = 0;
  h->master_ns = monotonic_ns();
  wire::store_release_u64(&h->step_id, step_id);
}

Coordinator::Coordinator(CoordinatorConfig cfg) : cfg_(std::move(cfg)) { layout_ = wire::segment_layout(cfg_.geo); }

Coordinator::~Coordinator() { shutdown(); }

void Coordinator::launch() {
  const std::string name =
      cfg_.shm_name.empty() ? "/zstep-" + std::to_string(getpid()) + "-" + std::to_string(g_segment_counter++)
                            : (cfg_.shm_name[0] == '/' ? cfg_.shm_name : "/" + cfg_.shm_name);
  arena_ = ShmArena::create(name, layout_.total_bytes);
  auto sb = reinterpret_cast<wire::Superblock*>(arena_.base());
  sb->magic = wire::kMagic;
  sb->version = wire::kVersion;
  sb->layout_hash = wire::layout_hash(layout_);
  sb->world_size = cfg_.geo.world_size;
  sb->max_seqs = cfg_.geo.max_seqs;
  sb->max_step_tokens = cfg_.geo.max_step_tokens;
  sb->max_pages_per_seq = cfg_.geo.max_pages_per_seq;
  sb->page_size = cfg_.geo.page_size;
  sb->vocab_size = cfg_.geo.vocab_size;
  sb->plan_offset = layout_.plan_offset;
  sb->plan_slot_bytes = layout_.plan.bytes;
  sb->result_offset = layout_.result_offset;
  sb->result_slot_bytes = layout_.result.bytes;
  sb->total_bytes = layout_.total_bytes;
  sb->master_pid = uint32_t(getpid());
  const int W = int(cfg_.geo.world_size);
  for (int r = 0; r < W; ++r) {
    plan_efd_.push_back(EventFd::create());
    done_efd_.push_back(EventFd::create());
  }
  for (int r = 0; r < W; ++r) {
    std::vector<std::string> args = cfg_.worker_argv;
    args.push_back("--shm-fd");
    args.push_back(std::to_string(arena_.fd()));
    args.push_back("--shm-bytes");
    args.push_back(std::to_string(layout_.total_bytes));
    args.push_back("--plan-fd");
    args.push_back(std::to_string(plan_efd_[r].fd()));
    args.push_back("--done-fd");
    args.push_back(std::to_string(done_efd_[r].fd()));
    args.push_back("--rank");
    args.push_back(std::to_string(r));
    args.push_back("--world-size");
    args.push_back(std::to_string(W));
    const pid_t parent = getpid();
    const pid_t pid = fork();
    if (pid < 0) throw std::runtime_error("fork failed");
    if (pid == 0) {
      // Child: die with the master; keep the transport fds across exec.
      prctl(PR_SET_PDEATHSIG, SIGKILL);
      if (getppid() != parent) _exit(1);
      clear_cloexec(arena_.fd());
      clear_cloexec(plan_efd_[r].fd());
      clear_cloexec(done_efd_[r].fd());
      // The workers' process group is hosted by their own rank 0.  A master started from
      // inside a torchrun job inherits TORCHELASTIC_USE_AGENT_STORE=True, which would make
      // every worker a store client of a server that never starts (a hang at init).
      unsetenv("TORCHELASTIC_USE_AGENT_STORE");
      for (auto& kv : cfg_.env) setenv(kv.first.c_str(), kv.second.c_str(), 1);
      std::vector<char*> argv;
      for (auto& a : args) argv.push_back(const_cast<char*>(a.c_str()));
      argv.push_back(nullptr);
      execvp(argv[0], argv.data());
      _exit(127);
    }
    pids_.push_back(pid);
  }
  arena_.unlink_now();  // the fd keeps the segment alive; no /dev/shm entry remains
  launched_ = true;
  // Wait for READY from every rank.
  const uint64_t deadline = monotonic_ns() + uint64_t(cfg_.ready_timeout_ms) * 1000000ull;
  for (int r = 0; r < W; ++r) {
    auto ws = reinterpret_cast<wire::WorkerState*>(arena_.base() + wire::kSuperblockBytes + r * wire::kWorkerStateBytes);
    while (wire::load_acquire_u32(&ws->status) != wire::kWorkerReady) {
      std::string why;
      if (!healthy(&why)) throw std::runtime_error("worker failed during startup: " + why);
      if (monotonic_ns() > deadline) {
        set_abort("startup timeout");
        throw std::runtime_error("workers did not become ready in time");
      }
      done_efd_[r].wait(cfg_.slice_ms);
    }
  }
}

bool Coordinator::healthy(std::string* why) {
  for (size_t r = 0; r < pids_.size(); ++r) {
    int st = 0;
    const pid_t w = waitpid(pids_[r], &st, WNOHANG);
    if (w == pids_[r]) {
      *why = "rank " + std::to_string(r) + " exited (status " + std::to_string(st) + ")";
      pids_[r] = -1;
      return false;
    }
    if (pids_[r] < 0) {
      *why = "rank " + std::to_string(r) + " is gone";
      return false;
    }
    auto ws = reinterpret_cast<wire::WorkerState*>(arena_.base() + wire::kSuperblockBytes + r * wire::kWorkerStateBytes);
    if (wire::load_acquire_u32(&ws->status) == wire::kWorkerError) {
      *why = "rank " + std::to_string(r) + " reported error " + std::to_string(ws->error_code);
      return false;
    }
    const uint64_t hb = __atomic_load_n(&ws->heartbeat_ns, __ATOMIC_ACQUIRE);
    if (hb != 0 && monotonic_ns() > hb + uint64_t(cfg_.heartbeat_timeout_ms) * 1000000ull) {
      *why = "rank " + std::to_string(r) + " heartbeat stalled";
      return false;
    }
  }
  return true;
}

void Coordinator::set_abort(const std::string& why) {
  if (arena_.valid()) {
    auto sb = reinterpret_cast<wire::Superblock*>(arena_.base());
    wire::store_release_u32(&sb->abort_word, 1);
    for (auto& e : plan_efd_) e.signal();
  }
  if (error_.empty()) error_ = why;
}

bool Coordinator::wait_all(uint64_t step_id, int timeout_ms) {
  const uint64_t deadline = monotonic_ns() + uint64_t(timeout_ms) * 1000000ull;
  for (size_t r = 0; r < done_efd_.size(); ++r) {
    auto ws = reinterpret_cast<wire::WorkerState*>(arena_.base() + wire::kSuperblockBytes + r * wire::kWorkerStateBytes);
    while (__atomic_load_n(&ws->ready_step, __ATOMIC_ACQUIRE) < step_id) {
      std::string why;
      if (!healthy(&why)) {
        set_abort(why);
        return false;
      }
      if (monotonic_ns() > deadline) {
        set_abort("step " + std::to_string(step_id) + " timed out on rank " + std::to_string(r));
        return false;
      }
      done_efd_[r].wait(cfg_.slice_ms);
    }
  }
  return true;
}

void Coordinator::write_plan(const engine::StepPlan& plan, uint8_t* slot, uint64_t step_id) {
  write_plan_slot(layout_, plan, slot, step_id);
}

bool Coordinator::submit(const engine::StepPlan& plan) {
  if (!launched_ || !error_.empty()) return false;
  if (inflight_.size() >= (size_t)wire::kPlanSlots) {
    error_ = "more steps in flight than plan slots";
    return false;
  }
  const uint64_t t0 = monotonic_ns();
  const uint64_t step = ++step_id_;
  uint8_t* slot = arena_.base() + layout_.plan_offset + (step % wire::kPlanSlots) * layout_.plan.bytes;
  try {
    write_plan(plan, slot, step);
  } catch (const std::exception& e) {
    error_ = e.what();
    return false;
  }
  for (auto& e : plan_efd_) e.signal();
  publish_ns_total += monotonic_ns() - t0;
  inflight_.push_back(step);
  return true;
}

bool Coordinator::collect(engine::StepResult* result) {
  if (inflight_.empty()) return false;
  const uint64_t step = inflight_.front();
  inflight_.pop_front();
  const uint64_t t1 = monotonic_ns();
  if (!wait_all(step, cfg_.step_timeout_ms)) return false;
  wait_ns_total += monotonic_ns() - t1;
  ++steps;
  const uint8_t* rs = arena_.base() + layout_.result_offset + (step % wire::kResultSlots) * layout_.result.bytes;
  auto rh = reinterpret_cast<const wire::StepResultHeader*>(rs);
  if (wire::load_acquire_u64(const_cast<uint64_t*>(&rh->step_id)) != step) {
    error_ = "result slot not published for step " + std::to_string(step);
    return false;
  }
  result->status = rh->status;
  result->gpu_exec_us = rh->gpu_exec_us;
  const auto* outs = reinterpret_cast<const wire::SeqStepOutput*>(rs + layout_.result.outputs);
  result->outputs.assign(outs, outs + rh->num_seqs);
  return true;
}

bool Coordinator::execute(const engine::StepPlan& plan, engine::StepResult* result) {
  return submit(plan) && collect(result);
}

void Coordinator::shutdown() {
  if (!launched_) return;
  launched_ = false;
  // Ask politely with a Shutdown step, then make sure every child is gone.
  engine::StepPlan p;
  p.opcode = wire::kOpShutdown;
  const uint64_t step = ++step_id_;
  try {
    write_plan(p, arena_.base() + layout_.plan_offset + (step % wire::kPlanSlots) * layout_.plan.bytes, step);
    for (auto& e : plan_efd_) e.signal();
  } catch (...) {
  }
  const uint64_t deadline = monotonic_ns() + 10ull * 1000000000ull;
  for (pid_t& pid : pids_) {
    if (pid <= 0) continue;
    while (true) {
      int st = 0;
      if (waitpid(pid, &st, WNOHANG) == pid) break;
      if (monotonic_ns() > deadline) {
        kill(pid, SIGKILL);
        waitpid(pid, &st, 0);
        break;
      }
      usleep(10000);
    }
    pid = -1;
  }
}

}  // namespace zs
