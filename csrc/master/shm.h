// POSIX shared-memory segment and eventfd wrappers (RAII) for the master <-> worker
// transport.  The master creates the segment exclusively (O_EXCL, mode 0600), passes
// its file descriptor to the workers it spawns and unlinks the name right after, so a
// crash never leaves a stale /dev/shm entry behind.
//
// Reference parity: crates/zs-shm/src/arena.rs (create/open/unlink_now :73-158) and
// eventfd.rs (wait_until :94).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>

namespace zs {

class ShmArena {
 public:
  ShmArena() = default;
  ~ShmArena();
  ShmArena(const ShmArena&) = delete;
  ShmArena& operator=(const ShmArena&) = delete;
  ShmArena(ShmArena&& o) noexcept;
  ShmArena& operator=(ShmArena&& o) noexcept;

  // Create a new zero-filled segment (fails if the name exists).
  static ShmArena create(const std::string& name, size_t bytes);
  // Map an existing segment by name or by an inherited file descriptor.
  static ShmArena open(const std::string& name, bool read_only = false);
  static ShmArena from_fd(int fd, size_t bytes, bool read_only = false);

  void unlink_now();  // remove the name; the mapping stays valid
  uint8_t* base() const { return base_; }
  size_t size() const { return size_; }
  int fd() const { return fd_; }
  const std::string& name() const { return name_; }
  bool valid() const { return base_ != nullptr; }

 private:
  void reset();
  std::string name_;
  int fd_ = -1;
  uint8_t* base_ = nullptr;
  size_t size_ = 0;
  bool owner_ = false;
  bool unlinked_ = false;
};

class EventFd {
 public:
  EventFd() = default;
  explicit EventFd(int fd) : fd_(fd) {}
  ~EventFd();
  EventFd(const EventFd&) = delete;
  EventFd& operator=(const EventFd&) = delete;
  EventFd(EventFd&& o) noexcept : fd_(o.fd_) { o.fd_ = -1; }
  EventFd& operator=(EventFd&& o) noexcept;

  static EventFd create();
  void signal(uint64_t n = 1) const;
  // Wait until the counter is nonzero or `timeout_ms` elapses; returns the drained
  // counter value (0 on timeout).
  uint64_t wait(int timeout_ms) const;
  uint64_t drain() const;
  int fd() const { return fd_; }
  int release() {
    const int f = fd_;
    fd_ = -1;
    return f;
  }

 private:
  int fd_ = -1;
};

uint64_t monotonic_ns();

}  // namespace zs
