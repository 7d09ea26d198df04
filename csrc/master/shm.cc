#include "shm.h"

#include <errno.h>
#include <fcntl.h>
#include <poll.h>
#include <sys/eventfd.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace zs {

uint64_t monotonic_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return uint64_t(ts.tv_sec) * 1000000000ull + uint64_t(ts.tv_nsec);
}

static std::runtime_error sys_error(const std::string& what) {
  return std::runtime_error(what + ": " + std::strerror(errno));
}

ShmArena::~ShmArena() { reset(); }

ShmArena::ShmArena(ShmArena&& o) noexcept { *this = std::move(o); }

ShmArena& ShmArena::operator=(ShmArena&& o) noexcept {
  if (this != &o) {
    reset();
    name_ = std::move(o.name_);
    fd_ = o.fd_;
    base_ = o.base_;
    size_ = o.size_;
    owner_ = o.owner_;
    unlinked_ = o.unlinked_;
    o.fd_ = -1;
    o.base_ = nullptr;
    o.size_ = 0;
    o.owner_ = false;
  }
  return *this;
}

void ShmArena::reset() {
  if (base_) munmap(base_, size_);
  if (fd_ >= 0) close(fd_);
  if (owner_ && !unlinked_ && !name_.empty()) shm_unlink(name_.c_str());
  base_ = nullptr;
  fd_ = -1;
  size_ = 0;
  owner_ = false;
}

ShmArena ShmArena::create(const std::string& name, size_t bytes) {
  ShmArena a;
  a.name_ = name;
  a.fd_ = shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
  if (a.fd_ < 0) throw sys_error("shm_open(" + name + ")");
  a.owner_ = true;
  if (ftruncate(a.fd_, off_t(bytes)) != 0) throw sys_error("ftruncate");
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, a.fd_, 0);
  if (p == MAP_FAILED) throw sys_error("mmap");
  a.base_ = static_cast<uint8_t*>(p);
  a.size_ = bytes;
  std::memset(a.base_, 0, bytes);
  return a;
}

ShmArena ShmArena::open(const std::string& name, bool read_only) {
  const int fd = shm_open(name.c_str(), read_only ? O_RDONLY : O_RDWR, 0600);
  if (fd < 0) throw sys_error("shm_open(" + name + ")");
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    throw sys_error("fstat");
  }
  ShmArena a = from_fd(fd, size_t(st.st_size), read_only);
  a.name_ = name;
  return a;
}

ShmArena ShmArena::from_fd(int fd, size_t bytes, bool read_only) {
  ShmArena a;
  a.fd_ = fd;
  void* p = mmap(nullptr, bytes, read_only ? PROT_READ : (PROT_READ | PROT_WRITE), MAP_SHARED, fd, 0);
  if (p == MAP_FAILED) throw sys_error("mmap");
  a.base_ = static_cast<uint8_t*>(p);
  a.size_ = bytes;
  return a;
}

void ShmArena::unlink_now() {
  if (!name_.empty() && !unlinked_) {
    shm_unlink(name_.c_str());
    unlinked_ = true;
  }
}

EventFd::~EventFd() {
  if (fd_ >= 0) close(fd_);
}

EventFd& EventFd::operator=(EventFd&& o) noexcept {
  if (this != &o) {
    if (fd_ >= 0) close(fd_);
    fd_ = o.fd_;
    o.fd_ = -1;
  }
  return *this;
}

EventFd EventFd::create() {
  const int fd = eventfd(0, EFD_NONBLOCK | EFD_CLOEXEC);
  if (fd < 0) throw sys_error("eventfd");
  return EventFd(fd);
}

void EventFd::signal(uint64_t n) const {
  if (fd_ < 0) return;
  ssize_t r;
  do {
    r = ::write(fd_, &n, sizeof(n));
  } while (r < 0 && errno == EINTR);
}

uint64_t EventFd::drain() const {
  uint64_t v = 0;
  if (fd_ < 0) return 0;
  ssize_t r;
  do {
    r = ::read(fd_, &v, sizeof(v));
  } while (r < 0 && errno == EINTR);
  return r == sizeof(v) ? v : 0;
}

uint64_t EventFd::wait(int timeout_ms) const {
  if (fd_ < 0) return 0;
  const uint64_t v = drain();
  if (v) return v;
  pollfd p{fd_, POLLIN, 0};
  int r;
  do {
    r = ::poll(&p, 1, timeout_ms);
  } while (r < 0 && errno == EINTR);
  if (r <= 0) return 0;
  return drain();
}

}  // namespace zs
