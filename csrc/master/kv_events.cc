#include "kv_events.h"

#include <arpa/inet.h>
#include <errno.h>
#include <netdb.h>
#include <poll.h>
#include <string.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <unistd.h>

#include <chrono>

namespace zs {
namespace kvev {

namespace {

// ------------------------------------------------------------------ msgpack writer
void mp_u8(std::string& o, uint8_t v) { o += (char)v; }
void mp_be(std::string& o, uint64_t v, int bytes) {
  for (int i = bytes - 1; i >= 0; --i) o += (char)((v >> (8 * i)) & 0xFF);
}
void mp_str(std::string& o, const std::string& s) {
  if (s.size() < 32) {
    mp_u8(o, 0xA0 | (uint8_t)s.size());
  } else if (s.size() < 256) {
    mp_u8(o, 0xD9);
    mp_u8(o, (uint8_t)s.size());
  } else {
    mp_u8(o, 0xDA);
    mp_be(o, s.size(), 2);
  }
  o += s;
}
void mp_bin(std::string& o, const std::string& b) {
  mp_u8(o, 0xC4);
  mp_u8(o, (uint8_t)b.size());
  o += b;
}
void mp_array(std::string& o, size_t n) {
  if (n < 16) {
    mp_u8(o, 0x90 | (uint8_t)n);
  } else {
    mp_u8(o, 0xDC);
    mp_be(o, n, 2);
  }
}
void mp_map(std::string& o, size_t n) { mp_u8(o, 0x80 | (uint8_t)n); }
void mp_f64(std::string& o, double d) {
  uint64_t u;
  memcpy(&u, &d, 8);
  mp_u8(o, 0xCB);
  mp_be(o, u, 8);
}

std::string key_bytes(uint64_t k) {
  std::string b;
  mp_be(b, k, 8);
  return b;
}

bool write_all(int fd, const std::string& s) {
  size_t off = 0;
  while (off < s.size()) {
    const ssize_t n = ::send(fd, s.data() + off, s.size() - off, MSG_NOSIGNAL);
    if (n < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    off += (size_t)n;
  }
  return true;
}

bool read_exact(int fd, size_t n, std::string* out, int timeout_ms) {
  out->clear();
  while (out->size() < n) {
    pollfd p{fd, POLLIN, 0};
    if (::poll(&p, 1, timeout_ms) <= 0) return false;
    char buf[256];
    const ssize_t r = ::recv(fd, buf, std::min(sizeof(buf), n - out->size()), 0);
    if (r <= 0) return false;
    out->append(buf, (size_t)r);
  }
  return true;
}

// ZMTP frame: flags (bit0 MORE, bit1 LONG, bit2 COMMAND), size (1 or 8 bytes), body.
std::string frame(const std::string& body, bool more, bool command = false) {
  std::string f;
  uint8_t flags = (more ? 1 : 0) | (command ? 4 : 0);
  if (body.size() > 255) {
    f += (char)(flags | 2);
    mp_be(f, body.size(), 8);
  } else {
    f += (char)flags;
    f += (char)body.size();
  }
  return f + body;
}

std::string greeting() {
  std::string g(64, '\0');
  g[0] = (char)0xFF;
  g[9] = 0x7F;
  g[10] = 3;  // major
  g[11] = 0;  // minor
  memcpy(&g[12], "NULL", 4);
  return g;  // as-server = 0, filler zeros
}

std::string ready_command(const char* socket_type) {
  std::string body;
  body += (char)5;
  body += "READY";
  body += (char)11;
  body += "Socket-Type";
  mp_be(body, strlen(socket_type), 4);
  body += socket_type;
  return frame(body, false, true);
}

}  // namespace

std::string encode_batch(const kv::KvEvent& ev, double ts) {
  std::string o;
  mp_array(o, 2);
  mp_f64(o, ts);
  mp_array(o, 1);
  if (ev.kind == kv::KvEvent::kAllCleared) {
    mp_map(o, 1);
    mp_str(o, "type");
    mp_str(o, "AllBlocksCleared");
    return o;
  }
  const bool stored = ev.kind == kv::KvEvent::kStored;
  mp_map(o, stored ? 3 : 2);
  mp_str(o, "type");
  mp_str(o, stored ? "BlockStored" : "BlockRemoved");
  mp_str(o, "block_hashes");
  mp_array(o, ev.block_keys.size());
  for (uint64_t k : ev.block_keys) mp_bin(o, key_bytes(k));
  if (stored) {
    mp_str(o, "medium");
    mp_str(o, "GPU");
  }
  return o;
}

Publisher::Publisher(std::string endpoint, std::string topic, size_t queue_cap)
    : endpoint_(std::move(endpoint)), topic_(std::move(topic)), cap_(queue_cap) {}

Publisher::~Publisher() { stop(); }

bool Publisher::connect_tcp(std::string* error) {
  const std::string hp = endpoint_.substr(6);
  const size_t c = hp.rfind(':');
  if (c == std::string::npos) {
    *error = "kv events endpoint needs tcp://host:port";
    return false;
  }
  addrinfo hints{}, *res = nullptr;
  hints.ai_family = AF_INET;
  hints.ai_socktype = SOCK_STREAM;
  if (getaddrinfo(hp.substr(0, c).c_str(), hp.substr(c + 1).c_str(), &hints, &res) != 0 || !res) {
    *error = "cannot resolve " + hp;
    return false;
  }
  fd_ = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
  const bool ok = fd_ >= 0 && ::connect(fd_, res->ai_addr, res->ai_addrlen) == 0;
  freeaddrinfo(res);
  if (!ok) {
    *error = "connect " + hp + ": " + strerror(errno);
    return false;
  }
  // Greeting exchange, then READY commands (NULL security mechanism).
  std::string peer;
  if (!write_all(fd_, greeting()) || !read_exact(fd_, 64, &peer, 5000) || (uint8_t)peer[0] != 0xFF ||
      peer[10] < 3) {
    *error = "ZMTP greeting failed";
    return false;
  }
  if (!write_all(fd_, ready_command("PUB"))) {
    *error = "ZMTP handshake failed";
    return false;
  }
  std::string hdr, body;
  if (!read_exact(fd_, 2, &hdr, 5000)) {
    *error = "no READY from subscriber";
    return false;
  }
  size_t len = (uint8_t)hdr[1];
  if ((uint8_t)hdr[0] & 2) {
    std::string rest;
    if (!read_exact(fd_, 7, &rest, 5000)) return false;
    len = 0;
    const std::string all = hdr.substr(1) + rest;
    for (char ch : all) len = (len << 8) | (uint8_t)ch;
  }
  if (!read_exact(fd_, len, &body, 5000) || body.compare(1, 5, "READY") != 0) {
    *error = "bad READY from subscriber";
    return false;
  }
  return true;
}

void Publisher::poll_subscriptions() {
  if (fd_ < 0) return;
  while (true) {
    pollfd p{fd_, POLLIN, 0};
    if (::poll(&p, 1, 0) <= 0) return;
    char buf[1024];
    const ssize_t n = ::recv(fd_, buf, sizeof(buf), MSG_DONTWAIT);
    if (n <= 0) return;
    rx_.append(buf, (size_t)n);
    while (rx_.size() >= 2) {
      const uint8_t flags = (uint8_t)rx_[0];
      size_t hdr = 2, len = (uint8_t)rx_[1];
      if (flags & 2) {
        if (rx_.size() < 9) break;
        hdr = 9;
        len = 0;
        for (int i = 1; i < 9; ++i) len = (len << 8) | (uint8_t)rx_[i];
      }
      if (rx_.size() < hdr + len) break;
      const std::string body = rx_.substr(hdr, len);
      rx_.erase(0, hdr + len);
      if (!(flags & 4) && !body.empty() && body[0] == 1) subs_.push_back(body.substr(1));        // subscribe
      if (!(flags & 4) && !body.empty() && body[0] == 0) {                                        // unsubscribe
        for (auto it = subs_.begin(); it != subs_.end(); ++it)
          if (*it == body.substr(1)) {
            subs_.erase(it);
            break;
          }
      }
      if ((flags & 4) && body.size() > 10 && body.compare(1, 9, "SUBSCRIBE") == 0) subs_.push_back(body.substr(10));
    }
  }
}

bool Publisher::send_frames(const std::vector<std::string>& parts) {
  std::string out;
  for (size_t i = 0; i < parts.size(); ++i) out += frame(parts[i], i + 1 < parts.size());
  return write_all(fd_, out);
}

bool Publisher::start(std::string* error) {
  if (endpoint_.rfind("file://", 0) == 0) {
    file_ = fopen(endpoint_.substr(7).c_str(), "ab");
    if (!file_) {
      *error = "cannot open " + endpoint_;
      return false;
    }
  } else if (endpoint_.rfind("tcp://", 0) == 0) {
    if (!connect_tcp(error)) return false;
  } else {
    *error = "kv events endpoint must be tcp://host:port or file://path";
    return false;
  }
  kv::KvEvent cleared;
  cleared.kind = kv::KvEvent::kAllCleared;
  publish(cleared);  // a fresh cache starts empty
  th_ = std::thread([this] { run(); });
  return true;
}

void Publisher::publish(const kv::KvEvent& ev) {
  struct timeval tv;
  gettimeofday(&tv, nullptr);
  std::string batch = encode_batch(ev, (double)tv.tv_sec + tv.tv_usec * 1e-6);
  {
    std::lock_guard<std::mutex> lk(mu_);
    if (q_.size() >= cap_) {
      q_.pop_front();
      dropped_.fetch_add(1);
    }
    q_.push_back(std::move(batch));
  }
  cv_.notify_one();
}

void Publisher::run() {
  while (true) {
    std::string batch;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait_for(lk, std::chrono::milliseconds(50), [&] { return stop_.load() || !q_.empty(); });
      if (q_.empty()) {
        if (stop_.load()) break;
        lk.unlock();
        poll_subscriptions();
        continue;
      }
      batch = std::move(q_.front());
      q_.pop_front();
    }
    if (file_) {
      std::string len;
      mp_be(len, batch.size(), 4);
      fwrite(len.data(), 1, 4, file_);
      fwrite(batch.data(), 1, batch.size(), file_);
      fflush(file_);
      sent_.fetch_add(1);
      continue;
    }
    // PUB semantics: deliver to matching subscriptions; wait briefly for the first one.
    for (int i = 0; i < 100 && subs_.empty() && !stop_.load(); ++i) {
      poll_subscriptions();
      if (subs_.empty()) usleep(10000);
    }
    poll_subscriptions();
    bool match = false;
    for (const auto& s : subs_) match |= topic_.compare(0, s.size(), s) == 0;
    if (!match) {
      dropped_.fetch_add(1);
      continue;
    }
    std::string seq;
    mp_be(seq, seq_++, 8);
    if (send_frames({topic_, seq, batch})) sent_.fetch_add(1);
    else dropped_.fetch_add(1);
  }
}

void Publisher::stop() {
  if (stop_.exchange(true)) return;
  cv_.notify_all();
  if (th_.joinable()) th_.join();
  if (fd_ >= 0) ::close(fd_);
  if (file_) fclose(file_);
  fd_ = -1;
  file_ = nullptr;
}

}  // namespace kvev
}  // namespace zs
