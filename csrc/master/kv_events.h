// Prefix-cache KV events (BlockStored / BlockRemoved / AllBlocksCleared) for external
// KV-aware routers.
//
// Encoding: one msgpack batch per event, `[ts_f64, [{"type": ..., "block_hashes":
// [bin8, ...], "medium": "GPU"}]]`; a block hash is the 8-byte external key of the block
// (the SHA-256 CBOR chain of kv.h), big-endian.
// Transport: a ZMTP 3.0 PUB socket (NULL mechanism) that connects to `tcp://host:port`
// and sends multipart messages [topic, sequence (u64 big-endian), batch] to subscribers
// whose subscription prefix matches the topic; or `file://path`, which appends
// length-prefixed (u32 big-endian) batches.  Publishing never blocks the engine: events
// go through a bounded queue to a background thread (overflow drops the oldest and is
// counted).
//
// Reference parity: crates/zs-server/src/serve/kv_events.rs:25 (encode_kv_event_batch),
// :69 (KvEventPublisher::spawn).
#pragma once

#include <stdint.h>

#include <atomic>
#include <condition_variable>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "kv.h"

namespace zs {
namespace kvev {

// msgpack batch of one event at unix time `ts`.
std::string encode_batch(const kv::KvEvent& ev, double ts);

class Publisher {
 public:
  // endpoint: "tcp://host:port" or "file://path".
  Publisher(std::string endpoint, std::string topic, size_t queue_cap = 4096);
  ~Publisher();
  bool start(std::string* error);
  void publish(const kv::KvEvent& ev);
  void stop();
  uint64_t sent() const { return sent_.load(); }
  uint64_t dropped() const { return dropped_.load(); }
  kv::KvEventSink sink() {
    return [this](const kv::KvEvent& e) { publish(e); };
  }

 private:
  void run();
  bool connect_tcp(std::string* error);
  bool send_frames(const std::vector<std::string>& parts);
  void poll_subscriptions();

  std::string endpoint_, topic_;
  size_t cap_;
  int fd_ = -1;
  FILE* file_ = nullptr;
  std::vector<std::string> subs_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<std::string> q_;
  std::thread th_;
  std::atomic<bool> stop_{false};
  std::atomic<uint64_t> sent_{0}, dropped_{0};
  uint64_t seq_ = 0;
  std::string rx_;  // partial frames from the subscriber
};

}  // namespace kvev
}  // namespace zs
