// OpenAI-compatible HTTP/1.1 + SSE front end of the master.
//
// Routes: POST /v1/chat/completions (streaming and not), GET /v1/models, probes
// (/livez, /health, /ready), GET /metrics (Prometheus text), POST /admin/drain.
// Auth: with an API key every /v1, /metrics and /admin route needs
// `Authorization: Bearer <key>` (constant-time compare); without one, /admin/drain
// (and /metrics unless remote metrics are allowed) is served to loopback peers only.
// An optional admin port (bound to 127.0.0.1) serves only the probes, /metrics and
// /admin.  Requests take the id from `x-nebula-request-id` / `x-request-id` (echoed)
// or get a generated one; a client that disconnects mid-stream cancels its request.
//
// One thread per connection (blocking sockets); each response closes the connection.
//
// Reference parity: crates/zs-server/src/serve.rs (router :154, probes, ChatRequest
// :340, reject_unsupported :415, resolve_sampling_params :482, CancelGuard :724,
// chat_completions :771), serve/auth.rs, serve/metrics.rs:65.
#pragma once

#include <stdint.h>

#include <atomic>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "serve_loop.h"
#include "tokenizer.h"

namespace zs {
namespace http {

struct ServerConfig {
  std::string host = "127.0.0.1";
  int port = 43537;              // 0 = pick a free port
  int admin_port = -1;           // -1 = none, 0 = pick a free port
  std::string api_key;
  std::string served_model_name = "zstep";
  uint32_t max_model_len = 32768;
  bool allow_remote_metrics = true;
  tok::TemplateFormat template_format = tok::TemplateFormat::kChatML;
  size_t max_body_bytes = 16u << 20;
  int max_connections = 4096;
};

class HttpServer {
 public:
  HttpServer(ServerConfig cfg, serve::ServeLoop* loop, const tok::Tokenizer* tokenizer);
  ~HttpServer();
  bool start(std::string* error);
  void stop();
  int port() const { return port_; }
  int admin_port() const { return admin_port_; }
  // Drain: stop admitting; in-flight streams finish (probes report it).
  void request_drain();
  size_t active_connections() const { return active_.load(); }

  // Prometheus text exposition of the loop's counters and engine stats.
  static std::string render_metrics(serve::ServeLoop* loop, const ServerConfig& cfg);

 private:
  struct Conn;
  bool listen_on(const std::string& host, int port, int* fd, int* bound_port, std::string* error);
  void accept_loop(int fd, bool admin_only);
  void handle(int fd, bool loopback_peer, bool admin_only);

  ServerConfig cfg_;
  serve::ServeLoop* loop_;
  const tok::Tokenizer* tok_;
  int listen_fd_ = -1, admin_fd_ = -1;
  int port_ = 0, admin_port_ = -1;
  std::atomic<bool> stop_{false};
  std::atomic<size_t> active_{0};
  std::atomic<uint64_t> counter_{0};
  std::vector<std::thread> acceptors_;
  uint64_t created_ = 0;
};

bool constant_time_eq(const std::string& a, const std::string& b);

}  // namespace http
}  // namespace zs
