#include "http_server.h"

#include <arpa/inet.h>
#include <errno.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <string.h>
#include <sys/socket.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <map>

#include "json.h"
#include "shm.h"

namespace zs {
namespace http {

using json::Value;

bool constant_time_eq(const std::string& a, const std::string& b) {
  // Length is not secret; compare every byte of the expected token regardless.
  unsigned char diff = a.size() == b.size() ? 0 : 1;
  for (size_t i = 0; i < b.size(); ++i) diff |= (unsigned char)((i < a.size() ? a[i] : 0) ^ b[i]);
  return diff == 0;
}

namespace {

struct Request {
  std::string method, path, query, body;
  std::map<std::string, std::string> headers;  // lower-case names
  const std::string& header(const std::string& k) const {
    static const std::string empty;
    auto it = headers.find(k);
    return it == headers.end() ? empty : it->second;
  }
};

const char* reason(int code) {
  switch (code) {
    case 200: return "OK";
    case 400: return "Bad Request";
    case 401: return "Unauthorized";
    case 403: return "Forbidden";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 413: return "Payload Too Large";
    case 429: return "Too Many Requests";
    case 500: return "Internal Server Error";
    case 503: return "Service Unavailable";
  }
  return "Error";
}

bool write_all(int fd, const std::string& data) {
  size_t off = 0;
  while (off < data.size()) {
    const ssize_t n = ::send(fd, data.data() + off, data.size() - off, MSG_NOSIGNAL);
    if (n < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    off += (size_t)n;
  }
  return true;
}

bool send_response(int fd, int code, const std::string& body, const std::string& ctype,
                   const std::vector<std::pair<std::string, std::string>>& extra = {}) {
  // Plain string building, no C++ streams: this code also runs inside processes that
  // load a second C++ runtime, where stream locale facets are not safe to share.
  std::string h = "HTTP/1.1 " + std::to_string(code) + " " + reason(code) + "\r\nContent-Type: " + ctype +
                  "\r\nContent-Length: " + std::to_string(body.size()) + "\r\nConnection: close\r\n";
  for (const auto& kv : extra) h += kv.first + ": " + kv.second + "\r\n";
  h += "\r\n";
  return write_all(fd, h + body);
}

std::string num(double v) {
  char b[40];
  snprintf(b, sizeof(b), "%.9g", v);
  return b;
}

bool send_json(int fd, int code, const Value& v, const std::vector<std::pair<std::string, std::string>>& extra = {}) {
  return send_response(fd, code, v.dump(), "application/json", extra);
}

Value error_body(const std::string& type, const std::string& code, const std::string& message) {
  Value e = Value::object();
  e.set("message", message);
  e.set("type", type);
  e.set("param", Value());
  e.set("code", code);
  Value root = Value::object();
  root.set("error", e);
  return root;
}

bool send_error(int fd, int status, const std::string& type, const std::string& code, const std::string& message,
                const std::vector<std::pair<std::string, std::string>>& extra = {}) {
  return send_json(fd, status, error_body(type, code, message), extra);
}

bool bad_request(int fd, const std::string& message) {
  return send_error(fd, 400, "invalid_request_error", "invalid_parameter", message);
}

// Reads one request (headers + Content-Length body).  Returns an HTTP status on
// malformed input (0 = ok, -1 = connection closed).
int read_request(int fd, size_t max_body, Request* req) {
  std::string buf;
  char tmp[16384];
  size_t hdr_end = std::string::npos;
  while (hdr_end == std::string::npos) {
    const ssize_t n = ::recv(fd, tmp, sizeof(tmp), 0);
    if (n <= 0) {
      if (n < 0 && errno == EINTR) continue;
      return -1;
    }
    buf.append(tmp, (size_t)n);
    hdr_end = buf.find("\r\n\r\n");
    if (hdr_end == std::string::npos && buf.size() > 65536) return 413;
  }
  // Request line and header lines, split on CRLF.
  std::vector<std::string> lines;
  for (size_t a = 0; a <= hdr_end;) {
    size_t b = buf.find("\r\n", a);
    if (b == std::string::npos || b > hdr_end) b = hdr_end;
    lines.push_back(buf.substr(a, b - a));
    a = b + 2;
    if (b == hdr_end) break;
  }
  if (lines.empty()) return 400;
  {
    const std::string& line = lines[0];
    const size_t s1 = line.find(' ');
    const size_t s2 = s1 == std::string::npos ? std::string::npos : line.find(' ', s1 + 1);
    if (s1 == std::string::npos || s2 == std::string::npos) return 400;
    req->method = line.substr(0, s1);
    const std::string target = line.substr(s1 + 1, s2 - s1 - 1);
    if (req->method.empty() || target.empty()) return 400;
    const size_t q = target.find('?');
    req->path = target.substr(0, q);
    if (q != std::string::npos) req->query = target.substr(q + 1);
  }
  for (size_t li = 1; li < lines.size(); ++li) {
    const std::string& line = lines[li];
    const size_t c = line.find(':');
    if (c == std::string::npos) continue;
    std::string k = line.substr(0, c), v = line.substr(c + 1);
    for (auto& ch : k) ch = (char)tolower((unsigned char)ch);
    const size_t a = v.find_first_not_of(" \t");
    v = a == std::string::npos ? std::string() : v.substr(a);
    while (!v.empty() && (v.back() == ' ' || v.back() == '\t')) v.pop_back();
    req->headers[k] = v;
  }
  size_t len = 0;
  const std::string& cl = req->header("content-length");
  if (!cl.empty()) {
    char* end = nullptr;
    const unsigned long long v = strtoull(cl.c_str(), &end, 10);
    if (end == cl.c_str() || *end != '\0') return 400;
    if (v > max_body) return 413;
    len = (size_t)v;
  }
  req->body = buf.substr(hdr_end + 4);
  while (req->body.size() < len) {
    const ssize_t n = ::recv(fd, tmp, sizeof(tmp), 0);
    if (n <= 0) {
      if (n < 0 && errno == EINTR) continue;
      return -1;
    }
    req->body.append(tmp, (size_t)n);
  }
  req->body.resize(len);
  return 0;
}

bool peer_closed(int fd) {
  pollfd p{fd, POLLIN | POLLRDHUP, 0};
  if (::poll(&p, 1, 0) <= 0) return false;
  if (p.revents & (POLLRDHUP | POLLHUP | POLLERR)) return true;
  if (p.revents & POLLIN) {
    char c;
    const ssize_t n = ::recv(fd, &c, 1, MSG_PEEK | MSG_DONTWAIT);
    return n == 0;
  }
  return false;
}

std::string bearer_token(const Request& r) {
  const std::string& a = r.header("authorization");
  if (a.size() > 7 && strncasecmp(a.c_str(), "Bearer ", 7) == 0) return a.substr(7);
  return {};
}

Value token_bytes_json(const std::string& s) {
  Value b = Value::array();
  for (unsigned char c : s) b.push(Value((int)c));
  return b;
}

// ------------------------------------------------------------------ chat request
struct ChatParams {
  std::vector<tok::ChatMessage> messages;
  int64_t max_tokens = -1;
  bool stream = false, include_usage = false, ignore_eos = false, logprobs = false;
  int top_logprobs = 0;
  std::vector<std::string> stop;
  double temperature = 0.0, top_p = 1.0, presence = 0.0, frequency = 0.0, repetition = 1.0;
  int top_k = 0;
  bool has_seed = false;
  uint64_t seed = 0;
  bool thinking = false;
  std::string reasoning_effort;
  std::string user;  // opaque end-user id (logged only)
};

bool parse_content(const Value& c, std::string* out, std::string* err) {
  if (c.is_string()) {
    *out = c.as_string();
    return true;
  }
  if (c.is_null()) {
    out->clear();
    return true;
  }
  if (c.is_array()) {
    std::string s;
    for (const auto& part : c.items()) {
      if (!part.is_object() || part.get("type").as_string() != "text" || !part.get("text").is_string()) {
        *err = "only text content parts are supported";
        return false;
      }
      s += part.get("text").as_string();
    }
    *out = std::move(s);
    return true;
  }
  *err = "message content must be a string or a list of text parts";
  return false;
}

// Returns "" on success, else the 400 message.
std::string parse_chat(const Value& body, ChatParams* p) {
  if (!body.is_object()) return "request body must be a JSON object";
  static const char* kKnown[] = {"model", "messages", "max_tokens", "max_completion_tokens", "stream",
                                 "stream_options", "stop", "temperature", "top_p", "top_k", "n", "seed",
                                 "ignore_eos", "tools", "tool_choice", "response_format", "logprobs",
                                 "top_logprobs", "presence_penalty", "frequency_penalty", "repetition_penalty",
                                 "reasoning_effort", "chat_template_kwargs", "user"};
  for (const auto& kv : body.members()) {
    bool known = false;
    for (const char* k : kKnown) known |= kv.first == k;
    if (!known && !kv.second.is_null()) return "unsupported parameter `" + kv.first + "`";
  }
  if (!body.get("tools").is_null() || !body.get("tool_choice").is_null()) return "tool calling is not supported";
  if (body.get("user").is_string()) p->user = body.get("user").as_string();
  if (!body.get("response_format").is_null()) return "response_format is not supported";
  const Value& n = body.get("n");
  if (!n.is_null() && (!n.is_int() || n.as_int() != 1)) return "n=" + n.dump() + " is not supported";
  const Value& msgs = body.get("messages");
  if (!msgs.is_array() || msgs.size() == 0) return "messages must be a non-empty array";
  for (const auto& m : msgs.items()) {
    if (!m.is_object() || !m.get("role").is_string()) return "each message needs a string role";
    tok::ChatMessage cm;
    cm.role = m.get("role").as_string();
    if (cm.role != "system" && cm.role != "user" && cm.role != "assistant")
      return "unsupported message role `" + cm.role + "`";
    std::string err;
    if (!parse_content(m.get("content"), &cm.content, &err)) return err;
    if (m.get("reasoning_content").is_string()) cm.reasoning = m.get("reasoning_content").as_string();
    p->messages.push_back(std::move(cm));
  }
  for (const char* k : {"max_tokens", "max_completion_tokens"}) {
    const Value& v = body.get(k);
    if (v.is_null()) continue;
    if (!v.is_int() || v.as_int() < 1) return "max_tokens / max_completion_tokens must be >= 1";
    p->max_tokens = v.as_int();
  }
  if (!body.get("stream").is_null()) {
    if (!body.get("stream").is_bool()) return "stream must be a boolean";
    p->stream = body.get("stream").as_bool();
  }
  const Value& so = body.get("stream_options");
  if (!so.is_null()) {
    if (!so.is_object()) return "stream_options must be an object";
    for (const auto& kv : so.members())
      if (kv.first != "include_usage") return "unsupported stream_options parameter `" + kv.first + "`";
    p->include_usage = so.get("include_usage").is_bool() && so.get("include_usage").as_bool();
  }
  const Value& stop = body.get("stop");
  if (stop.is_string()) {
    p->stop.push_back(stop.as_string());
  } else if (stop.is_array()) {
    if (stop.size() > 4) return "stop accepts at most 4 sequences";
    for (const auto& s : stop.items()) {
      if (!s.is_string()) return "stop must be a string or a list of strings";
      p->stop.push_back(s.as_string());
    }
  } else if (!stop.is_null()) {
    return "stop must be a string or a list of strings";
  }
  auto num = [&](const char* k, double lo, double hi, double* out, const char* msg) -> std::string {
    const Value& v = body.get(k);
    if (v.is_null()) return "";
    if (!v.is_number() || !std::isfinite(v.as_double()) || v.as_double() < lo || v.as_double() > hi) return msg;
    *out = v.as_double();
    return "";
  };
  std::string e;
  if (!(e = num("temperature", 0.0, 2.0, &p->temperature, "temperature must be finite and within [0.0, 2.0]")).empty()) return e;
  if (!(e = num("top_p", 1e-9, 1.0, &p->top_p, "top_p must be finite and within (0.0, 1.0]")).empty()) return e;
  if (!(e = num("presence_penalty", -2.0, 2.0, &p->presence, "presence_penalty must be finite and within [-2.0, 2.0]")).empty()) return e;
  if (!(e = num("frequency_penalty", -2.0, 2.0, &p->frequency, "frequency_penalty must be finite and within [-2.0, 2.0]")).empty()) return e;
  if (!(e = num("repetition_penalty", 1e-6, 10.0, &p->repetition, "repetition_penalty must be within (0, 10]")).empty()) return e;
  const Value& tk = body.get("top_k");
  if (!tk.is_null()) {
    if (!tk.is_int() || tk.as_int() < -1) return "top_k must be -1, 0 (disabled), or >= 1";
    p->top_k = tk.as_int() <= 0 ? 0 : (int)tk.as_int();
  }
  const Value& seed = body.get("seed");
  if (!seed.is_null()) {
    if (!seed.is_int()) return "seed must be an integer";
    p->has_seed = true;
    p->seed = (uint64_t)seed.as_int();
  }
  if (!body.get("ignore_eos").is_null()) p->ignore_eos = body.get("ignore_eos").as_bool();
  if (!body.get("logprobs").is_null()) p->logprobs = body.get("logprobs").as_bool();
  const Value& tl = body.get("top_logprobs");
  if (!tl.is_null()) {
    if (!p->logprobs) return "top_logprobs can only be specified when logprobs is true";
    if (!tl.is_int() || tl.as_int() < 0 || tl.as_int() > 5) return "top_logprobs must be between 0 and 5";
    p->top_logprobs = (int)tl.as_int();
  }
  const Value& re = body.get("reasoning_effort");
  if (re.is_string()) p->reasoning_effort = re.as_string();
  const Value& kw = body.get("chat_template_kwargs");
  if (!kw.is_null()) {
    if (!kw.is_object()) return "chat_template_kwargs must be an object";
    for (const auto& kv : kw.members()) {
      if (kv.first == "enable_thinking") {
        p->thinking = kv.second.is_bool() && kv.second.as_bool();
      } else if (kv.first == "thinking_mode") {
        p->thinking = kv.second.is_string() && kv.second.as_string() == "thinking";
      } else {
        return "unsupported chat_template_kwargs parameter `" + kv.first + "`";
      }
    }
  }
  return "";
}

const char* finish_name(engine::Finish f, bool stop_hit) {
  if (stop_hit) return "stop";
  switch (f) {
    case engine::Finish::kStop: return "stop";
    case engine::Finish::kLength: return "length";
    case engine::Finish::kCancelled: return "stop";
    case engine::Finish::kError: return "error";
    default: return nullptr;
  }
}

}  // namespace

// ------------------------------------------------------------------ server
HttpServer::HttpServer(ServerConfig cfg, serve::ServeLoop* loop, const tok::Tokenizer* tokenizer)
    : cfg_(std::move(cfg)), loop_(loop), tok_(tokenizer) {
  created_ = (uint64_t)time(nullptr);
}

HttpServer::~HttpServer() { stop(); }

bool HttpServer::listen_on(const std::string& host, int port, int* fd, int* bound_port, std::string* error) {
  *fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (*fd < 0) {
    *error = std::string("socket: ") + strerror(errno);
    return false;
  }
  int one = 1;
  setsockopt(*fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in addr{};
  addr.sin_family = AF_INET;
  addr.sin_port = htons((uint16_t)port);
  if (inet_pton(AF_INET, host.c_str(), &addr.sin_addr) != 1) {
    *error = "bad bind address " + host;
    ::close(*fd);
    return false;
  }
  if (::bind(*fd, (sockaddr*)&addr, sizeof(addr)) != 0 || ::listen(*fd, 1024) != 0) {
    *error = "bind " + host + ":" + std::to_string(port) + ": " + strerror(errno);
    ::close(*fd);
    return false;
  }
  socklen_t len = sizeof(addr);
  getsockname(*fd, (sockaddr*)&addr, &len);
  *bound_port = ntohs(addr.sin_port);
  return true;
}

bool HttpServer::start(std::string* error) {
  if (!listen_on(cfg_.host, cfg_.port, &listen_fd_, &port_, error)) return false;
  if (cfg_.admin_port >= 0 && !listen_on("127.0.0.1", cfg_.admin_port, &admin_fd_, &admin_port_, error)) return false;
  acceptors_.emplace_back([this] { accept_loop(listen_fd_, false); });
  if (admin_fd_ >= 0) acceptors_.emplace_back([this] { accept_loop(admin_fd_, true); });
  return true;
}

void HttpServer::stop() {
  if (stop_.exchange(true)) return;
  for (int fd : {listen_fd_, admin_fd_})
    if (fd >= 0) ::shutdown(fd, SHUT_RDWR);
  for (auto& t : acceptors_)
    if (t.joinable()) t.join();
  for (int fd : {listen_fd_, admin_fd_})
    if (fd >= 0) ::close(fd);
  // Let open connections notice and finish (they hold no server-owned state beyond `this`).
  for (int i = 0; i < 500 && active_.load() > 0; ++i) usleep(10000);
}

void HttpServer::request_drain() { loop_->drain(); }

void HttpServer::accept_loop(int fd, bool admin_only) {
  while (!stop_.load()) {
    pollfd p{fd, POLLIN, 0};
    const int r = ::poll(&p, 1, 100);
    if (r <= 0) continue;
    sockaddr_in peer{};
    socklen_t len = sizeof(peer);
    const int c = ::accept4(fd, (sockaddr*)&peer, &len, SOCK_CLOEXEC);
    if (c < 0) continue;
    if ((int)active_.load() >= cfg_.max_connections) {
      send_error(c, 503, "server_error", "overloaded", "too many connections");
      ::close(c);
      continue;
    }
    int one = 1;
    setsockopt(c, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    const bool loopback = (ntohl(peer.sin_addr.s_addr) >> 24) == 127;
    active_.fetch_add(1);
    std::thread([this, c, loopback, admin_only] {
      handle(c, loopback, admin_only);
      ::close(c);
      active_.fetch_sub(1);
    }).detach();
  }
}

std::string HttpServer::render_metrics(serve::ServeLoop* loop, const ServerConfig& cfg) {
  std::string o;
  const auto st = loop->stats();
  auto& m = loop->metrics();
  const std::string model = "model_name=\"" + cfg.served_model_name + "\"";
  const std::string lbl = "{" + model + "}";
  auto head = [&](const char* name, const char* help, const char* type) {
    o += std::string("# HELP zstep:") + name + " " + help + "\n# TYPE zstep:" + name + " " + type + "\n";
  };
  auto gauge = [&](const char* name, const char* help, double v) {
    head(name, help, "gauge");
    o += std::string("zstep:") + name + lbl + " " + num(v) + "\n";
  };
  auto counter = [&](const char* name, const char* help, double v) {
    head(name, help, "counter");
    o += std::string("zstep:") + name + lbl + " " + num(v) + "\n";
  };
  auto hist = [&](const char* name, const char* help, const serve::Histogram& h) {
    head(name, help, "histogram");
    const auto c = h.counts();
    uint64_t cum = 0;
    for (size_t i = 0; i < h.bounds().size(); ++i) {
      cum += c[i];
      o += std::string("zstep:") + name + "_bucket{" + model + ",le=\"" + num(h.bounds()[i]) + "\"} " +
           std::to_string(cum) + "\n";
    }
    cum += c.back();
    o += std::string("zstep:") + name + "_bucket{" + model + ",le=\"+Inf\"} " + std::to_string(cum) + "\n";
    o += std::string("zstep:") + name + "_sum" + lbl + " " + num(h.sum()) + "\n";
    o += std::string("zstep:") + name + "_count" + lbl + " " + std::to_string(h.count()) + "\n";
  };
  gauge("num_requests_running", "Requests in the running batch.", st.running);
  gauge("num_requests_waiting", "Requests waiting for admission.", st.waiting);
  gauge("kv_cache_usage_perc", "Fraction of device KV pages in use.", st.kv_usage);
  gauge("engine_state", "0 starting, 1 ready, 2 draining, 3 faulted.", (double)(int)loop->state());
  counter("num_preemptions_total", "Preempted requests.", (double)st.preemptions);
  counter("prompt_tokens_total", "Prompt tokens of finished requests.", (double)m.prompt_tokens.load());
  counter("generation_tokens_total", "Generated tokens.", (double)m.generation_tokens.load());
  counter("prefix_cache_queries_total", "Prompt tokens looked up in the prefix cache.", (double)st.prefix_query_tokens);
  counter("prefix_cache_hits_total", "Prompt tokens served from the prefix cache.", (double)st.prefix_hit_tokens);
  counter("prefix_cache_evictions_total", "Prefix cache nodes evicted.", (double)st.prefix_evictions);
  head("request_outcomes_total", "Finished requests by outcome.", "counter");
  const std::pair<const char*, uint64_t> outcomes[] = {{"stop", m.requests_ok.load()},
                                                       {"length", m.requests_length.load()},
                                                       {"cancelled", m.requests_cancelled.load()},
                                                       {"error", m.requests_error.load()},
                                                       {"rejected", m.requests_rejected.load()}};
  for (const auto& kv : outcomes)
    o += "zstep:request_outcomes_total{" + model + ",outcome=\"" + kv.first + "\"} " + std::to_string(kv.second) + "\n";
  // Kept for dashboards built on the reference's metric set: nothing is JIT-compiled at run
  // time here (every kernel is built ahead of time for sm_100a), so it stays 0.
  counter("triton_recompilations_total", "Runtime kernel recompilations (always 0: kernels are prebuilt).", 0.0);
  if (st.spec_drafts > 0 || st.spec_verify_rows > 0) {
    counter("spec_decode_num_drafts_total", "Verify steps with drafts.", (double)st.spec_verify_steps);
    counter("spec_decode_num_draft_tokens_total", "Draft tokens proposed.", (double)st.spec_drafts);
    counter("spec_decode_num_accepted_tokens_total", "Draft tokens accepted.", (double)st.spec_accepted);
    gauge("spec_decode_mean_acceptance_length", "Mean tokens per verify step (accepted + bonus).",
          st.spec_verify_steps ? 1.0 + (double)st.spec_accepted / (double)st.spec_verify_steps : 0.0);
  }
  if (st.dram_capacity > 0) {
    gauge("dram_kv_capacity_blocks", "Host DRAM prefix-cache tier capacity.", (double)st.dram_capacity);
    gauge("dram_kv_occupied_blocks", "Blocks resident in the host DRAM tier.", (double)st.dram_occupied);
    counter("dram_kv_offloads_total", "Blocks demoted from HBM to host DRAM.", (double)st.dram_offloads);
    counter("dram_kv_reloads_total", "Blocks reloaded from host DRAM into HBM.", (double)st.dram_reloads);
    counter("dram_kv_evictions_total", "Blocks dropped from the full host DRAM tier.", (double)st.dram_evictions);
    counter("dram_kv_hit_tokens_total", "Prompt tokens served from the host DRAM tier.", (double)st.dram_hit_tokens);
  }
  hist("time_to_first_token_seconds", "Time to first token.", m.ttft);
  hist("time_per_output_token_seconds", "Time per output token after the first.", m.tpot);
  hist("e2e_request_latency_seconds", "End-to-end request latency.", m.e2e);
  return o;
}

void HttpServer::handle(int fd, bool loopback, bool admin_only) {
  Request req;
  const int rc = read_request(fd, cfg_.max_body_bytes, &req);
  if (rc < 0) return;
  if (rc > 0) {
    send_error(fd, rc, "invalid_request_error", "bad_request", rc == 413 ? "request too large" : "malformed request");
    return;
  }
  std::string rid = req.header("x-nebula-request-id");
  if (rid.empty()) rid = req.header("x-request-id");
  if (rid.empty()) {
    char buf[64];
    snprintf(buf, sizeof(buf), "chatcmpl-%llx-%llx", (unsigned long long)monotonic_ns(),
             (unsigned long long)counter_.fetch_add(1));
    rid = buf;
  }
  const std::vector<std::pair<std::string, std::string>> rid_hdr = {{"x-request-id", rid}};
  const serve::EngineState state = loop_->state();
  auto status_json = [](const char* s) {
    Value v = Value::object();
    v.set("status", s);
    return v;
  };
  // Probes.
  if (req.path == "/livez") {
    send_response(fd, 200, "ok", "text/plain");
    return;
  }
  if (req.path == "/health") {
    if (state == serve::EngineState::kReady) send_json(fd, 200, status_json("ok"));
    else if (state == serve::EngineState::kDraining) send_json(fd, 200, status_json("draining"));
    else send_json(fd, 503, status_json(serve::state_name(state)));
    return;
  }
  if (req.path == "/ready") {
    if (state == serve::EngineState::kReady) send_json(fd, 200, status_json("ready"));
    else send_json(fd, 503, status_json(serve::state_name(state)));
    return;
  }
  const bool authed = !cfg_.api_key.empty() && constant_time_eq(bearer_token(req), cfg_.api_key);
  auto unauthorized = [&] {
    send_error(fd, 401, "invalid_request_error", "invalid_api_key", "missing or invalid Authorization Bearer token",
               {{"WWW-Authenticate", "Bearer"}});
  };
  // Ops routes: the key when one is set, else loopback (metrics may be remote).
  if (req.path == "/metrics" || req.path == "/admin/drain") {
    const bool is_metrics = req.path == "/metrics";
    if (!cfg_.api_key.empty()) {
      if (!authed) return unauthorized();
    } else if (!loopback && !(is_metrics && cfg_.allow_remote_metrics)) {
      send_error(fd, 403, "invalid_request_error", "forbidden", "ops routes are served to loopback peers only");
      return;
    }
    if (is_metrics) {
      send_response(fd, 200, render_metrics(loop_, cfg_), "text/plain; version=0.0.4");
    } else {
      if (req.method != "POST") {
        send_error(fd, 405, "invalid_request_error", "method_not_allowed", "use POST");
        return;
      }
      request_drain();
      send_json(fd, 200, status_json("draining"));
    }
    return;
  }
  if (admin_only) {
    send_error(fd, 404, "invalid_request_error", "not_found", "not found");
    return;
  }
  if (req.path != "/v1/models" && req.path != "/v1/chat/completions") {
    send_error(fd, 404, "invalid_request_error", "not_found", "no route for " + req.path);
    return;
  }
  if (!cfg_.api_key.empty() && !authed) return unauthorized();
  if (state != serve::EngineState::kReady) {
    send_error(fd, 503, "server_error", serve::state_name(state), std::string("engine is ") + serve::state_name(state),
               rid_hdr);
    return;
  }
  if (req.path == "/v1/models") {
    Value model = Value::object();
    model.set("id", cfg_.served_model_name);
    model.set("object", "model");
    model.set("created", created_);
    model.set("owned_by", "zstep");
    model.set("max_model_len", cfg_.max_model_len);
    Value data = Value::array();
    data.push(model);
    Value root = Value::object();
    root.set("object", "list");
    root.set("data", data);
    send_json(fd, 200, root, rid_hdr);
    return;
  }
  if (req.method != "POST") {
    send_error(fd, 405, "invalid_request_error", "method_not_allowed", "use POST", rid_hdr);
    return;
  }
  // ------------------------------------------------------------ chat completions
  Value body;
  std::string perr;
  if (!json::parse(req.body, &body, &perr)) {
    bad_request(fd, "invalid JSON body: " + perr);
    return;
  }
  ChatParams cp;
  const std::string verr = parse_chat(body, &cp);
  if (!verr.empty()) {
    bad_request(fd, verr);
    return;
  }
  tok::TemplateOptions topt;
  topt.format = cfg_.template_format;
  topt.thinking = cp.thinking;
  topt.reasoning_effort = cp.reasoning_effort;
  std::string prompt, terr;
  if (!tok::render_chat(cp.messages, topt, &prompt, &terr)) {
    bad_request(fd, terr);
    return;
  }
  std::vector<int32_t> ids = tok_->encode(prompt);
  if (ids.empty()) {
    bad_request(fd, "empty prompt");
    return;
  }
  if (ids.size() >= cfg_.max_model_len) {
    send_error(fd, 400, "invalid_request_error", "context_length_exceeded",
               "prompt has " + std::to_string(ids.size()) + " tokens; max_model_len is " +
                   std::to_string(cfg_.max_model_len));
    return;
  }
  const int64_t room = (int64_t)cfg_.max_model_len - (int64_t)ids.size();
  if (cp.max_tokens > room) {
    send_error(fd, 400, "invalid_request_error", "context_length_exceeded",
               "prompt + max_tokens exceeds max_model_len " + std::to_string(cfg_.max_model_len));
    return;
  }
  engine::Request er;
  er.id = loop_->next_request_id();
  er.prompt = ids;
  er.max_tokens = (uint32_t)(cp.max_tokens > 0 ? cp.max_tokens : room);
  er.ignore_eos = cp.ignore_eos;
  er.eos_ids = tok_->eos_ids();
  er.sampling.temperature = (float)cp.temperature;
  er.sampling.top_p = (float)cp.top_p;
  er.sampling.top_k = cp.top_k;
  er.sampling.presence_penalty = (float)cp.presence;
  er.sampling.frequency_penalty = (float)cp.frequency;
  er.sampling.repetition_penalty = (float)cp.repetition;
  er.sampling.seed = cp.temperature <= 0.0 ? 0 : (cp.has_seed ? cp.seed : (monotonic_ns() ^ (er.id * 0x9E3779B97F4A7C15ull)));
  er.sampling.logprobs = cp.logprobs ? cp.top_logprobs : -1;
  std::shared_ptr<serve::RequestStream> stream;
  const serve::SubmitError se = loop_->submit(er, &stream);
  if (se == serve::SubmitError::kOverloaded) {
    send_error(fd, 429, "server_error", "overloaded", "waiting queue is full; retry later", rid_hdr);
    return;
  }
  if (se != serve::SubmitError::kOk) {
    send_error(fd, 503, "server_error", "unavailable", "engine is not accepting requests", rid_hdr);
    return;
  }
  // One line per accepted request (the W3C trace context passes through for correlation).
  {
    const std::string tp = req.header("traceparent");
    fprintf(stderr,
            "zstep_serve request_id=%s traceparent=%s loop_id=%llu prompt_tokens=%zu max_tokens=%u stream=%s "
            "stops=%zu seed=%s user=%s\n",
            rid.c_str(), tp.empty() ? "-" : tp.c_str(), (unsigned long long)er.id, er.prompt.size(), er.max_tokens,
            cp.stream ? "true" : "false", cp.stop.size(), cp.has_seed ? std::to_string(cp.seed).c_str() : "-",
            cp.user.empty() ? "-" : cp.user.c_str());
  }

  const uint64_t created = (uint64_t)time(nullptr);
  tok::StreamDecoder dec(tok_, cp.stop);
  auto chunk = [&](Value delta, const char* finish, Value logprobs) {
    Value choice = Value::object();
    choice.set("index", 0);
    choice.set("delta", std::move(delta));
    choice.set("logprobs", std::move(logprobs));
    choice.set("finish_reason", finish ? Value(finish) : Value());
    Value choices = Value::array();
    choices.push(std::move(choice));
    Value c = Value::object();
    c.set("id", rid);
    c.set("object", "chat.completion.chunk");
    c.set("created", created);
    c.set("model", cfg_.served_model_name);
    c.set("choices", std::move(choices));
    return "data: " + c.dump() + "\n\n";
  };
  auto lp_entries = [&](const serve::StreamEvent& ev, Value* content) {
    for (size_t k = 0; k < ev.tokens.size(); ++k) {
      const std::string t = tok_->token_bytes(ev.tokens[k]);
      Value e = Value::object();
      e.set("token", tok::sanitize_utf8(t));
      e.set("logprob", k < ev.logprobs.size() ? (double)ev.logprobs[k] : 0.0);
      e.set("bytes", token_bytes_json(t));
      Value tops = Value::array();
      if (k < ev.top_logprobs.size()) {
        int taken = 0;
        for (const auto& pr : ev.top_logprobs[k]) {
          if (taken++ >= cp.top_logprobs) break;
          const std::string tt = tok_->token_bytes(pr.first);
          Value te = Value::object();
          te.set("token", tok::sanitize_utf8(tt));
          te.set("logprob", (double)pr.second);
          te.set("bytes", token_bytes_json(tt));
          tops.push(std::move(te));
        }
      }
      e.set("top_logprobs", std::move(tops));
      content->push(std::move(e));
    }
  };

  bool client_gone = false;
  if (cp.stream) {
    std::string head = "HTTP/1.1 200 OK\r\nContent-Type: text/event-stream\r\nCache-Control: no-cache\r\n"
                       "Connection: close\r\nx-request-id: " + rid + "\r\n\r\n";
    Value d0 = Value::object();
    d0.set("role", "assistant");
    d0.set("content", "");
    client_gone = !write_all(fd, head + chunk(std::move(d0), nullptr, Value()));
  }
  std::string text;
  Value all_lp = Value::array();
  uint32_t prompt_tokens = (uint32_t)ids.size(), completion = 0, cached = 0;
  const char* finish = nullptr;
  bool stop_hit = false, failed = false;
  std::string fail_msg;
  while (!client_gone) {
    serve::StreamEvent ev;
    if (!stream->pop(&ev, 100)) {
      if (peer_closed(fd)) client_gone = true;
      continue;
    }
    std::string delta;
    if (!stop_hit) {
      for (int32_t t : ev.tokens) {
        delta += dec.push(t);
        if (dec.stopped()) {
          stop_hit = true;
          break;
        }
      }
    }
    completion += (uint32_t)ev.tokens.size();
    Value lp;
    if (cp.logprobs && !ev.tokens.empty()) {
      Value content = Value::array();
      lp_entries(ev, &content);
      if (cp.stream) {
        lp = Value::object();
        lp.set("content", std::move(content));
      } else {
        for (const auto& e : content.items()) all_lp.push(e);
      }
    }
    const bool done = ev.finish != engine::Finish::kNone || stop_hit;
    if (done && !stop_hit) delta += dec.finish();
    if (ev.finish == engine::Finish::kError) {
      failed = true;
      fail_msg = ev.error;
    }
    if (ev.finish != engine::Finish::kNone) {
      prompt_tokens = ev.prompt_tokens ? ev.prompt_tokens : prompt_tokens;
      cached = ev.cached_tokens;
      if (ev.completion_tokens) completion = ev.completion_tokens;
    }
    text += delta;
    if (cp.stream && (!delta.empty() || !lp.is_null())) {
      Value d = Value::object();
      d.set("content", delta);
      if (!write_all(fd, chunk(std::move(d), nullptr, std::move(lp)))) client_gone = true;
    }
    if (done) {
      if (stop_hit && ev.finish == engine::Finish::kNone) loop_->cancel(er.id);  // stop string: end early
      finish = finish_name(ev.finish == engine::Finish::kNone ? engine::Finish::kStop : ev.finish, stop_hit);
      break;
    }
  }
  if (client_gone) {
    loop_->cancel(er.id);
    return;
  }
  Value usage = Value::object();
  usage.set("prompt_tokens", prompt_tokens);
  usage.set("completion_tokens", completion);
  usage.set("total_tokens", prompt_tokens + completion);
  Value ptd = Value::object();
  ptd.set("cached_tokens", cached);
  usage.set("prompt_tokens_details", ptd);
  if (cp.stream) {
    std::string tail;
    if (failed) {
      tail += "data: " + error_body("server_error", "engine_error", fail_msg).dump() + "\n\n";
    } else {
      tail += chunk(Value::object(), finish, Value());
    }
    if (cp.include_usage) {
      Value c = Value::object();
      c.set("id", rid);
      c.set("object", "chat.completion.chunk");
      c.set("created", created);
      c.set("model", cfg_.served_model_name);
      c.set("choices", Value::array());
      c.set("usage", usage);
      tail += "data: " + c.dump() + "\n\n";
    }
    tail += "data: [DONE]\n\n";
    write_all(fd, tail);
    return;
  }
  if (failed) {
    send_error(fd, 500, "server_error", "engine_error", fail_msg, rid_hdr);
    return;
  }
  Value msg = Value::object();
  msg.set("role", "assistant");
  msg.set("content", text);
  Value choice = Value::object();
  choice.set("index", 0);
  choice.set("message", msg);
  if (cp.logprobs) {
    Value lp = Value::object();
    lp.set("content", all_lp);
    choice.set("logprobs", lp);
  } else {
    choice.set("logprobs", Value());
  }
  choice.set("finish_reason", finish ? Value(finish) : Value("stop"));
  Value choices = Value::array();
  choices.push(choice);
  Value root = Value::object();
  root.set("id", rid);
  root.set("object", "chat.completion");
  root.set("created", created);
  root.set("model", cfg_.served_model_name);
  root.set("choices", choices);
  root.set("usage", usage);
  send_json(fd, 200, root, rid_hdr);
}

}  // namespace http
}  // namespace zs
