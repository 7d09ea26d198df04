// `zstep` command line: `zstep serve` (OpenAI-compatible HTTP/SSE server) and
// `zstep run` (offline generation, greedy parity check, benchmark tiers).
//
// The master is this process; GPU (or CPU) workers are `python -m
// zstep_b200.runtime.worker` processes spawned by the shared-memory coordinator, one per
// tensor-parallel rank.  `--mock` replaces the workers by a deterministic scripted
// backend (no GPU, no Python) for API and control-plane testing.
//
// Reference parity: crates/zs-server/src/serve/cli.rs (SERVE_USAGE :6-49,
// validate_known_flags :143, parse_with_env :273, engine_config :622),
// crates/zs-server/src/lib.rs (USAGE :176, run_greedy_verification :417,
// run_engine :696), crates/zs-scheduler/src/serving/report.rs (tiers, provenance).
#include <limits.h>
#include <signal.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <fstream>
#include <map>
#include <set>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "coordinator.h"
#include "engine.h"
#include "http_server.h"
#include "json.h"
#include "kv_events.h"
#include "serve_loop.h"
#include "shm.h"
#include "tokenizer.h"

using namespace zs;

extern char** environ;

namespace {

const char* kServeUsage =
    "zstep serve - persistent OpenAI-compatible HTTP/SSE engine\n"
    "Usage: zstep serve --model-dir <PATH> [OPTIONS]\n"
    "  --model-dir PATH             Model directory (config.json, tokenizer.json, weights)\n"
    "  --model NAME                 Worker model: preset name or directory (default: --model-dir)\n"
    "  --served-model-name ID       Model id on /v1/models (default: directory basename)\n"
    "  --host IP                    Bind address (default 127.0.0.1)\n"
    "  --port PORT                  Bind port (default 43537; 0 = any free port)\n"
    "  --api-key TOKEN              Bearer token for /v1/*, /admin/*, /metrics (or ZSTEP_API_KEY)\n"
    "  --admin-port PORT            Loopback-only port for probes, /metrics and /admin\n"
    "  --allow-remote-metrics | --no-allow-remote-metrics\n"
    "  --world-size N               Tensor-parallel workers 1..8 (default 1)\n"
    "  --device cuda|cpu            Worker device (default cuda)\n"
    "  --max-model-len N            Max prompt + output tokens (default 32768)\n"
    "  --max-seqs N                 Max concurrent sequences (default 128)\n"
    "  --max-step-tokens N          Max tokens per step (default 4096)\n"
    "  --max-prefill-chunk N        Max prefill chunk (default 2048)\n"
    "  --page-block-tokens N        KV page size (default 16)\n"
    "  --num-kv-pages N             KV pages per GPU (default: --gpu-memory-utilization x 32768 / 0.95)\n"
    "  --gpu-memory-utilization F   KV page calibration factor in (0, 1] (default 0.95)\n"
    "  --kv-cache-dtype auto|bf16   KV cache dtype (the caches are bf16; fp8 is rejected)\n"
    "  --tokenizer-mode auto|chatml|deepseek|deepseek_v41\n"
    "  --enable-prefix-caching | --no-enable-prefix-caching   (default on)\n"
    "  --apc-node-pages N           Pages per prefix-cache node (default 8)\n"
    "  --apc-gdn-node-tokens 64|128 Prefix-cache node size in tokens for recurrent (GDN) models\n"
    "  --num-ckpt-slots N           Recurrent-state checkpoint slots (default 64 with APC)\n"
    "  --dram-kv-blocks N           Host DRAM tier of the prefix cache, in blocks (default 0 = off;\n"
    "                               attention-only models; implies --apc-node-pages 1)\n"
    "  --dram-loading-area-ratio R  Share of HBM pages kept free for DRAM reloads (default 0.10;\n"
    "                               alias --kv-loading-area-ratio)\n"
    "  --in-flight-depth 0|1        Publish the next decode step before processing the current one (default 0)\n"
    "  --max-waiting-requests N     Bounded waiting queue (default 1024)\n"
    "  --prefill-policy srpt|fifo   (default srpt)\n"
    "  --prefill-starvation-cap-ms N  Wait after which the oldest prompt preempts SRPT (default 60000, 0 = off)\n"
    "  --max-mixed-step-tokens N    Cap of steps mixing decode rows and prefill chunks (default 3072 for\n"
    "                               DeepSeek-style models, 0 = off)\n"
    "  --dynamic-prefill-budget | --no-dynamic-prefill-budget   Ramp that cap to --max-step-tokens as the\n"
    "                               prefill backlog grows from 2048 to 16384 tokens (default on with srpt)\n"
    "  --drain-timeout-secs N       SIGTERM drain grace period (default 30)\n"
    "  --python PATH                Python for workers (default: python3)\n"
    "  --worker-root PATH           Directory containing the zstep_b200 package\n"
    "  --ready-timeout-secs N       Worker start-up timeout (default 1800)\n"
    "  --step-timeout-secs N        Per-step timeout (default 300)\n"
    "  --speculative-method none|ngram|mtp|dspark\n"
    "  --num-speculative-tokens K   Draft tokens per verify step 1..7\n"
    "  --prompt-lookup-max N        Longest n-gram suffix tried for ngram drafts (default 5)\n"
    "  --prompt-lookup-min N        Shortest n-gram suffix tried (default 2)\n"
    "  --allreduce-blocks N / --allreduce-threads N   Accepted for compatibility; the NVLink\n"
    "                               collectives size their own grids\n"
    "  --kv-events-endpoint ADDR    Publish prefix-cache events: tcp://host:port (ZMTP PUB) or file://path\n"
    "  --kv-events-topic TOPIC      Topic of published events (default <served-model-name>/0)\n"
    "  --mock                       Scripted backend instead of workers (no GPU)\n";

const char* kRunUsage =
    "zstep run - offline generation / parity / benchmark\n"
    "Usage: zstep run --model-dir <PATH> [OPTIONS]\n"
    "  (all engine/worker options of `zstep serve`, plus)\n"
    "  --prompt-ids 1,2,3           Generate from these token ids\n"
    "  --prompt TEXT                Generate from this text (chat template applied)\n"
    "  --max-tokens N               Tokens to generate (default 32)\n"
    "  --verify-greedy-json PATH    {\"prompts\": [[ids]], \"expected\": [[ids]]}: exit 1 on mismatch; or the\n"
    "                               multi-case form {\"cases\": [{name, prompt_token_ids, max_tokens,\n"
    "                               expected_greedy_token_ids, top2_steps?, require_exact?,\n"
    "                               max_mismatch_margin?}]}: each case alone, all batched, all chunked\n"
    "  --verify-output-json PATH    Also write the parity report to PATH\n"
    "  --require-exact-greedy BOOL  Multi-case form: fail on any token difference (default false)\n"
    "  --require-exact-cases LIST   Multi-case form: cases that must match exactly\n"
    "  --max-greedy-mismatch-margin F  Multi-case form: fail when a run diverges at a step whose\n"
    "                               top-1 minus top-2 logit margin exceeds F\n"
    "  --metrics-output PATH        Also write the JSON report to PATH\n"
    "  --warmup-prompts N           Untimed 512->64 prompts at concurrency 16 before --bench-tiers (default 0)\n"
    "  --heartbeat-timeout-ms N     Per-worker heartbeat stall timeout (default 5000)\n"
    "  --shm-name NAME              POSIX shared-memory object name (default: unique per run)\n"
    "  --max-pages-per-seq N        Page-table capacity (sets --max-model-len to N x page size)\n"
    "  --max-decoder-rows N         Decoder rows per step (= --max-step-tokens here; must not be smaller)\n"
    "  Aliases: --max-new-tokens = --max-tokens, --repeats = --bench-repeats, --steps = --micro-steps,\n"
    "  --hidden-size / --output-features / --router-experts / --router-top-k = --micro-*;\n"
    "  `zstep --model-dir ...` without a subcommand is `zstep run`; tiers may be separated by ';'\n"
    "  --bench-tiers SPEC[,SPEC]    label:concurrency:prompts:input_len:output_len[:prefix_len:num_prefixes]\n"
    "                               (with prefix fields, prompt i = shared prefix i % num_prefixes + input_len ids)\n"
    "  --bench-repeats N            Interleaved repeats per tier (default 1)\n"
    "  --micro-steps N              Control-plane benchmark: N synthetic micro-steps per token count on the\n"
    "                               `micro` worker model (no --model-dir needed); reports round-trip latency;\n"
    "                               the default mode (200 steps) when neither a model nor a mode is given\n"
    "  --token-counts LIST          Rows per micro-step, comma separated (default 6,48,192)\n"
    "  --micro-hidden N / --micro-features N / --micro-experts N / --micro-topk N   micro-step model shape\n"
    "  --seed N                     Prompt seed (default 0)\n";

struct Args {
  std::map<std::string, std::string> kv;
  std::set<std::string> flags;
  bool has(const std::string& k) const { return kv.count(k) || flags.count(k); }
  std::string get(const std::string& k, const std::string& d = "") const {
    auto it = kv.find(k);
    return it == kv.end() ? d : it->second;
  }
  long num(const std::string& k, long d) const {
    auto it = kv.find(k);
    if (it == kv.end()) return d;
    char* end = nullptr;
    const long v = strtol(it->second.c_str(), &end, 10);
    if (end == it->second.c_str() || *end) {
      fprintf(stderr, "zstep: --%s expects an integer, got `%s`\n", k.c_str(), it->second.c_str());
      exit(2);
    }
    return v;
  }
};

const std::set<std::string> kValueFlags = {
    "model-dir", "model", "served-model-name", "host", "port", "api-key", "admin-port", "world-size", "device",
    "max-model-len", "max-seqs", "max-step-tokens", "max-prefill-chunk", "page-block-tokens", "num-kv-pages",
    "tokenizer-mode", "apc-node-pages", "num-ckpt-slots", "dram-kv-blocks", "dram-loading-area-ratio",
    "micro-steps", "token-counts", "in-flight-depth", "micro-hidden", "micro-features", "micro-experts", "micro-topk", "max-waiting-requests", "prefill-policy",
    "drain-timeout-secs", "python", "worker-root", "ready-timeout-secs", "step-timeout-secs", "speculative-method",
    "num-speculative-tokens", "prompt-ids", "prompt", "max-tokens", "verify-greedy-json", "bench-tiers",
    "bench-repeats", "seed", "kv-events-endpoint", "kv-events-topic", "gpu-memory-utilization", "kv-cache-dtype",
    "apc-gdn-node-tokens", "kv-loading-area-ratio", "prefill-starvation-cap-ms", "max-mixed-step-tokens",
    "prompt-lookup-max", "prompt-lookup-min", "allreduce-blocks", "allreduce-threads", "max-new-tokens", "repeats",
    "steps", "hidden-size", "output-features", "router-experts", "router-top-k", "heartbeat-timeout-ms", "shm-name",
    "max-decoder-rows", "max-pages-per-seq", "warmup-prompts", "metrics-output", "verify-output-json",
    "require-exact-greedy", "require-exact-cases", "max-greedy-mismatch-margin"};

// --tokenizer-mode: auto (DeepSeek template when the vocabulary has its turn markers, else
// ChatML), chatml, deepseek (also spelled deepseek_v41).  Returns false on another value.
bool template_format(const Args& a, const tok::Tokenizer& t, bool has_tokenizer, tok::TemplateFormat* out) {
  const std::string mode = a.get("tokenizer-mode", "auto");
  if (mode == "chatml") {
    *out = tok::TemplateFormat::kChatML;
  } else if (mode == "deepseek" || mode == "deepseek_v41") {
    *out = tok::TemplateFormat::kDeepSeek;
  } else if (mode == "auto") {
    *out = has_tokenizer && t.token_id("<｜User｜>") >= 0 ? tok::TemplateFormat::kDeepSeek
                                                          : tok::TemplateFormat::kChatML;
  } else {
    return false;
  }
  return true;
}

// Flag names of the reference's `zstep run` that mean the same as one of ours.
void apply_aliases(Args* a) {
  static const std::pair<const char*, const char*> kAlias[] = {
      {"max-new-tokens", "max-tokens"}, {"repeats", "bench-repeats"},       {"steps", "micro-steps"},
      {"hidden-size", "micro-hidden"},  {"output-features", "micro-features"}, {"router-experts", "micro-experts"},
      {"router-top-k", "micro-topk"}};
  for (const auto& [from, to] : kAlias) {
    auto it = a->kv.find(from);
    if (it == a->kv.end()) continue;
    if (!a->kv.count(to)) a->kv[to] = it->second;
    a->kv.erase(it);
  }
}
// Model families without per-slot recurrent state: DeepSeek-style presets, or an HF
// directory whose config.json has MLA fields.
bool attention_only_model(const std::string& model) {
  if (model.rfind("deepseek", 0) == 0) return true;
  FILE* f = fopen((model + "/config.json").c_str(), "rb");
  if (!f) return false;
  std::string text;
  char buf[4096];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) text.append(buf, n);
  fclose(f);
  return text.find("\"kv_lora_rank\"") != std::string::npos;
}

const std::set<std::string> kBoolFlags = {"allow-remote-metrics", "no-allow-remote-metrics", "enable-prefix-caching",
                                          "no-enable-prefix-caching", "dynamic-prefill-budget",
                                          "no-dynamic-prefill-budget", "mock", "help"};

bool parse_args(int argc, char** argv, int start, Args* a, std::string* err) {
  for (int i = start; i < argc; ++i) {
    std::string s = argv[i];
    if (s.rfind("--", 0) != 0) {
      *err = "unexpected argument `" + s + "`";
      return false;
    }
    s = s.substr(2);
    std::string val;
    const size_t eq = s.find('=');
    const bool inline_val = eq != std::string::npos;
    if (inline_val) {
      val = s.substr(eq + 1);
      s = s.substr(0, eq);
    }
    if (kBoolFlags.count(s)) {
      if (inline_val) {
        *err = "--" + s + " takes no value";
        return false;
      }
      a->flags.insert(s);
    } else if (kValueFlags.count(s)) {
      if (!inline_val) {
        if (i + 1 >= argc) {
          *err = "--" + s + " needs a value";
          return false;
        }
        val = argv[++i];
      }
      a->kv[s] = val;
    } else {
      *err = "unknown flag --" + s;
      return false;
    }
  }
  return true;
}

std::string basename_of(const std::string& p) {
  std::string s = p;
  while (!s.empty() && s.back() == '/') s.pop_back();
  const size_t k = s.rfind('/');
  return k == std::string::npos ? s : s.substr(k + 1);
}

std::string self_root() {
  char buf[PATH_MAX];
  const ssize_t n = readlink("/proc/self/exe", buf, sizeof(buf) - 1);
  if (n <= 0) return ".";
  buf[n] = 0;
  std::string p = buf;  // <root>/zstep_b200/bin/zstep
  for (int k = 0; k < 3; ++k) {
    const size_t s = p.rfind('/');
    if (s == std::string::npos) return ".";
    p = p.substr(0, s);
  }
  return p.empty() ? "/" : p;
}

struct Built {
  std::shared_ptr<engine::Engine> engine;
  std::shared_ptr<Coordinator> coord;
  tok::Tokenizer tokenizer;
  bool has_tokenizer = false;
  engine::Config cfg;
};

// Engine + backend from the common flags.
bool build_engine(const Args& a, Built* b, std::string* err) {
  const bool micro = a.has("micro-steps");
  const std::string dir = a.get("model-dir");
  if (dir.empty() && !micro) {
    *err = "--model-dir is required";
    return false;
  }
  if (micro) {
    // the micro-step model needs no checkpoint or tokenizer
  } else if (b->tokenizer.load_dir(dir, err)) {
    b->has_tokenizer = true;
  } else if (!a.has("prompt-ids") && !a.has("bench-tiers") && !a.has("verify-greedy-json")) {
    return false;  // text serving needs the tokenizer
  }
  err->clear();
  engine::Config& c = b->cfg;
  c.max_seqs = (uint32_t)a.num("max-seqs", 128);
  c.max_step_tokens = (uint32_t)a.num("max-step-tokens", 4096);
  c.max_prefill_chunk = (uint32_t)a.num("max-prefill-chunk", 2048);
  c.page_size = (uint32_t)a.num("page-block-tokens", 16);
  double util = 0.95;
  if (a.has("gpu-memory-utilization")) {
    char* end = nullptr;
    util = strtod(a.get("gpu-memory-utilization").c_str(), &end);
    if (end == a.get("gpu-memory-utilization").c_str() || *end || !(util > 0.0) || util > 1.0) {
      *err = "--gpu-memory-utilization must be in (0, 1]";
      return false;
    }
  }
  // Calibration as a scale of the default page count (32768 pages x 16 tokens of bf16 KV
  // fit beside the weights on one 180 GB GPU at 0.95).
  c.num_pages = (uint32_t)a.num("num-kv-pages", std::max<long>(128, std::lround(util / 0.95 * 32768.0)));
  const std::string kv_dtype = a.get("kv-cache-dtype", "auto");
  if (kv_dtype != "auto" && kv_dtype != "bf16" && kv_dtype != "bfloat16") {
    *err = "--kv-cache-dtype `" + kv_dtype + "` is not supported: the KV caches are bf16 (pass auto or bf16)";
    return false;
  }
  c.max_model_len = (uint32_t)a.num("max-model-len", 32768);
  if (a.has("max-pages-per-seq") && !a.has("max-model-len")) {
    const long mp = a.num("max-pages-per-seq", 1);
    if (mp < 1) {
      *err = "--max-pages-per-seq must be >= 1";
      return false;
    }
    c.max_model_len = uint32_t(mp) * c.page_size;
  }
  if (a.has("max-decoder-rows") && a.num("max-decoder-rows", 0) < (long)c.max_step_tokens) {
    *err = "--max-decoder-rows must be >= --max-step-tokens (a step's rows are its tokens here)";
    return false;
  }
  c.prefix_caching = !a.has("no-enable-prefix-caching");
  c.dram_blocks = (uint32_t)a.num("dram-kv-blocks", 0);
  c.in_flight_depth = (uint32_t)a.num("in-flight-depth", 0);
  if (c.in_flight_depth > 1) {
    *err = "--in-flight-depth must be 0 or 1";
    return false;
  }
  c.pages_per_node = (uint32_t)a.num("apc-node-pages", c.dram_blocks ? 1 : 8);
  // Attention-only models (the DeepSeek-style family) keep no per-slot recurrent state.
  c.recurrent_state = !attention_only_model(a.get("model", dir));
  if (a.has("apc-gdn-node-tokens")) {
    const long t = a.num("apc-gdn-node-tokens", 128);
    if ((t != 64 && t != 128) || t % c.page_size) {
      *err = "--apc-gdn-node-tokens must be 64 or 128 (and a multiple of --page-block-tokens)";
      return false;
    }
    if (c.recurrent_state && !a.has("apc-node-pages")) c.pages_per_node = uint32_t(t / c.page_size);
  }
  c.num_ckpt_slots = (uint32_t)a.num("num-ckpt-slots", c.prefix_caching && c.recurrent_state ? 64 : 0);
  if (a.has("dram-loading-area-ratio")) c.dram_loading_area = strtod(a.get("dram-loading-area-ratio").c_str(), nullptr);
  if (a.has("kv-loading-area-ratio")) c.dram_loading_area = strtod(a.get("kv-loading-area-ratio").c_str(), nullptr);
  if (c.dram_blocks > 0) {
    if (!c.prefix_caching || c.pages_per_node != 1 || c.recurrent_state) {
      *err = "--dram-kv-blocks needs prefix caching, --apc-node-pages 1 and an attention-only model";
      return false;
    }
    if (!(c.dram_loading_area > 0.0) || c.dram_loading_area > 0.5) {
      *err = "--dram-loading-area-ratio must be in (0, 0.5]";
      return false;
    }
  }
  c.prefill_policy = a.get("prefill-policy", "srpt");
  const long starve = a.num("prefill-starvation-cap-ms", 60000);
  const long mixed = a.num("max-mixed-step-tokens", c.recurrent_state ? 0 : 3072);
  if (starve < 0 || mixed < 0) {
    *err = "--prefill-starvation-cap-ms and --max-mixed-step-tokens must be >= 0";
    return false;
  }
  // FIFO keeps the plain arrival order: no starvation promotion, a fixed mixed-step cap.
  c.starvation_ms = c.prefill_policy == "srpt" ? uint32_t(starve) : 0;
  c.max_mixed_step_tokens = uint32_t(mixed);
  c.dynamic_prefill_budget = a.has("dynamic-prefill-budget") ||
                             (c.prefill_policy == "srpt" && !a.has("no-dynamic-prefill-budget"));
  c.max_waiting = (uint32_t)a.num("max-waiting-requests", 1024);
  c.spec_method = a.get("speculative-method", "none");
  c.num_spec_tokens = (uint32_t)a.num("num-speculative-tokens", c.spec_method == "none" ? 0 : 3);
  const long la_max = a.num("prompt-lookup-max", 5), la_min = a.num("prompt-lookup-min", 2);
  if (la_min < 1 || la_max < la_min) {
    *err = "--prompt-lookup-min must be >= 1 and <= --prompt-lookup-max";
    return false;
  }
  c.ngram_min = uint32_t(la_min);
  c.ngram_max = uint32_t(la_max);
  for (const char* k : {"allreduce-blocks", "allreduce-threads"})
    if (a.has(k)) {
      if (a.num(k, 1) < 1) {
        *err = std::string("--") + k + " must be >= 1";
        return false;
      }
      fprintf(stderr, "zstep: --%s accepted and ignored: the NVLink collectives size their own grids\n", k);
    }
  if (c.max_seqs < 1 || c.max_seqs > 512) {  // 512: the largest decode CUDA-graph bucket
    *err = "--max-seqs must be within 1..512";
    return false;
  }
  if (c.max_step_tokens < c.max_seqs) {
    *err = "--max-step-tokens must be >= --max-seqs";
    return false;
  }
  if (c.prefill_policy != "srpt" && c.prefill_policy != "fifo") {
    *err = "--prefill-policy must be srpt or fifo";
    return false;
  }
  if (c.spec_method != "none" && c.spec_method != "ngram" && c.spec_method != "mtp" && c.spec_method != "dspark") {
    *err = "--speculative-method must be none, ngram, mtp or dspark";
    return false;
  }
  if (c.spec_method != "none" && (c.num_spec_tokens < 1 || c.num_spec_tokens > 7)) {
    *err = "--num-speculative-tokens must be within 1..7";
    return false;
  }
  const long world = a.num("world-size", 1);
  if (world < 1 || world > 8) {
    *err = "--world-size must be within 1..8";
    return false;
  }
  std::shared_ptr<engine::Backend> backend;
  if (a.has("mock")) {
    const int32_t vocab = b->has_tokenizer ? (int32_t)b->tokenizer.vocab_size() : 1000;
    const int32_t eos = b->has_tokenizer && !b->tokenizer.eos_ids().empty() ? b->tokenizer.eos_ids()[0] : -1;
    backend = serve::make_mock_backend(0, std::max<int32_t>(2, std::min<int32_t>(vocab, 256)), eos, 0);
  } else {
    CoordinatorConfig cc;
    cc.geo.world_size = (uint32_t)world;
    cc.geo.max_seqs = c.max_seqs;
    cc.geo.max_step_tokens = c.max_step_tokens;
    cc.geo.page_size = c.page_size;
    cc.geo.max_pages_per_seq = (c.max_model_len + c.page_size - 1) / c.page_size;
    cc.geo.vocab_size = 0;
    const std::string py = a.get("python", "python3");
    cc.worker_argv = {py,
                      "-m",
                      "zstep_b200.runtime.worker",
                      "--model",
                      micro ? std::string("micro") : a.get("model", dir),
                      "--device",
                      a.get("device", "cuda"),
                      "--num-pages",
                      std::to_string(c.num_pages),
                      "--max-model-len",
                      std::to_string(c.max_model_len),
                      "--num-ckpt-slots",
                      std::to_string(c.num_ckpt_slots),
                      "--spec-method",
                      c.spec_method,
                      "--num-spec-tokens",
                      std::to_string(c.num_spec_tokens),
                      "--dram-kv-blocks",
                      std::to_string(c.dram_blocks)};
    if (micro)
      for (const char* k : {"micro-hidden", "micro-features", "micro-experts", "micro-topk"})
        if (a.has(k)) {
          cc.worker_argv.push_back(std::string("--") + k);
          cc.worker_argv.push_back(a.get(k));
        }
    const std::string root = a.get("worker-root", self_root());
    const char* pp = getenv("PYTHONPATH");
    cc.env["PYTHONPATH"] = root + (pp ? std::string(":") + pp : std::string());
    cc.env["MASTER_ADDR"] = "127.0.0.1";
    cc.env["MASTER_PORT"] = std::to_string(29500 + (getpid() % 20000));
    cc.ready_timeout_ms = (int)a.num("ready-timeout-secs", 1800) * 1000;
    cc.heartbeat_timeout_ms = (int)a.num("heartbeat-timeout-ms", 5000);
    cc.shm_name = a.get("shm-name", "");
    cc.step_timeout_ms = (int)a.num("step-timeout-secs", 300) * 1000;
    b->coord = std::make_shared<Coordinator>(cc);
    b->coord->launch();
    if (!b->coord->error().empty()) {
      *err = "worker start-up failed: " + b->coord->error();
      return false;
    }
    backend = b->coord;
  }
  b->engine = std::make_shared<engine::Engine>(c, backend);
  return true;
}

volatile sig_atomic_t g_signal = 0;
void on_signal(int sig) { g_signal = sig; }

// ------------------------------------------------------------------ serve
int cmd_serve(const Args& a) {
  if (a.has("help")) {
    fputs(kServeUsage, stdout);
    return 0;
  }
  Built b;
  std::string err;
  if (!build_engine(a, &b, &err)) {
    fprintf(stderr, "zstep serve: %s\n\n%s", err.c_str(), kServeUsage);
    return 2;
  }
  if (!b.has_tokenizer) {
    fprintf(stderr, "zstep serve: tokenizer.json not found in --model-dir\n");
    return 2;
  }
  std::unique_ptr<kvev::Publisher> kv_pub;
  if (a.has("kv-events-endpoint")) {
    const std::string topic = a.get("kv-events-topic", a.get("served-model-name", basename_of(a.get("model-dir"))) + "/0");
    kv_pub.reset(new kvev::Publisher(a.get("kv-events-endpoint"), topic));
    if (!kv_pub->start(&err)) {
      fprintf(stderr, "zstep serve: %s\n", err.c_str());
      return 1;
    }
    b.engine->set_event_sink(kv_pub->sink());
  }
  serve::ServeLoop loop(b.engine, b.coord, b.cfg.max_waiting);
  http::ServerConfig sc;
  sc.host = a.get("host", "127.0.0.1");
  sc.port = (int)a.num("port", 43537);
  sc.admin_port = a.has("admin-port") ? (int)a.num("admin-port", 0) : -1;
  sc.api_key = a.get("api-key", getenv("ZSTEP_API_KEY") ? getenv("ZSTEP_API_KEY") : "");
  sc.served_model_name = a.get("served-model-name", basename_of(a.get("model-dir")));
  sc.max_model_len = b.cfg.max_model_len;
  const char* arm = getenv("ZSTEP_ALLOW_REMOTE_METRICS");
  sc.allow_remote_metrics = !(a.has("no-allow-remote-metrics") || (arm && std::string(arm) == "0"));
  if (!template_format(a, b.tokenizer, b.has_tokenizer, &sc.template_format)) {
    fprintf(stderr, "zstep serve: --tokenizer-mode must be auto, chatml, deepseek or deepseek_v41\n");
    return 2;
  }
  http::HttpServer server(sc, &loop, &b.tokenizer);
  if (!server.start(&err)) {
    fprintf(stderr, "zstep serve: %s\n", err.c_str());
    return 1;
  }
  loop.start();
  signal(SIGTERM, on_signal);
  signal(SIGINT, on_signal);
  signal(SIGPIPE, SIG_IGN);
  fprintf(stderr, "zstep serve: listening on %s:%d (model %s)\n", sc.host.c_str(), server.port(),
          sc.served_model_name.c_str());
  printf("{\"event\": \"ready\", \"port\": %d, \"admin_port\": %d}\n", server.port(), server.admin_port());
  fflush(stdout);
  while (!g_signal && loop.state() != serve::EngineState::kFaulted) usleep(50000);
  // Drain: stop admitting, let in-flight requests finish within the grace period.
  server.request_drain();
  const long grace_ms = a.num("drain-timeout-secs", 30) * 1000;
  for (long t = 0; t < grace_ms && !loop.idle(); t += 50) usleep(50000);
  server.stop();
  loop.shutdown();
  if (kv_pub) kv_pub->stop();
  if (b.coord) b.coord->shutdown();
  return loop.state() == serve::EngineState::kFaulted ? 1 : 0;
}

// ------------------------------------------------------------------ run
std::vector<int32_t> parse_ids(const std::string& s) {
  std::vector<int32_t> out;
  std::stringstream ss(s);
  std::string tok;
  while (std::getline(ss, tok, ',')) {
    if (!tok.empty()) out.push_back((int32_t)strtol(tok.c_str(), nullptr, 10));
  }
  return out;
}

// Runs requests to completion; returns tokens per request id.
std::map<uint64_t, std::vector<int32_t>> drive(engine::Engine& e, std::string* err) {
  std::map<uint64_t, std::vector<int32_t>> out;
  while (e.has_work()) {
    for (auto& ev : e.step()) out[ev.request_id].insert(out[ev.request_id].end(), ev.tokens.begin(), ev.tokens.end());
    if (e.poisoned()) {
      *err = e.error();
      break;
    }
  }
  return out;
}

std::string git_sha(const std::string& root) {
  if (const char* e = getenv("ZSTEP_GIT_SHA")) return e;
  std::ifstream h(root + "/.git/HEAD");
  std::string line;
  if (!std::getline(h, line)) return "unknown";
  if (line.rfind("ref: ", 0) == 0) {
    std::ifstream r(root + "/.git/" + line.substr(5));
    std::string sha;
    if (std::getline(r, sha)) return sha;
    return "unknown";
  }
  return line;
}

json::Value provenance(const std::string& root) {
  json::Value p = json::Value::object();
  p.set("git_sha", git_sha(root));
  p.set("unix_time", (int64_t)time(nullptr));
  char host[256] = {0};
  gethostname(host, sizeof(host) - 1);
  p.set("hostname", std::string(host));
  json::Value env = json::Value::object();
  for (char** e = environ; *e; ++e) {
    std::string kv = *e;
    if (kv.rfind("ZSTEP_", 0) != 0 && kv.rfind("NCCL_", 0) != 0 && kv.rfind("CUDA_", 0) != 0) continue;
    const size_t eq = kv.find('=');
    std::string k = kv.substr(0, eq), v = eq == std::string::npos ? "" : kv.substr(eq + 1);
    std::string up = k;
    for (auto& ch : up) ch = (char)toupper(ch);
    if (up.find("KEY") != std::string::npos || up.find("TOKEN") != std::string::npos ||
        up.find("SECRET") != std::string::npos || up.find("PASSWORD") != std::string::npos)
      v = "<redacted>";
    env.set(k, v);
  }
  p.set("env", env);
  return p;
}

double mean_of(const std::vector<double>& v) {
  double s = 0;
  for (double x : v) s += x;
  return v.empty() ? 0 : s / v.size();
}
double std_of(const std::vector<double>& v) {
  if (v.size() < 2) return 0;
  const double m = mean_of(v);
  double s = 0;
  for (double x : v) s += (x - m) * (x - m);
  return std::sqrt(s / (v.size() - 1));
}
double pct(std::vector<double> v, double q) {
  if (v.empty()) return 0;
  std::sort(v.begin(), v.end());
  return v[std::min(v.size() - 1, (size_t)(q * (v.size() - 1) + 0.5))];
}

struct Tier {
  std::string label;
  int conc = 1, prompts = 1, in = 128, out = 128;
  int prefix_len = 0, num_prefixes = 0;  // shared random prefixes: prompt i = prefix[i % n] + in random ids
};

json::Value run_tier(engine::Engine& e, const Tier& t, uint64_t seed, int32_t vocab, std::string* err) {
  const int32_t hi = std::max<int32_t>(11, vocab - 10);
  auto prompts = engine::random_prompts(seed, (size_t)t.prompts, (size_t)t.in, 10, hi);
  if (t.prefix_len > 0 && t.num_prefixes > 0) {
    const auto prefixes = engine::random_prompts(seed ^ 0x5EC0DEull, (size_t)t.num_prefixes, (size_t)t.prefix_len, 10, hi);
    for (size_t i = 0; i < prompts.size(); ++i) {
      std::vector<int32_t> p = prefixes[i % prefixes.size()];
      p.insert(p.end(), prompts[i].begin(), prompts[i].end());
      prompts[i].swap(p);
    }
  }
  const engine::EngineStats st0 = e.stats();
  std::map<uint64_t, double> t_submit, t_first, t_last;
  std::map<uint64_t, uint32_t> produced;
  size_t next = 0, done = 0;
  uint64_t id_base = seed << 20;
  const double t0 = (double)monotonic_ns() * 1e-9;
  uint64_t gen_tokens = 0;
  while (done < prompts.size()) {
    while (next < prompts.size() && (int)(next - done) < t.conc) {
      engine::Request r;
      r.id = id_base + next;
      r.prompt = prompts[next];
      r.max_tokens = (uint32_t)t.out;
      r.ignore_eos = true;
      if (!e.submit(r)) break;
      t_submit[r.id] = (double)monotonic_ns() * 1e-9;
      ++next;
    }
    auto evs = e.step();
    if (e.poisoned()) {
      *err = e.error();
      break;
    }
    const double now = (double)monotonic_ns() * 1e-9;
    for (auto& ev : evs) {
      if (!ev.tokens.empty()) {
        if (!t_first.count(ev.request_id)) t_first[ev.request_id] = now;
        t_last[ev.request_id] = now;
        produced[ev.request_id] += (uint32_t)ev.tokens.size();
        gen_tokens += ev.tokens.size();
      }
      if (ev.finish != engine::Finish::kNone) ++done;
    }
  }
  const double wall = (double)monotonic_ns() * 1e-9 - t0;
  std::vector<double> ttft, tpot;
  for (auto& kv : t_first) {
    ttft.push_back((kv.second - t_submit[kv.first]) * 1e3);
    const uint32_t n = produced[kv.first];
    if (n > 1) tpot.push_back((t_last[kv.first] - kv.second) * 1e3 / (n - 1));
  }
  json::Value r = json::Value::object();
  r.set("label", t.label);
  r.set("concurrency", t.conc);
  r.set("num_prompts", t.prompts);
  r.set("input_len", t.in);
  r.set("output_len", t.out);
  r.set("wall_s", wall);
  r.set("output_tok_s", gen_tokens / std::max(wall, 1e-9));
  r.set("total_tok_s", (gen_tokens + (double)t.prompts * t.in) / std::max(wall, 1e-9));
  r.set("mean_ttft_ms", mean_of(ttft));
  r.set("p50_ttft_ms", pct(ttft, 0.5));
  r.set("p99_ttft_ms", pct(ttft, 0.99));
  r.set("mean_tpot_ms", mean_of(tpot));
  r.set("p50_tpot_ms", pct(tpot, 0.5));
  const engine::EngineStats st1 = e.stats();
  if (t.prefix_len > 0) {
    r.set("shared_prefix_len", t.prefix_len);
    r.set("num_prefixes", t.num_prefixes);
  }
  r.set("engine_steps", (int64_t)(st1.steps - st0.steps));
  r.set("run_ahead_steps", (int64_t)(st1.run_ahead_steps - st0.run_ahead_steps));
  const uint64_t steps = st1.spec_verify_steps - st0.spec_verify_steps;
  if (steps > 0) {
    r.set("spec_verify_steps", (int64_t)steps);
    r.set("mean_acceptance_length", 1.0 + (double)(st1.spec_accepted - st0.spec_accepted) / (double)steps);
  }
  return r;
}

// Writes a report to stdout and, with --metrics-output, to that file too.
void emit(const Args& a, const json::Value& v) {
  const std::string text = v.dump();
  printf("%s\n", text.c_str());
  if (a.has("metrics-output")) {
    std::ofstream f(a.get("metrics-output"));
    f << text << "\n";
  }
}

// One greedy generation pass: every prompt submitted at once (ignore EOS), with the top-2
// log-probabilities of each step; margin = top-1 minus top-2 (NaN when not reported).
struct GreedyRun {
  std::vector<int32_t> tokens;
  std::vector<double> margin;
};

std::vector<GreedyRun> greedy_pass(engine::Engine& e, const std::vector<std::vector<int32_t>>& prompts,
                                   const std::vector<uint32_t>& lens, uint64_t id0, std::string* err) {
  for (size_t i = 0; i < prompts.size(); ++i) {
    engine::Request r;
    r.id = id0 + i;
    r.prompt = prompts[i];
    r.max_tokens = lens[i];
    r.ignore_eos = true;
    r.sampling.logprobs = 2;
    e.submit(r);
  }
  std::vector<GreedyRun> out(prompts.size());
  while (e.has_work()) {
    for (auto& ev : e.step()) {
      if (ev.request_id < id0 || ev.request_id >= id0 + prompts.size()) continue;
      GreedyRun& g = out[ev.request_id - id0];
      for (size_t j = 0; j < ev.tokens.size(); ++j) {
        g.tokens.push_back(ev.tokens[j]);
        const bool has2 = j < ev.top_logprobs.size() && ev.top_logprobs[j].size() >= 2;
        g.margin.push_back(has2 ? (double)ev.top_logprobs[j][0].second - ev.top_logprobs[j][1].second : NAN);
      }
    }
    if (e.poisoned()) {
      *err = e.error();
      break;
    }
  }
  return out;
}

json::Value match_report(const std::vector<int32_t>& want, const GreedyRun& got) {
  size_t first = want.size(), same = 0;
  for (size_t i = 0; i < want.size(); ++i) {
    const bool eq = i < got.tokens.size() && got.tokens[i] == want[i];
    same += eq ? 1 : 0;
    if (!eq && first == want.size()) first = i;
  }
  json::Value r = json::Value::object();
  r.set("exact_prefix_match_tokens", (int64_t)first);
  r.set("exact_token_matches", (int64_t)same);
  r.set("total_tokens", (int64_t)want.size());
  r.set("exact_token_match_rate", want.empty() ? 1.0 : (double)same / (double)want.size());
  r.set("all_matched", first == want.size());
  if (first < want.size()) {
    r.set("first_mismatch_token_index", (int64_t)first);
    if (first < got.margin.size() && !std::isnan(got.margin[first]))
      r.set("zstep_top1_minus_top2_margin", got.margin[first]);
  }
  return r;
}

// First step where two passes differ: {token_index, left/right tokens and margins}, or null.
json::Value pair_mismatch(const char* ln, const GreedyRun& l, const char* rn, const GreedyRun& r, double* margin) {
  *margin = NAN;
  const size_t n = std::max(l.tokens.size(), r.tokens.size());
  for (size_t i = 0; i < n; ++i) {
    const int32_t a = i < l.tokens.size() ? l.tokens[i] : -1, b = i < r.tokens.size() ? r.tokens[i] : -1;
    if (a == b) continue;
    json::Value m = json::Value::object();
    m.set("token_index", (int64_t)i);
    m.set("left_mode", std::string(ln));
    m.set("right_mode", std::string(rn));
    m.set("left_token", (int64_t)a);
    m.set("right_token", (int64_t)b);
    const double ml = i < l.margin.size() ? l.margin[i] : NAN, mr = i < r.margin.size() ? r.margin[i] : NAN;
    if (!std::isnan(ml)) m.set("left_margin", ml);
    if (!std::isnan(mr)) m.set("right_margin", mr);
    *margin = std::isnan(ml) ? mr : std::isnan(mr) ? ml : std::max(ml, mr);
    return m;
  }
  return json::Value();
}

bool parse_bool(const std::string& s, bool* out) {
  if (s == "true" || s == "1" || s == "yes") return (*out = true), true;
  if (s == "false" || s == "0" || s == "no") return (*out = false), true;
  return false;
}

// The multi-case greedy parity check: each case alone and unchunked, all cases batched and
// unchunked, all cases batched with the configured prefill chunk; every pass against the
// expected tokens and against each other, then the gates.  Returns the exit code.
int verify_cases(const Args& a, engine::Engine& e, const json::Value& v, const std::string& root) {
  struct Case {
    std::string name;
    std::vector<int32_t> prompt, want;
    uint32_t max_tokens = 0;
    bool require_exact = false;
    double margin_limit = NAN;
  };
  std::vector<Case> cases;
  for (const auto& c : v.get("cases").items()) {
    Case k;
    k.name = c.get("name").as_string();
    for (const auto& t : c.get("prompt_token_ids").items()) k.prompt.push_back((int32_t)t.as_int());
    for (const auto& t : c.get("expected_greedy_token_ids").items()) k.want.push_back((int32_t)t.as_int());
    k.max_tokens = (uint32_t)c.get("max_tokens").as_int();
    k.require_exact = c.get("require_exact").is_bool() && c.get("require_exact").as_bool();
    if (c.get("max_mismatch_margin").is_number()) k.margin_limit = c.get("max_mismatch_margin").as_double();
    const size_t top2 = c.get("top2_steps").is_array() ? c.get("top2_steps").size() : 0;
    std::string bad;
    if (k.prompt.empty() || k.max_tokens == 0) bad = "has an empty prompt or zero output length";
    else if (k.want.size() != k.max_tokens) bad = "expected token count differs from max_tokens";
    else if (top2 && top2 != k.max_tokens) bad = "has a top2_steps count that differs from max_tokens";
    if (!bad.empty()) {
      fprintf(stderr, "zstep run: case `%s` %s\n", k.name.c_str(), bad.c_str());
      return 2;
    }
    cases.push_back(std::move(k));
  }
  if (cases.empty()) {
    fprintf(stderr, "zstep run: the greedy reference has no cases\n");
    return 2;
  }
  bool exact_all = false;
  if (a.has("require-exact-greedy") && !parse_bool(a.get("require-exact-greedy"), &exact_all)) {
    fprintf(stderr, "zstep run: --require-exact-greedy takes true or false\n");
    return 2;
  }
  double margin_flag = NAN;
  if (a.has("max-greedy-mismatch-margin")) margin_flag = strtod(a.get("max-greedy-mismatch-margin").c_str(), nullptr);
  std::vector<std::vector<int32_t>> prompts;
  std::vector<uint32_t> lens;
  for (const auto& k : cases) {
    prompts.push_back(k.prompt);
    lens.push_back(k.max_tokens);
  }
  std::string err;
  const uint32_t chunk = e.config().max_prefill_chunk;
  e.set_max_prefill_chunk(UINT32_MAX);
  uint64_t id = 1;
  std::vector<GreedyRun> single;
  for (size_t i = 0; i < cases.size() && err.empty(); ++i) {
    single.push_back(greedy_pass(e, {prompts[i]}, {lens[i]}, id, &err)[0]);
    id += 1;
  }
  std::vector<GreedyRun> batched, chunked;
  if (err.empty()) batched = greedy_pass(e, prompts, lens, id, &err);
  id += cases.size();
  e.set_max_prefill_chunk(chunk);
  if (err.empty()) chunked = greedy_pass(e, prompts, lens, id, &err);
  json::Value rep = json::Value::object();
  rep.set("git_sha", git_sha(root));
  rep.set("vllm_version", v.get("vllm_version").is_string() ? v.get("vllm_version").as_string() : std::string());
  rep.set("max_prefill_chunk", (int64_t)chunk);
  if (!err.empty()) {
    rep.set("error", err);
    emit(a, rep);
    return 1;
  }
  bool all = true, b_vs_s = true, c_vs_b = true;
  std::string gate;
  json::Value cv = json::Value::array();
  std::set<std::string> names;
  for (size_t i = 0; i < cases.size(); ++i) {
    const Case& k = cases[i];
    names.insert(k.name);
    const json::Value ms = match_report(k.want, single[i]), mb = match_report(k.want, batched[i]),
                      mc = match_report(k.want, chunked[i]);
    double m_sb, m_bc;
    const json::Value sb = pair_mismatch("single", single[i], "batched", batched[i], &m_sb);
    const json::Value bc = pair_mismatch("batched", batched[i], "chunked", chunked[i], &m_bc);
    b_vs_s = b_vs_s && sb.is_null();
    c_vs_b = c_vs_b && bc.is_null();
    const bool ok = ms.get("all_matched").as_bool() && mb.get("all_matched").as_bool() &&
                    mc.get("all_matched").as_bool() && sb.is_null() && bc.is_null();
    all = all && ok;
    json::Value r = json::Value::object();
    r.set("name", k.name);
    r.set("all_matched", ok);
    r.set("single_match", ms);
    r.set("batched_match", mb);
    r.set("chunked_match", mc);
    r.set("single_vs_batched_first_mismatch", sb);
    r.set("batched_vs_chunked_first_mismatch", bc);
    for (const auto& [key, run] : {std::pair<const char*, const GreedyRun*>{"single_generated_token_ids", &single[i]},
                                   {"batched_generated_token_ids", &batched[i]},
                                   {"chunked_generated_token_ids", &chunked[i]}}) {
      json::Value t = json::Value::array();
      for (int32_t x : run->tokens) t.push((int64_t)x);
      r.set(key, t);
    }
    cv.push(r);
    if (!gate.empty()) continue;
    if (k.require_exact && !ok) gate = "case `" + k.name + "` had token mismatches (reference require_exact=true)";
    const double limit = std::isnan(margin_flag) ? k.margin_limit : margin_flag;
    if (gate.empty() && !std::isnan(limit)) {
      const json::Value& m = ms.get("zstep_top1_minus_top2_margin");
      if (m.is_number() && m.as_double() > limit)
        gate = "case `" + k.name + "` diverged from the reference with margin " + std::to_string(m.as_double());
      for (double pm : {m_sb, m_bc})
        if (gate.empty() && !std::isnan(pm) && pm > limit)
          gate = "case `" + k.name + "` diverged between passes with margin " + std::to_string(pm);
    }
  }
  if (gate.empty() && exact_all && !all) gate = "greedy parity report had token mismatches (--require-exact-greedy=true)";
  if (gate.empty() && a.has("require-exact-cases")) {
    std::stringstream ss(a.get("require-exact-cases"));
    std::string name;
    while (gate.empty() && std::getline(ss, name, ',')) {
      if (name.empty()) continue;
      if (!names.count(name)) {
        gate = "--require-exact-cases names unknown case `" + name + "`";
        break;
      }
      for (const auto& c : cv.items())
        if (c.get("name").as_string() == name && !c.get("all_matched").as_bool())
          gate = "case `" + name + "` had token mismatches (--require-exact-cases)";
    }
  }
  rep.set("all_matched", all);
  rep.set("batched_vs_single_exact_match", b_vs_s);
  rep.set("chunked_vs_unchunked_exact_match", c_vs_b);
  rep.set("cases", cv);
  rep.set("gate", gate.empty() ? std::string("ok") : gate);
  emit(a, rep);
  if (a.has("verify-output-json")) {
    std::ofstream f(a.get("verify-output-json"));
    f << rep.dump() << "\n";
  }
  if (!gate.empty()) fprintf(stderr, "zstep run: %s\n", gate.c_str());
  return gate.empty() ? 0 : 1;
}

int cmd_run(const Args& a) {
  if (a.has("help")) {
    fputs(kRunUsage, stdout);
    return 0;
  }
  Built b;
  std::string err;
  if (!build_engine(a, &b, &err)) {
    fprintf(stderr, "zstep run: %s\n\n%s", err.c_str(), kRunUsage);
    return 2;
  }
  signal(SIGPIPE, SIG_IGN);
  int rc = 0;
  engine::Engine& e = *b.engine;
  const std::string root = a.get("worker-root", self_root());
  if (a.has("micro-steps")) {
    // Control-plane benchmark: synthetic plans (one 1-row sequence per token) straight
    // through the coordinator; the host clock measures publish -> all ranks done -> result.
    if (!b.coord) {
      fprintf(stderr, "zstep run: --micro-steps needs workers (not --mock)\n");
      return 2;
    }
    const int steps = (int)a.num("micro-steps", 200);
    std::vector<int> counts;
    {
      std::string list = a.get("token-counts", "6,48,192");
      size_t p0 = 0;
      while (p0 <= list.size()) {
        const size_t p1 = list.find(',', p0);
        const std::string item = list.substr(p0, p1 == std::string::npos ? std::string::npos : p1 - p0);
        if (!item.empty()) counts.push_back(atoi(item.c_str()));
        if (p1 == std::string::npos) break;
        p0 = p1 + 1;
      }
    }
    json::Value tiers = json::Value::array();
    for (int m : counts) {
      if (m < 1 || (uint32_t)m > b.cfg.max_seqs || (uint32_t)m > b.cfg.max_step_tokens) {
        fprintf(stderr, "zstep run: token count %d must be within 1..min(--max-seqs, --max-step-tokens)\n", m);
        rc = 2;
        break;
      }
      engine::StepPlan p;
      p.query_start.push_back(0);
      for (int i = 0; i < m; ++i) {
        p.token_ids.push_back(i + 1);
        p.positions.push_back(i);
        p.row_slot.push_back(i);
        p.query_start.push_back(i + 1);
        p.seq_slot.push_back(i);
        p.seq_len.push_back(1);
        p.sample_row.push_back(i);
        p.sampling.push_back(wire::SamplingParams{});
        p.restore_slot.push_back(-1);
        p.spec_width.push_back(0);
      }
      std::vector<double> lat_us, gpu_us;
      for (int s = 0; s < steps + 5 && err.empty(); ++s) {
        engine::StepResult res;
        const uint64_t t0 = monotonic_ns();
        if (!b.coord->execute(p, &res)) {
          err = b.coord->error();
          break;
        }
        const uint64_t t1 = monotonic_ns();
        if (s >= 5) {  // warm-up steps excluded
          lat_us.push_back((t1 - t0) * 1e-3);
          gpu_us.push_back((double)res.gpu_exec_us);
        }
      }
      if (!err.empty()) break;
      json::Value t = json::Value::object();
      t.set("token_count", m);
      t.set("steps", steps);
      t.set("p50_step_us", pct(lat_us, 0.5));
      t.set("p99_step_us", pct(lat_us, 0.99));
      t.set("mean_step_us", mean_of(lat_us));
      t.set("mean_gpu_us", mean_of(gpu_us));
      t.set("mean_overhead_us", mean_of(lat_us) - mean_of(gpu_us));
      t.set("steps_per_s", 1e6 / std::max(mean_of(lat_us), 1e-9));
      tiers.push(t);
    }
    json::Value report = json::Value::object();
    report.set("micro_steps", tiers);
    report.set("world_size", (int64_t)a.num("world-size", 1));
    report.set("provenance", provenance(root));
    if (!err.empty()) report.set("error", err);
    emit(a, report);
    if (b.coord) b.coord->shutdown();
    return err.empty() && rc == 0 ? 0 : 1;
  }
  if (a.has("verify-greedy-json")) {
    std::ifstream f(a.get("verify-greedy-json"));
    std::stringstream ss;
    ss << f.rdbuf();
    json::Value v;
    if (!json::parse(ss.str(), &v, &err)) {
      fprintf(stderr, "zstep run: bad --verify-greedy-json: %s\n", err.c_str());
      return 2;
    }
    if (v.has("cases")) {
      const int code = verify_cases(a, e, v, root);
      if (b.coord) b.coord->shutdown();
      return code;
    }
    const auto& prompts = v.get("prompts");
    const auto& expected = v.get("expected");
    for (size_t i = 0; i < prompts.size(); ++i) {
      engine::Request r;
      r.id = i + 1;
      for (const auto& t : prompts[i].items()) r.prompt.push_back((int32_t)t.as_int());
      r.max_tokens = (uint32_t)(i < expected.size() ? expected[i].size() : a.num("max-tokens", 32));
      r.ignore_eos = true;
      e.submit(r);
    }
    auto out = drive(e, &err);
    int mismatches = 0;
    json::Value rep = json::Value::array();
    for (size_t i = 0; i < prompts.size(); ++i) {
      std::vector<int32_t> exp;
      if (i < expected.size())
        for (const auto& t : expected[i].items()) exp.push_back((int32_t)t.as_int());
      const auto& got = out[i + 1];
      const bool ok = got == exp;
      mismatches += ok ? 0 : 1;
      json::Value r = json::Value::object();
      r.set("index", (int64_t)i);
      r.set("match", ok);
      json::Value g = json::Value::array();
      for (int32_t t : got) g.push(t);
      r.set("tokens", g);
      rep.push(r);
    }
    json::Value root_v = json::Value::object();
    root_v.set("verify_greedy", rep);
    root_v.set("mismatches", mismatches);
    emit(a, root_v);
    if (a.has("verify-output-json")) {
      std::ofstream vf(a.get("verify-output-json"));
      vf << root_v.dump() << "\n";
    }
    rc = (mismatches || !err.empty()) ? 1 : 0;
  } else if (a.has("bench-tiers")) {
    std::vector<Tier> tiers;
    std::string specs = a.get("bench-tiers");
    std::replace(specs.begin(), specs.end(), ';', ',');  // the reference separates tiers with ';'
    std::stringstream ss(specs);
    std::string spec;
    while (std::getline(ss, spec, ',')) {
      std::vector<std::string> f;
      std::stringstream s2(spec);
      std::string part;
      while (std::getline(s2, part, ':')) f.push_back(part);
      if (f.size() != 5 && f.size() != 7) {
        fprintf(stderr, "zstep run: tier `%s` is not label:conc:prompts:in:out[:prefix_len:num_prefixes]\n",
                spec.c_str());
        return 2;
      }
      Tier t{f[0], atoi(f[1].c_str()), atoi(f[2].c_str()), atoi(f[3].c_str()), atoi(f[4].c_str())};
      if (f.size() == 7) {
        t.prefix_len = atoi(f[5].c_str());
        t.num_prefixes = atoi(f[6].c_str());
        if (t.prefix_len < 1 || t.num_prefixes < 1) {
          fprintf(stderr, "zstep run: tier `%s` has non-positive prefix fields\n", spec.c_str());
          return 2;
        }
      }
      if (t.conc < 1 || t.prompts < 1 || t.in < 1 || t.out < 1) {
        fprintf(stderr, "zstep run: tier `%s` has non-positive fields\n", spec.c_str());
        return 2;
      }
      tiers.push_back(t);
    }
    const int repeats = (int)a.num("bench-repeats", 1);
    const int32_t vocab = b.has_tokenizer ? (int32_t)b.tokenizer.vocab_size() : 1000;
    if (const long w = a.num("warmup-prompts", 0); w > 0) {  // untimed, report discarded
      Tier wt{"warmup", 16, (int)w, 512, 64};
      run_tier(e, wt, a.num("seed", 0) + 7777, vocab, &err);
    }
    std::map<std::string, std::vector<json::Value>> runs;
    for (int rep = 0; rep < repeats && err.empty(); ++rep)  // interleaved: tier order repeats
      for (const auto& t : tiers) runs[t.label].push_back(run_tier(e, t, a.num("seed", 0) + rep, vocab, &err));
    json::Value report = json::Value::object();
    json::Value tv = json::Value::array();
    for (const auto& t : tiers) {
      std::vector<double> tps, ttft, tpot;
      json::Value reps = json::Value::array();
      for (const auto& r : runs[t.label]) {
        tps.push_back(r.get("output_tok_s").as_double());
        ttft.push_back(r.get("p50_ttft_ms").as_double());
        tpot.push_back(r.get("p50_tpot_ms").as_double());
        reps.push(r);
      }
      json::Value agg = json::Value::object();
      agg.set("label", t.label);
      agg.set("output_tok_s_mean", mean_of(tps));
      agg.set("output_tok_s_std", std_of(tps));
      agg.set("p50_ttft_ms_mean", mean_of(ttft));
      agg.set("p50_tpot_ms_mean", mean_of(tpot));
      agg.set("runs", reps);
      tv.push(agg);
    }
    report.set("tiers", tv);
    report.set("provenance", provenance(root));
    if (!err.empty()) report.set("error", err);
    emit(a, report);
    rc = err.empty() ? 0 : 1;
  } else {
    engine::Request r;
    r.id = 1;
    if (a.has("prompt-ids")) {
      r.prompt = parse_ids(a.get("prompt-ids"));
    } else if (a.has("prompt") && b.has_tokenizer) {
      std::string prompt;
      tok::TemplateOptions to;
      if (!template_format(a, b.tokenizer, b.has_tokenizer, &to.format)) {
        fprintf(stderr, "zstep run: --tokenizer-mode must be auto, chatml, deepseek or deepseek_v41\n");
        return 2;
      }
      if (!tok::render_chat({{"user", a.get("prompt"), ""}}, to, &prompt, &err)) {
        fprintf(stderr, "zstep run: %s\n", err.c_str());
        return 2;
      }
      r.prompt = b.tokenizer.encode(prompt);
      r.eos_ids = b.tokenizer.eos_ids();
    } else {
      fprintf(stderr, "zstep run: give --prompt-ids, --prompt, --verify-greedy-json or --bench-tiers\n");
      return 2;
    }
    r.max_tokens = (uint32_t)a.num("max-tokens", 32);
    e.submit(r);
    auto out = drive(e, &err);
    json::Value res = json::Value::object();
    json::Value toks = json::Value::array();
    for (int32_t t : out[1]) toks.push(t);
    res.set("tokens", toks);
    if (b.has_tokenizer) res.set("text", tok::sanitize_utf8(b.tokenizer.decode(out[1])));
    if (!err.empty()) res.set("error", err);
    emit(a, res);
    rc = err.empty() ? 0 : 1;
  }
  if (b.coord) b.coord->shutdown();
  return rc;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2 || !strcmp(argv[1], "--help") || !strcmp(argv[1], "-h")) {
    printf("zstep <serve|run> [OPTIONS]\n\n%s\n%s", kServeUsage, kRunUsage);
    return argc < 2 ? 2 : 0;
  }
  // `zstep --model-dir ... --bench-tiers ...` (options first) is `zstep run`.
  const bool implicit_run = strncmp(argv[1], "--", 2) == 0;
  const std::string sub = implicit_run ? "run" : argv[1];
  Args a;
  std::string err;
  if (sub != "serve" && sub != "run") {
    fprintf(stderr, "zstep: unknown subcommand `%s` (serve | run)\n", sub.c_str());
    return 2;
  }
  if (!parse_args(argc, argv, implicit_run ? 1 : 2, &a, &err)) {
    fprintf(stderr, "zstep %s: %s\n\n%s", sub.c_str(), err.c_str(), sub == "serve" ? kServeUsage : kRunUsage);
    return 2;
  }
  apply_aliases(&a);
  // `zstep run` with no model and no mode is the control-plane micro-step benchmark (200
  // steps), as in the reference.
  if (sub == "run" && !a.has("model-dir") && !a.has("micro-steps") && !a.has("prompt-ids") && !a.has("prompt") &&
      !a.has("bench-tiers") && !a.has("verify-greedy-json") && !a.has("help") && !a.has("mock"))
    a.kv["micro-steps"] = "200";
  try {
    return sub == "serve" ? cmd_serve(a) : cmd_run(a);
  } catch (const std::exception& ex) {
    fprintf(stderr, "zstep %s: %s\n", sub.c_str(), ex.what());
    return 1;
  }
}
