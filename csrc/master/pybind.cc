// Python bindings of the C++ control plane (module zstep_b200._master).  Tests and the
// offline engine API drive the real C++ engine / coordinator / KV code through this.
#include <unistd.h>

#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "coordinator.h"
#include "engine.h"
#include "http_server.h"
#include "kv_events.h"
#include "serve_loop.h"
#include "tokenizer.h"
#include "kv.h"
#include "sha256.h"
#include "wire.h"

namespace py = pybind11;
using namespace zs;

namespace {

// Backend that hands the staged plan to a Python callable (tests, in-process runners).
class PyBackend : public engine::Backend {
 public:
  explicit PyBackend(py::function fn) : fn_(std::move(fn)) {}
  bool execute(const engine::StepPlan& p, engine::StepResult* r) override {
    py::gil_scoped_acquire g;
    py::dict d;
    d["opcode"] = p.opcode;
    d["flags"] = p.flags;
    d["bucket"] = p.bucket;
    d["token_ids"] = p.token_ids;
    d["positions"] = p.positions;
    d["row_slot"] = p.row_slot;
    d["query_start"] = p.query_start;
    d["seq_slot"] = p.seq_slot;
    d["seq_len"] = p.seq_len;
    d["sample_row"] = p.sample_row;
    d["dirty_rows"] = p.dirty_rows;
    d["dirty_pages"] = p.dirty_pages;
    d["ckpt_row"] = p.ckpt_row;
    d["ckpt_slot"] = p.ckpt_slot;
    d["restore_slot"] = p.restore_slot;
    d["spec_width"] = p.spec_width;
    py::list sp;
    for (auto& s : p.sampling)
      sp.append(py::make_tuple(s.temperature, s.top_p, s.top_k, s.presence_penalty, s.frequency_penalty,
                               s.repetition_penalty, s.seed, s.logprobs));
    d["sampling"] = sp;
    try {
      py::object res = fn_(d);
      if (res.is_none()) {
        err_ = "backend returned None";
        return false;
      }
      py::list outs = res.cast<py::list>();
      r->outputs.clear();
      for (auto o : outs) {
        wire::SeqStepOutput so{};
        py::dict od = o.cast<py::dict>();
        std::vector<int32_t> toks = od["tokens"].cast<std::vector<int32_t>>();
        so.num_tokens = int32_t(std::min<size_t>(toks.size(), wire::kMaxSpecTokens));
        for (int i = 0; i < so.num_tokens; ++i) so.tokens[i] = toks[i];
        if (od.contains("logprobs")) {
          auto lp = od["logprobs"].cast<std::vector<float>>();
          for (int i = 0; i < so.num_tokens && i < int(lp.size()); ++i) so.logprobs[i] = lp[i];
        }
        if (od.contains("drafts")) {
          auto dr = od["drafts"].cast<std::vector<int32_t>>();
          so.num_drafts = int32_t(std::min<size_t>(dr.size(), wire::kMaxSpecTokens));
          for (int i = 0; i < so.num_drafts; ++i) so.next_drafts[i] = dr[i];
        }
        r->outputs.push_back(so);
      }
      r->status = 0;
      return true;
    } catch (py::error_already_set& e) {
      err_ = e.what();
      return false;
    }
  }
  std::string error() const override { return err_; }

 private:
  py::function fn_;
  std::string err_;
};

py::dict layout_dict(const wire::Geometry& g) {
  const auto s = wire::segment_layout(g);
  py::dict d;
  const auto& p = s.plan;
  d["header"] = p.header;
  d["token_ids"] = p.token_ids;
  d["positions"] = p.positions;
  d["row_slot"] = p.row_slot;
  d["query_start"] = p.query_start;
  d["seq_slot"] = p.seq_slot;
  d["seq_len"] = p.seq_len;
  d["sample_row"] = p.sample_row;
  d["sampling"] = p.sampling;
  d["dirty_rows"] = p.dirty_rows;
  d["dirty_pages"] = p.dirty_pages;
  d["ckpt_row"] = p.ckpt_row;
  d["ckpt_slot"] = p.ckpt_slot;
  d["restore_slot"] = p.restore_slot;
  d["spec_width"] = p.spec_width;
  d["kv_ops"] = p.kv_ops;
  d["plan_bytes"] = p.bytes;
  d["max_ckpt"] = p.max_ckpt;
  d["result_outputs"] = s.result.outputs;
  d["result_bytes"] = s.result.bytes;
  d["plan_offset"] = s.plan_offset;
  d["result_offset"] = s.result_offset;
  d["total_bytes"] = s.total_bytes;
  d["layout_hash"] = wire::layout_hash(s);
  d["sizeof_superblock"] = sizeof(wire::Superblock);
  d["sizeof_worker_state"] = sizeof(wire::WorkerState);
  d["sizeof_step_header"] = sizeof(wire::StepHeader);
  d["sizeof_sampling"] = sizeof(wire::SamplingParams);
  d["sizeof_result_header"] = sizeof(wire::StepResultHeader);
  d["sizeof_seq_output"] = sizeof(wire::SeqStepOutput);
  return d;
}

py::dict event_dict(const engine::TokenEvent& e) {
  py::dict d;
  d["request_id"] = e.request_id;
  d["tokens"] = e.tokens;
  d["logprobs"] = e.logprobs;
  d["finish"] = int(e.finish);
  d["prompt_tokens"] = e.prompt_tokens;
  d["completion_tokens"] = e.completion_tokens;
  d["cached_tokens"] = e.cached_tokens;
  d["first"] = e.first;
  return d;
}

}  // namespace

PYBIND11_MODULE(_master, m) {
  m.doc() = "zstep_b200 C++ control plane";

  // ---------------------------------------------------------------- wire
  py::class_<wire::Geometry>(m, "Geometry")
      .def(py::init<>())
      .def_readwrite("world_size", &wire::Geometry::world_size)
      .def_readwrite("max_seqs", &wire::Geometry::max_seqs)
      .def_readwrite("max_step_tokens", &wire::Geometry::max_step_tokens)
      .def_readwrite("max_pages_per_seq", &wire::Geometry::max_pages_per_seq)
      .def_readwrite("page_size", &wire::Geometry::page_size)
      .def_readwrite("vocab_size", &wire::Geometry::vocab_size);
  m.def("layout", &layout_dict);
  m.def("select_bucket", &wire::select_bucket);
  m.attr("MAGIC") = wire::kMagic;
  m.attr("VERSION") = wire::kVersion;
  m.attr("ABORT_OFFSET") = wire::kAbortOffset;
  m.attr("DECODE_BUCKETS") = std::vector<uint32_t>(wire::kDecodeBuckets.begin(), wire::kDecodeBuckets.end());

  // ---------------------------------------------------------------- hashing
  m.def("sha256", [](py::bytes b) {
    std::string s = b;
    auto h = sha256(s.data(), s.size());
    return py::bytes(reinterpret_cast<const char*>(h.data()), h.size());
  });
  m.def("block_hashes", [](const std::vector<int32_t>& toks, size_t block, const std::string& seed) {
    std::vector<py::bytes> out;
    for (auto& h : kv::compute_block_hashes(toks, block, seed))
      out.emplace_back(reinterpret_cast<const char*>(h.data()), h.size());
    return out;
  });
  m.def("external_keys", [](const std::vector<int32_t>& toks, size_t block, const std::string& seed) {
    std::vector<uint64_t> out;
    for (auto& h : kv::compute_block_hashes(toks, block, seed)) out.push_back(kv::external_key(h));
    return out;
  });

  // ---------------------------------------------------------------- kv
  py::class_<kv::BlockLease>(m, "BlockLease")
      .def("ids", &kv::BlockLease::ids)
      .def("__len__", &kv::BlockLease::size)
      .def("release", &kv::BlockLease::release)
      .def("take_front", &kv::BlockLease::take_front)
      .def("absorb", [](kv::BlockLease& self, kv::BlockLease& other) { self.absorb(std::move(other)); });
  py::class_<kv::BlockPool>(m, "BlockPool")
      .def(py::init<int32_t, int32_t>(), py::arg("num_blocks"), py::arg("first_id") = 0)
      .def("allocate", &kv::BlockPool::allocate)
      .def("available", &kv::BlockPool::available)
      .def("capacity", &kv::BlockPool::capacity);
  py::class_<kv::PrefixLease>(m, "PrefixLease")
      .def("pages", &kv::PrefixLease::pages)
      .def("matched_nodes", &kv::PrefixLease::matched_nodes)
      .def("matched_tokens", &kv::PrefixLease::matched_tokens)
      .def("leaf_aux", &kv::PrefixLease::leaf_aux)
      .def("leaf_node", &kv::PrefixLease::leaf_node)
      .def("release", &kv::PrefixLease::release);
  py::class_<kv::PrefixVictim>(m, "PrefixVictim")
      .def_readonly("pages", &kv::PrefixVictim::pages)
      .def_readonly("tokens", &kv::PrefixVictim::tokens)
      .def_readonly("aux_slot", &kv::PrefixVictim::aux_slot);
  py::class_<kv::PrefixTree>(m, "PrefixTree")
      .def(py::init<uint32_t, uint32_t, std::string>(), py::arg("block_tokens"), py::arg("pages_per_node") = 1,
           py::arg("seed") = "42")
      .def("match", &kv::PrefixTree::match, py::arg("tokens"), py::arg("max_nodes") = SIZE_MAX)
      .def("peek", &kv::PrefixTree::peek, py::arg("tokens"), py::arg("max_nodes") = SIZE_MAX)
      .def("insert",
           [](kv::PrefixTree& t, uint64_t parent, const std::vector<int32_t>& toks, kv::BlockLease& pages,
              kv::BlockLease* aux) {
             kv::BlockLease none;
             bool created = false;
             const uint64_t id = t.insert(parent, toks.data(), pages, aux ? *aux : none, &created);
             return py::make_tuple(id, created);
           },
           py::arg("parent"), py::arg("tokens"), py::arg("pages"), py::arg("aux") = nullptr)
      .def("pin_chain", &kv::PrefixTree::pin_chain)
      .def("evict_lru", &kv::PrefixTree::evict_lru)
      .def("aux_of", &kv::PrefixTree::aux_of)
      .def("cached_nodes", &kv::PrefixTree::cached_nodes)
      .def("cached_pages", &kv::PrefixTree::cached_pages)
      .def("evictable_pages", &kv::PrefixTree::evictable_pages)
      .def("node_tokens", &kv::PrefixTree::node_tokens)
      .def("clear", &kv::PrefixTree::clear)
      .def("set_event_sink", [](kv::PrefixTree& t, py::function fn) {
        t.set_event_sink([fn](const kv::KvEvent& e) {
          py::gil_scoped_acquire g;
          fn(int(e.kind), e.block_keys, e.parent_key, e.tokens);
        });
      });
  py::class_<kv::HybridAliasTable>(m, "HybridAliasTable")
      .def(py::init<>())
      .def("insert", &kv::HybridAliasTable::insert)
      .def("remove_by_anchor", &kv::HybridAliasTable::remove_by_anchor)
      .def("slot_for_anchor", &kv::HybridAliasTable::slot_for_anchor)
      .def("anchor_for_slot", &kv::HybridAliasTable::anchor_for_slot)
      .def("__len__", &kv::HybridAliasTable::size);
  py::class_<kv::SubPageAllocator>(m, "SubPageAllocator")
      .def(py::init<uint32_t, uint32_t, uint32_t>())
      .def("allocate", &kv::SubPageAllocator::allocate)
      .def("release", &kv::SubPageAllocator::release)
      .def("active", &kv::SubPageAllocator::active);

  // ---------------------------------------------------------------- engine
  py::class_<engine::Config>(m, "EngineConfig")
      .def(py::init<>())
      .def_readwrite("max_seqs", &engine::Config::max_seqs)
      .def_readwrite("max_step_tokens", &engine::Config::max_step_tokens)
      .def_readwrite("max_prefill_chunk", &engine::Config::max_prefill_chunk)
      .def_readwrite("page_size", &engine::Config::page_size)
      .def_readwrite("num_pages", &engine::Config::num_pages)
      .def_readwrite("max_model_len", &engine::Config::max_model_len)
      .def_readwrite("prefix_caching", &engine::Config::prefix_caching)
      .def_readwrite("pages_per_node", &engine::Config::pages_per_node)
      .def_readwrite("recurrent_state", &engine::Config::recurrent_state)
      .def_readwrite("num_ckpt_slots", &engine::Config::num_ckpt_slots)
      .def_readwrite("prefill_policy", &engine::Config::prefill_policy)
      .def_readwrite("starvation_steps", &engine::Config::starvation_steps)
      .def_readwrite("starvation_ms", &engine::Config::starvation_ms)
      .def_readwrite("max_mixed_step_tokens", &engine::Config::max_mixed_step_tokens)
      .def_readwrite("dynamic_prefill_budget", &engine::Config::dynamic_prefill_budget)
      .def_readwrite("backlog_low_tokens", &engine::Config::backlog_low_tokens)
      .def_readwrite("backlog_high_tokens", &engine::Config::backlog_high_tokens)
      .def_readwrite("max_waiting", &engine::Config::max_waiting)
      .def_readwrite("spec_method", &engine::Config::spec_method)
      .def_readwrite("num_spec_tokens", &engine::Config::num_spec_tokens)
      .def_readwrite("ngram_min", &engine::Config::ngram_min)
      .def_readwrite("ngram_max", &engine::Config::ngram_max)
      .def_readwrite("kv_hash_seed", &engine::Config::kv_hash_seed)
      .def_readwrite("dram_blocks", &engine::Config::dram_blocks)
      .def_readwrite("dram_loading_area", &engine::Config::dram_loading_area)
      .def_readwrite("in_flight_depth", &engine::Config::in_flight_depth);
  py::class_<engine::EngineStats>(m, "EngineStats")
      .def_readonly("waiting", &engine::EngineStats::waiting)
      .def_readonly("running", &engine::EngineStats::running)
      .def_readonly("kv_usage", &engine::EngineStats::kv_usage)
      .def_readonly("steps", &engine::EngineStats::steps)
      .def_readonly("decode_steps", &engine::EngineStats::decode_steps)
      .def_readonly("prefill_tokens", &engine::EngineStats::prefill_tokens)
      .def_readonly("decode_tokens", &engine::EngineStats::decode_tokens)
      .def_readonly("prefix_queries", &engine::EngineStats::prefix_queries)
      .def_readonly("prefix_hit_tokens", &engine::EngineStats::prefix_hit_tokens)
      .def_readonly("prefix_query_tokens", &engine::EngineStats::prefix_query_tokens)
      .def_readonly("prefix_evictions", &engine::EngineStats::prefix_evictions)
      .def_readonly("spec_drafts", &engine::EngineStats::spec_drafts)
      .def_readonly("spec_accepted", &engine::EngineStats::spec_accepted)
      .def_readonly("spec_verify_steps", &engine::EngineStats::spec_verify_steps)
      .def_readonly("dram_capacity", &engine::EngineStats::dram_capacity)
      .def_readonly("dram_occupied", &engine::EngineStats::dram_occupied)
      .def_readonly("dram_offloads", &engine::EngineStats::dram_offloads)
      .def_readonly("dram_reloads", &engine::EngineStats::dram_reloads)
      .def_readonly("dram_evictions", &engine::EngineStats::dram_evictions)
      .def_readonly("dram_hit_tokens", &engine::EngineStats::dram_hit_tokens)
      .def_readonly("run_ahead_steps", &engine::EngineStats::run_ahead_steps)
      .def_readonly("last_gpu_us", &engine::EngineStats::last_gpu_us);
  py::class_<engine::Engine, std::shared_ptr<engine::Engine>>(m, "Engine")
      .def(py::init([](engine::Config cfg, py::function backend, bool async_backend) {
             auto be = std::make_shared<PyBackend>(backend);
             be->set_async(async_backend);  // tests: let the engine run ahead (steps still run at submit)
             return std::make_shared<engine::Engine>(cfg, be);
           }),
           py::arg("config"), py::arg("backend"), py::arg("async_backend") = false)
      .def("submit",
           [](engine::Engine& e, uint64_t id, std::vector<int32_t> prompt, uint32_t max_tokens, bool ignore_eos,
              std::vector<int32_t> eos, float temperature, float top_p, int32_t top_k, uint64_t seed) {
             engine::Request r;
             r.id = id;
             r.prompt = std::move(prompt);
             r.max_tokens = max_tokens;
             r.ignore_eos = ignore_eos;
             r.eos_ids = std::move(eos);
             r.sampling.temperature = temperature;
             r.sampling.top_p = top_p;
             r.sampling.top_k = top_k;
             r.sampling.seed = seed;
             return e.submit(std::move(r));
           },
           py::arg("id"), py::arg("prompt"), py::arg("max_tokens") = 16, py::arg("ignore_eos") = false,
           py::arg("eos") = std::vector<int32_t>{}, py::arg("temperature") = 0.f, py::arg("top_p") = 1.f,
           py::arg("top_k") = 0, py::arg("seed") = 0)
      .def("cancel", &engine::Engine::cancel)
      .def("step",
           [](engine::Engine& e) {
             std::vector<engine::TokenEvent> evs;
             {
               py::gil_scoped_release nogil;
               evs = e.step();
             }
             py::list out;
             for (auto& ev : evs) out.append(event_dict(ev));
             return out;
           })
      .def("has_work", &engine::Engine::has_work)
      .def("poisoned", &engine::Engine::poisoned)
      .def("error", &engine::Engine::error)
      .def("stats", &engine::Engine::stats)
      .def("free_pages", &engine::Engine::free_pages)
      .def("free_slots", &engine::Engine::free_slots)
      .def("free_ckpt_slots", &engine::Engine::free_ckpt_slots)
      .def("cached_prefix_nodes", [](engine::Engine& e) { return e.prefix_tree() ? e.prefix_tree()->cached_nodes() : 0; });


  // ---------------------------------------------------------------- tokenizer
  py::class_<tok::Tokenizer, std::shared_ptr<tok::Tokenizer>>(m, "Tokenizer")
      .def(py::init<>())
      .def("load_dir",
           [](tok::Tokenizer& t, const std::string& d) {
             std::string err;
             if (!t.load_dir(d, &err)) throw std::runtime_error(err);
           })
      .def("load_json",
           [](tok::Tokenizer& t, const std::string& j) {
             std::string err;
             if (!t.load_json(j, &err)) throw std::runtime_error(err);
           })
      .def("encode", &tok::Tokenizer::encode)
      .def("decode",
           [](const tok::Tokenizer& t, const std::vector<int32_t>& ids, bool skip) {
             return py::bytes(t.decode(ids, skip));
           },
           py::arg("ids"), py::arg("skip_special") = true)
      .def("token_bytes", [](const tok::Tokenizer& t, int32_t id) { return py::bytes(t.token_bytes(id)); })
      .def("token_id", &tok::Tokenizer::token_id)
      .def("is_special", &tok::Tokenizer::is_special)
      .def("vocab_size", &tok::Tokenizer::vocab_size)
      .def("eos_ids", &tok::Tokenizer::eos_ids)
      .def("set_eos_ids", &tok::Tokenizer::set_eos_ids)
      .def_static("pre_split", [](const std::string& text) {
        py::list out;
        for (auto& p : tok::Tokenizer::pre_split(text)) out.append(py::bytes(p));
        return out;
      });
  m.def("render_chat",
        [](std::vector<std::tuple<std::string, std::string, std::string>> msgs, const std::string& format, bool thinking,
           bool add_bos, const std::string& effort) {
          std::vector<tok::ChatMessage> ms;
          for (auto& t : msgs) ms.push_back({std::get<0>(t), std::get<1>(t), std::get<2>(t)});
          tok::TemplateOptions o;
          o.format = format == "deepseek" ? tok::TemplateFormat::kDeepSeek : tok::TemplateFormat::kChatML;
          o.thinking = thinking;
          o.add_bos = add_bos;
          o.reasoning_effort = effort;
          std::string prompt, err;
          if (!tok::render_chat(ms, o, &prompt, &err)) throw std::invalid_argument(err);
          return prompt;
        },
        py::arg("messages"), py::arg("format") = "chatml", py::arg("thinking") = false, py::arg("add_bos") = true,
        py::arg("reasoning_effort") = "");
  py::class_<tok::StreamDecoder>(m, "StreamDecoder")
      .def(py::init([](std::shared_ptr<tok::Tokenizer> t, std::vector<std::string> stop) {
             return new tok::StreamDecoder(t.get(), std::move(stop));
           }),
           py::keep_alive<1, 2>())
      .def("push", [](tok::StreamDecoder& d, int32_t id) { return py::bytes(d.push(id)); })
      .def("finish", [](tok::StreamDecoder& d) { return py::bytes(d.finish()); })
      .def("stopped", &tok::StreamDecoder::stopped);

  // ---------------------------------------------------------------- online server (mock backend)
  struct MockServer {
    std::shared_ptr<tok::Tokenizer> tok;
    std::shared_ptr<engine::Engine> engine;
    std::unique_ptr<serve::ServeLoop> loop;
    std::unique_ptr<http::HttpServer> server;
  };
  py::class_<MockServer, std::shared_ptr<MockServer>>(m, "MockServer")
      .def("port", [](MockServer& s) { return s.server->port(); })
      .def("admin_port", [](MockServer& s) { return s.server->admin_port(); })
      .def("state", [](MockServer& s) { return std::string(serve::state_name(s.loop->state())); })
      .def("set_state", [](MockServer& s, int st) { s.loop->set_state((serve::EngineState)st); })
      .def("drain", [](MockServer& s) { s.server->request_drain(); })
      .def("idle", [](MockServer& s) { return s.loop->idle(); })
      .def("free_pages", [](MockServer& s) { return s.engine->free_pages(); })
      .def("free_slots", [](MockServer& s) { return s.engine->free_slots(); })
      .def("metrics_text", [](MockServer& s) { return http::HttpServer::render_metrics(s.loop.get(), http::ServerConfig()); })
      .def("stop", [](MockServer& s) {
        py::gil_scoped_release nogil;
        s.server->stop();
        s.loop->shutdown();
      });
  m.def("serve_mock",
        [](std::shared_ptr<tok::Tokenizer> t, engine::Config cfg, int port, std::string api_key, int admin_port,
           std::string model_name, size_t max_waiting, int32_t mock_high, int32_t eos_every, bool allow_remote_metrics,
           std::string template_format, int step_delay_us, int32_t mock_low, int64_t fail_after) {
          auto ms = std::make_shared<MockServer>();
          ms->tok = t;
          const int32_t eos = t->eos_ids().empty() ? -1 : t->eos_ids()[0];
          auto backend = serve::make_mock_backend(mock_low, mock_high, eos, eos_every);
          if (step_delay_us > 0) {
            struct Slow : engine::Backend {
              std::shared_ptr<engine::Backend> inner;
              int us;
              bool execute(const engine::StepPlan& p, engine::StepResult* r) override {
                usleep(us);
                return inner->execute(p, r);
              }
            };
            auto slow = std::make_shared<Slow>();
            slow->inner = backend;
            slow->us = step_delay_us;
            backend = slow;
          }
          if (fail_after >= 0) {
            // Fault injection: the backend fails every step after its first `fail_after`,
            // as a dead worker or a kernel error would.
            struct Failing : engine::Backend {
              std::shared_ptr<engine::Backend> inner;
              int64_t left;
              bool execute(const engine::StepPlan& p, engine::StepResult* r) override {
                if (left-- <= 0) return false;
                return inner->execute(p, r);
              }
              std::string error() const override { return "injected backend fault"; }
            };
            auto failing = std::make_shared<Failing>();
            failing->inner = backend;
            failing->left = fail_after;
            backend = failing;
          }
          ms->engine = std::make_shared<engine::Engine>(cfg, backend);
          ms->loop.reset(new serve::ServeLoop(ms->engine, nullptr, max_waiting));
          http::ServerConfig sc;
          sc.port = port;
          sc.api_key = api_key;
          sc.admin_port = admin_port;
          sc.served_model_name = model_name;
          sc.max_model_len = cfg.max_model_len;
          sc.allow_remote_metrics = allow_remote_metrics;
          sc.template_format = template_format == "deepseek" ? tok::TemplateFormat::kDeepSeek : tok::TemplateFormat::kChatML;
          ms->server.reset(new http::HttpServer(sc, ms->loop.get(), t.get()));
          std::string err;
          if (!ms->server->start(&err)) throw std::runtime_error(err);
          ms->loop->start();
          return ms;
        },
        py::arg("tokenizer"), py::arg("config"), py::arg("port") = 0, py::arg("api_key") = "",
        py::arg("admin_port") = -1, py::arg("model_name") = "zstep-mock", py::arg("max_waiting") = 64,
        py::arg("mock_high") = 256, py::arg("eos_every") = 0, py::arg("allow_remote_metrics") = true,
        py::arg("template_format") = "chatml", py::arg("step_delay_us") = 0, py::arg("mock_low") = 0,
        py::arg("fail_after") = -1);
  m.def("mock_next_token", &serve::mock_next_token);


  // ---------------------------------------------------------------- KV events
  auto mk_event = [](int kind, std::vector<uint64_t> keys) {
    kv::KvEvent e;
    e.kind = kind == 0 ? kv::KvEvent::kStored : kind == 1 ? kv::KvEvent::kRemoved : kv::KvEvent::kAllCleared;
    e.block_keys = std::move(keys);
    return e;
  };
  m.def("encode_kv_batch",
        [mk_event](int kind, std::vector<uint64_t> keys, double ts) {
          return py::bytes(kvev::encode_batch(mk_event(kind, std::move(keys)), ts));
        });
  py::class_<kvev::Publisher, std::shared_ptr<kvev::Publisher>>(m, "KvEventPublisher")
      .def(py::init<std::string, std::string, size_t>(), py::arg("endpoint"), py::arg("topic"),
           py::arg("queue_cap") = 4096)
      .def("start",
           [](kvev::Publisher& p) {
             std::string err;
             bool ok;
             {
               py::gil_scoped_release nogil;
               ok = p.start(&err);
             }
             if (!ok) throw std::runtime_error(err);
           })
      .def("publish",
           [mk_event](kvev::Publisher& p, int kind, std::vector<uint64_t> keys) { p.publish(mk_event(kind, keys)); })
      .def("stop",
           [](kvev::Publisher& p) {
             py::gil_scoped_release nogil;
             p.stop();
           })
      .def("sent", &kvev::Publisher::sent)
      .def("dropped", &kvev::Publisher::dropped);

  // ---------------------------------------------------------------- coordinator engine
  m.def("make_shm_engine",
        [](engine::Config cfg, wire::Geometry geo, std::vector<std::string> argv, std::map<std::string, std::string> env,
           int ready_timeout_ms, int step_timeout_ms, int heartbeat_timeout_ms) {
          CoordinatorConfig cc;
          cc.geo = geo;
          cc.worker_argv = std::move(argv);
          cc.env = std::move(env);
          cc.ready_timeout_ms = ready_timeout_ms;
          cc.step_timeout_ms = step_timeout_ms;
          cc.heartbeat_timeout_ms = heartbeat_timeout_ms;
          auto coord = std::make_shared<Coordinator>(cc);
          {
            py::gil_scoped_release nogil;
            coord->launch();
          }
          auto eng = std::make_shared<engine::Engine>(cfg, coord);
          return py::make_tuple(eng, py::cast(coord));
        });
  py::class_<Coordinator, std::shared_ptr<Coordinator>>(m, "Coordinator")
      .def("shutdown", [](Coordinator& c) {
        py::gil_scoped_release nogil;
        c.shutdown();
      })
      .def("pids", &Coordinator::pids)
      .def("error", &Coordinator::error)
      .def("steps", [](Coordinator& c) { return c.steps; })
      .def("publish_ns_total", [](Coordinator& c) { return c.publish_ns_total; })
      .def("wait_ns_total", [](Coordinator& c) { return c.wait_ns_total; });
}
