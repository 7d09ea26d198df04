// Torch bindings of the zstep_b200 kernel library (module zstep_b200._C).
//
// Each binding validates devices/dtypes/contiguity, converts tensors to raw pointers
// and calls the C ABI in zs_kernels.h on the current CUDA stream.  Any non-zero return
// code raises, so a missing or rejected kernel is never silently replaced.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <algorithm>
#include <optional>

#include "zs_kernels.h"

namespace {

using Tensor = at::Tensor;
using OptT = std::optional<Tensor>;

template <typename T = void>
T* ptr(const Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
template <typename T = void>
T* optptr(const OptT& t) {
  return t.has_value() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}
void check_opt(const OptT& t, const char* name) {
  if (t.has_value()) check_cuda(*t, name);
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void rc(int code, const char* what) { TORCH_CHECK(code == 0, what, " failed with code ", code); }

void gemm_mxf8(const Tensor& a, const Tensor& sfa, const Tensor& b, const Tensor& sfb, int64_t k,
               int64_t n_pad, int64_t n_valid, int64_t groups, int64_t m_rows,
               const OptT& group_count, const OptT& group_offset, const OptT& chunk_prefix,
               int64_t epi_mode, const Tensor& out, int64_t ldo, const OptT& out_sf,
               const OptT& row_dst, const OptT& row_scale, const OptT& err, int64_t max_items,
               int64_t block_n, int64_t k_splits, int64_t split_stride, int64_t a_tiled,
               int64_t fix_splits, const OptT& ws, const OptT& tile_sem, const OptT& row_temp,
               const OptT& row_seed, const OptT& row_pos, int64_t id_offset, const OptT& sample_any,
               int64_t a_fp4, const std::vector<int64_t>& push_part, const OptT& push_epoch, int64_t push_rank,
               int64_t push_mode, int64_t last_m0, int64_t last_mt) {
  check_cuda(a, "a");
  check_cuda(sfa, "sfa");
  check_cuda(b, "b");
  check_cuda(sfb, "sfb");
  check_cuda(out, "out");
  check_opt(group_count, "group_count");
  check_opt(group_offset, "group_offset");
  check_opt(chunk_prefix, "chunk_prefix");
  TORCH_CHECK(a.element_size() == 1 && b.element_size() == 1, "a/b must be 8-bit");
  TORCH_CHECK(a.numel() * (a_fp4 ? 2 : 1) >= groups * n_pad * k, "a too small");
  TORCH_CHECK(!a_fp4 || a_tiled, "MXFP4 weights must be pre-tiled");
  TORCH_CHECK(b.numel() % k == 0, "b must be [rows, k]");
  GemmMxf8Args p{};
  p.a = ptr<const uint8_t>(a);
  p.sfa = ptr<const uint8_t>(sfa);
  p.b = ptr<const uint8_t>(b);
  p.sfb = ptr<const uint8_t>(sfb);
  p.k = (int)k;
  p.n_pad = (int)n_pad;
  p.n_valid = (int)n_valid;
  p.groups = (int)groups;
  p.b_rows = (int)(b.numel() / k);
  p.m_rows = (int)m_rows;
  p.group_count = optptr<const int>(group_count);
  p.group_offset = optptr<const int>(group_offset);
  p.chunk_prefix = optptr<const int>(chunk_prefix);
  p.max_items = (int)max_items;
  p.epi_mode = (int)epi_mode;
  p.out = ptr(out);
  p.ldo = (int)ldo;
  p.out_sf = optptr<uint8_t>(out_sf);
  p.row_dst = optptr<const int>(row_dst);
  p.row_scale = optptr<const float>(row_scale);
  p.err = optptr<int>(err);
  p.block_n = (int)block_n;
  p.chunk_rows = (int)block_n;
  p.k_splits = (int)k_splits;
  p.split_stride = split_stride;
  p.a_tiled = (int)a_tiled;
  p.a_fp4 = (int)a_fp4;
  p.fix_splits = (int)fix_splits;
  if (row_temp.has_value()) {
    TORCH_CHECK(row_seed.has_value() && row_pos.has_value(), "sampling needs row_temp, row_seed and row_pos");
    TORCH_CHECK(row_temp->scalar_type() == at::kFloat && row_seed->scalar_type() == at::kLong &&
                    row_pos->scalar_type() == at::kInt,
                "row_temp f32, row_seed i64, row_pos i32");
    p.row_temp = ptr<const float>(*row_temp);
    p.row_seed = ptr<const long long>(*row_seed);
    p.row_pos = ptr<const int>(*row_pos);
  }
  p.id_offset = (int)id_offset;
  p.sample_any = optptr<const float>(sample_any);
  TORCH_CHECK(push_part.size() <= 8, "at most 8 push targets");
  for (size_t q = 0; q < push_part.size(); ++q) p.push_part[q] = reinterpret_cast<void*>(push_part[q]);
  p.push_world = (int)push_part.size();
  p.push_epoch = optptr<const uint32_t>(push_epoch);
  p.push_rank = (int)push_rank;
  p.push_rows = (int)m_rows;
  p.push_mode = (int)push_mode;
  p.last_m0 = (int)last_m0;
  p.last_mt = (int)last_mt;
  if (fix_splits > 1) {
    TORCH_CHECK(ws.has_value() && tile_sem.has_value(), "split-K needs ws and tile_sem");
    TORCH_CHECK(ws->scalar_type() == at::kFloat && tile_sem->scalar_type() == at::kInt, "ws f32, tile_sem i32");
    p.ws = ptr<float>(*ws);
    p.tile_sem = ptr<int>(*tile_sem);
    const int64_t tile_floats = fix_splits * 128 * (block_n == 32 ? 32 : 128);
    p.max_tiles = (int)std::min<int64_t>(tile_sem->numel(), ws->numel() / tile_floats);
  }
  if (k_splits > 1)
    TORCH_CHECK(out.numel() >= (k_splits - 1) * split_stride + m_rows * ldo, "split-K out too small");
  TORCH_CHECK(p.chunk_prefix == nullptr || (p.group_count && p.group_offset), "grouped mode args");
  if (p.chunk_prefix == nullptr) {
    TORCH_CHECK(m_rows <= p.b_rows, "m_rows > rows of b");
    // kEpiPushLL stores into the all-reduce's receive buffers, never into `out`.
    if (k_splits <= 1 && epi_mode != kEpiPushLL)
      TORCH_CHECK(out.numel() >= m_rows * ldo, "out too small for m_rows x ldo");
  }
  rc(zs_gemm_mxf8(&p, stream()), "zs_gemm_mxf8");
}

void quant_mxf8(const Tensor& x, const Tensor& q, const Tensor& sf) {
  check_cuda(x, "x");
  check_cuda(q, "q");
  check_cuda(sf, "sf");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2, "x must be bf16 [rows, k]");
  const int rows = (int)x.size(0), k = (int)x.size(1);
  TORCH_CHECK(q.numel() >= (int64_t)rows * k, "q too small");
  TORCH_CHECK(sf.numel() >= (int64_t)((rows + 127) / 128) * (k / 128) * 512, "sf too small");
  rc(zs_quant_mxf8(ptr(x), rows, k, k, ptr<uint8_t>(q), ptr<uint8_t>(sf), stream()), "zs_quant_mxf8");
}

void add_rmsnorm_quant(const Tensor& residual, const OptT& delta, int64_t n_terms,
                       int64_t d_row_stride, int64_t d_term_stride, const Tensor& weight,
                       double w_offset, double eps, int64_t rows, const OptT& normed,
                       const OptT& q, const OptT& sf, const OptT& term_index, const OptT& term_scale) {
  check_cuda(residual, "residual");
  check_opt(delta, "delta");
  check_opt(normed, "normed");
  check_opt(q, "q");
  check_opt(sf, "sf");
  const int hidden = (int)residual.size(-1);
  TORCH_CHECK(residual.numel() >= rows * hidden, "residual too small");
  const int f32 = delta.has_value() && delta->scalar_type() == at::kFloat ? 1 : 0;
  if (delta.has_value())
    TORCH_CHECK(f32 || delta->scalar_type() == at::kBFloat16, "delta must be bf16 or f32");
  rc(zs_add_rmsnorm_quant(ptr(residual), optptr(delta), (int)n_terms, d_row_stride, d_term_stride, f32,
                          optptr<const int>(term_index), optptr<const float>(term_scale), ptr(weight), (float)w_offset, (float)eps, (int)rows, hidden,
                          optptr(normed), optptr<uint8_t>(q), optptr<uint8_t>(sf), stream()),
     "zs_add_rmsnorm_quant");
}

void embed_rmsnorm_quant(const Tensor& ids, const Tensor& embed, const Tensor& hidden,
                         const Tensor& weight, double w_offset, double eps, int64_t rows,
                         const OptT& normed, const OptT& q, const OptT& sf) {
  check_cuda(ids, "ids");
  check_cuda(embed, "embed");
  check_cuda(hidden, "hidden");
  TORCH_CHECK(ids.scalar_type() == at::kInt, "ids must be int32");
  rc(zs_embed_rmsnorm_quant(ptr<const int>(ids), ptr(embed), ptr(hidden), ptr(weight),
                            (float)w_offset, (float)eps, (int)rows, (int)embed.size(1),
                            optptr(normed), optptr<uint8_t>(q), optptr<uint8_t>(sf), stream()),
     "zs_embed_rmsnorm_quant");
}

void argmax_reduce(const Tensor& keys, int64_t rows, int64_t tiles, const OptT& ids,
                   const OptT& vals, const OptT& out_keys) {
  check_cuda(keys, "keys");
  rc(zs_argmax_reduce(ptr<const unsigned long long>(keys), (int)rows, (int)tiles,
                      optptr<int>(ids), optptr<float>(vals), optptr<unsigned long long>(out_keys),
                      stream()),
     "zs_argmax_reduce");
}

void gdn(bool prefill, const Tensor& proj, int64_t num_k_heads, int64_t num_v_heads,
         const Tensor& conv_w, const Tensor& conv_state, const Tensor& ssm_state,
         const Tensor& a_log, const Tensor& dt_bias, const Tensor& norm_w, double eps,
         const Tensor& slots, const Tensor& positions, int64_t rows, const OptT& out_bf16,
         const OptT& out_q, const OptT& out_sf, const OptT& seq_start, int64_t num_seqs,
         const OptT& ckpt_rows, const OptT& ckpt_slots, int64_t max_ckpt, const OptT& err,
         const OptT& out_slots = std::nullopt, int64_t impl = 0, int64_t max_seq_rows = 0) {
  check_cuda(proj, "proj");
  check_cuda(ssm_state, "ssm_state");
  check_cuda(conv_state, "conv_state");
  TORCH_CHECK(ssm_state.scalar_type() == at::kFloat, "ssm_state must be f32");
  TORCH_CHECK(a_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat,
              "a_log/dt_bias must be f32");
  GdnArgs g{};
  g.proj = ptr(proj);
  g.ld_proj = (int)proj.size(-1);
  g.num_k_heads = (int)num_k_heads;
  g.num_v_heads = (int)num_v_heads;
  g.head_k = 128;
  g.head_v = 128;
  g.conv_w = ptr(conv_w);
  g.conv_state = ptr(conv_state);
  g.ssm_state = ptr<float>(ssm_state);
  g.a_log = ptr<const float>(a_log);
  g.dt_bias = ptr<const float>(dt_bias);
  g.norm_w = ptr(norm_w);
  g.eps = (float)eps;
  g.slots = ptr<const int>(slots);
  g.positions = ptr<const int>(positions);
  g.rows = (int)rows;
  g.out_bf16 = optptr(out_bf16);
  g.out_q = optptr<uint8_t>(out_q);
  g.out_sf = optptr<uint8_t>(out_sf);
  g.seq_start = optptr<const int>(seq_start);
  g.num_seqs = (int)num_seqs;
  g.ckpt_rows = optptr<const int>(ckpt_rows);
  g.ckpt_slots = optptr<const int>(ckpt_slots);
  g.max_ckpt = (int)max_ckpt;
  g.err = optptr<int>(err);
  g.out_slots = optptr<const int>(out_slots);
  g.impl = (int)impl;
  g.max_seq_rows = (int)max_seq_rows;
  rc(prefill ? zs_gdn_prefill(&g, stream()) : zs_gdn_decode(&g, stream()), "zs_gdn");
}

AttnArgs make_attn(const Tensor& qkv, int64_t num_q_heads, int64_t num_kv_heads,
                   int64_t rotary_dim, double rope_theta, const Tensor& q_norm_w,
                   const Tensor& k_norm_w, double eps, const Tensor& k_cache,
                   const Tensor& v_cache, int64_t page_size, const Tensor& page_table,
                   const Tensor& slots, const Tensor& positions, int64_t rows,
                   const Tensor& q_out, const Tensor& gate_out) {
  check_cuda(qkv, "qkv");
  check_cuda(k_cache, "k_cache");
  check_cuda(v_cache, "v_cache");
  check_cuda(page_table, "page_table");
  TORCH_CHECK(page_table.scalar_type() == at::kInt, "page_table must be int32");
  AttnArgs a{};
  a.qkv = ptr(qkv);
  a.ld_qkv = (int)qkv.size(-1);
  a.num_q_heads = (int)num_q_heads;
  a.num_kv_heads = (int)num_kv_heads;
  a.head_dim = 256;
  a.rotary_dim = (int)rotary_dim;
  a.rope_theta = (float)rope_theta;
  a.q_norm_w = ptr(q_norm_w);
  a.k_norm_w = ptr(k_norm_w);
  a.eps = (float)eps;
  a.k_cache = ptr(k_cache);
  a.v_cache = ptr(v_cache);
  a.page_size = (int)page_size;
  a.page_table = ptr<const int>(page_table);
  a.max_pages = (int)page_table.size(1);
  a.slots = ptr<const int>(slots);
  a.positions = ptr<const int>(positions);
  a.rows = (int)rows;
  a.q_out = ptr(q_out);
  a.gate_out = ptr(gate_out);
  return a;
}

void attn_prologue(const Tensor& qkv, int64_t num_q_heads, int64_t num_kv_heads,
                   int64_t rotary_dim, double rope_theta, const Tensor& q_norm_w,
                   const Tensor& k_norm_w, double eps, const Tensor& k_cache,
                   const Tensor& v_cache, int64_t page_size, const Tensor& page_table,
                   const Tensor& slots, const Tensor& positions, int64_t rows,
                   const Tensor& q_out, const Tensor& gate_out) {
  AttnArgs a = make_attn(qkv, num_q_heads, num_kv_heads, rotary_dim, rope_theta, q_norm_w,
                         k_norm_w, eps, k_cache, v_cache, page_size, page_table, slots,
                         positions, rows, q_out, gate_out);
  rc(zs_attn_prologue(&a, stream()), "zs_attn_prologue");
}

void attn_decode(const Tensor& q_out, const Tensor& gate_out, int64_t num_q_heads,
                 int64_t num_kv_heads, const Tensor& k_cache, const Tensor& v_cache,
                 int64_t page_size, const Tensor& page_table, const Tensor& slots,
                 const Tensor& seq_lens, int64_t rows, const Tensor& partial, int64_t num_splits,
                 double sm_scale, const OptT& out_bf16, const OptT& out_q, const OptT& out_sf, int64_t impl,
                 const OptT& err, const OptT& seq_start, int64_t num_seqs) {
  check_cuda(q_out, "q_out");
  check_cuda(partial, "partial");
  TORCH_CHECK(!seq_start.has_value() || (num_seqs >= 0 && seq_start->numel() > num_seqs),
              "seq_start must hold num_seqs + 1 row offsets");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == page_size, "k_cache must be [pages, kv_heads, page, 256]");
  TORCH_CHECK(partial.numel() >= rows * num_q_heads * num_splits * 260, "partial too small");
  AttnArgs a{};
  a.num_q_heads = (int)num_q_heads;
  a.num_kv_heads = (int)num_kv_heads;
  a.head_dim = 256;
  a.k_cache = ptr(k_cache);
  a.v_cache = ptr(v_cache);
  a.page_size = (int)page_size;
  a.page_table = ptr<const int>(page_table);
  a.max_pages = (int)page_table.size(1);
  a.slots = ptr<const int>(slots);
  a.seq_lens = ptr<const int>(seq_lens);
  a.rows = (int)rows;
  a.q_out = ptr(q_out);
  a.gate_out = ptr(gate_out);
  a.partial = ptr<float>(partial);
  a.num_splits = (int)num_splits;
  a.sm_scale = (float)sm_scale;
  a.out_bf16 = optptr(out_bf16);
  a.out_q = optptr<uint8_t>(out_q);
  a.out_sf = optptr<uint8_t>(out_sf);
  a.impl = (int)impl;
  a.err = optptr<int>(err);
  a.seq_start = optptr<const int>(seq_start);
  a.num_seqs = seq_start.has_value() ? (int)num_seqs : 0;
  rc(zs_attn_decode(&a, stream()), "zs_attn_decode");
}

void moe_route(const Tensor& logits, int64_t rows, int64_t num_experts, int64_t top_k,
               bool norm_topk, int64_t scoring, const OptT& bias, int64_t n_group,
               int64_t topk_group, double routed_scale, int64_t shared_gate_col,
               int64_t expert_begin, int64_t expert_end, bool has_shared, const Tensor& topk_ids,
               const Tensor& topk_w, const Tensor& group_count, const Tensor& group_offset,
               const Tensor& chunk_prefix, const Tensor& pair_slot, const Tensor& row_dst,
               const Tensor& row_scale, const Tensor& x_q, const Tensor& x_sf,
               const Tensor& xg_q, const Tensor& xg_sf, const OptT& err, int64_t ld_logits,
               int64_t logit_splits, int64_t logit_split_stride, int64_t chunk_rows, const OptT& pair_src,
               const OptT& pair_w) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat, "logits must be f32");
  MoeRouteArgs a{};
  a.logits = ptr<const float>(logits);
  a.ld_logits = (int)ld_logits;
  a.logit_splits = (int)logit_splits;
  a.logit_split_stride = logit_split_stride;
  a.chunk_rows = (int)chunk_rows;
  TORCH_CHECK(logits.numel() >= (logit_splits > 1 ? (logit_splits - 1) * logit_split_stride : 0) +
                                    rows * ld_logits, "logits too small");
  a.rows = (int)rows;
  a.num_experts = (int)num_experts;
  a.top_k = (int)top_k;
  a.norm_topk = norm_topk ? 1 : 0;
  a.scoring = (int)scoring;
  a.bias = optptr<const float>(bias);
  a.n_group = (int)n_group;
  a.topk_group = (int)topk_group;
  a.routed_scale = (float)routed_scale;
  a.shared_gate_col = (int)shared_gate_col;
  a.expert_begin = (int)expert_begin;
  a.expert_end = (int)expert_end;
  a.has_shared = has_shared ? 1 : 0;
  a.topk_ids = ptr<int>(topk_ids);
  a.topk_w = ptr<float>(topk_w);
  a.group_count = ptr<int>(group_count);
  a.group_offset = ptr<int>(group_offset);
  a.chunk_prefix = ptr<int>(chunk_prefix);
  a.pair_slot = ptr<int>(pair_slot);
  a.row_dst = ptr<int>(row_dst);
  a.row_scale = ptr<float>(row_scale);
  a.pair_src = optptr<int>(pair_src);
  a.pair_w = optptr<float>(pair_w);
  TORCH_CHECK(a.pair_src == nullptr || a.pair_w != nullptr, "pair_src needs pair_w");
  a.max_grouped_rows = (int)(xg_q.numel() / x_q.size(-1));
  a.x_q = ptr<const uint8_t>(x_q);
  a.x_sf = ptr<const uint8_t>(x_sf);
  a.hidden = (int)x_q.size(-1);
  a.xg_q = ptr<uint8_t>(xg_q);
  a.xg_sf = ptr<uint8_t>(xg_sf);
  a.err = optptr<int>(err);
  rc(zs_moe_route(&a, stream()), "zs_moe_route");
}

void fused_allreduce_norm(int64_t rank, int64_t world, int64_t protocol, const Tensor& delta, int64_t n_terms,
                          int64_t row_stride, int64_t term_stride, const std::vector<int64_t>& part,
                          const std::vector<int64_t>& out, const std::vector<int64_t>& flags, const Tensor& epoch,
                          const Tensor& grid_counter, const Tensor& residual, const Tensor& weight, double w_offset,
                          double eps, int64_t rows, const OptT& normed, const OptT& q, const OptT& sf, const OptT& err,
                          const OptT& term_index, const OptT& term_scale, int64_t timeout_ms, bool pushed,
                          const std::vector<int64_t>& mc) {
  TORCH_CHECK(world >= 1 && world <= 8 && (int64_t)part.size() == world &&
                  (out.empty() || (int64_t)out.size() == world) && (flags.empty() || (int64_t)flags.size() == world),
              "bad world / pointer lists");
  TORCH_CHECK(mc.empty() || mc.size() == 3, "mc: multicast addresses of part, out and flags");
  check_cuda(delta, "delta");
  check_cuda(residual, "residual");
  FusedArArgs a{};
  a.rank = (int)rank;
  a.world = (int)world;
  a.protocol = (int)protocol;
  a.delta = ptr(delta);
  a.n_terms = (int)n_terms;
  a.row_stride = row_stride;
  a.term_stride = term_stride;
  a.delta_f32 = delta.scalar_type() == at::kFloat ? 1 : 0;
  for (int r = 0; r < world; ++r) {
    a.part[r] = reinterpret_cast<void*>(part[r]);
    if (!out.empty()) a.out[r] = reinterpret_cast<void*>(out[r]);
    if (!flags.empty()) a.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
  }
  a.epoch = ptr<uint32_t>(epoch);
  a.grid_counter = ptr<uint32_t>(grid_counter);
  a.residual = ptr(residual);
  a.weight = ptr(weight);
  a.w_offset = (float)w_offset;
  a.eps = (float)eps;
  a.rows = (int)rows;
  a.hidden = (int)residual.size(-1);
  a.normed = optptr(normed);
  a.q = optptr<uint8_t>(q);
  a.sf = optptr<uint8_t>(sf);
  a.err = optptr<int>(err);
  a.term_index = optptr<const int>(term_index);
  a.term_scale = optptr<const float>(term_scale);
  a.timeout_ms = (unsigned int)timeout_ms;
  a.pushed = pushed ? 1 : 0;
  if (!mc.empty()) {
    a.mc_part = reinterpret_cast<void*>(mc[0]);
    a.mc_out = reinterpret_cast<void*>(mc[1]);
    a.mc_flags = reinterpret_cast<uint32_t*>(mc[2]);
  }
  rc(zs_fused_allreduce_norm(&a, stream()), "zs_fused_allreduce_norm");
}

void allreduce_sum_f32(int64_t rank, int64_t world, const Tensor& data, int64_t rows, int64_t max_rows,
                       const std::vector<int64_t>& buf, const Tensor& epoch, const Tensor& grid_counter,
                       const OptT& err, int64_t timeout_ms, const std::vector<int64_t>& part,
                       const std::vector<int64_t>& out, const std::vector<int64_t>& flags) {
  TORCH_CHECK(world >= 1 && world <= 8 && (int64_t)buf.size() == world, "bad world ", world, " / buffer list");
  check_cuda(data, "data");
  TORCH_CHECK(data.scalar_type() == at::kFloat && data.dim() == 2, "data: f32 [rows, cols]");
  SumArArgs a{};
  a.rank = (int)rank;
  a.world = (int)world;
  a.data = ptr<float>(data);
  a.rows = (int)rows;
  a.cols = (int)data.size(1);
  a.max_rows = (int)max_rows;
  for (int r = 0; r < world; ++r) a.buf[r] = reinterpret_cast<void*>(buf[r]);
  a.epoch = ptr<uint32_t>(epoch);
  a.grid_counter = ptr<uint32_t>(grid_counter);
  a.err = optptr<int>(err);
  a.timeout_ms = (unsigned int)timeout_ms;
  if (!part.empty()) {
    TORCH_CHECK((int64_t)part.size() == world && (int64_t)out.size() == world && (int64_t)flags.size() == world,
                "plain fp32 sum: part / out / flags per rank");
    a.plain = 1;
    for (int r = 0; r < world; ++r) {
      a.part[r] = reinterpret_cast<void*>(part[r]);
      a.out[r] = reinterpret_cast<void*>(out[r]);
      a.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
    }
  }
  rc(zs_allreduce_sum_f32(&a, stream()), "zs_allreduce_sum_f32");
}

void allreduce_argmax(int64_t rank, int64_t world, int64_t rows, int64_t max_rows, const Tensor& tile_keys,
                      int64_t tiles, int64_t id_offset, const std::vector<int64_t>& lines, const Tensor& epoch,
                      const Tensor& grid_counter, const OptT& out_ids, const OptT& out_vals, const OptT& err,
                      int64_t timeout_ms) {
  TORCH_CHECK(world >= 1 && world <= 8 && (int64_t)lines.size() == world, "bad world / pointer lists");
  check_cuda(tile_keys, "tile_keys");
  TORCH_CHECK(tile_keys.scalar_type() == at::kLong && tile_keys.numel() >= rows * tiles, "tile_keys: i64 [rows, tiles]");
  ArgmaxArArgs a{};
  a.rank = (int)rank;
  a.world = (int)world;
  a.rows = (int)rows;
  a.max_rows = (int)max_rows;
  a.tile_keys = ptr<const unsigned long long>(tile_keys);
  a.tiles = (int)tiles;
  a.id_offset = (int)id_offset;
  for (int r = 0; r < world; ++r) a.lines[r] = reinterpret_cast<void*>(lines[r]);
  a.epoch = ptr<uint32_t>(epoch);
  a.grid_counter = ptr<uint32_t>(grid_counter);
  a.out_ids = optptr<int>(out_ids);
  a.out_vals = optptr<float>(out_vals);
  a.err = optptr<int>(err);
  a.timeout_ms = (unsigned int)timeout_ms;
  rc(zs_allreduce_argmax(&a, stream()), "zs_allreduce_argmax");
}

void spec_verify(int64_t n, int64_t k, int64_t dummy_slot, const Tensor& ids, const Tensor& targets,
                 const Tensor& pos, const Tensor& slot, const Tensor& record, const Tensor& rep_start,
                 const Tensor& rep_idx, const Tensor& rep_slot, const Tensor& rep_pos, const Tensor& mtp_ids,
                 const Tensor& mtp_pos, const Tensor& mtp_slot, const Tensor& mtp_len, const Tensor& last_row) {
  const int64_t rows = n * (k + 1);
  for (const Tensor* t : {&ids, &targets, &pos, &slot, &rep_slot, &rep_pos, &mtp_ids, &mtp_pos, &mtp_slot, &mtp_len}) {
    check_cuda(*t, "spec_verify operand");
    TORCH_CHECK(t->scalar_type() == at::kInt && t->numel() >= rows, "spec_verify: int32 [n*(k+1)] operands");
  }
  check_cuda(record, "record");
  check_cuda(rep_start, "rep_start");
  check_cuda(rep_idx, "rep_idx");
  check_cuda(last_row, "last_row");
  TORCH_CHECK(record.scalar_type() == at::kInt && record.numel() >= n * (k + 2), "record: int32 [n, k+2]");
  TORCH_CHECK(rep_start.scalar_type() == at::kInt && rep_start.numel() >= n + 1, "rep_start: int32 [n+1]");
  TORCH_CHECK(rep_idx.scalar_type() == at::kLong && rep_idx.numel() >= rows, "rep_idx: int64 [n*(k+1)]");
  TORCH_CHECK(last_row.scalar_type() == at::kLong && last_row.numel() >= n, "last_row: int64 [n]");
  SpecVerifyArgs a{};
  a.n = (int)n;
  a.k = (int)k;
  a.dummy_slot = (int)dummy_slot;
  a.ids = ptr<const int>(ids);
  a.targets = ptr<const int>(targets);
  a.pos = ptr<const int>(pos);
  a.slot = ptr<const int>(slot);
  a.record = ptr<int>(record);
  a.rep_start = ptr<int>(rep_start);
  a.rep_idx = ptr<long long>(rep_idx);
  a.rep_slot = ptr<int>(rep_slot);
  a.rep_pos = ptr<int>(rep_pos);
  a.mtp_ids = ptr<int>(mtp_ids);
  a.mtp_pos = ptr<int>(mtp_pos);
  a.mtp_slot = ptr<int>(mtp_slot);
  a.mtp_len = ptr<int>(mtp_len);
  a.last_row = ptr<long long>(last_row);
  rc(zs_spec_verify(&a, stream()), "zs_spec_verify");
}

// Expert-parallel dispatch (which = 0) or combine (which = 1); offs = the six byte
// offsets of the symmetric block (flags, counts, q, sf, meta, comb).
void ep_call(int64_t which, int64_t rank, int64_t world, int64_t tokens, int64_t max_tokens, int64_t hidden,
             int64_t top_k, int64_t num_experts, int64_t recv_cap, int64_t chunk_rows, const Tensor& topk_ids,
             const Tensor& topk_w, const OptT& x, const std::vector<int64_t>& sym, const std::vector<int64_t>& offs,
             const Tensor& cnt, const Tensor& pair_slot, const Tensor& bar, const Tensor& epoch,
             const Tensor& group_count, const Tensor& group_offset, const Tensor& chunk_prefix,
             const Tensor& recv_rows, const OptT& y, int64_t ldy, const OptT& residual, const OptT& out,
             const OptT& err, int64_t timeout_ms) {
  TORCH_CHECK(world >= 1 && world <= EP_MAX_WORLD && (int64_t)sym.size() == world, "bad world ", world,
              " or symmetric pointer list of ", sym.size());
  TORCH_CHECK(offs.size() == 6, "offs: flags, counts, q, sf, meta, comb");
  check_cuda(topk_ids, "topk_ids");
  TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_w.scalar_type() == at::kFloat, "topk ids int32, weights f32");
  TORCH_CHECK(topk_ids.is_contiguous() && topk_w.is_contiguous(), "topk tensors must be contiguous");
  EpArgs a{};
  a.rank = (int)rank;
  a.world = (int)world;
  a.tokens = (int)tokens;
  a.max_tokens = (int)max_tokens;
  a.hidden = (int)hidden;
  a.top_k = (int)top_k;
  a.num_experts = (int)num_experts;
  a.recv_cap = (int)recv_cap;
  a.chunk_rows = (int)chunk_rows;
  a.topk_ids = ptr<const int>(topk_ids);
  a.topk_w = ptr<const float>(topk_w);
  if (x) {
    TORCH_CHECK(x->scalar_type() == at::kBFloat16 && x->is_contiguous() && x->size(-1) == hidden, "x: bf16 [tokens, hidden]");
    a.x = ptr(*x);
  }
  for (int r = 0; r < world; ++r) a.sym[r] = reinterpret_cast<char*>(sym[r]);
  a.off_flags = offs[0];
  a.off_counts = offs[1];
  a.off_q = offs[2];
  a.off_sf = offs[3];
  a.off_meta = offs[4];
  a.off_comb = offs[5];
  a.cnt = ptr<int>(cnt);
  a.pair_slot = ptr<int>(pair_slot);
  a.bar = ptr<unsigned long long>(bar);
  a.epoch = ptr<uint32_t>(epoch);
  a.group_count = ptr<int>(group_count);
  a.group_offset = ptr<int>(group_offset);
  a.chunk_prefix = ptr<int>(chunk_prefix);
  a.recv_rows = ptr<int>(recv_rows);
  if (y) {
    TORCH_CHECK(y->scalar_type() == at::kBFloat16 && y->stride(-1) == 1, "y: bf16 rows");
    a.y = ptr(*y);
    a.y_rows = (int)y->size(0);
  }
  a.ldy = ldy;
  if (residual) {
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->is_contiguous(), "residual: bf16 [tokens, hidden]");
    a.residual = ptr(*residual);
  }
  if (out) {
    TORCH_CHECK(out->scalar_type() == at::kBFloat16 && out->is_contiguous(), "out: bf16 [tokens, hidden]");
    a.out = ptr(*out);
  }
  a.err = optptr<int>(err);
  a.timeout_ms = (unsigned int)timeout_ms;
  if (which == 0)
    rc(zs_ep_dispatch(&a, stream()), "zs_ep_dispatch");
  else
    rc(zs_ep_combine(&a, stream()), "zs_ep_combine");
}

int64_t symm_alloc(int64_t bytes) {
  void* p = nullptr;
  rc(zs_symm_alloc((size_t)bytes, &p), "zs_symm_alloc");
  return reinterpret_cast<int64_t>(p);
}

py::bytes ipc_handle(int64_t p) {
  char h[64];
  rc(zs_ipc_handle(reinterpret_cast<void*>(p), h), "zs_ipc_handle");
  return py::bytes(h, 64);
}

int64_t ipc_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == 64, "IPC handle must be 64 bytes");
  void* p = nullptr;
  rc(zs_ipc_open(s.data(), &p), "zs_ipc_open");
  return reinterpret_cast<int64_t>(p);
}

// Non-owning tensor view of device memory at `p` (lifetime managed by the caller).
Tensor tensor_from_ptr(int64_t p, std::vector<int64_t> sizes, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, device);
  return at::from_blob(reinterpret_cast<void*>(p), sizes, opts);
}

}  // namespace


// ------------------------------------------------------------------ DeepSeek-style layers
void mhc_partial(const Tensor& x, int64_t rows, int64_t hidden, const Tensor& fn, int64_t mode, const OptT& y,
                 const OptT& mix_prev, const OptT& ids, const OptT& embed, const Tensor& partial) {
  check_cuda(x, "x");
  check_cuda(fn, "fn");
  check_cuda(partial, "partial");
  TORCH_CHECK(x.scalar_type() == at::kFloat && fn.scalar_type() == at::kFloat, "mhc: x and fn must be fp32");
  MhcPartialArgs a{};
  a.x = ptr<float>(x);
  a.rows = (int)rows;
  a.hidden = (int)hidden;
  a.m = (int)fn.size(0);
  a.fn = ptr<const float>(fn);
  a.mode = (int)mode;
  a.y = optptr<const float>(y);
  a.mix_prev = optptr<const float>(mix_prev);
  a.ids = optptr<const int>(ids);
  a.embed = optptr<const __nv_bfloat16>(embed);
  a.partial = ptr<float>(partial);
  TORCH_CHECK(mode != 1 || (a.y && a.mix_prev), "mhc_partial mode 1 needs y and mix_prev");
  TORCH_CHECK(mode != 2 || (a.ids && a.embed), "mhc_partial mode 2 needs ids and embed");
  TORCH_CHECK(x.numel() >= rows * 4 * hidden, "mhc_partial: x too small");
  TORCH_CHECK(partial.numel() >= rows * zs_mhc_slices((int)hidden) * (a.m + 1), "mhc_partial: partial too small");
  rc(zs_mhc_partial(&a, stream()), "zs_mhc_partial");
}

void mhc_finalize(const Tensor& x, int64_t rows, int64_t hidden, const Tensor& partial, const Tensor& base,
                  const Tensor& scale, double eps, int64_t iters, const OptT& mix_out, const Tensor& weight,
                  const Tensor& q, const Tensor& sf) {
  check_cuda(x, "x");
  check_cuda(q, "q");
  MhcFinalizeArgs a{};
  a.x = ptr<const float>(x);
  a.rows = (int)rows;
  a.hidden = (int)hidden;
  a.m = (int)base.numel();
  a.slices = zs_mhc_slices((int)hidden);
  a.partial = ptr<const float>(partial);
  a.base = ptr<const float>(base);
  a.scale = ptr<const float>(scale);
  a.eps = (float)eps;
  a.sinkhorn_iters = (int)iters;
  a.mix_out = optptr<float>(mix_out);
  a.weight = ptr<const __nv_bfloat16>(weight);
  a.q = ptr<uint8_t>(q);
  a.sf = ptr<uint8_t>(sf);
  TORCH_CHECK(a.m == 4 || a.mix_out, "mhc_finalize: a 24-logit site needs mix_out");
  TORCH_CHECK(q.numel() >= rows * hidden, "mhc_finalize: q too small");
  rc(zs_mhc_finalize(&a, stream()), "zs_mhc_finalize");
}

void rms_quant(const Tensor& x, int64_t width, const Tensor& w, double eps, int64_t rows, const Tensor& q,
               const Tensor& sf) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1, "rms_quant: bf16 rows with unit stride");
  TORCH_CHECK(q.numel() >= rows * width, "rms_quant: q too small");
  rc(zs_rms_quant(ptr(x), (int)x.stride(0), (int)width, ptr(w), (float)eps, (int)rows, ptr<uint8_t>(q),
                  ptr<uint8_t>(sf), stream()),
     "zs_rms_quant");
}

void mla_prologue(const Tensor& proj, int64_t off_kva, int64_t off_ik, int64_t off_iw, const Tensor& qi,
                  int64_t off_iq, int64_t rows, int64_t heads, int64_t nope, int64_t rope, int64_t kv_lora,
                  int64_t index_heads, int64_t index_dim, const Tensor& kv_norm, const Tensor& ik_norm, double eps,
                  double theta, const Tensor& slots, const Tensor& positions, const Tensor& page_table,
                  int64_t page_size, const Tensor& ckv_cache, const Tensor& ik_cache, const Tensor& q_pe,
                  const Tensor& iq, const Tensor& iw) {
  check_cuda(proj, "proj");
  check_cuda(ckv_cache, "ckv_cache");
  check_cuda(ik_cache, "ik_cache");
  TORCH_CHECK(page_table.scalar_type() == at::kInt, "page_table must be int32");
  MlaPrologueArgs a{};
  a.proj = ptr<const __nv_bfloat16>(proj);
  a.ld_proj = (int)proj.stride(0);
  a.off_kva = (int)off_kva;
  a.off_ik = (int)off_ik;
  a.off_iw = (int)off_iw;
  a.qi = ptr<const __nv_bfloat16>(qi);
  a.ld_qi = (int)qi.stride(0);
  a.off_iq = (int)off_iq;
  a.rows = (int)rows;
  a.heads = (int)heads;
  a.qk_dim = (int)(nope + rope);
  a.nope = (int)nope;
  a.rope = (int)rope;
  a.kv_lora = (int)kv_lora;
  a.index_heads = (int)index_heads;
  a.index_dim = (int)index_dim;
  a.kv_norm = ptr<const __nv_bfloat16>(kv_norm);
  a.ik_norm = ptr<const __nv_bfloat16>(ik_norm);
  a.eps = (float)eps;
  a.theta = (float)theta;
  a.iw_scale = (float)(1.0 / std::sqrt((double)index_heads));
  a.slot = ptr<const int>(slots);
  a.pos = ptr<const int>(positions);
  a.page_table = ptr<const int>(page_table);
  a.max_pages = (int)page_table.size(1);
  a.page_size = (int)page_size;
  a.ckv_cache = ptr<__nv_bfloat16>(ckv_cache);
  a.ik_cache = ptr<__nv_bfloat16>(ik_cache);
  a.q_pe = ptr<__nv_bfloat16>(q_pe);
  a.iq = ptr<__nv_bfloat16>(iq);
  a.iw = ptr<float>(iw);
  rc(zs_mla_prologue(&a, stream()), "zs_mla_prologue");
}

void mla_absorb_q(const Tensor& qi, int64_t qk_dim, int64_t nope, const Tensor& w_uk, int64_t heads, int64_t rows,
                  const Tensor& q_lat) {
  check_cuda(qi, "qi");
  check_cuda(w_uk, "w_uk");
  const int kl = (int)w_uk.size(-1);
  TORCH_CHECK(q_lat.numel() >= rows * heads * kl, "mla_absorb_q: q_lat too small");
  rc(zs_mla_absorb_q(ptr(qi), (int)qi.stride(0), (int)qk_dim, (int)nope, ptr(w_uk), kl, (int)heads, (int)rows,
                     ptr(q_lat), stream()),
     "zs_mla_absorb_q");
}

void mla_attn(const Tensor& q_lat, const Tensor& q_pe, const Tensor& ckv_cache, const Tensor& page_table,
              int64_t page_size, const Tensor& slots, const Tensor& sel, const Tensor& n_sel, int64_t rows,
              int64_t heads, int64_t splits, double sm_scale, const Tensor& partial, int64_t impl,
              const OptT& err) {
  check_cuda(q_lat, "q_lat");
  check_cuda(partial, "partial");
  TORCH_CHECK(impl >= 0 && impl <= 2, "mla_attn: impl is 0 / 1 (SIMT) or 2 (tensor cores)");
  MlaAttnArgs a{};
  a.impl = (int)impl;
  a.err = optptr<int>(err);
  a.q_lat = ptr<const __nv_bfloat16>(q_lat);
  a.q_pe = ptr<const __nv_bfloat16>(q_pe);
  a.ckv_cache = ptr<const __nv_bfloat16>(ckv_cache);
  a.page_table = ptr<const int>(page_table);
  a.max_pages = (int)page_table.size(1);
  a.page_size = (int)page_size;
  a.slot = ptr<const int>(slots);
  a.sel = ptr<const int>(sel);
  a.ld_sel = (int)sel.stride(0);
  a.n_sel = ptr<const int>(n_sel);
  a.rows = (int)rows;
  a.heads = (int)heads;
  a.kv_lora = 512;
  a.rope = (int)(ckv_cache.size(-1) - 512);
  a.splits = (int)splits;
  a.sm_scale = (float)sm_scale;
  a.partial = ptr<float>(partial);
  TORCH_CHECK(partial.numel() >= rows * heads * splits * (512 + 4), "mla_attn: partial too small");
  rc(zs_mla_attn(&a, stream()), "zs_mla_attn");
}

void mla_up(const Tensor& partial, int64_t rows, int64_t heads, int64_t splits, const Tensor& w_uv_t, const Tensor& q,
            const Tensor& sf) {
  MlaUpArgs a{};
  a.partial = ptr<const float>(partial);
  a.rows = (int)rows;
  a.heads = (int)heads;
  a.splits = (int)splits;
  a.v_dim = (int)w_uv_t.size(-1);
  a.w_uv_t = ptr<const __nv_bfloat16>(w_uv_t);
  a.q = ptr<uint8_t>(q);
  a.sf = ptr<uint8_t>(sf);
  TORCH_CHECK(q.numel() >= rows * heads * a.v_dim, "mla_up: q too small");
  rc(zs_mla_up(&a, stream()), "zs_mla_up");
}

void dsa_index(const Tensor& iq, const Tensor& iw, const Tensor& ik_cache, const Tensor& page_table,
               int64_t page_size, const Tensor& slots, const Tensor& ctx_len, int64_t rows, int64_t index_heads,
               int64_t topk, int64_t max_ctx, const Tensor& scores, const Tensor& sel, const Tensor& n_sel,
               const OptT& err) {
  check_cuda(iq, "iq");
  check_cuda(scores, "scores");
  TORCH_CHECK(ik_cache.size(-1) == 128, "dsa_index: index dim must be 128");
  TORCH_CHECK(max_ctx <= scores.size(1), "dsa_index: scores buffer narrower than the context");
  TORCH_CHECK(topk <= sel.size(1), "dsa_index: sel buffer narrower than top-k");
  DsaScoresArgs s{};
  s.iq = ptr<const __nv_bfloat16>(iq);
  s.iw = ptr<const float>(iw);
  s.ik_cache = ptr<const __nv_bfloat16>(ik_cache);
  s.page_table = ptr<const int>(page_table);
  s.max_pages = (int)page_table.size(1);
  s.page_size = (int)page_size;
  s.slot = ptr<const int>(slots);
  s.ctx_len = ptr<const int>(ctx_len);
  s.rows = (int)rows;
  s.index_heads = (int)index_heads;
  s.topk = (int)topk;
  s.scale = (float)(1.0 / std::sqrt(128.0));
  s.scores = ptr<float>(scores);
  s.ld_scores = (int)scores.stride(0);
  s.err = optptr<int>(err);
  rc(zs_dsa_scores(&s, (int)max_ctx, stream()), "zs_dsa_scores");
  DsaTopkArgs k{};
  k.scores = s.scores;
  k.ld_scores = s.ld_scores;
  k.ctx_len = s.ctx_len;
  k.rows = (int)rows;
  k.topk = (int)topk;
  k.sel = ptr<int>(sel);
  k.ld_sel = (int)sel.stride(0);
  k.n_sel = ptr<int>(n_sel);
  rc(zs_dsa_topk(&k, stream()), "zs_dsa_topk");
}

void gather_sum(const Tensor& rows_in, const Tensor& src, const Tensor& w, int64_t rows, const Tensor& y) {
  check_cuda(rows_in, "rows_in");
  const int k1 = (int)src.size(-1);
  const int hidden = (int)rows_in.size(-1);
  TORCH_CHECK(y.numel() >= rows * hidden, "gather_sum: y too small");
  rc(zs_gather_sum(ptr(rows_in), ptr<const int>(src), ptr<const float>(w), k1, hidden, (int)rows, ptr<float>(y),
                   stream()),
     "zs_gather_sum");
}


void sample_rows(const Tensor& logits, int64_t vocab, int64_t rows, const Tensor& temperature, const OptT& top_k,
                 const OptT& top_p, const OptT& presence, const OptT& frequency, const OptT& repetition,
                 const Tensor& seed, const OptT& hist, const OptT& hist_len, int64_t top_n, const Tensor& out_token,
                 const OptT& out_logprob, const OptT& out_top_ids, const OptT& out_top_lp) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(-1) == 1, "sample: fp32 logits rows");
  TORCH_CHECK(seed.scalar_type() == at::kLong, "sample: int64 seeds");
  SampleArgs a{};
  a.logits = ptr<float>(logits);
  a.ld = (int)logits.stride(0);
  a.vocab = (int)vocab;
  a.rows = (int)rows;
  a.temperature = ptr<const float>(temperature);
  a.top_k = optptr<const int>(top_k);
  a.top_p = optptr<const float>(top_p);
  a.presence = optptr<const float>(presence);
  a.frequency = optptr<const float>(frequency);
  a.repetition = optptr<const float>(repetition);
  a.seed = ptr<const unsigned long long>(seed);
  a.hist = optptr<const int>(hist);
  a.hist_ld = hist.has_value() ? (int)hist->stride(0) : 0;
  a.hist_len = optptr<const int>(hist_len);
  a.want_logprobs = out_logprob.has_value() ? 1 : 0;
  a.top_n = (int)top_n;
  a.out_token = ptr<int>(out_token);
  a.out_logprob = optptr<float>(out_logprob);
  a.out_top_ids = optptr<int>(out_top_ids);
  a.out_top_lp = optptr<float>(out_top_lp);
  TORCH_CHECK(!a.want_logprobs || top_n == 0 || (a.out_top_ids && a.out_top_lp), "sample: top-N outputs");
  rc(zs_sample(&a, stream()), "zs_sample");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("sample", &sample_rows, py::arg("logits"), py::arg("vocab"), py::arg("rows"), py::arg("temperature"),
        py::arg("top_k"), py::arg("top_p"), py::arg("presence"), py::arg("frequency"), py::arg("repetition"),
        py::arg("seed"), py::arg("hist"), py::arg("hist_len"), py::arg("top_n"), py::arg("out_token"),
        py::arg("out_logprob"), py::arg("out_top_ids"), py::arg("out_top_lp"));
  m.def("mhc_partial", &mhc_partial, py::arg("x"), py::arg("rows"), py::arg("hidden"), py::arg("fn"), py::arg("mode"),
        py::arg("y") = py::none(), py::arg("mix_prev") = py::none(), py::arg("ids") = py::none(),
        py::arg("embed") = py::none(), py::arg("partial"));
  m.def("mhc_slices", &zs_mhc_slices);
  m.def("set_pdl", [](bool on) { zs_set_pdl(on ? 1 : 0); });
  m.def("pdl_enabled", []() { return zs_pdl_enabled() != 0; });
  m.def("mhc_finalize", &mhc_finalize, py::arg("x"), py::arg("rows"), py::arg("hidden"), py::arg("partial"),
        py::arg("base"), py::arg("scale"), py::arg("eps"), py::arg("iters"), py::arg("mix_out"), py::arg("weight"),
        py::arg("q"), py::arg("sf"));
  m.def("rms_quant", &rms_quant);
  m.def("mla_prologue", &mla_prologue);
  m.def("mla_absorb_q", &mla_absorb_q);
  m.def("mla_attn", &mla_attn, py::arg("q_lat"), py::arg("q_pe"), py::arg("ckv_cache"), py::arg("page_table"),
        py::arg("page_size"), py::arg("slots"), py::arg("sel"), py::arg("n_sel"), py::arg("rows"), py::arg("heads"),
        py::arg("splits"), py::arg("sm_scale"), py::arg("partial"), py::arg("impl") = 1, py::arg("err") = py::none());
  m.def("mla_up", &mla_up);
  m.def("dsa_index", &dsa_index, py::arg("iq"), py::arg("iw"), py::arg("ik_cache"), py::arg("page_table"),
        py::arg("page_size"), py::arg("slots"), py::arg("ctx_len"), py::arg("rows"), py::arg("index_heads"),
        py::arg("topk"), py::arg("max_ctx"), py::arg("scores"), py::arg("sel"), py::arg("n_sel"),
        py::arg("err") = py::none());
  m.def("gather_sum", &gather_sum);

  m.def("fused_allreduce_norm", &fused_allreduce_norm, py::arg("rank"), py::arg("world"), py::arg("protocol"),
        py::arg("delta"), py::arg("n_terms"), py::arg("row_stride"), py::arg("term_stride"), py::arg("part"),
        py::arg("out"), py::arg("flags"), py::arg("epoch"), py::arg("grid_counter"), py::arg("residual"),
        py::arg("weight"), py::arg("w_offset"), py::arg("eps"), py::arg("rows"), py::arg("normed"), py::arg("q"),
        py::arg("sf"), py::arg("err"), py::arg("term_index") = py::none(), py::arg("term_scale") = py::none(),
        py::arg("timeout_ms") = 0, py::arg("pushed") = false, py::arg("mc") = std::vector<int64_t>{});
  m.def("allreduce_sum_f32", &allreduce_sum_f32, py::arg("rank"), py::arg("world"), py::arg("data"), py::arg("rows"),
        py::arg("max_rows"), py::arg("buf"), py::arg("epoch"), py::arg("grid_counter"), py::arg("err"),
        py::arg("timeout_ms") = 0, py::arg("part") = std::vector<int64_t>{}, py::arg("out") = std::vector<int64_t>{},
        py::arg("flags") = std::vector<int64_t>{});
  m.def("allreduce_argmax", &allreduce_argmax, py::arg("rank"), py::arg("world"), py::arg("rows"),
        py::arg("max_rows"), py::arg("tile_keys"), py::arg("tiles"), py::arg("id_offset"), py::arg("lines"),
        py::arg("epoch"), py::arg("grid_counter"), py::arg("out_ids"), py::arg("out_vals"), py::arg("err"),
        py::arg("timeout_ms") = 0);
  m.def("ep_call", &ep_call, py::arg("which"), py::arg("rank"), py::arg("world"), py::arg("tokens"),
        py::arg("max_tokens"), py::arg("hidden"), py::arg("top_k"), py::arg("num_experts"), py::arg("recv_cap"),
        py::arg("chunk_rows"), py::arg("topk_ids"), py::arg("topk_w"), py::arg("x"), py::arg("sym"), py::arg("offs"),
        py::arg("cnt"), py::arg("pair_slot"), py::arg("bar"), py::arg("epoch"), py::arg("group_count"),
        py::arg("group_offset"), py::arg("chunk_prefix"), py::arg("recv_rows"), py::arg("y"), py::arg("ldy"),
        py::arg("residual"), py::arg("out"), py::arg("err"), py::arg("timeout_ms") = 0);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_free", [](int64_t p) { rc(zs_symm_free(reinterpret_cast<void*>(p)), "zs_symm_free"); });
  m.def("symm_memset", [](int64_t p, int64_t bytes) {
    TORCH_CHECK(cudaMemsetAsync(reinterpret_cast<void*>(p), 0, (size_t)bytes, stream()) == cudaSuccess,
                "cudaMemsetAsync failed");
  });
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", [](int64_t p) { rc(zs_ipc_close(reinterpret_cast<void*>(p)), "zs_ipc_close"); });
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.doc() = "zstep_b200 sm_100a kernels";
  m.def("gemm_mxf8", &gemm_mxf8, py::arg("a"), py::arg("sfa"), py::arg("b"), py::arg("sfb"), py::arg("k"),
        py::arg("n_pad"), py::arg("n_valid"), py::arg("groups"), py::arg("m_rows"), py::arg("group_count"),
        py::arg("group_offset"), py::arg("chunk_prefix"), py::arg("epi_mode"), py::arg("out"), py::arg("ldo"),
        py::arg("out_sf"), py::arg("row_dst"), py::arg("row_scale"), py::arg("err"), py::arg("max_items"),
        py::arg("block_n"), py::arg("k_splits"), py::arg("split_stride"), py::arg("a_tiled"),
        py::arg("fix_splits") = 1, py::arg("ws") = py::none(), py::arg("tile_sem") = py::none(),
        py::arg("row_temp") = py::none(), py::arg("row_seed") = py::none(), py::arg("row_pos") = py::none(),
        py::arg("id_offset") = 0, py::arg("sample_any") = py::none(), py::arg("a_fp4") = 0,
        py::arg("push_part") = std::vector<int64_t>{}, py::arg("push_epoch") = py::none(), py::arg("push_rank") = 0,
        py::arg("push_mode") = 1, py::arg("last_m0") = 0, py::arg("last_mt") = 0);
  m.def("quant_mxf8", &quant_mxf8);
  m.def("spec_verify", &spec_verify);
  m.def("add_rmsnorm_quant", &add_rmsnorm_quant, py::arg("residual"), py::arg("delta"), py::arg("n_terms"),
        py::arg("d_row_stride"), py::arg("d_term_stride"), py::arg("weight"), py::arg("w_offset"), py::arg("eps"),
        py::arg("rows"), py::arg("normed"), py::arg("q"), py::arg("sf"), py::arg("term_index") = py::none(),
        py::arg("term_scale") = py::none());
  m.def("embed_rmsnorm_quant", &embed_rmsnorm_quant);
  m.def("argmax_reduce", &argmax_reduce);
  m.def("gdn_decode", [](const Tensor& proj, int64_t hk, int64_t hv, const Tensor& conv_w,
                         const Tensor& conv_state, const Tensor& ssm_state, const Tensor& a_log,
                         const Tensor& dt_bias, const Tensor& norm_w, double eps,
                         const Tensor& slots, const Tensor& positions, int64_t rows,
                         const OptT& out_bf16, const OptT& out_q, const OptT& out_sf,
                         const OptT& err) {
    gdn(false, proj, hk, hv, conv_w, conv_state, ssm_state, a_log, dt_bias, norm_w, eps, slots,
        positions, rows, out_bf16, out_q, out_sf, std::nullopt, 0, std::nullopt, std::nullopt, 0,
        err);
  });
  m.def("gdn_prefill", [](const Tensor& proj, int64_t hk, int64_t hv, const Tensor& conv_w,
                          const Tensor& conv_state, const Tensor& ssm_state, const Tensor& a_log,
                          const Tensor& dt_bias, const Tensor& norm_w, double eps,
                          const Tensor& slots, const Tensor& positions, int64_t rows,
                          const OptT& out_bf16, const OptT& out_q, const OptT& out_sf,
                          const Tensor& seq_start, int64_t num_seqs, const OptT& ckpt_rows,
                          const OptT& ckpt_slots, int64_t max_ckpt, const OptT& err, const OptT& out_slots,
                          int64_t impl, int64_t max_seq_rows) {
    gdn(true, proj, hk, hv, conv_w, conv_state, ssm_state, a_log, dt_bias, norm_w, eps, slots,
        positions, rows, out_bf16, out_q, out_sf, seq_start, num_seqs, ckpt_rows, ckpt_slots,
        max_ckpt, err, out_slots, impl, max_seq_rows);
  }, py::arg("proj"), py::arg("hk"), py::arg("hv"), py::arg("conv_w"), py::arg("conv_state"), py::arg("ssm_state"),
     py::arg("a_log"), py::arg("dt_bias"), py::arg("norm_w"), py::arg("eps"), py::arg("slots"), py::arg("positions"),
     py::arg("rows"), py::arg("out_bf16"), py::arg("out_q"), py::arg("out_sf"), py::arg("seq_start"),
     py::arg("num_seqs"), py::arg("ckpt_rows"), py::arg("ckpt_slots"), py::arg("max_ckpt"), py::arg("err"),
     py::arg("out_slots") = py::none(), py::arg("impl") = 0, py::arg("max_seq_rows") = 0);
  m.def("attn_prologue", &attn_prologue);
  m.def("attn_decode", &attn_decode, py::arg("q_out"), py::arg("gate_out"), py::arg("num_q_heads"),
        py::arg("num_kv_heads"), py::arg("k_cache"), py::arg("v_cache"), py::arg("page_size"), py::arg("page_table"),
        py::arg("slots"), py::arg("seq_lens"), py::arg("rows"), py::arg("partial"), py::arg("num_splits"),
        py::arg("sm_scale"), py::arg("out_bf16"), py::arg("out_q"), py::arg("out_sf"), py::arg("impl") = 0,
        py::arg("err") = py::none(), py::arg("seq_start") = py::none(), py::arg("num_seqs") = 0);
  m.def("moe_route", &moe_route, py::arg("logits"), py::arg("rows"), py::arg("num_experts"), py::arg("top_k"),
        py::arg("norm_topk"), py::arg("scoring"), py::arg("bias"), py::arg("n_group"), py::arg("topk_group"),
        py::arg("routed_scale"), py::arg("shared_gate_col"), py::arg("expert_begin"), py::arg("expert_end"),
        py::arg("has_shared"), py::arg("topk_ids"), py::arg("topk_w"), py::arg("group_count"),
        py::arg("group_offset"), py::arg("chunk_prefix"), py::arg("pair_slot"), py::arg("row_dst"),
        py::arg("row_scale"), py::arg("x_q"), py::arg("x_sf"), py::arg("xg_q"), py::arg("xg_sf"), py::arg("err"),
        py::arg("ld_logits"), py::arg("logit_splits"), py::arg("logit_split_stride"), py::arg("chunk_rows"),
        py::arg("pair_src") = py::none(), py::arg("pair_w") = py::none());
}
