"""DeepSeek-style MLA + DSA + mHC MoE runner on B200 kernels.

Flat model code over preallocated buffers, like the Qwen3.5 runner: weights are packed
once into the MXFP8 GEMM layout, every step is a fixed launch sequence that a CUDA graph
captures per decode bucket.  Per layer (decode or varlen prefill), with the residual kept
as n = 4 fp32 mHC streams X:

  mHC site  : partial mixing sums (fused with the previous site's stream update
              X <- res @ X + post * y) -> Sinkhorn/sigmoid mixing + collapse pre @ X +
              RMSNorm + MXFP8 quant
  attention : [q_a | kv_a | index k | index w] GEMM -> q_a RMSNorm + quant ->
              [q_b (local heads) | index q] GEMM -> prologue (latent + index caches,
              RoPE) -> q_nope absorption into the latent space -> indexer scores +
              deterministic top-k -> split-KV latent attention -> merge + W_UV
              up-projection + MXFP8 -> o_proj GEMM (f32) -> sum over ranks
  FFN       : dense (layer < first_k_dense_replace): gate/up GEMM with SiLU*up + MXFP8
              epilogue -> down GEMM;  MoE: router GEMM -> sigmoid grouped top-k with
              correction bias + grouped scatter -> grouped gate/up (SiLU) -> grouped
              down -> weighted gather of each token's expert rows -> sum over ranks
  head      : final collapse site (sigmoid pre only) -> lm_head GEMM + fused argmax

Parallelism: attention heads (and the dense FFN's intermediate) are split over the tp
ranks; experts are placed by expert parallelism over the same ranks (expert e lives on
rank e // (E / tp)); every rank holds the replicated residual streams, so dispatch is
local and the combine is the same sum over ranks as the attention output.

The reference serves this family through vLLM with its own kernels swapped in
(worker/zstep_worker/models/deepseek_v41.py:408 DeepSeekV41StepRunner, :1043 TP
collectives, :1444 decode graphs); zstep_b200/models/deepseek_ref.py is the fp32 oracle.
"""

from __future__ import annotations

import math

import torch

from ..config import DeepSeekConfig
from ..ops import _ext
from ..ops import mx
from ..utils.env import runtime_config
from .deepseek_weights import DeepSeekRandomWeights
from .qwen35 import (DECODE_BUCKETS, EPI_BF16, EPI_F32, EPI_SILU, PackedLinear, Qwen35Runner, _pad128,
                     interleave_gate_up, pack_linear)


def pack_linear_fp4(w: torch.Tensor, C) -> PackedLinear:
    """Expert weights [G, N, K] -> MXFP4: packed e2m1 pre-tiled into 8 KiB chunks per
    (128-row tile, 128-K tile) plus the usual e8m0 scale atoms.  The GEMM widens each
    chunk to e4m3 in shared memory, so HBM carries half the bytes of MXFP8."""
    if w.dim() == 2:
        w = w.unsqueeze(0)
    g, n, k = w.shape
    npad = _pad128(n)
    flat = torch.zeros(g, npad, k, dtype=torch.bfloat16, device=w.device)
    flat[:, :n] = w
    flat = flat.reshape(g * npad, k)
    packed, code = mx.quantize_fp4(flat)
    return PackedLinear(q=mx.tile_weight_fp4(packed), sf=mx.atoms_from_codes(code), n=n, n_pad=npad, k=k, groups=g,
                        fp4=True)


class DeepSeekRunner:
    """Single-process DeepSeek-style model runner for one GPU (tp_rank of tp_size)."""

    # Shared machinery of the Qwen runner (staging, graphs, GEMM dispatch, lm_head).
    stage = Qwen35Runner.stage
    staged_bytes = Qwen35Runner.staged_bytes
    set_pages = Qwen35Runner.set_pages
    bucket_for = Qwen35Runner.bucket_for
    capture_decode_graph = Qwen35Runner.capture_decode_graph
    decode_step = Qwen35Runner.decode_step
    check_error = Qwen35Runner.check_error
    _gemm = Qwen35Runner._gemm
    _fix_splits = Qwen35Runner._fix_splits
    _dense_bn = Qwen35Runner._dense_bn
    _gather_sf = Qwen35Runner._gather_sf
    _lm_head_argmax = Qwen35Runner._lm_head_argmax
    lm_head_rows = Qwen35Runner.lm_head_rows
    set_sampling = Qwen35Runner.set_sampling
    clear_sampling = Qwen35Runner.clear_sampling

    def __init__(self, cfg: DeepSeekConfig, *, device="cuda", weights=None, max_seqs: int = 64,
                 max_prefill_tokens: int = 2048, num_pages: int = 4096, page_size: int = 16,
                 max_model_len: int = 4096, tp_rank: int = 0, tp_size: int = 1, collectives=None, seed: int = 0,
                 num_ckpt_slots: int = 0, num_spec_tokens: int = 0):
        self.cfg = c = cfg
        assert c.kv_lora_rank == 512 and c.qk_rope_head_dim == 64 and c.qk_nope_head_dim == 128 \
            and c.v_head_dim == 128 and c.index_head_dim == 128 and c.hc_mult == 4, \
            "the MLA/DSA/mHC kernels serve kv_lora 512, rope 64, nope/v 128, index dim 128, 4 streams"
        assert c.num_attention_heads % tp_size == 0 and c.num_attention_heads // tp_size <= 16
        assert c.n_routed_experts % tp_size == 0 and c.intermediate_size % (64 * tp_size) == 0
        self.dev = torch.device(device)
        self.C = _ext.load()
        self.tp_rank, self.tp = tp_rank, tp_size
        self.coll = collectives
        self.page_size = page_size
        self.max_seqs = max_seqs
        self.max_model_len = max_model_len
        self.max_pages = (max_model_len + page_size - 1) // page_size
        self.num_pages = num_pages
        self.max_prefill_tokens = max_prefill_tokens
        self.eps = c.rms_norm_eps
        self.hl = c.num_attention_heads // tp_size
        self.e_local = c.n_routed_experts // tp_size
        self.e_begin = tp_rank * self.e_local
        self.groups = self.e_local + 1  # + shared expert
        self.top_k = c.num_experts_per_tok
        self.scoring = {"sigmoid": 1, "sqrtsoftplus": 2}[c.scoring_func]  # route kernel's scoring mode
        self.mla_impl = runtime_config().mla_impl  # latent attention: 1 SIMT, 2 tensor cores
        self.k1 = self.top_k + 1
        self.num_slots = max_seqs + 1
        self.dummy_slot = max_seqs
        self.num_spec = num_spec_tokens
        self.spec = None
        self.spec_slot_base = 0  # no recurrent state: verify needs no spare slots
        src = weights or DeepSeekRandomWeights(cfg, seed=seed)
        self._load_weights(src)
        self._alloc_state()
        self._alloc_buffers()
        if self.num_spec:
            from .deepseek_spark import DSparkDrafter

            self.spec = DSparkDrafter(self, src)
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}

    # ------------------------------------------------------------------ weights
    def _load_weights(self, src) -> None:
        c, C, dev, r, tp = self.cfg, self.C, self.dev, self.tp_rank, self.tp
        get = lambda n: src.get(n, dev)  # noqa: E731
        f32 = lambda n: get(n).float().contiguous()  # noqa: E731
        bf = lambda n: get(n).to(torch.bfloat16).contiguous()  # noqa: E731
        self.embed = bf("embed")
        self.final_norm = bf("final_norm")
        vs = c.vocab_size // tp
        self.vocab_local = vs
        self.lm_head = pack_linear(get("lm_head")[r * vs:(r + 1) * vs], C)
        self.hc_head = (f32("hc_head.fn"), f32("hc_head.base"), f32("hc_head.scale"))
        self.layers = []
        for i in range(c.num_hidden_layers):
            p = f"layers.{i}."
            L = {"hc_attn": (f32(p + "hc_attn.fn"), f32(p + "hc_attn.base"), f32(p + "hc_attn.scale")),
                 "hc_ffn": (f32(p + "hc_ffn.fn"), f32(p + "hc_ffn.base"), f32(p + "hc_ffn.scale"))}
            L.update(self._load_layer(src, p, c.is_dense(i)))
            self.layers.append(L)
            torch.cuda.synchronize(dev)

    def _load_layer(self, src, p: str, dense: bool) -> dict:
        """MLA attention (this rank's heads), indexer and FFN (dense slice or local experts)
        of the layer with name prefix `p`."""
        c, C, dev, r, tp = self.cfg, self.C, self.dev, self.tp_rank, self.tp
        get = lambda n: src.get(n, dev)  # noqa: E731
        bf = lambda n: get(n).to(torch.bfloat16).contiguous()  # noqa: E731
        hl = self.hl
        nope, vd, qk = c.qk_nope_head_dim, c.v_head_dim, c.qk_head_dim
        L = {"attn_norm": bf(p + "attn_norm"), "ffn_norm": bf(p + "ffn_norm")}
        L["proj_a"] = pack_linear(torch.cat([get(p + "mla.q_a"), get(p + "mla.kv_a"), get(p + "idx.wk"),
                                             get(p + "idx.w")], 0), C)
        q_b = get(p + "mla.q_b")[r * hl * qk:(r + 1) * hl * qk]
        L["proj_q"] = pack_linear(torch.cat([q_b, get(p + "idx.wq")], 0), C)
        L["q_a_norm"], L["kv_a_norm"], L["idx_k_norm"] = bf(p + "mla.q_a_norm"), bf(p + "mla.kv_a_norm"), \
            bf(p + "idx.k_norm")
        kv_b = get(p + "mla.kv_b").reshape(c.num_attention_heads, nope + vd, c.kv_lora_rank)[r * hl:(r + 1) * hl]
        L["w_uk"] = kv_b[:, :nope].to(torch.bfloat16).contiguous()                   # [hl, nope, kl]
        L["w_uv_t"] = kv_b[:, nope:].transpose(1, 2).to(torch.bfloat16).contiguous()  # [hl, kl, v]
        L["o_proj"] = pack_linear(get(p + "mla.o_proj")[:, r * hl * vd:(r + 1) * hl * vd].contiguous(), C)
        if dense:
            Fl = c.intermediate_size // tp
            sl = slice(r * Fl, (r + 1) * Fl)
            L["dense"] = True
            L["gate_up"] = pack_linear(interleave_gate_up(get(p + "mlp.gate")[sl][None],
                                                          get(p + "mlp.up")[sl][None]), C)
            L["down"] = pack_linear(get(p + "mlp.down")[:, sl].contiguous(), C)
        else:
            L["dense"] = False
            L.update(self._load_moe(src, p))
        return L

    def _load_moe(self, src, p: str) -> dict:
        c, C, dev = self.cfg, self.C, self.dev
        H = c.hidden_size
        eb, ee = self.e_begin, self.e_begin + self.e_local
        ex = lambda n, e: src.get_expert(p + "moe." + n, e, dev)  # noqa: E731
        gate = torch.stack([ex("gate", e) for e in range(eb, ee)] + [src.get(p + "moe.shared.gate", dev)])
        up = torch.stack([ex("up", e) for e in range(eb, ee)] + [src.get(p + "moe.shared.up", dev)])
        packer = pack_linear_fp4 if c.expert_format == "mxfp4" else pack_linear
        out = {"router": pack_linear(src.get(p + "moe.router", dev), C),
               "bias": src.get(p + "moe.bias", dev).float().contiguous(),
               "gate_up": packer(interleave_gate_up(gate, up), C)}
        del gate, up
        sd = src.get(p + "moe.shared.down", dev)
        if self.tp > 1:
            # Tensor-parallel shared expert: this rank's intermediate columns only (its
            # gate/up tiles are selected in the grouped GEMM, the other columns of the down
            # projection are zero), summed over ranks by the sublayer all-reduce.
            c0, c1 = self.shared_cols()
            mask = torch.zeros(1, sd.shape[1], dtype=sd.dtype, device=dev)
            mask[:, c0:c1] = 1
            sd = sd * mask
        down = torch.stack([ex("down", e) for e in range(eb, ee)] + [sd])
        out["down"] = packer(down, C)
        return out

    def shared_cols(self) -> tuple[int, int]:
        """This rank's intermediate columns of the shared expert."""
        n = self.cfg.moe_intermediate_size * self.cfg.n_shared_experts // self.tp
        return self.tp_rank * n, (self.tp_rank + 1) * n

    # ------------------------------------------------------------------ state
    def _alloc_state(self) -> None:
        c, dev = self.cfg, self.dev
        L = c.num_hidden_layers
        self.ckv_cache = torch.zeros(L, self.num_pages, self.page_size, c.kv_cache_dim, dtype=torch.bfloat16,
                                     device=dev)
        self.ik_cache = torch.zeros(L, self.num_pages, self.page_size, c.index_head_dim, dtype=torch.bfloat16,
                                    device=dev)
        self.page_table = torch.zeros(self.num_slots, self.max_pages, dtype=torch.int32, device=dev)

    def _alloc_buffers(self) -> None:
        c, dev = self.cfg, self.dev
        H, hl = c.hidden_size, self.hl
        R = max(self.max_seqs, self.max_prefill_tokens)
        Rp = _pad128(R)
        self.R = R
        if self.tp > 1 and hasattr(self.coll, "reserve"):
            self.coll.reserve(R, H)  # symmetric buffers of the NVLink sublayer sums
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        u8 = dict(dtype=torch.uint8, device=dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.num_sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.use_fix_splits = False
        self.wa = self.layers[0]["proj_a"].n
        self.wq = self.layers[0]["proj_q"].n
        self.off_kva = c.q_lora_rank
        self.off_ik = self.off_kva + c.kv_cache_dim
        self.off_iw = self.off_ik + c.index_head_dim
        self.off_iq = hl * c.qk_head_dim
        b = {}
        b["X"] = torch.zeros(R, 4, H, **f32)
        self.hc_slices = self.C.mhc_slices(H)
        b["hcp"] = torch.zeros(R * self.hc_slices * (c.hc_mix_dim + 1), **f32)
        b["mix"] = torch.zeros(R, 4 + 16, **f32)
        b["y"] = torch.zeros(R, H, **f32)
        b["xq"] = torch.zeros(Rp, H, **u8)
        b["xsf"] = torch.zeros(mx.atoms_bytes(Rp, H), **u8)
        b["proj_a"] = torch.zeros(R, self.wa, **bf)
        b["qa_q"] = torch.zeros(Rp, c.q_lora_rank, **u8)
        b["qa_sf"] = torch.zeros(mx.atoms_bytes(Rp, c.q_lora_rank), **u8)
        b["qi"] = torch.zeros(R, self.wq, **bf)
        b["q_pe"] = torch.zeros(R, hl, c.qk_rope_head_dim, **bf)
        b["iq"] = torch.zeros(R, c.index_n_heads, c.index_head_dim, **bf)
        b["iw"] = torch.zeros(R, c.index_n_heads, **f32)
        b["q_lat"] = torch.zeros(R, hl, c.kv_lora_rank, **bf)
        b["scores"] = torch.zeros(R, self.max_model_len, **f32)
        b["sel"] = torch.zeros(R, c.index_topk, **i32)
        b["n_sel"] = torch.zeros(R, **i32)
        self.max_splits = 32
        b["attn_part"] = torch.zeros(max(R, self.max_seqs * self.max_splits) * hl * (c.kv_lora_rank + 4), **f32)
        b["o_q"] = torch.zeros(Rp, hl * c.v_head_dim, **u8)
        b["o_sf"] = torch.zeros(mx.atoms_bytes(Rp, hl * c.v_head_dim), **u8)
        dense = [L for L in self.layers if L["dense"]]
        if dense:
            Fl = c.intermediate_size // self.tp
            b["act_d"] = torch.zeros(Rp, Fl, **u8)
            b["act_d_sf"] = torch.zeros(mx.atoms_bytes(Rp, Fl), **u8)
        moe = [L for L in self.layers if not L["dense"]]
        if moe:
            nr = moe[0]["router"].n_pad
            G = self.groups
            b["logits"] = torch.zeros(R * nr, **f32)
            b["topk_ids"] = torch.zeros(R, self.top_k, **i32)
            b["topk_w"] = torch.zeros(R, self.top_k, **f32)
            b["gcount"] = torch.zeros(G, **i32)
            b["goff"] = torch.zeros(G, **i32)
            b["gpre"] = torch.zeros(G + 1, **i32)
            b["pair_slot"] = torch.zeros(R, self.k1, **i32)
            mg = _pad128(R * self.k1) + 128 * G
            b["row_dst"] = torch.zeros(mg, **i32)
            b["row_scale"] = torch.zeros(mg, **f32)
            b["xg"] = torch.zeros(mg, H, **u8)
            b["xg_sf"] = torch.zeros(mx.atoms_bytes(mg, H), **u8)
            I = c.moe_intermediate_size
            b["act"] = torch.zeros(mg, I, **u8)
            b["act_sf"] = torch.zeros(mx.atoms_bytes(mg, I), **u8)
            b["moe_y"] = torch.zeros(mg, H, **bf)
            b["pair_src"] = torch.zeros(R, self.k1, **i32)
            b["pair_w"] = torch.zeros(R, self.k1, **f32)
        vt = self.lm_head.n_pad // 128
        self.vocab_tiles = vt
        self.lm_rows = self.max_seqs * (1 + self.num_spec)  # verify steps score every verify row
        b["samp_temp"] = torch.zeros(R, **f32)
        b["samp_seed"] = torch.zeros(R, dtype=torch.int64, device=dev)
        b["samp_pos"] = torch.zeros(R, **i32)
        b["samp_any"] = torch.zeros(1, **f32)
        b["gemm_ws"] = torch.zeros(1, **f32)
        b["gemm_sem"] = torch.zeros(1, **i32)
        b["lm_keys"] = torch.zeros(self.lm_rows, vt, dtype=torch.int64, device=dev)
        b["out_ids"] = torch.zeros(self.lm_rows, **i32)
        b["out_vals"] = torch.zeros(self.lm_rows, **f32)
        b["out_keys"] = torch.zeros(self.lm_rows, dtype=torch.int64, device=dev)
        b["err"] = torch.zeros(1, **i32)
        b["xq_last"] = torch.zeros(_pad128(self.lm_rows), H, **u8)
        b["inputs"] = torch.zeros(4, R, **i32)
        b["in_ids"], b["in_pos"], b["in_slot"], b["in_len"] = b["inputs"].unbind(0)
        self.host_inputs = torch.zeros(4, R, dtype=torch.int32, pin_memory=True)
        b["seq_start"] = torch.zeros(self.max_seqs + 1, **i32)
        self.buf = b

    # ------------------------------------------------------------------ helpers
    def _moe_bn(self, rows: int) -> int:
        return 32 if rows * self.top_k <= 32 * self.cfg.n_routed_experts else 128

    def _reduce(self, rows: int) -> None:
        if self.tp > 1:
            self.coll.allreduce_sum(self.buf["y"][:rows])

    def _attn_splits(self, rows: int) -> int:
        return int(max(1, min(self.max_splits, math.ceil(2 * self.num_sms / max(rows, 1)))))

    def pad_decode_inputs(self, n: int, bucket: int) -> None:
        if bucket > n:
            b = self.buf
            b["in_ids"][n:bucket] = 0
            b["in_pos"][n:bucket] = 0
            b["in_slot"][n:bucket] = self.dummy_slot
            b["in_len"][n:bucket] = 1

    # ------------------------------------------------------------------ sublayers
    def _site(self, rows: int, hc, norm_w, mix_out=True) -> None:
        """Finalize an mHC site: mixing coefficients, collapse, RMSNorm, MXFP8 -> xq."""
        b, c = self.buf, self.cfg
        fn, base, scale = hc
        self.C.mhc_finalize(b["X"], rows, c.hidden_size, b["hcp"], base, scale, self.eps, c.hc_sinkhorn_iters,
                            b["mix"] if mix_out else None, norm_w, b["xq"], b["xsf"])

    def _advance(self, rows: int, next_fn) -> None:
        """Apply the finished sublayer's stream update and start the next site's sums."""
        b, c = self.buf, self.cfg
        self.C.mhc_partial(b["X"], rows, c.hidden_size, next_fn, 1, y=b["y"], mix_prev=b["mix"], partial=b["hcp"])

    def _attention(self, li: int, L, rows: int, decode: bool, caches=None) -> None:
        """MLA + DSA sublayer -> buf["y"] (fp32, reduced over ranks).  `caches` (latent,
        index) overrides layer li's paged caches (the DSpark head keeps its own)."""
        c, C, b = self.cfg, self.C, self.buf
        hl = self.hl
        ckv, ik = caches if caches is not None else (self.ckv_cache[li], self.ik_cache[li])
        pos, slot, lens = b["in_pos"][:rows], b["in_slot"][:rows], b["in_len"][:rows]
        proj_a = b["proj_a"][:rows]
        self._gemm(L["proj_a"], b["xq"], b["xsf"], rows, proj_a, self.wa)
        C.rms_quant(proj_a, c.q_lora_rank, L["q_a_norm"], self.eps, rows, b["qa_q"], b["qa_sf"])
        qi = b["qi"][:rows]
        self._gemm(L["proj_q"], b["qa_q"], b["qa_sf"], rows, qi, self.wq)
        C.mla_prologue(proj_a, self.off_kva, self.off_ik, self.off_iw, qi, self.off_iq, rows, hl,
                       c.qk_nope_head_dim, c.qk_rope_head_dim, c.kv_lora_rank, c.index_n_heads, c.index_head_dim,
                       L["kv_a_norm"], L["idx_k_norm"], self.eps, c.rope_theta, slot, pos, self.page_table,
                       self.page_size, ckv, ik, b["q_pe"], b["iq"], b["iw"])
        C.mla_absorb_q(qi, c.qk_head_dim, c.qk_nope_head_dim, L["w_uk"], hl, rows, b["q_lat"])
        C.dsa_index(b["iq"], b["iw"], ik, self.page_table, self.page_size, slot, lens, rows,
                    c.index_n_heads, c.index_topk, self.max_model_len, b["scores"], b["sel"], b["n_sel"], b["err"])
        splits = self._attn_splits(rows) if decode else 1
        C.mla_attn(b["q_lat"], b["q_pe"], ckv, self.page_table, self.page_size, slot, b["sel"],
                   b["n_sel"], rows, hl, splits, c.qk_head_dim ** -0.5, b["attn_part"], impl=self.mla_impl,
                   err=b["err"])
        C.mla_up(b["attn_part"], rows, hl, splits, L["w_uv_t"], b["o_q"], b["o_sf"])
        self._gemm(L["o_proj"], b["o_q"], b["o_sf"], rows, b["y"], c.hidden_size, EPI_F32)
        self._reduce(rows)

    def _ffn(self, L, rows: int) -> None:
        c, C, b = self.cfg, self.C, self.buf
        H = c.hidden_size
        if L["dense"]:
            Fl = c.intermediate_size // self.tp
            self._gemm(L["gate_up"], b["xq"], b["xsf"], rows, b["act_d"], Fl, EPI_SILU, out_sf=b["act_d_sf"])
            self._gemm(L["down"], b["act_d"], b["act_d_sf"], rows, b["y"], H, EPI_F32)
        else:
            E = c.n_routed_experts
            nr = L["router"].n_pad
            self._gemm(L["router"], b["xq"], b["xsf"], rows, b["logits"], nr, EPI_F32)
            C.moe_route(b["logits"], rows, E, self.top_k, True, self.scoring, L["bias"], c.n_group, c.topk_group,
                        c.routed_scaling_factor, -1, self.e_begin, self.e_begin + self.e_local, True, b["topk_ids"],
                        b["topk_w"], b["gcount"], b["goff"], b["gpre"], b["pair_slot"], b["row_dst"], b["row_scale"],
                        b["xq"], b["xsf"], b["xg"], b["xg_sf"], b["err"], nr, 1, rows * nr, self._moe_bn(rows),
                        b["pair_src"], b["pair_w"])
            I = c.moe_intermediate_size
            c0, c1 = self.shared_cols()
            self._gemm(L["gate_up"], b["xg"], b["xg_sf"], rows, b["act"], I, EPI_SILU, grouped=True,
                       out_sf=b["act_sf"], last_tiles=(c0 // 64, (c1 - c0) // 64) if self.tp > 1 else None)
            self._gemm(L["down"], b["act"], b["act_sf"], rows, b["moe_y"], H, EPI_BF16, grouped=True)
            C.gather_sum(b["moe_y"], b["pair_src"], b["pair_w"], rows, b["y"])
        self._reduce(rows)

    def _layers(self, rows: int, decode: bool) -> None:
        c, C, b = self.cfg, self.C, self.buf
        H = c.hidden_size
        C.mhc_partial(b["X"], rows, H, self.layers[0]["hc_attn"][0], 2, ids=b["in_ids"][:rows], embed=self.embed,
                      partial=b["hcp"])
        aux = {li: j for j, li in enumerate(self.spec.aux)} if self.spec is not None and not decode else {}
        for li, L in enumerate(self.layers):
            self._site(rows, L["hc_attn"], L["attn_norm"])
            self._attention(li, L, rows, decode)
            self._advance(rows, L["hc_ffn"][0])
            self._site(rows, L["hc_ffn"], L["ffn_norm"])
            if li in aux:
                self.spec.capture(aux[li], rows)
            self._ffn(L, rows)
            nxt = self.layers[li + 1]["hc_attn"][0] if li + 1 < len(self.layers) else self.hc_head[0]
            self._advance(rows, nxt)
        self._site(rows, self.hc_head, self.final_norm, mix_out=False)

    def paged_caches(self) -> list[torch.Tensor]:
        """Device tensors indexed [layer, page, ...]: what a host DRAM tier slot holds."""
        return [self.ckv_cache, self.ik_cache]

    def copy_recurrent_state(self, src_slot: int, dst_slot: int) -> None:
        """No recurrent state: every cached quantity lives in the paged latent / index caches."""

    def checkpoint_args(self, ckpt_rows, ckpt_slots, query_start):
        return None

    # ------------------------------------------------------------------ public step API
    def decode_forward(self, rows: int) -> torch.Tensor:
        self._layers(rows, decode=True)
        self._lm_head_argmax(rows)
        return self.buf["out_ids"][:rows]

    def prefill_forward(self, rows: int, num_seqs: int, ckpt=None) -> torch.Tensor:
        b = self.buf
        self._layers(rows, decode=False)
        last = b["seq_start"][1:num_seqs + 1].long() - 1
        return self.lm_head_rows(last, b["xq_last"])


__all__ = ["DeepSeekRunner", "pack_linear_fp4", "DECODE_BUCKETS"]
