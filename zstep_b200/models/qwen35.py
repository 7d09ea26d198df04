"""Qwen3.5 hybrid (GatedDeltaNet + gated GQA + MoE) runner on B200 kernels.

Flat model code: weights are packed once into the MXFP8 GEMM layout (e4m3 rows padded
to 128 + e8m0 scale atoms), every intermediate lives in a preallocated buffer, and a
decode step is a fixed sequence of sm_100a kernel launches that is captured into one
CUDA graph per batch bucket.  Per layer (decode or varlen prefill):

  GDN layer : in_proj GEMM -> fused conv/delta-rule/gated-norm kernel (MXFP8 out)
              -> out_proj GEMM -> residual add + RMSNorm + MXFP8 quant
  GQA layer : qkv GEMM -> q/k norm + partial RoPE + paged KV write -> split-KV gated
              attention (MXFP8 out) -> o_proj GEMM -> residual add + RMSNorm + quant
  MoE       : router GEMM (f32 logits) -> top-k + grouped scatter -> grouped gate/up
              GEMM with SiLU*up + MXFP8 epilogue -> grouped down GEMM scattering
              weight-scaled rows -> combine of the 9 pair rows + residual + RMSNorm
  head      : lm_head GEMM with a fused per-tile argmax -> row argmax

The shared expert is expert group E of the grouped GEMMs (every token visits it with
weight sigmoid(shared gate)), so routed and shared experts stream in one launch.

Tensor parallel (tp > 1): attention/GDN heads and the dense projections are sharded
(column-parallel in, row-parallel out), experts are sharded by expert id over the
replicated activations, and the row-parallel partial sums are reduced by the
collective layer's fused all-reduce + residual + RMSNorm (parallel/collectives.py).

Reference parity: worker/zstep_worker/models/qwen35_moe.py (runner, 1021-1168 decode
forward, 1236 varlen prefill, 1404 graph capture, 484-524 state allocation).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..config import Qwen35Config
from ..ops import _ext
from ..utils.env import runtime_config
from ..ops import mx
from .weights import RandomWeights

EPI_BF16, EPI_F32, EPI_SILU, EPI_SCATTER, EPI_ARGMAX, EPI_PUSH = 0, 1, 2, 3, 4, 5

DECODE_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512)


def _pad128(n: int) -> int:
    return (n + 127) // 128 * 128


@dataclass
class PackedLinear:
    """MXFP8 weight in the GEMM layout: q e4m3 pre-tiled into contiguous 128x128-byte
    blocks ([groups*n_pad/128][k/128][128][128]), sf scale atoms."""

    q: torch.Tensor
    sf: torch.Tensor
    n: int
    n_pad: int
    k: int
    groups: int = 1
    fp4: bool = False   # q holds packed e2m1 tiles ([..][k/128][128 rows][64 B]); widened in the GEMM


def pack_linear(w: torch.Tensor, C) -> PackedLinear:
    """w [N, K] or [G, N, K] (bf16, on the GPU) -> PackedLinear (quantized by the GPU kernel)."""
    if w.dim() == 2:
        w = w.unsqueeze(0)
    g, n, k = w.shape
    npad = _pad128(n)
    if npad != n:
        wp = torch.zeros(g, npad, k, dtype=torch.bfloat16, device=w.device)
        wp[:, :n] = w
    else:
        wp = w.to(torch.bfloat16).contiguous()
    flat = wp.reshape(g * npad, k)
    q = torch.empty(g * npad, k, dtype=torch.uint8, device=w.device)
    sf = torch.empty(mx.atoms_bytes(g * npad, k), dtype=torch.uint8, device=w.device)
    C.quant_mxf8(flat, q, sf)
    return PackedLinear(q=mx.tile_weight(q), sf=sf, n=n, n_pad=npad, k=k, groups=g)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[G, I, K] gate and up -> [G, 2I, K] with 128-row tiles [gate 64 rows ; up 64 rows]."""
    g, i, k = gate.shape
    assert i % 64 == 0
    return torch.stack([gate.reshape(g, i // 64, 64, k), up.reshape(g, i // 64, 64, k)], dim=2).reshape(g, 2 * i, k)


class Qwen35Runner:
    """Single-process model runner for one GPU (tp_rank of tp_size)."""

    def __init__(self, cfg: Qwen35Config, *, device="cuda", weights=None, max_seqs: int = 256,
                 max_prefill_tokens: int = 4096, num_pages: int = 4096, page_size: int = 16,
                 max_model_len: int = 4096, num_ckpt_slots: int = 0, tp_rank: int = 0, tp_size: int = 1,
                 collectives=None, seed: int = 0, num_spec_tokens: int = 0):
        self.cfg = cfg
        self.dev = torch.device(device)
        self.C = _ext.load()
        self.tp_rank, self.tp = tp_rank, tp_size
        self.coll = collectives
        self.page_size = page_size
        self.max_seqs = max_seqs
        self.max_pages = (max_model_len + page_size - 1) // page_size
        self.num_pages = num_pages
        self.max_prefill_tokens = max_prefill_tokens
        self.eps = cfg.rms_norm_eps
        assert cfg.linear_key_head_dim == 128 and cfg.linear_value_head_dim == 128, "GDN kernels need 128-dim heads"
        assert cfg.head_dim == 256, "attention kernels need head_dim 256"
        assert cfg.hidden_size % 2048 == 0
        # Local (per-rank) head counts.
        self.hk = cfg.linear_num_key_heads // tp_size
        self.hv = cfg.linear_num_value_heads // tp_size
        self.hq = cfg.num_attention_heads // tp_size
        self.hkv = max(1, cfg.num_key_value_heads // tp_size)
        self.kv_rep = tp_size // cfg.num_key_value_heads if tp_size > cfg.num_key_value_heads else 1
        E = cfg.num_experts
        assert E % tp_size == 0
        self.e_local = E // tp_size
        self.e_begin = tp_rank * self.e_local
        # Shared expert: replicated gate/up, down output-sharded by rank (only rank r writes
        # its 1/tp slice of the hidden dim; the all-reduce then sums the slices).
        assert cfg.shared_expert_intermediate_size == cfg.moe_intermediate_size
        assert cfg.shared_expert_intermediate_size % (64 * tp_size) == 0, "shared expert tiles must split over ranks"
        self.groups = self.e_local + 1
        self.top_k = cfg.num_experts_per_tok
        self.k1 = self.top_k + 1
        # Speculative decoding keeps one extra recurrent-state slot per request slot: a
        # verify step writes its final state there and leaves the pre-step state intact.
        self.num_spec = num_spec_tokens if cfg.mtp_num_hidden_layers > 0 else 0
        self.spec_slot_base = max_seqs + num_ckpt_slots
        self.num_slots = self.spec_slot_base + (max_seqs if self.num_spec else 0) + 1  # last = padding dummy
        self.dummy_slot = self.num_slots - 1
        src = weights or RandomWeights(cfg, seed=seed)
        self._load_weights(src)
        self._alloc_state()
        self._alloc_buffers()
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.spec = None
        if self.num_spec:
            from .qwen35_spec import SpecDecoder

            self.spec = SpecDecoder(self, src)

    # ------------------------------------------------------------------ weights
    def _shard_rows(self, t: torch.Tensor, parts: list[int]) -> torch.Tensor:
        """Column-parallel shard of a fused projection made of consecutive row blocks."""
        out, o = [], 0
        for p in parts:
            blk = t[o:o + p]
            n = p // self.tp
            out.append(blk[self.tp_rank * n:(self.tp_rank + 1) * n])
            o += p
        return torch.cat(out, 0)

    def _load_weights(self, src) -> None:
        cfg, C, dev, tp, r = self.cfg, self.C, self.dev, self.tp, self.tp_rank
        get = lambda n: src.get(n, dev)  # noqa: E731
        H = cfg.hidden_size
        self.embed = get("embed").to(torch.bfloat16).contiguous()
        self.final_norm = get("final_norm").to(torch.bfloat16).contiguous()
        lm = get("lm_head")
        vs = cfg.vocab_size // tp
        self.vocab_local = vs
        self.lm_head = pack_linear(lm[r * vs:(r + 1) * vs], C)
        del lm
        self.layers = []
        Hk, Hv, dk, dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, 128, 128
        Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        for i in range(cfg.num_hidden_layers):
            p = f"layers.{i}."
            L = {"type": cfg.layer_types[i]}
            L["input_norm"] = get(p + "input_norm").to(torch.bfloat16)
            L["post_norm"] = get(p + "post_norm").to(torch.bfloat16)
            if L["type"] == "linear_attention":
                w = get(p + "gdn.in_proj")
                w = self._shard_rows(w, [Hk * dk, Hk * dk, Hv * dv, Hv * dv, Hv, Hv])
                L["in_proj"] = pack_linear(w, C)
                cw = get(p + "gdn.conv_w")
                L["conv_w"] = self._shard_rows(cw, [Hk * dk, Hk * dk, Hv * dv]).to(torch.bfloat16).contiguous()
                L["a_log"] = get(p + "gdn.a_log").float()[r * self.hv:(r + 1) * self.hv].contiguous()
                L["dt_bias"] = get(p + "gdn.dt_bias").float()[r * self.hv:(r + 1) * self.hv].contiguous()
                L["gnorm"] = get(p + "gdn.norm").to(torch.bfloat16).contiguous()
                wo = get(p + "gdn.out_proj")
                L["out_proj"] = pack_linear(wo[:, r * self.hv * dv:(r + 1) * self.hv * dv].contiguous(), C)
            else:
                L.update(self._load_attn(get, p))
            L.update(self._load_moe(get, p))
            self.layers.append(L)
            torch.cuda.synchronize(dev)
        self.gdn_index = {i: j for j, i in enumerate(cfg.gdn_layers)}
        self.attn_index = {i: j for j, i in enumerate(cfg.attn_layers)}

    def _load_attn(self, get, p: str) -> dict:
        cfg, C, r = self.cfg, self.C, self.tp_rank
        Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        w = get(p + "attn.qkv")
        q = w[:Hq * 2 * D][r * self.hq * 2 * D:(r + 1) * self.hq * 2 * D]
        kvh = (r * Hkv) // self.tp if self.tp > Hkv else r * self.hkv
        k = w[Hq * 2 * D:Hq * 2 * D + Hkv * D][kvh * D:(kvh + self.hkv) * D]
        v = w[Hq * 2 * D + Hkv * D:][kvh * D:(kvh + self.hkv) * D]
        out = {"qkv": pack_linear(torch.cat([q, k, v], 0), C),
               "q_norm": get(p + "attn.q_norm").to(torch.bfloat16).contiguous(),
               "k_norm": get(p + "attn.k_norm").to(torch.bfloat16).contiguous()}
        wo = get(p + "attn.o_proj")
        out["o_proj"] = pack_linear(wo[:, r * self.hq * D:(r + 1) * self.hq * D].contiguous(), C)
        return out

    def _load_moe(self, get, p: str) -> dict:
        cfg, C = self.cfg, self.C
        H, E = cfg.hidden_size, cfg.num_experts
        router = get(p + "moe.router")
        sg = get(p + "moe.shared_gate")
        out = {"router": pack_linear(torch.cat([router, sg], 0), C)}
        eb, ee = self.e_begin, self.e_begin + self.e_local
        gate = torch.cat([get(p + "moe.gate")[eb:ee], get(p + "moe.shared.gate")[None]], 0)
        up = torch.cat([get(p + "moe.up")[eb:ee], get(p + "moe.shared.up")[None]], 0)
        out["gate_up"] = pack_linear(interleave_gate_up(gate, up), C)
        del gate, up
        down = get(p + "moe.down")[eb:ee]
        sd = get(p + "moe.shared.down")
        if self.tp > 1:
            # Tensor-parallel shared expert: rank r computes the intermediate columns
            # [r*I/tp, (r+1)*I/tp) (its 128-row tiles of the interleaved gate/up, selected in
            # the grouped GEMM by last_m0/last_mt) and the down projection over those columns
            # only (the other columns' weights are zero), so the all-reduce sums the slices.
            sl = self.shared_cols()
            mask = torch.zeros(1, sd.shape[1], dtype=sd.dtype, device=sd.device)
            mask[:, sl[0]:sl[1]] = 1
            sd = sd * mask
        out["down"] = pack_linear(torch.cat([down, sd[None]], 0), C)
        return out

    def shared_cols(self) -> tuple[int, int]:
        """This rank's intermediate columns of the shared expert."""
        n = self.cfg.shared_expert_intermediate_size // self.tp
        return self.tp_rank * n, (self.tp_rank + 1) * n

    # ------------------------------------------------------------------ state
    def _alloc_state(self) -> None:
        cfg, dev = self.cfg, self.dev
        nG, nA = len(cfg.gdn_layers), len(cfg.attn_layers)
        conv_dim = 2 * self.hk * 128 + self.hv * 128
        self.conv_dim = conv_dim
        self.conv_state = torch.zeros(nG, self.num_slots, 2, conv_dim, 3, dtype=torch.bfloat16, device=dev)
        self.ssm_state = torch.zeros(nG, self.num_slots, self.hv, 128, 128, dtype=torch.float32, device=dev)
        kv_shape = (nA, self.num_pages, self.hkv, self.page_size, cfg.head_dim)  # head-major pages
        self.k_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev)
        # Page table: one row per request slot (+ dummy row).  Page 0 is the dummy page.
        self.page_table = torch.zeros(self.num_slots, self.max_pages, dtype=torch.int32, device=dev)

    def _alloc_buffers(self) -> None:
        cfg, dev = self.cfg, self.dev
        H = cfg.hidden_size
        R = max(self.max_seqs, self.max_prefill_tokens)
        Rp = _pad128(R)
        self.R = R
        if self.tp > 1 and hasattr(self.coll, "reserve"):
            self.coll.reserve(R, H)  # collective: symmetric buffers for the fused all-reduce
        i32 = dict(dtype=torch.int32, device=dev)
        self.gdn_w = 2 * self.hk * 128 + 2 * self.hv * 128 + 2 * self.hv
        self.qkv_w = (2 * self.hq + 2 * self.hkv) * cfg.head_dim
        self.mid_w = max(self.hv * 128, self.hq * cfg.head_dim)
        b = {}
        b["hidden"] = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
        # Sampling parameters of the lm_head rows (temperature 0 = greedy).
        b["samp_temp"] = torch.zeros(R, dtype=torch.float32, device=dev)
        b["samp_seed"] = torch.zeros(R, dtype=torch.int64, device=dev)
        b["samp_pos"] = torch.zeros(R, dtype=torch.int32, device=dev)
        b["samp_any"] = torch.zeros(1, dtype=torch.float32, device=dev)  # max temperature of the batch
        # In-kernel split-K: fp32 partial tiles + per-tile arrival counters (kept zero).
        b["gemm_ws"] = torch.zeros(8 << 20, dtype=torch.float32, device=dev)
        b["gemm_sem"] = torch.zeros(16384, dtype=torch.int32, device=dev)
        self.num_sms = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 148
        # In-kernel split-K for dense GEMMs with few output tiles.  Off by default: on the
        # decode shapes measured so far it did not beat the unsplit kernel.
        self.use_fix_splits = runtime_config().gemm_fix_splits
        # Varlen prefill attention: 0 = tensor-core kernel, 1 = SIMT kernel (per-row causal lengths).
        self.prefill_attn_impl = 0
        b["xq"] = torch.zeros(Rp, H, dtype=torch.uint8, device=dev)
        b["xsf"] = torch.zeros(mx.atoms_bytes(Rp, H), dtype=torch.uint8, device=dev)
        b["proj"] = torch.zeros(R * max(self.gdn_w, self.qkv_w), dtype=torch.bfloat16, device=dev)
        b["midq"] = torch.zeros(Rp * self.mid_w, dtype=torch.uint8, device=dev)
        b["midsf"] = torch.zeros(mx.atoms_bytes(Rp, self.mid_w), dtype=torch.uint8, device=dev)
        # Row-parallel projection output: f32 split-K partials [splits, rows, H].
        self.max_ksplit = 16
        b["delta_f32"] = torch.zeros(max(R * H, self.max_ksplit * self.max_seqs * H), dtype=torch.float32,
                                     device=dev)
        b["q_out"] = torch.zeros(R, self.hq, cfg.head_dim, dtype=torch.bfloat16, device=dev)
        b["gate_out"] = torch.zeros(R, self.hq, cfg.head_dim, dtype=torch.bfloat16, device=dev)
        self.max_splits = 16
        b["partial"] = torch.zeros(max(R * self.hq, self.max_seqs * self.hq * self.max_splits) * 260,
                                   dtype=torch.float32, device=dev)
        nr = self.layers[0]["router"].n_pad
        b["logits"] = torch.zeros(max(R * nr, self.max_ksplit * self.max_seqs * nr), dtype=torch.float32, device=dev)
        G = self.groups
        b["topk_ids"] = torch.zeros(R, self.top_k, **i32)
        b["topk_w"] = torch.zeros(R, self.top_k, dtype=torch.float32, device=dev)
        b["gcount"] = torch.zeros(G, **i32)
        b["goff"] = torch.zeros(G, **i32)
        b["gpre"] = torch.zeros(G + 1, **i32)
        b["pair_slot"] = torch.zeros(R, self.k1, **i32)
        mg = _pad128(R * self.k1) + 128 * G
        self.max_grouped = mg
        b["row_dst"] = torch.zeros(mg, **i32)
        b["row_scale"] = torch.zeros(mg, dtype=torch.float32, device=dev)
        b["xg"] = torch.zeros(mg, H, dtype=torch.uint8, device=dev)
        b["xg_sf"] = torch.zeros(mx.atoms_bytes(mg, H), dtype=torch.uint8, device=dev)
        I = cfg.moe_intermediate_size
        b["act"] = torch.zeros(mg, I, dtype=torch.uint8, device=dev)
        b["act_sf"] = torch.zeros(mx.atoms_bytes(mg, I), dtype=torch.uint8, device=dev)
        # Expert outputs in grouped-row order; each token gathers its pairs' rows (pair_src)
        # weighted by its routing weights (pair_w) inside the residual/all-reduce kernel.
        b["moe_y"] = torch.zeros(mg, H, dtype=torch.bfloat16, device=dev)
        b["pair_src"] = torch.zeros(R, self.k1, **i32)
        b["pair_w"] = torch.zeros(R, self.k1, dtype=torch.float32, device=dev)
        vt = self.lm_head.n_pad // 128
        self.vocab_tiles = vt
        # lm_head rows: one per sequence; with speculative decoding every verify row and
        # every MTP catch-up row (up to a whole step's rows).
        self.lm_rows = R if self.num_spec else self.max_seqs
        b["lm_keys"] = torch.zeros(self.lm_rows, vt, dtype=torch.int64, device=dev)
        b["out_ids"] = torch.zeros(self.lm_rows, **i32)
        b["out_vals"] = torch.zeros(self.lm_rows, dtype=torch.float32, device=dev)
        b["out_keys"] = torch.zeros(self.lm_rows, dtype=torch.int64, device=dev)
        b["err"] = torch.zeros(1, **i32)
        b["xq_last"] = torch.zeros(_pad128(self.lm_rows), H, dtype=torch.uint8, device=dev)
        # Step inputs (static so graphs can read them): ids, positions, slots, seq_lens,
        # packed as one [4, R] block so a step's inputs arrive in a single H2D copy.
        b["inputs"] = torch.zeros(4, R, **i32)
        b["in_ids"], b["in_pos"], b["in_slot"], b["in_len"] = b["inputs"].unbind(0)
        self.host_inputs = torch.zeros(4, R, dtype=torch.int32, pin_memory=True)
        b["seq_start"] = torch.zeros(self.max_seqs + 1, **i32)
        b["last_rows"] = torch.zeros(self.max_seqs, dtype=torch.int64, device=dev)
        self.buf = b

    # ------------------------------------------------------------------ kernels
    def _gemm(self, w: PackedLinear, xq, xsf, rows: int, out, ldo: int, epi=EPI_BF16, grouped=False,
              out_sf=None, row_dst=None, row_scale=None, k_splits: int = 1, last_tiles=None, bn=None, **sampling):
        b = self.buf
        if grouped:
            bn = self._moe_bn(rows)
            m0, mt = last_tiles if last_tiles is not None else (0, 0)
            self.C.gemm_mxf8(w.q, w.sf, xq, xsf, w.k, w.n_pad, w.n, w.groups, 0, b["gcount"], b["goff"], b["gpre"],
                             epi, out, ldo, out_sf, row_dst, row_scale, b["err"], 0, bn, 1, 0, 1, a_fp4=int(w.fp4),
                             last_m0=m0, last_mt=mt)
        else:
            if bn is None:
                bn = self._dense_bn(rows, w) if k_splits == 1 else (32 if rows <= 32 else 128)
            tiles = -(-rows // bn) * (w.n_pad // 128)
            fs = self._fix_splits(tiles, tiles, w.k // 128, bn) if (k_splits == 1 and self.use_fix_splits) else 1
            self.C.gemm_mxf8(w.q, w.sf, xq, xsf, w.k, w.n_pad, w.n, 1, rows, None, None, None, epi, out, ldo,
                             out_sf, row_dst, row_scale, b["err"], 0, bn, k_splits, rows * ldo, 1,
                             fs, b["gemm_ws"], b["gemm_sem"], a_fp4=int(w.fp4), **sampling)

    def _dense_bn(self, rows: int, w: PackedLinear, k_splits: int = 1) -> int:
        """Token tile of a dense GEMM.  One CTA streams its weight tiles at a bounded rate, so
        a GEMM with few 128-token work items leaves most SMs idle; 32-token items multiply
        the CTAs (the weight tile is re-read from L2 per item) until about half the SMs
        have work.  ZSTEP_GEMM_DENSE_BN pins 32 or 128."""
        forced = runtime_config().gemm_dense_bn
        if forced:
            return forced
        if rows <= 32:
            return 32
        # Measured on B200 at 256 rows: 32-token items win up to ~32 128-token items
        # (e.g. 15.4 vs 17.0 us at 1536 x 2048) and lose beyond (21.6 vs 17.4 us at 3088 x 2048).
        items128 = -(-rows // 128) * (w.n_pad // 128) * max(1, k_splits)
        return 32 if rows <= 512 and items128 * 4 <= self.num_sms else 128

    def _fix_splits(self, max_tiles: int, items: int, k_tiles: int, bn: int) -> int:
        """In-kernel split-K factor for a dense GEMM: double while all split items still fit
        in one wave (the splits of a tile wait for each other), each split keeps >= 2 K
        tiles, and the workspace holds every tile.  A single CTA streams only ~100 GB/s,
        so a GEMM with few output tiles needs the extra CTAs to approach HBM bandwidth."""
        s = 1
        cap = self.buf["gemm_ws"].numel()
        while (items * s * 2 <= self.num_sms and s * 2 <= 8 and k_tiles % (s * 2) == 0 and k_tiles // (s * 2) >= 2
               and max_tiles * s * 2 * 128 * bn <= cap and max_tiles <= self.buf["gemm_sem"].numel()):
            s *= 2
        return s

    def _moe_bn(self, rows: int) -> int:
        """Token chunk of the grouped expert GEMMs: 32 while the average expert sees a few
        tokens (decode), 128 for prefill-sized batches."""
        return 32 if rows * self.top_k <= 32 * self.cfg.num_experts else 128

    def _split_plan(self, w: PackedLinear, rows: int, cap: int | None = None) -> tuple[int, int]:
        """(token tile, K splits) of a dense GEMM whose consumer sums f32 split-K partials
        (decode only): for each tile, split K until about one wave of work items; keep the
        tile with more items, the 128-token one on a tie (fewer weight re-reads).  Measured
        on B200: the router (384 x 2048) runs best as 32-token x 4 splits, a 2048 x 4096
        projection as 128-token x 4 splits."""
        if rows > self.max_seqs:
            return (32 if rows <= 32 else 128), 1
        k_tiles = w.k // 128
        limit = min(self.max_ksplit, k_tiles, cap or self.max_ksplit)
        best = None
        for bn in ((32,) if rows <= 32 else (128, 32)):
            items = ((rows + bn - 1) // bn) * (w.n_pad // 128)
            s = 1
            while items * s * 2 <= 160 and s * 2 <= limit:
                s *= 2
            if best is None or items * s > best[2]:
                best = (bn, s, items * s)
        return best[0], best[1]

    def _mid(self, width: int) -> torch.Tensor:
        rp = _pad128(self.R)
        return self.buf["midq"][: rp * width].view(rp, width)

    def _attn_splits(self, rows: int, decode: bool, ctx: int | None = None) -> int:
        if not decode:
            return 1
        ctas = max(rows * self.hkv, 1)
        if self.hq // self.hkv >= 4:
            # Tensor-core decode (one CTA per SM, a dependent chain per 128-key tile): about
            # two waves of CTAs, each split keeping >= 8 tiles to amortise its first load.
            ctx = ctx or self.max_pages * self.page_size
            return int(max(1, min(self.max_splits, math.ceil(296 / ctas), max(1, ctx // 1024))))
        return int(max(1, min(self.max_splits, math.ceil(1200 / ctas))))

    def _proj_out(self, w: PackedLinear, xq, xsf, rows: int, norm_w, hidden=None) -> None:
        """Row-parallel output projection (GDN out_proj / attention o_proj), then residual
        add + RMSNorm (+ all-reduce across ranks).  Tensor parallel at decode sizes: the
        GEMM epilogue pushes its bf16 partial tiles straight into the fused all-reduce's
        receive slots over NVLink, and the all-reduce only reduces and normalises.
        Otherwise: f32 split-K partials, reduced by the next kernel."""
        H = self.cfg.hidden_size
        b = self.buf
        tgt = self.coll.push_target(rows) if self.tp > 1 and hasattr(self.coll, "push_target") else None
        if tgt is not None:
            proto, parts, ep = tgt
            self.C.gemm_mxf8(w.q, w.sf, xq, xsf, w.k, w.n_pad, w.n, 1, rows, None, None, None, EPI_PUSH,
                             b["delta_f32"], H, None, None, None, b["err"], 0, 32, 1, 0, 1,
                             push_part=parts, push_epoch=ep, push_rank=self.tp_rank, push_mode=proto)
            self.coll.allreduce_add_rmsnorm(b["delta_f32"], 1, H, 0, b["hidden"] if hidden is None else hidden,
                                            norm_w, self.eps, rows, b["xq"], b["xsf"], protocol=proto, pushed=True)
            return
        bn, s = self._split_plan(w, rows)
        self._gemm(w, xq, xsf, rows, self.buf["delta_f32"], H, EPI_F32, k_splits=s, bn=bn)
        self._row_parallel_reduce(self.buf["delta_f32"], rows, s, norm_w, rows * H, H, hidden=hidden)

    def _row_parallel_reduce(self, delta_rows: torch.Tensor, rows: int, n_terms: int, norm_w, term_stride: int,
                             row_stride: int, term_index=None, term_scale=None, hidden=None):
        """hidden += sum of delta terms (all-reduced across tp ranks), then RMSNorm -> xq.
        With ``term_index`` [rows, n_terms] the terms are gathered rows of delta (negative:
        not produced on this rank), scaled by ``term_scale``."""
        b, H = self.buf, self.cfg.hidden_size
        hidden = b["hidden"] if hidden is None else hidden
        if self.tp > 1:
            self.coll.allreduce_add_rmsnorm(delta_rows, n_terms, row_stride, term_stride, hidden, norm_w,
                                            self.eps, rows, b["xq"], b["xsf"], term_index=term_index,
                                            term_scale=term_scale)
            return
        self.C.add_rmsnorm_quant(hidden, delta_rows, n_terms, row_stride, term_stride, norm_w, 1.0, self.eps,
                                 rows, None, b["xq"], b["xsf"], term_index, term_scale)

    def _layers(self, rows: int, decode: bool, num_seqs: int = 0, ckpt=None, gdn_out_slots=None,
                proj_store=None, max_seq_rows: int = 0) -> None:
        """All decoder layers over the staged rows.  Varlen (prefill / verify) steps may
        redirect each sequence's final GDN state (`gdn_out_slots`) and keep every GDN layer's
        input projection (`proj_store[layer]`) for a later replay; `max_seq_rows` (a bound
        on the rows of any sequence, 0 if unknown) lets a verify step's few rows per
        sequence run on the streaming GDN kernel."""
        cfg, C, b = self.cfg, self.C, self.buf
        H = cfg.hidden_size
        pos, slot, lens = b["in_pos"][:rows], b["in_slot"][:rows], b["in_len"][:rows]
        C.embed_rmsnorm_quant(b["in_ids"][:rows], self.embed, b["hidden"], self.layers[0]["input_norm"], 1.0,
                              self.eps, rows, None, b["xq"], b["xsf"])
        for li, L in enumerate(self.layers):
            if L["type"] == "linear_attention":
                gi = self.gdn_index[li]
                if proj_store is not None:
                    proj = proj_store[gi][:rows]
                else:
                    proj = b["proj"][:rows * self.gdn_w].view(rows, self.gdn_w)
                self._gemm(L["in_proj"], b["xq"], b["xsf"], rows, proj, self.gdn_w)
                midq = self._mid(self.hv * 128)
                args = (proj, self.hk, self.hv, L["conv_w"], self.conv_state[gi], self.ssm_state[gi], L["a_log"],
                        L["dt_bias"], L["gnorm"], self.eps, slot, pos, rows, None, midq, b["midsf"])
                if decode:
                    C.gdn_decode(*args, b["err"])
                else:
                    ck_rows, ck_slots, max_ck = ckpt if ckpt is not None else (None, None, 0)
                    C.gdn_prefill(*args, b["seq_start"][:num_seqs + 1], num_seqs, ck_rows, ck_slots, max_ck,
                                  b["err"], gdn_out_slots, max_seq_rows=max_seq_rows)
                self._proj_out(L["out_proj"], midq, b["midsf"], rows, L["post_norm"])
            else:
                ai = self.attn_index[li]
                qkv = b["proj"][:rows * self.qkv_w].view(rows, self.qkv_w)
                self._gemm(L["qkv"], b["xq"], b["xsf"], rows, qkv, self.qkv_w)
                C.attn_prologue(qkv, self.hq, self.hkv, cfg.rotary_dim, cfg.rope_theta, L["q_norm"], L["k_norm"],
                                self.eps, self.k_cache[ai], self.v_cache[ai], self.page_size, self.page_table, slot,
                                pos, rows, b["q_out"], b["gate_out"])
                midq = self._mid(self.hq * cfg.head_dim)
                splits = self._attn_splits(rows, decode)
                # Varlen steps pass their sequence boundaries: the tensor-core kernel then
                # serves several query rows of a sequence from each K/V tile it loads.
                grouped = not decode and num_seqs > 0
                C.attn_decode(b["q_out"], b["gate_out"], self.hq, self.hkv, self.k_cache[ai], self.v_cache[ai],
                              self.page_size, self.page_table, slot, lens, rows, b["partial"], splits,
                              1.0 / math.sqrt(cfg.head_dim), None, midq, b["midsf"],
                              impl=0 if decode else self.prefill_attn_impl,
                              seq_start=b["seq_start"][:num_seqs + 1] if grouped else None,
                              num_seqs=num_seqs if grouped else 0)
                self._proj_out(L["o_proj"], midq, b["midsf"], rows, L["post_norm"])
            self._moe(L, rows)
            next_w = self.layers[li + 1]["input_norm"] if li + 1 < len(self.layers) else self.final_norm
            self._row_parallel_reduce(b["moe_y"], rows, self.k1, next_w, 0, H, term_index=b["pair_src"],
                                      term_scale=b["pair_w"])

    def _moe(self, L, rows: int) -> None:
        cfg, C, b = self.cfg, self.C, self.buf
        E = cfg.num_experts
        nr = L["router"].n_pad
        # Router logits: split-K partials summed by the routing kernel (or one term when the
        # GEMM reduces its splits in-kernel).
        bn, s = (None, 1) if self.use_fix_splits else self._split_plan(L["router"], rows, cap=4)
        self._gemm(L["router"], b["xq"], b["xsf"], rows, b["logits"], nr, EPI_F32, k_splits=s, bn=bn)
        C.moe_route(b["logits"], rows, E, self.top_k, cfg.norm_topk_prob, 0, None, 1, 1, 1.0, E,
                    self.e_begin, self.e_begin + self.e_local, True, b["topk_ids"], b["topk_w"], b["gcount"],
                    b["goff"], b["gpre"], b["pair_slot"], b["row_dst"], b["row_scale"], b["xq"], b["xsf"], b["xg"],
                    b["xg_sf"], b["err"], nr, s, rows * nr, self._moe_bn(rows), b["pair_src"], b["pair_w"])
        I = cfg.moe_intermediate_size
        # Shared expert (last group): this rank's 128-row gate/up tiles only (64 columns each).
        c0, c1 = self.shared_cols()
        self._gemm(L["gate_up"], b["xg"], b["xg_sf"], rows, b["act"], I, EPI_SILU, grouped=True, out_sf=b["act_sf"],
                   last_tiles=(c0 // 64, (c1 - c0) // 64) if self.tp > 1 else None)
        self._gemm(L["down"], b["act"], b["act_sf"], rows, b["moe_y"], cfg.hidden_size, EPI_BF16, grouped=True)

    def _lm_head_argmax(self, rows: int, xq=None, xsf=None, pos=None, head=None) -> None:
        if rows > self.lm_rows:
            raise ValueError(f"lm_head over {rows} rows exceeds the {self.lm_rows}-row output buffers")
        """Greedy (temperature 0) or sampled next token of each row: the lm_head GEMM's
        epilogue reduces each vocab tile to one packed key of the (Gumbel-perturbed, for
        sampling rows) logits; the keys are then max-reduced locally or across ranks."""
        b = self.buf
        xq = b["xq"] if xq is None else xq
        xsf = b["xsf"] if xsf is None else xsf
        self._gemm(self.lm_head if head is None else head, xq, xsf, rows, b["lm_keys"], self.vocab_tiles, EPI_ARGMAX,
                   row_temp=b["samp_temp"], row_seed=b["samp_seed"], row_pos=b["in_pos"] if pos is None else pos,
                   id_offset=self.tp_rank * self.vocab_local, sample_any=b["samp_any"])
        if self.tp > 1:
            self.coll.argmax_allreduce(b["lm_keys"], rows, self.vocab_tiles, self.tp_rank * self.vocab_local,
                                       b["out_ids"], b["out_vals"])
        else:
            self.C.argmax_reduce(b["lm_keys"], rows, self.vocab_tiles, b["out_ids"], b["out_vals"], b["out_keys"])

    # ------------------------------------------------------------------ public step API
    def decode_forward(self, rows: int) -> torch.Tensor:
        """Run one decode step over the first `rows` staged inputs; returns out_ids[:rows]."""
        self._layers(rows, decode=True)
        self._lm_head_argmax(rows)
        return self.buf["out_ids"][:rows]

    def prefill_forward(self, rows: int, num_seqs: int, ckpt=None) -> torch.Tensor:
        """Varlen prefill over `rows` staged tokens in `num_seqs` sequences (seq_start staged).
        Returns the greedy next token of each sequence (from its last row)."""
        b = self.buf
        self._layers(rows, decode=False, num_seqs=num_seqs, ckpt=ckpt)
        # lm_head only on each sequence's last row: gather those normed rows.
        last = b["seq_start"][1:num_seqs + 1].long() - 1
        return self.lm_head_rows(last, b["xq_last"])

    def lm_head_rows(self, row_idx: torch.Tensor, xq_buf: torch.Tensor) -> torch.Tensor:
        """Next token of the selected rows of the last forward (normed MXFP8 rows gathered
        into `xq_buf`, then the lm_head GEMM + argmax / sampling)."""
        b, H = self.buf, self.cfg.hidden_size
        n = int(row_idx.numel())
        if n > self.lm_rows or n > xq_buf.shape[0]:
            raise ValueError(f"lm_head over {n} rows exceeds the {self.lm_rows}-row output buffers")
        codes = self._gather_sf(b["xsf"], row_idx, H)
        xq_buf[:n] = b["xq"][row_idx]
        sf = mx.atoms_from_codes(codes)
        self.last_lm_sf = sf  # scale atoms of the gathered rows (the full sampling head reuses them)
        b["samp_pos"][:n] = b["in_pos"][row_idx]
        self._lm_head_argmax(n, xq_buf, sf, pos=b["samp_pos"])
        return b["out_ids"][:n]

    def set_sampling(self, temperatures, seeds) -> None:
        """Per-sequence temperature (0 = greedy) and seed for the next steps' lm_head.
        Sequence i of a decode step is row i; of a prefill step, its last row."""
        n = len(temperatures)
        self.buf["samp_temp"][:n].copy_(torch.tensor(temperatures, dtype=torch.float32))
        self.buf["samp_seed"][:n].copy_(torch.tensor([s & 0x7FFFFFFFFFFFFFFF for s in seeds], dtype=torch.int64))
        self.buf["samp_temp"][n:].zero_()
        self.buf["samp_any"].fill_(max([0.0] + [float(t) for t in temperatures]))

    def clear_sampling(self) -> None:
        self.buf["samp_temp"].zero_()
        self.buf["samp_any"].zero_()

    def _gather_sf(self, atoms: torch.Tensor, rows_idx: torch.Tensor, k: int):
        """Gather scale codes of selected rows from an atom buffer (device ops)."""
        nkb = k // 32
        rb = rows_idx // 128
        rr = rows_idx % 128
        kb = torch.arange(nkb, device=atoms.device)
        off = (rb[:, None] * (k // 128) + kb[None, :] // 4) * 512 + (rr[:, None] % 32) * 16 + (rr[:, None] // 32) * 4 \
            + kb[None, :] % 4
        return atoms[off]

    def stage(self, ids, positions, slots, seq_lens=None, seq_start=None) -> int:
        """Write step inputs into the pinned staging block and copy it to the device in one
        H2D transfer (4 x R int32).  Returns the number of rows."""
        b, h = self.buf, self.host_inputs
        n = len(ids)
        h[0, :n] = torch.as_tensor(ids, dtype=torch.int32)
        h[1, :n] = torch.as_tensor(positions, dtype=torch.int32)
        h[2, :n] = torch.as_tensor(slots, dtype=torch.int32)
        if seq_lens is None:
            h[3, :n] = h[1, :n] + 1
        else:
            h[3, :n] = torch.as_tensor(seq_lens, dtype=torch.int32)
        for i in range(4):
            b["inputs"][i, :n].copy_(h[i, :n], non_blocking=True)
        if seq_start is not None:
            b["seq_start"][:len(seq_start)].copy_(torch.as_tensor(seq_start, dtype=torch.int32))
        self._staged_rows = n
        return n

    def staged_bytes(self) -> int:
        """Host->device bytes moved by the last stage() call."""
        return 4 * 4 * getattr(self, "_staged_rows", 0)

    def paged_caches(self) -> list[torch.Tensor]:
        """Device tensors indexed [layer, page, ...] (the attention layers' K and V)."""
        return [self.k_cache, self.v_cache]

    def copy_recurrent_state(self, src_slot: int, dst_slot: int) -> None:
        """Restore a checkpoint: GDN state and both conv-window buffers of every layer."""
        self.ssm_state[:, dst_slot].copy_(self.ssm_state[:, src_slot])
        self.conv_state[:, dst_slot].copy_(self.conv_state[:, src_slot])

    def checkpoint_args(self, ckpt_rows, ckpt_slots, query_start):
        """Per-sequence checkpoint tables for the GDN prefill kernel: for sequence s,
        entries [s*max_ck, (s+1)*max_ck) list (global row, checkpoint slot) pairs in row
        order, -1 padded."""
        rows = [int(x) for x in ckpt_rows]
        slots = [int(x) for x in ckpt_slots]
        qs = [int(x) for x in query_start]
        n = len(qs) - 1
        per = [[] for _ in range(n)]
        for r, s in sorted(zip(rows, slots)):
            for i in range(n):
                if qs[i] <= r < qs[i + 1]:
                    per[i].append((r, s))
                    break
        max_ck = max(1, max(len(p) for p in per))
        rt = torch.full((n, max_ck), -1, dtype=torch.int32)
        st = torch.zeros((n, max_ck), dtype=torch.int32)
        for i, p in enumerate(per):
            for j, (r, s) in enumerate(p):
                rt[i, j], st[i, j] = r, s
        return rt.to(self.dev), st.to(self.dev), max_ck

    def set_pages(self, slot: int, pages: list[int]) -> None:
        self.page_table[slot, :len(pages)] = torch.as_tensor(pages, dtype=torch.int32, device=self.dev)

    def bucket_for(self, n: int) -> int:
        for bk in DECODE_BUCKETS:
            if bk >= n and bk <= self.max_seqs:
                return bk
        return self.max_seqs

    def pad_decode_inputs(self, n: int, bucket: int) -> None:
        """Point padding rows [n, bucket) at the dummy slot/page (their outputs are ignored)."""
        if bucket > n:
            b = self.buf
            b["in_ids"][n:bucket] = 0
            b["in_pos"][n:bucket] = 1
            b["in_slot"][n:bucket] = self.dummy_slot
            b["in_len"][n:bucket] = 1

    def capture_decode_graph(self, bucket: int) -> None:
        """Capture one decode step over `bucket` rows into a CUDA graph."""
        b = self.buf
        saved = b["inputs"].clone()
        self.pad_decode_inputs(0, bucket)
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.decode_forward(bucket)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.decode_forward(bucket)
        self.graphs[bucket] = g
        b["inputs"].copy_(saved)  # capture ran on dummy rows; restore the staged step

    def decode_step(self, n: int) -> torch.Tensor:
        """Replay the graph of the bucket that fits n staged rows (captured on demand)."""
        bucket = self.bucket_for(n)
        self.pad_decode_inputs(n, bucket)
        if bucket not in self.graphs:
            self.capture_decode_graph(bucket)
            self.pad_decode_inputs(n, bucket)
        self.graphs[bucket].replay()
        return self.buf["out_ids"][:n]

    def check_error(self) -> int:
        err = int(self.buf["err"].item())
        if not err and self.coll is not None and hasattr(self.coll, "check_error"):
            err = self.coll.check_error()
        return err
