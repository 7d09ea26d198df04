"""DSpark draft head for the DeepSeek-style runner: block-parallel drafts from the target's
auxiliary hidden states, with a low-rank Markov correction between draft positions.

Context: after every target step the head stores, for each row the target accepted, a
context entry at that row's position: the MXFP8 FFN-site inputs of the auxiliary target
layers (captured during the target forward) are concatenated, combined by ``fc`` into one
hidden row, normalised, and projected by the draft layer's own MLA projection into its
own latent and index caches (same page table as the target).

Draft: each drafting sequence feeds a block of K rows at positions p+1..p+K: its newest
token then K-1 filler tokens.  The draft layer (MLA + DSA attention over the stored
contexts and the whole block, i.e. non-causal inside the block because every block row's
attention length is p+1+K; then a dense FFN; plain residual) and its final norm give one
hidden row per block row.  Draft k is the greedy token of
    lm_head(h_k) + markov_w2 . markov_w1[previous token],
evaluated as ONE GEMM over the concatenated row [h_k | markov_w1[prev]] against
[lm_head | markov_w2] with the fused argmax epilogue (vocab-sharded and rank-reduced like
the target's lm_head), so the K steps only chain through the previous token.

Reference parity: worker/zstep_worker/models/deepseek_v41_dspark.py (DeepSeekV41DSparkDrafter
:36: block of [anchor, noise...] :387, Markov head over base logits :123, context KV from
combined auxiliary hidden states :233, draft :471).
"""

from __future__ import annotations

import torch

from ..ops import mx
from .qwen35 import EPI_BF16, EPI_F32, EPI_SILU, _pad128, pack_linear


class DSparkDrafter:
    context_only = True  # a context entry needs only its own target row

    def __init__(self, runner, src):
        r = self.r = runner
        c, C, dev = r.cfg, r.C, r.dev
        self.K = r.num_spec
        if r.R < r.max_seqs * self.K:
            raise ValueError(f"DSpark blocks need {r.max_seqs * self.K} staged rows; raise max_prefill_tokens")
        get = lambda n: src.get(n, dev)  # noqa: E731
        bf = lambda n: get(n).to(torch.bfloat16).contiguous()  # noqa: E731
        H = c.hidden_size
        self.aux = tuple(c.dspark_aux())
        na = len(self.aux)
        self.fc = pack_linear(get("dspark.fc"), C)  # [H, na*H], replicated
        self.L = r._load_layer(src, "layers.dspark.", dense=True)
        self.final_norm = bf("dspark.final_norm")
        self.noise = c.vocab_size - 1 if c.dspark_noise_token < 0 else c.dspark_noise_token
        self.rank_m = c.dspark_markov_rank
        self.w1 = bf("dspark.markov_w1")  # [V, rank] (replicated: indexed by the previous token)
        vs, tr = r.vocab_local, r.tp_rank
        head = torch.cat([get("lm_head")[tr * vs:(tr + 1) * vs], get("dspark.markov_w2")[tr * vs:(tr + 1) * vs]], 1)
        self.head = pack_linear(head.contiguous(), C)  # [V/tp, H + rank]
        del head
        self.ckv = torch.zeros(r.num_pages, r.page_size, c.kv_cache_dim, dtype=torch.bfloat16, device=dev)
        self.ik = torch.zeros(r.num_pages, r.page_size, c.index_head_dim, dtype=torch.bfloat16, device=dev)
        R, Rp = r.R, _pad128(r.R)
        u8 = dict(dtype=torch.uint8, device=dev)
        self.aux_q = torch.zeros(na, R, H, **u8)
        self.aux_codes = torch.zeros(na, R, H // 32, **u8)
        self.fc_q = torch.zeros(Rp, na * H, **u8)
        self.fc_sf = torch.zeros(mx.atoms_bytes(Rp, na * H), **u8)
        self.h = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
        ms = _pad128(r.max_seqs)
        self.cat_q = torch.zeros(ms, H + self.rank_m, **u8)
        self.cat_sf = torch.zeros(mx.atoms_bytes(ms, H + self.rank_m), **u8)
        self.mk_q = torch.zeros(ms, self.rank_m, **u8)
        self.mk_sf = torch.zeros(mx.atoms_bytes(ms, self.rank_m), **u8)
        self._rows = torch.arange(R, device=dev)

    # ------------------------------------------------------------------ target side
    def capture(self, j: int, rows: int) -> None:
        """Keep the MXFP8 FFN-site input of auxiliary layer j (called by the target forward)."""
        r = self.r
        H = r.cfg.hidden_size
        self.aux_q[j, :rows].copy_(r.buf["xq"][:rows])
        self.aux_codes[j, :rows].copy_(r._gather_sf(r.buf["xsf"], self._rows[:rows], H))

    def forward(self, rows: int, num_seqs: int, lm_rows: torch.Tensor, verify_slots, ckpt=None) -> torch.Tensor:
        """Target forward over the staged varlen rows (auxiliary states captured); returns the
        next token at each of `lm_rows`."""
        r = self.r
        r._layers(rows, decode=False)
        return r.lm_head_rows(lm_rows, r.buf["xq_last"])

    def replay(self, row_groups, slots, positions) -> None:
        """No recurrent state: rejected rows' cache entries are overwritten before use."""

    # ------------------------------------------------------------------ contexts
    def store_contexts(self, positions: list[int], slots: list[int], rows_t: torch.Tensor) -> None:
        """Context entries at `positions` of `slots` from target rows `rows_t` of the last
        forward (auxiliary states -> fc -> draft layer's attention norm -> MLA prologue)."""
        r, C, b, c, L = self.r, self.r.C, self.r.buf, self.r.cfg, self.L
        n = len(positions)
        if n == 0:
            return
        H, na = c.hidden_size, len(self.aux)
        self.fc_q[:n].copy_(self.aux_q[:, rows_t].permute(1, 0, 2).reshape(n, na * H))
        codes = self.aux_codes[:, rows_t].permute(1, 0, 2).reshape(n, na * H // 32)
        sf = mx.atoms_from_codes(codes)
        self.fc_sf[:sf.numel()].copy_(sf)
        r._gemm(self.fc, self.fc_q, self.fc_sf, n, self.h, H, EPI_BF16)
        C.rms_quant(self.h, H, L["attn_norm"], r.eps, n, b["xq"], b["xsf"])
        r.stage([0] * n, positions, slots)
        proj_a = b["proj_a"][:n]
        r._gemm(L["proj_a"], b["xq"], b["xsf"], n, proj_a, r.wa)
        # Only the latent and index-key entries matter here; the query-side outputs of the
        # prologue (from whatever qi holds) are discarded.
        C.mla_prologue(proj_a, r.off_kva, r.off_ik, r.off_iw, b["qi"][:n], r.off_iq, n, r.hl, c.qk_nope_head_dim,
                       c.qk_rope_head_dim, c.kv_lora_rank, c.index_n_heads, c.index_head_dim, L["kv_a_norm"],
                       L["idx_k_norm"], r.eps, c.rope_theta, b["in_slot"][:n], b["in_pos"][:n], r.page_table,
                       r.page_size, self.ckv, self.ik, b["q_pe"], b["iq"], b["iw"])

    # ------------------------------------------------------------------ drafts
    def _block(self, anchors: list[int], pos_next: list[int], slots: list[int]) -> torch.Tensor:
        """Draft layer over the K-row blocks; returns the final-normed MXFP8 rows in b["xq"]."""
        r, C, b, c, L = self.r, self.r.C, self.r.buf, self.r.cfg, self.L
        K, H = self.K, c.hidden_size
        ids, pos, sl, lens = [], [], [], []
        for a, p, s in zip(anchors, pos_next, slots):
            ids += [a] + [self.noise] * (K - 1)
            pos += list(range(p, p + K))
            sl += [s] * K
            lens += [p + K] * K  # every block row sees the whole block (and the context)
        rows = len(ids)
        r.stage(ids, pos, sl, seq_lens=lens)
        h = self.h[:rows]
        torch.index_select(r.embed, 0, b["in_ids"][:rows].long(), out=h)
        C.rms_quant(h, H, L["attn_norm"], r.eps, rows, b["xq"], b["xsf"])
        r._attention(-1, L, rows, False, caches=(self.ckv, self.ik))
        h.copy_(h.float() + b["y"][:rows])  # residual add in fp32, stored bf16
        C.rms_quant(h, H, L["ffn_norm"], r.eps, rows, b["xq"], b["xsf"])
        Fl = c.intermediate_size // r.tp
        r._gemm(L["gate_up"], b["xq"], b["xsf"], rows, b["act_d"], Fl, EPI_SILU, out_sf=b["act_d_sf"])
        r._gemm(L["down"], b["act_d"], b["act_d_sf"], rows, b["y"], H, EPI_F32)
        r._reduce(rows)
        h.copy_(h.float() + b["y"][:rows])
        C.rms_quant(h, H, self.final_norm, r.eps, rows, b["xq"], b["xsf"])
        return rows

    def _step(self, n: int, k: int, prev: torch.Tensor) -> torch.Tensor:
        """Draft k of every block: greedy token of [h | w1[prev]] . [lm_head | w2]^T."""
        r, C, b, c = self.r, self.r.C, self.r.buf, self.r.cfg
        H, K = c.hidden_size, self.K
        sel = self._rows[:n] * K + k
        C.quant_mxf8(self.w1[prev.long()].contiguous(), self.mk_q[:n], self.mk_sf)
        self.cat_q[:n, :H] = b["xq"][sel]
        self.cat_q[:n, H:] = self.mk_q[:n]
        codes = torch.cat([r._gather_sf(b["xsf"], sel, H), mx.codes_from_atoms(self.mk_sf, n, self.rank_m)], 1)
        sf = mx.atoms_from_codes(codes)
        self.cat_sf[:sf.numel()].copy_(sf)
        b["samp_pos"][:n] = b["in_pos"][sel]
        r._lm_head_argmax(n, self.cat_q, self.cat_sf, pos=b["samp_pos"], head=self.head)
        return b["out_ids"][:n].clone()

    def draft(self, ids, positions, slots, hidden_rows: torch.Tensor, last_of_seq: list[int]) -> list[list[int]]:
        """Store the accepted rows as contexts, then one block per drafting sequence
        (`last_of_seq[i]` = its newest row in `ids` / `positions`).  Returns K drafts each."""
        self.store_contexts(positions, slots, hidden_rows)
        anchors = [ids[j] for j in last_of_seq]
        pos_next = [positions[j] + 1 for j in last_of_seq]
        sl = [slots[j] for j in last_of_seq]
        n = len(anchors)
        if n == 0:
            return []
        b = self.r.buf
        self._block(anchors, pos_next, sl)
        any_s = b["samp_any"].clone()  # drafts are greedy
        b["samp_any"].zero_()
        prev = torch.tensor(anchors, dtype=torch.int32, device=self.r.dev)
        out = []
        for k in range(self.K):
            prev = self._step(n, k, prev)
            out.append(prev)
        b["samp_any"].copy_(any_s)
        return torch.stack(out, 1).cpu().tolist()

    def catch_up(self, ids, positions, slots, hidden_rows: torch.Tensor) -> None:
        """Steps without drafting sequences still store their accepted rows as contexts."""
        self.store_contexts(positions, slots, hidden_rows)
