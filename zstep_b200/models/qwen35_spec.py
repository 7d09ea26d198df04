"""Speculative decoding for the Qwen3.5 runner: multi-token-prediction (MTP) drafts,
verify forward and recurrent-state roll-back.

A verify step feeds each sequence its last token plus K drafts.  The target model runs
them as one varlen forward (causal attention from per-row context lengths; the GatedDeltaNet
layers step through the rows in order), the lm_head scores every verify row, and the host
accepts the longest draft prefix that matches the target's greedy tokens plus one bonus
token.

Roll-back: recurrent state cannot be rewound, so a verify step writes each verify
sequence's final GDN state to a spare slot and leaves the pre-step state untouched; every GDN
layer's input projection of the step is kept.  After acceptance the GDN recurrence is
replayed over the accepted rows only, in place on the pre-step slot (the outputs of the
replay are discarded: the verify pass already produced them).  Attention needs no roll-back:
KV written at rejected positions is overwritten before it is read.

MTP head (one full-attention MoE layer, own KV cache, shared embedding and lm_head):
draft_{t+2} = head(norm_e(embed(token_{t+1})), norm_h(hidden_t)).  After every target
step the head first catches up over the rows the target just accepted (their embeddings and
the target's hidden states), which also yields the first draft; K-1 more single-row steps
chain the head's own hidden state.

Reference parity: worker/zstep_worker/models/qwen35_mtp.py:47 (Qwen35MtpDrafter,
_forward_gpu :219, draft :511), qwen35_moe.py:1861 (_rollback_recurrent_states),
worker/zstep_worker/spec_decode.py:41 (verify_greedy).
"""

from __future__ import annotations

import torch

from ..ops import mx
from .qwen35 import EPI_BF16, _pad128, pack_linear


class SpecDecoder:
    context_only = False  # an MTP entry at row p needs the token at p+1

    def __init__(self, runner, src):
        r = self.r = runner
        cfg, C, dev = r.cfg, r.C, r.dev
        self.K = r.num_spec
        get = lambda n: src.get(n, dev)  # noqa: E731
        H = cfg.hidden_size
        p = "mtp.layer."
        self.fc = pack_linear(get("mtp.fc"), C)  # [H, 2H], replicated on every rank
        self.norm_e = get("mtp.pre_fc_norm_embedding").to(torch.bfloat16).contiguous()
        self.norm_h = get("mtp.pre_fc_norm_hidden").to(torch.bfloat16).contiguous()
        self.norm = get("mtp.norm").to(torch.bfloat16).contiguous()
        L = {"type": "full_attention", "input_norm": get(p + "input_norm").to(torch.bfloat16),
             "post_norm": get(p + "post_norm").to(torch.bfloat16)}
        L.update(r._load_attn(get, p))
        L.update(r._load_moe(get, p))
        self.L = L
        kv_shape = (r.num_pages, r.hkv, r.page_size, cfg.head_dim)
        self.k_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev)
        R = r.R
        Rp = _pad128(R)
        bf = dict(dtype=torch.bfloat16, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.res = torch.zeros(R, H, **bf)      # MTP residual stream (its hidden output)
        self.hid = torch.zeros(R, H, **bf)      # hidden-state input rows
        self.emb = torch.zeros(R, H, **bf)
        self.emb_n = torch.zeros(R, H, **bf)
        self.hid_n = torch.zeros(R, H, **bf)
        self.fc_q = torch.zeros(Rp, 2 * H, dtype=torch.uint8, device=dev)
        self.fc_sf = torch.zeros(mx.atoms_bytes(Rp, 2 * H), dtype=torch.uint8, device=dev)
        self.ids = torch.zeros(R, **i32)
        self.pos = torch.zeros(R, **i32)
        self.slot = torch.zeros(R, **i32)
        self.lens = torch.zeros(R, **i32)
        nG = len(cfg.gdn_layers)
        self.proj_store = torch.zeros(nG, R, r.gdn_w, **bf)  # GDN input projections of a verify step
        self.fix_proj = torch.zeros(R, r.gdn_w, **bf)
        self.fix_seq_start = torch.zeros(r.max_seqs + 1, **i32)
        self.out_slots = torch.zeros(r.max_seqs, **i32)

    # ------------------------------------------------------------------ target side
    def forward(self, rows: int, num_seqs: int, lm_rows: torch.Tensor, verify_slots: list[int | None],
                ckpt=None) -> torch.Tensor:
        """Varlen target forward over the staged rows (seq_start staged).  Sequence i with
        verify_slots[i] set writes its final GDN state to that spare slot.  Returns the
        next token at each row of `lm_rows` (device int64 row indices)."""
        r = self.r
        seq_slots = r.buf["in_slot"][r.buf["seq_start"][:num_seqs].long()]
        out = seq_slots.clone()
        for i, vs in enumerate(verify_slots):
            if vs is not None:
                out[i] = vs
        self.out_slots[:num_seqs].copy_(out)
        r._layers(rows, decode=False, num_seqs=num_seqs, ckpt=ckpt, gdn_out_slots=self.out_slots[:num_seqs],
                  proj_store=self.proj_store)
        return r.lm_head_rows(lm_rows, r.buf["xq_last"])

    def replay(self, row_groups: list[tuple[int, int]], slots: list[int], positions: list[int]) -> None:
        """Re-run the GDN recurrence of every layer over rows [start, start+n) of the last
        forward for each (start, n) in `row_groups`, in place on the given slots, so each
        sequence's recurrent state ends right after its last accepted row."""
        r = self.r
        if not row_groups:
            return
        dev = r.dev
        idx, starts, slot_rows, pos_rows = [], [0], [], []
        for (st, n), sl, p0 in zip(row_groups, slots, positions):
            idx.extend(range(st, st + n))
            starts.append(starts[-1] + n)
            slot_rows.extend([sl] * n)
            pos_rows.extend(range(p0, p0 + n))
        rows = len(idx)
        idx_t = torch.tensor(idx, dtype=torch.long, device=dev)
        self.fix_seq_start[:len(starts)].copy_(torch.tensor(starts, dtype=torch.int32))
        self.slot[:rows].copy_(torch.tensor(slot_rows, dtype=torch.int32))
        self.pos[:rows].copy_(torch.tensor(pos_rows, dtype=torch.int32))
        midq = r._mid(r.hv * 128)
        for li in r.cfg.gdn_layers:
            gi = r.gdn_index[li]
            L = r.layers[li]
            torch.index_select(self.proj_store[gi], 0, idx_t, out=self.fix_proj[:rows])
            r.C.gdn_prefill(self.fix_proj[:rows], r.hk, r.hv, L["conv_w"], r.conv_state[gi], r.ssm_state[gi],
                            L["a_log"], L["dt_bias"], L["gnorm"], r.eps, self.slot[:rows], self.pos[:rows], rows,
                            None, midq, r.buf["midsf"], self.fix_seq_start[:len(starts)], len(row_groups), None, None,
                            0, r.buf["err"], max_seq_rows=max(n for _, n in row_groups))

    # ------------------------------------------------------------------ graph path
    # A steady-state verify step (every sequence carries K drafts, greedy, no checkpoint)
    # runs as one CUDA graph per sequence bucket: target forward, lm_head argmax, on-device
    # verify (csrc/kernels/sampling.cu spec_verify), replay of the accepted rows, draft-head
    # catch-up and the K-1 chained drafts, with no host round trip inside the step.
    def _graph_buffers(self) -> None:
        if hasattr(self, "g_record"):
            return
        r, K, dev = self.r, self.K, self.r.dev
        ms, R = r.max_seqs, r.R
        i32 = dict(dtype=torch.int32, device=dev)
        self.g_record = torch.zeros(ms, 2 * K + 2, **i32)  # acc_len | K+1 accepted tokens | K next drafts
        self.g_verify = torch.zeros(ms, K + 2, **i32)
        self.g_rep_start = torch.zeros(ms + 1, **i32)
        self.g_rep_idx = torch.zeros(R, dtype=torch.long, device=dev)
        self.g_rep_slot = torch.zeros(R, **i32)
        self.g_rep_pos = torch.zeros(R, **i32)
        self.g_last = torch.zeros(ms, dtype=torch.long, device=dev)
        self.g_graphs: dict[int, torch.cuda.CUDAGraph] = {}

    def graph_bucket(self, n: int) -> int | None:
        """Smallest decode bucket holding n verify sequences (None: too many rows)."""
        r = self.r
        bk = r.bucket_for(n)
        if bk < n or bk * (self.K + 1) > r.R or bk * (self.K + 1) > r.lm_rows:
            return None
        return bk

    def verify_step(self, nb: int) -> None:
        """One speculative step over nb sequences x (K+1) staged rows (seq_start and
        out_slots staged), device-only.  Result rows: self.g_record[:nb]."""
        r, C, b, K = self.r, self.r.C, self.r.buf, self.K
        R = nb * (K + 1)
        r._layers(R, decode=False, num_seqs=nb, gdn_out_slots=self.out_slots[:nb], proj_store=self.proj_store,
                  max_seq_rows=K + 1)
        r._lm_head_argmax(R)
        C.spec_verify(nb, K, r.dummy_slot, b["in_ids"], b["out_ids"], b["in_pos"], b["in_slot"], self.g_verify,
                      self.g_rep_start, self.g_rep_idx, self.g_rep_slot, self.g_rep_pos, self.ids, self.pos, self.slot,
                      self.lens, self.g_last)
        # Replay the GDN recurrence over the accepted rows, in place on the pre-step slots.
        midq = r._mid(r.hv * 128)
        for li in r.cfg.gdn_layers:
            gi = r.gdn_index[li]
            L = r.layers[li]
            torch.index_select(self.proj_store[gi], 0, self.g_rep_idx[:R], out=self.fix_proj[:R])
            C.gdn_prefill(self.fix_proj[:R], r.hk, r.hv, L["conv_w"], r.conv_state[gi], r.ssm_state[gi], L["a_log"],
                          L["dt_bias"], L["gnorm"], r.eps, self.g_rep_slot[:R], self.g_rep_pos[:R], R, None, midq,
                          b["midsf"], self.g_rep_start[:nb + 1], nb, None, None, 0, b["err"], max_seq_rows=K + 1)
        # Draft head: catch-up over every verify row (rows past a sequence's accepted
        # prefix point at the padding slot), then K-1 chained single-row steps.
        self.hid[:R].copy_(b["hidden"][:R])
        first = self.mtp(R)
        last = self.g_last[:nb]
        drafts = [first.index_select(0, last)]
        prev = self.res.index_select(0, last)
        pos0 = self.pos.index_select(0, last)
        slot0 = self.slot.index_select(0, last)
        for s in range(1, K):
            self.ids[:nb].copy_(drafts[-1])
            self.pos[:nb].copy_(pos0 + s)
            self.slot[:nb].copy_(slot0)
            self.lens[:nb].copy_(pos0 + s + 1)
            self.hid[:nb].copy_(prev)
            drafts.append(self.mtp(nb).clone())
            prev = self.res[:nb].clone()
        self.g_record[:nb, :K + 2].copy_(self.g_verify[:nb])
        self.g_record[:nb, K + 2:].copy_(torch.stack(drafts, 1))

    def run_verify_graph(self, nb: int) -> None:
        """Replay (capturing on first use) the verify-step graph of bucket nb."""
        self._graph_buffers()
        if nb not in self.g_graphs:
            r, b = self.r, self.r.buf
            saved = (b["inputs"].clone(), b["seq_start"].clone(), self.out_slots.clone())
            # Capture on padding rows only: every row and state slot is the dummy one.
            R = nb * (self.K + 1)
            b["in_ids"][:R] = 0
            b["in_pos"][:R] = 1
            b["in_slot"][:R] = r.dummy_slot
            b["in_len"][:R] = 2
            b["seq_start"][:nb + 1].copy_(torch.arange(nb + 1, device=r.dev, dtype=torch.int32) * (self.K + 1))
            self.out_slots[:nb] = r.dummy_slot
            s = torch.cuda.Stream(r.dev)
            s.wait_stream(torch.cuda.current_stream(r.dev))
            with torch.cuda.stream(s):
                for _ in range(2):
                    self.verify_step(nb)
            torch.cuda.current_stream(r.dev).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self.verify_step(nb)
            self.g_graphs[nb] = g
            b["inputs"].copy_(saved[0])
            b["seq_start"].copy_(saved[1])
            self.out_slots.copy_(saved[2])
        self.g_graphs[nb].replay()

    # ------------------------------------------------------------------ MTP head
    def mtp(self, rows: int) -> torch.Tensor:
        """MTP head over `rows` staged rows (self.ids / pos / slot / lens and self.hid).
        Returns the draft token of every row; self.res holds the head's hidden output."""
        r, C, b, L = self.r, self.r.C, self.r.buf, self.L
        cfg = r.cfg
        H, eps = cfg.hidden_size, r.eps
        C.embed_rmsnorm_quant(self.ids[:rows], r.embed, self.emb, self.norm_e, 1.0, eps, rows, self.emb_n, None, None)
        C.add_rmsnorm_quant(self.hid, None, 0, H, H, self.norm_h, 1.0, eps, rows, self.hid_n, None, None)
        fc_in = torch.cat([self.emb_n[:rows], self.hid_n[:rows]], dim=1)
        C.quant_mxf8(fc_in, self.fc_q[:rows], self.fc_sf)
        r._gemm(self.fc, self.fc_q, self.fc_sf, rows, self.res, H, EPI_BF16)
        C.add_rmsnorm_quant(self.res, None, 0, H, H, L["input_norm"], 1.0, eps, rows, None, b["xq"], b["xsf"])
        qkv = b["proj"][:rows * r.qkv_w].view(rows, r.qkv_w)
        r._gemm(L["qkv"], b["xq"], b["xsf"], rows, qkv, r.qkv_w)
        C.attn_prologue(qkv, r.hq, r.hkv, cfg.rotary_dim, cfg.rope_theta, L["q_norm"], L["k_norm"], eps, self.k_cache,
                        self.v_cache, r.page_size, r.page_table, self.slot[:rows], self.pos[:rows], rows, b["q_out"],
                        b["gate_out"])
        midq = r._mid(r.hq * cfg.head_dim)
        C.attn_decode(b["q_out"], b["gate_out"], r.hq, r.hkv, self.k_cache, self.v_cache, r.page_size, r.page_table,
                      self.slot[:rows], self.lens[:rows], rows, b["partial"], self._splits(rows),
                      cfg.head_dim ** -0.5, None, midq, b["midsf"])
        r._proj_out(L["o_proj"], midq, b["midsf"], rows, L["post_norm"], hidden=self.res)
        r._moe(L, rows)
        r._row_parallel_reduce(b["moe_y"], rows, r.k1, self.norm, 0, H, term_index=b["pair_src"],
                               term_scale=b["pair_w"], hidden=self.res)
        # Drafts are greedy: switch the lm_head's sampling off for these rows.
        any_s = b["samp_any"].clone()
        b["samp_any"].zero_()
        ids = r.lm_head_rows(torch.arange(rows, device=r.dev), b["xq_last"])
        b["samp_any"].copy_(any_s)
        return ids

    def _splits(self, rows: int) -> int:
        """Split-KV factor for the MTP attention, capped by the runner's partial buffer."""
        r = self.r
        cap = r.buf["partial"].numel() // (260 * max(1, rows * r.hq))
        return max(1, min(r._attn_splits(rows, True), cap))

    def stage_mtp(self, ids, positions, slots, hidden_rows: torch.Tensor | None = None,
                  hidden_src: torch.Tensor | None = None) -> int:
        """Stage MTP input rows: token ids, positions, request slots, and hidden states
        gathered from `hidden_src` at `hidden_rows` (device indices)."""
        n = len(ids)
        self.ids[:n].copy_(torch.tensor(ids, dtype=torch.int32))
        self.pos[:n].copy_(torch.tensor(positions, dtype=torch.int32))
        self.slot[:n].copy_(torch.tensor(slots, dtype=torch.int32))
        self.lens[:n].copy_(self.pos[:n] + 1)
        if hidden_rows is not None:
            torch.index_select(hidden_src, 0, hidden_rows, out=self.hid[:n])
        return n

    def catch_up(self, ids, positions, slots, hidden_rows: torch.Tensor) -> None:
        """Steps without drafting sequences: run the head over the accepted rows so its KV
        cache stays complete."""
        self.stage_mtp(ids, positions, slots, hidden_rows, self.r.buf["hidden"])
        self.mtp(len(ids))

    def draft(self, ids, positions, slots, hidden_rows: torch.Tensor, last_of_seq: list[int]) -> list[list[int]]:
        """Catch-up rows (one per accepted target row) then K-1 chained steps.  Returns the K
        drafts of each sequence; `last_of_seq[i]` is the catch-up row of sequence i's newest
        token."""
        r = self.r
        n = self.stage_mtp(ids, positions, slots, hidden_rows, r.buf["hidden"])
        first = self.mtp(n).clone()
        sel = torch.tensor(last_of_seq, dtype=torch.long, device=r.dev)
        drafts = [first[sel]]
        prev_hidden = self.res[sel].clone()
        pos = [positions[j] for j in last_of_seq]
        sl = [slots[j] for j in last_of_seq]
        for _ in range(self.K - 1):
            pos = [p + 1 for p in pos]
            tok = drafts[-1].tolist()
            m = self.stage_mtp(tok, pos, sl)
            self.hid[:m].copy_(prev_hidden)
            d = self.mtp(m).clone()
            drafts.append(d)
            prev_hidden = self.res[:m].clone()
        return torch.stack(drafts, 1).cpu().tolist()
