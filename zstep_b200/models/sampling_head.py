"""Full-distribution sampling head shared by the GPU runners.

Steps whose sequences ask for more than greedy or plain-temperature decoding (top-k,
top-p, presence / frequency / repetition penalties, log-probabilities) run the lm_head
GEMM in f32 over the rows the step just normed (still in the runner's MXFP8 buffers),
gather the vocabulary shards of all tensor-parallel ranks (NCCL all-gather), and sample
every row with the `sample` kernel (penalties, temperature, top-k, top-p, seeded draw,
log-probabilities).  A per-slot ring of the last 4096 generated tokens feeds the
penalties; a sequence's ring restarts when its prompt starts at position 0.

Reference parity: worker/zstep_worker/sampler.py:62 (SlotPenaltyState), :127
(sample_tp8_logits).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .qwen35 import EPI_F32

HIST = 4096


class SamplingHead:
    def __init__(self, runner):
        self.r = runner
        dev = runner.dev
        self.hist = torch.zeros(runner.num_slots, HIST, dtype=torch.int32, device=dev)
        self.hist_len = torch.zeros(runner.num_slots, dtype=torch.int32, device=dev)
        self.hist_pos = torch.zeros(runner.num_slots, dtype=torch.int32, device=dev)
        self.logits = None
        self.gathered = None

    def reset(self, slots) -> None:
        if len(slots):
            idx = torch.as_tensor(np.asarray(slots, dtype=np.int64), device=self.r.dev)
            self.hist_len[idx] = 0
            self.hist_pos[idx] = 0

    def _buffers(self, n: int):
        r = self.r
        vl = r.vocab_local
        if self.logits is None:
            self.logits = torch.empty(r.lm_rows, vl, dtype=torch.float32, device=r.dev)
            if r.tp > 1:
                self.gathered = torch.empty(r.tp, r.lm_rows, vl, dtype=torch.float32, device=r.dev)
        return self.logits[:n]

    def sample(self, n: int, xq, xsf, slots, params: np.ndarray, top_n: int = 0, record=None):
        """Rows 0..n-1 of (xq, xsf) are the normed lm_head inputs of sequences in `slots`;
        `params` the plan's sampling records; `record[i]` whether row i's token is a real
        generated token (goes into its slot's penalty ring).  Returns (tokens, logprobs,
        top_ids, top_lps) as host arrays (logprob fields None unless requested)."""
        r = self.r
        dev = r.dev
        logits = self._buffers(n)
        r._gemm(r.lm_head, xq, xsf, n, logits, r.vocab_local, EPI_F32)
        if r.tp > 1:
            g = self.gathered[:, :n]
            dist.all_gather_into_tensor(g, logits.contiguous())
            full = g.permute(1, 0, 2).reshape(n, r.tp * r.vocab_local)
        else:
            full = logits
        vocab = r.cfg.vocab_size
        f32 = lambda k: torch.as_tensor(np.ascontiguousarray(params[k][:n]), dtype=torch.float32).to(dev)  # noqa: E731
        temp, top_p = f32("temperature"), f32("top_p")
        pres, freq, rep = f32("presence"), f32("frequency"), f32("repetition")
        top_k = torch.as_tensor(np.ascontiguousarray(params["top_k"][:n]), dtype=torch.int32).to(dev)
        seed = torch.as_tensor(params["seed"][:n].astype(np.int64), dtype=torch.int64).to(dev)
        sl = torch.as_tensor(np.asarray(slots[:n], dtype=np.int64), device=dev)
        hist = self.hist.index_select(0, sl)
        hlen = self.hist_len.index_select(0, sl)
        tok = torch.empty(n, dtype=torch.int32, device=dev)
        want_lp = bool((params["logprobs"][:n] >= 0).any())
        lp = torch.empty(n, dtype=torch.float32, device=dev) if want_lp else None
        tids = torch.zeros(n, 5, dtype=torch.int32, device=dev) if want_lp else None
        tlps = torch.zeros(n, 5, dtype=torch.float32, device=dev) if want_lp else None
        r.C.sample(full, vocab, n, temp, top_k, top_p, pres, freq, rep, seed, hist, hlen,
                   min(5, max(0, top_n)) if want_lp else 0, tok, lp, tids, tlps)
        # record into the rings (generated tokens only)
        keep = np.ones(n, dtype=bool) if record is None else np.asarray(record[:n], dtype=bool)
        if keep.any():
            ki = torch.as_tensor(np.nonzero(keep)[0], device=dev)
            rs, rt = sl.index_select(0, ki), tok.index_select(0, ki)
            pos = self.hist_pos.index_select(0, rs).long()
            self.hist[rs, pos] = rt
            self.hist_pos.index_copy_(0, rs, (pos.int() + 1) % HIST)
            self.hist_len.index_copy_(0, rs, (self.hist_len.index_select(0, rs) + 1).clamp(max=HIST))
        out = (tok.cpu().numpy(), lp.cpu().numpy() if want_lp else None, tids.cpu().numpy() if want_lp else None,
               tlps.cpu().numpy() if want_lp else None)
        return out


def needs_full(params: np.ndarray, n: int) -> bool:
    """Whether a step's sampled rows need the full-distribution head."""
    p = params[:n]
    stoch = p["temperature"] > 0
    return bool(((stoch & ((p["top_k"] > 0) | (p["top_p"] < 1.0))) | (p["presence"] != 0) | (p["frequency"] != 0)
                 | (p["repetition"] != 1.0) | (p["logprobs"] >= 0)).any())
