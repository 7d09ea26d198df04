"""Micro-step model: a fixed synthetic step for measuring the control plane.

Each step derives bf16 activations from the plan alone, ((column + token + position +
slot) mod 1024) / 1024, then runs RMSNorm + MXFP8 quantization, one MXFP8 GEMM to
`features` columns, a sigmoid router top-k over the first `experts` columns whose weight
sum is added back to every column, a sum over the tensor-parallel ranks, and an argmax
per sampled row.  It exercises the same SHM plan / result path, collectives and kernel
launches as a model step while costing a few microseconds of GPU time, so `zstep run
--micro-steps` isolates the master <-> worker round trip.  On the CPU the same math runs
in PyTorch fp32 (no quantization).

Reference parity: worker/zstep_worker/runtime_loop.py:109-325 (MicroStep).
"""

from __future__ import annotations

import numpy as np
import torch

from ..runtime import wire


class MicroStepRunner:
    def __init__(self, args, rank: int, world: int, geo, device: str = "cuda", collectives=None):
        self.rank, self.world = rank, world
        self.H = getattr(args, "micro_hidden", 5120)
        self.F = getattr(args, "micro_features", 2048)
        self.E = getattr(args, "micro_experts", 384)
        self.K = getattr(args, "micro_topk", 6)
        if self.H % 128 or self.F % 128 or not 0 < self.K <= self.E <= self.F:
            raise ValueError("micro-step: hidden/features must be multiples of 128 and top_k <= experts <= features")
        self.dev = torch.device(device if device != "cuda" else f"cuda:{torch.cuda.current_device()}")
        self.coll = collectives
        g = torch.Generator(device="cpu").manual_seed(2026 + rank)
        self.norm_w = (1.0 + 0.02 * torch.randn(self.H, generator=g)).to(torch.bfloat16).to(self.dev)
        w = (0.02 * torch.randn(self.F, self.H, generator=g)).to(torch.bfloat16).to(self.dev)
        self.cols = torch.arange(self.H, device=self.dev, dtype=torch.int32)
        if self.dev.type == "cuda":
            from ..ops import _ext
            from ..ops import mx
            from .qwen35 import _pad128, pack_linear

            self.C = _ext.load()
            self.W = pack_linear(w, self.C)
            R = max(geo.max_step_tokens, 1)
            Rp = _pad128(R)
            self.xq = torch.zeros(Rp, self.H, dtype=torch.uint8, device=self.dev)
            self.xsf = torch.zeros(mx.atoms_bytes(Rp, self.H), dtype=torch.uint8, device=self.dev)
            self.out = torch.zeros(R, self.F, dtype=torch.float32, device=self.dev)
            self.err = torch.zeros(1, dtype=torch.int32, device=self.dev)
        else:
            self.w = w.float()
        self.start = torch.cuda.Event(enable_timing=True) if self.dev.type == "cuda" else None
        self.end = torch.cuda.Event(enable_timing=True) if self.dev.type == "cuda" else None
        self.last_gpu_us = 0

    def forward(self, tokens: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
        """Per-row output [rows, features] (fp32), identical on every rank."""
        rows = tokens.shape[0]
        act = ((self.cols[None, :] + tokens[:, None] + positions[:, None] + slots[:, None]) % 1024).to(torch.float32)
        act = (act * (1.0 / 1024.0)).to(torch.bfloat16)
        if self.dev.type == "cuda":
            self.C.rms_quant(act, self.H, self.norm_w, 1e-6, rows, self.xq, self.xsf)
            self.C.gemm_mxf8(self.W.q, self.W.sf, self.xq, self.xsf, self.W.k, self.W.n_pad, self.W.n, 1, rows, None,
                             None, None, 1, self.out, self.F, None, None, None, self.err, 0, 32 if rows <= 32 else 128,
                             1, rows * self.F, 1)
            y = self.out[:rows]
        else:
            x = act.float()
            x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * self.norm_w.float()
            y = x @ self.w.T
        score = torch.sigmoid(y[:, :self.E])
        topw = torch.topk(score, self.K, dim=-1).values
        y = y + (topw / topw.sum(-1, keepdim=True) * 1.5).sum(-1, keepdim=True)
        if self.world > 1:
            if self.coll is not None:
                self.coll.allreduce_sum(y)
            else:
                import torch.distributed as dist

                dist.all_reduce(y)
        return y

    def execute(self, plan: dict) -> np.ndarray:
        n = plan["num_seqs"]
        rows = plan["num_rows"]
        out = np.zeros(n, dtype=wire.SEQ_OUTPUT_DTYPE)
        if rows == 0:
            return out
        if self.start is not None:
            self.start.record()
        t = torch.from_numpy(plan["token_ids"][:rows]).to(self.dev, non_blocking=True)
        p = torch.from_numpy(plan["positions"][:rows]).to(self.dev, non_blocking=True)
        s = torch.from_numpy(plan["row_slot"][:rows]).to(self.dev, non_blocking=True)
        y = self.forward(t, p, s)
        rows_sel = [int(r) for r in plan["sample_row"][:n]]
        idx = torch.tensor([max(r, 0) for r in rows_sel], dtype=torch.long, device=self.dev)
        ids = y.index_select(0, idx).argmax(-1).cpu().numpy() if n else []
        if self.end is not None:
            self.end.record()
            self.end.synchronize()
            self.last_gpu_us = max(1, int(self.start.elapsed_time(self.end) * 1000))
        for i in range(n):
            out[i]["req_slot"] = int(plan["seq_slot"][i])
            if rows_sel[i] >= 0:
                out[i]["num_tokens"] = 1
                out[i]["tokens"][0] = int(ids[i])
        return out

    def close(self) -> None:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()
