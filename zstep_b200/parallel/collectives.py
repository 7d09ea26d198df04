"""Tensor-parallel collectives used by the model runners.

Two implementations share one interface:

* ``NcclCollectives`` -- the baseline: local term sum, ``dist.all_reduce`` over NCCL,
  then the residual-add + RMSNorm + MXFP8 kernel; global argmax via an int64 MAX
  all-reduce of packed (logit, ~id) keys.
* ``FusedCollectives`` (parallel/fused.py) -- the product path: one sm_100a kernel
  that pulls the peers' partial sums over NVLink (P2P loads from symmetric memory),
  reduces them in a fixed rank order (bit-identical on every rank), and applies the
  residual add, RMSNorm and MXFP8 quantization in the same pass.

``allreduce_add_rmsnorm`` takes the local contribution as ``n_terms`` partial terms
(split-K partials or MoE pair rows) addressed as ``delta[row*row_stride + t*term_stride
+ col]``; terms are summed in index order before the cross-rank reduction.

Reference parity: the reference's host-SHM all-reduce + add + RMSNorm
(worker/zstep_worker/kernels_sm120/shm_allreduce.py:437,514) and the TP=8 top-2
argmax exchange (csrc/qwen35_ops_kernels.cu:202).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

_SIGN = -(1 << 63)  # xor mask mapping unsigned key order onto signed int64 order


def local_term_sum(delta: torch.Tensor, rows: int, hidden: int, n_terms: int, row_stride: int,
                   term_stride: int) -> torch.Tensor:
    """Sum of the local partial terms as fp32 [rows, hidden] (fixed term order)."""
    view = torch.as_strided(delta, (n_terms, rows, hidden), (term_stride, row_stride, 1))
    acc = view[0].float()
    for t in range(1, n_terms):
        acc = acc + view[t].float()
    return acc


class NcclCollectives:
    def __init__(self, group=None, device=None):
        from ..ops import _ext

        self.C = _ext.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device

    def allreduce_add_rmsnorm(self, delta, n_terms: int, row_stride: int, term_stride: int, hidden_buf,
                              norm_w, eps: float, rows: int, xq, xsf) -> None:
        H = hidden_buf.shape[-1]
        acc = local_term_sum(delta, rows, H, n_terms, row_stride, term_stride).to(torch.bfloat16)
        dist.all_reduce(acc, group=self.group)
        self.C.add_rmsnorm_quant(hidden_buf, acc, 1, H, H, norm_w, 1.0, eps, rows, None, xq, xsf)

    def argmax_allreduce(self, keys, rows: int, tiles: int, id_offset: int, out_ids, out_vals) -> None:
        local = torch.empty(rows, dtype=torch.int64, device=keys.device)
        self.C.argmax_reduce(keys, rows, tiles, None, None, local)
        # Rebase ids to the global vocabulary: low word holds ~local_id.
        lid = (~local) & 0xFFFFFFFF
        gid = lid + id_offset
        k = (local & ~0xFFFFFFFF) | ((~gid) & 0xFFFFFFFF)
        k = k ^ _SIGN
        dist.all_reduce(k, op=dist.ReduceOp.MAX, group=self.group)
        k = k ^ _SIGN
        out_ids[:rows] = ((~k) & 0xFFFFFFFF).to(torch.int32)
        hi = (k >> 32) & 0xFFFFFFFF
        bits = torch.where(hi >= 0x80000000, hi & 0x7FFFFFFF, (~hi) & 0xFFFFFFFF).to(torch.int32)
        out_vals[:rows] = bits.view(torch.float32)
