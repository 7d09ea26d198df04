"""Tensor-parallel collectives used by the model runners.

Two implementations share one interface:

* ``NcclCollectives`` -- the baseline: local term sum, ``dist.all_reduce`` over NCCL,
  then the residual-add + RMSNorm + MXFP8 kernel; global argmax via an int64 MAX
  all-reduce of packed (logit, ~id) keys.
* ``FusedCollectives`` (parallel/fused.py) -- the product path: one sm_100a kernel
  that pushes each rank's partial sums into its peers' symmetric memory over NVLink
  (P2P stores of flag-carrying LL lines; every load is local), reduces them in a fixed
  rank order (bit-identical on every rank), and applies the residual add, RMSNorm and
  MXFP8 quantization in the same pass.

``allreduce_add_rmsnorm`` takes the local contribution as ``n_terms`` partial terms
(split-K partials or MoE pair rows) addressed as ``delta[row*row_stride + t*term_stride
+ col]``, or gathered (``term_index``/``term_scale``: the MoE expert outputs of each
token, weighted by its routing weights); terms are summed in index order before the
cross-rank reduction.

Reference parity: the reference's host-SHM all-reduce + add + RMSNorm
(worker/zstep_worker/kernels_sm120/shm_allreduce.py:437,514) and the TP=8 top-2
argmax exchange (csrc/qwen35_ops_kernels.cu:202).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

_SIGN = -(1 << 63)  # xor mask mapping unsigned key order onto signed int64 order


def local_term_sum(delta: torch.Tensor, rows: int, hidden: int, n_terms: int, row_stride: int,
                   term_stride: int, term_index: torch.Tensor | None = None,
                   term_scale: torch.Tensor | None = None) -> torch.Tensor:
    """Sum of the local partial terms as fp32 [rows, hidden] in term order.  With
    ``term_index`` term t of row r is row ``term_index[r, t]`` of delta (negative:
    skipped), scaled by ``term_scale[r, t]`` when given."""
    acc = None
    if term_index is None:
        view = torch.as_strided(delta, (n_terms, rows, hidden), (term_stride, row_stride, 1))
    else:
        n_src = (delta.numel() - hidden) // row_stride + 1
        src = torch.as_strided(delta, (n_src, hidden), (row_stride, 1))
    for t in range(n_terms):
        if term_index is None:
            v = view[t].float()
        else:
            idx = term_index[:rows, t].long()
            v = src[idx.clamp(min=0)].float() * (idx >= 0).unsqueeze(1)
        if term_scale is not None:
            v = v * term_scale[:rows, t:t + 1]
        acc = v if acc is None else acc + v
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
                              norm_w, eps: float, rows: int, xq, xsf, term_index=None, term_scale=None) -> None:
        H = hidden_buf.shape[-1]
        acc = local_term_sum(delta, rows, H, n_terms, row_stride, term_stride, term_index,
                             term_scale).to(torch.bfloat16)
        dist.all_reduce(acc, group=self.group)
        self.C.add_rmsnorm_quant(hidden_buf, acc, 1, H, H, norm_w, 1.0, eps, rows, None, xq, xsf)

    def allreduce_sum(self, t: torch.Tensor) -> None:
        """In-place sum over ranks (the row-parallel sublayer output of the mHC model)."""
        dist.all_reduce(t, group=self.group)

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


class LocalCollectives:
    """Single-process stand-in with the collective interface: every reduction sees only this
    rank's own contribution.  Used to time one rank's compute of a tensor-parallel layout on
    one GPU (the numbers then exclude communication); never for real outputs."""

    def __init__(self, device=None):
        from ..ops import _ext

        self.C = _ext.load()
        self.device = device

    def allreduce_add_rmsnorm(self, delta, n_terms: int, row_stride: int, term_stride: int, hidden_buf,
                              norm_w, eps: float, rows: int, xq, xsf, term_index=None, term_scale=None) -> None:
        self.C.add_rmsnorm_quant(hidden_buf, delta, n_terms, row_stride, term_stride, norm_w, 1.0, eps, rows, None,
                                 xq, xsf, term_index, term_scale)

    def allreduce_sum(self, t: torch.Tensor) -> None:
        pass

    def argmax_allreduce(self, keys, rows: int, tiles: int, id_offset: int, out_ids, out_vals) -> None:
        self.C.argmax_reduce(keys, rows, tiles, out_ids, out_vals, None)
