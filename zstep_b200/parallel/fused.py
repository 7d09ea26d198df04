"""Fused NVLink collectives for tensor parallelism (the product path).

Each rank allocates one symmetric block with ``cudaMalloc`` and shares it with its
peers through CUDA IPC; every rank then holds device pointers to all W blocks and the
sm_100a kernels in csrc/kernels/collective.cu load and store peer memory directly.
Block layout (all offsets 256-byte aligned)::

    [flags: 32 x u32][argmax keys: R x u64][rs words: (R+W) x H/2 x 8 B][ag words: R x H/2 x 8 B]
    [one-shot words: 2 x W x 8 x H/2 x 8 B][fp32 sum words: 2 x W x S x H x 8 B]

Reductions of at most 8 rows take the one-shot cluster kernel (one NVLink hop instead
of two; an 8-CTA cluster per row shares the RMSNorm statistics through distributed
shared memory).  ``allreduce_sum`` (the mHC model's fp32 sublayer outputs) is a one-shot
push of flag-in-data words for up to S = ``sum_rows`` rows and NCCL above that.

The all-reduce moves "flag-in-data" words (32 bits of payload + the call's epoch in one
8-byte store), so it needs no separate barrier; flags 16-31 belong to the argmax
exchange.  The epoch words and the completion counter are rank-local device memory; the
kernels advance them themselves, so every call (eager or CUDA-graph replay) uses fresh
flag values and nothing needs resetting between steps.

The collectives are issued by every rank in the same order (the model's layer order),
which is what the kernels' epochs rely on.  Waits are bounded: a peer that never
arrives makes the kernel record ``kErrPeerTimeout`` (2) in ``err`` and return.

Reference parity: worker/zstep_worker/kernels_sm120/shm_allreduce.py:437 (host-SHM
all-reduce + residual + RMSNorm) and csrc/qwen35_ops_kernels.cu:202 (TP argmax).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _ext
from ..utils.env import runtime_config

_ALIGN = 256


def _up(x: int, a: int = _ALIGN) -> int:
    return (x + a - 1) // a * a


class FusedCollectives:
    def __init__(self, device, group=None, max_rows: int = 0, hidden: int = 0, sum_rows: int = 64):
        self.C = _ext.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("fused collectives support up to 8 ranks (one NVLink domain)")
        self.device = torch.device(device)
        self.max_rows = 0
        self.hidden = 0
        self._base = 0
        self._peers: list[int] = []
        self.epoch = torch.zeros(4, dtype=torch.int32, device=self.device)  # [ar, argmax, one-shot ar, sum]
        self.grid = torch.zeros(3, dtype=torch.int32, device=self.device)  # completion counters per kernel
        self.sum_rows = sum_rows
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.local_keys = None
        self.timeout_ms = runtime_config().coll_timeout_ms  # bound on every cross-rank wait
        self.large_rows = 1024
        from .collectives import NcclCollectives

        self.nccl = NcclCollectives(group, self.device)
        if max_rows and hidden:
            self.reserve(max_rows, hidden)

    # ---------------------------------------------------------------- memory
    def reserve(self, max_rows: int, hidden: int) -> None:
        """Collective: allocate and exchange the symmetric block (all ranks, same args)."""
        if max_rows <= self.max_rows and hidden == self.hidden:
            return
        self.close()
        R, H = max_rows, hidden
        # Reduce-scatter and all-gather buffers hold flag-in-data words: 8 bytes per two
        # bf16 values (the reduce-scatter side is [world][ceil(R/world)][H/2]).
        self.off_keys = _up(32 * 4)
        self.off_part = self.off_keys + _up(R * 8)
        self.off_out = self.off_part + _up((R + self.world) * H * 4)
        self.off_small = self.off_out + _up(R * H * 4)
        self.off_sum = self.off_small + _up(2 * self.world * 8 * H * 4)
        self.nbytes = self.off_sum + _up(2 * self.world * self.sum_rows * H * 8)
        with torch.cuda.device(self.device):
            self._base = self.C.symm_alloc(self.nbytes)
            handle = self.C.ipc_handle(self._base)
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=self.group)
            self._peers = [self._base if r == self.rank else self.C.ipc_open(handles[r]) for r in range(self.world)]
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.max_rows, self.hidden = R, H
        self.flag_ptrs = [p for p in self._peers]
        self.key_ptrs = [p + self.off_keys for p in self._peers]
        self.part_ptrs = [p + self.off_part for p in self._peers]
        self.out_ptrs = [p + self.off_out for p in self._peers]
        self.small_ptrs = [p + self.off_small for p in self._peers]
        self.sum_ptrs = [p + self.off_sum for p in self._peers]
        self.local_keys = torch.zeros(R, dtype=torch.int64, device=self.device)

    def close(self) -> None:
        if not self._base:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no peer may still be reading our block
        for r, p in enumerate(self._peers):
            if r != self.rank:
                self.C.ipc_close(p)
        dist.barrier(group=self.group)
        self.C.symm_free(self._base)
        self._base, self._peers, self.max_rows = 0, [], 0

    def check_error(self) -> int:
        return int(self.err.item())

    # ---------------------------------------------------------------- ops
    def allreduce_add_rmsnorm(self, delta, n_terms: int, row_stride: int, term_stride: int, hidden_buf,
                              norm_w, eps: float, rows: int, xq, xsf, term_index=None, term_scale=None) -> None:
        """hidden_buf[:rows] += sum over ranks of the local term sums; then RMSNorm(norm_w)
        -> MXFP8 (xq, xsf).  Every rank ends with the same bf16 residual stream."""
        H = hidden_buf.shape[-1]
        if rows > self.max_rows or H != self.hidden:
            raise ValueError(f"fused all-reduce reserved for {self.max_rows}x{self.hidden}, got {rows}x{H}")
        if rows > self.large_rows:
            # Prefill-sized reductions are bandwidth-bound: the flag-in-data protocol moves
            # twice the bytes, so large ones go through NCCL's ring/NVLS kernels.
            self.nccl.allreduce_add_rmsnorm(delta, n_terms, row_stride, term_stride, hidden_buf, norm_w, eps, rows,
                                            xq, xsf, term_index=term_index, term_scale=term_scale)
            return
        if rows <= 8 and (H // 16) % 32 == 0:
            self.C.fused_allreduce_norm(self.rank, self.world, delta, n_terms, row_stride, term_stride,
                                        self.part_ptrs, self.out_ptrs, self.flag_ptrs, self.epoch[2:3], self.grid[1:2],
                                        hidden_buf, norm_w, 1.0, eps, rows, None, xq, xsf, self.err, term_index,
                                        term_scale, self.timeout_ms, oneshot=self.small_ptrs)
            return
        self.C.fused_allreduce_norm(self.rank, self.world, delta, n_terms, row_stride, term_stride, self.part_ptrs,
                                    self.out_ptrs, self.flag_ptrs, self.epoch[0:1], self.grid[0:1], hidden_buf, norm_w,
                                    1.0, eps, rows, None, xq, xsf, self.err, term_index, term_scale,
                                    self.timeout_ms)

    def allreduce_sum(self, t: torch.Tensor) -> None:
        """In-place fp32 sum over ranks of t [rows, hidden] (mHC sublayer outputs): one-shot
        over NVLink up to ``sum_rows`` rows, NCCL above (bandwidth-bound sizes)."""
        if t.dim() == 2 and t.shape[1] == self.hidden and t.shape[0] <= self.sum_rows and t.dtype == torch.float32 \
                and t.is_contiguous():
            self.C.allreduce_sum_f32(self.rank, self.world, t, t.shape[0], self.sum_rows, self.sum_ptrs,
                                     self.epoch[3:4], self.grid[2:3], self.err, self.timeout_ms)
            return
        self.nccl.allreduce_sum(t)

    def argmax_allreduce(self, keys, rows: int, tiles: int, id_offset: int, out_ids, out_vals) -> None:
        """Global greedy token per row from per-tile packed keys of this rank's vocab shard."""
        if rows > self.max_rows:
            raise ValueError(f"fused argmax reserved for {self.max_rows} rows, got {rows}")
        self.C.argmax_reduce(keys, rows, tiles, None, None, self.local_keys)
        self.C.allreduce_argmax(self.rank, self.world, rows, self.key_ptrs, self.flag_ptrs, self.epoch[1:2],
                                self.local_keys, id_offset, out_ids, out_vals, self.err, self.timeout_ms)
