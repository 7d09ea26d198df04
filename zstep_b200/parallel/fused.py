"""Fused NVLink collectives for tensor parallelism (the product path).

Each rank allocates one symmetric block with ``cudaMalloc`` and shares it with its
peers through CUDA IPC; every rank then holds device pointers to all W blocks and the
sm_100a kernels in csrc/kernels/collective.cu store into peer memory directly (every
protocol is push-based: kernels load only their own memory).  Block layout (all offsets
256-byte aligned; R = reserved rows, H = hidden, S = ``sum_rows``, Rl = LL two-shot rows)::

    [plain flags: 2 x 8 x FAR_CTAS u32][argmax lines: 2 x W x R x 16 B]
    [one-shot lines: 2 x W x 64 x H/4 x 16 B]
    [two-shot LL: (Rl + W) x H/4 x 16 B  +  Rl x H/4 x 16 B]
    [plain two-shot: (R + W) x H x 2 B  +  R x H x 2 B][fp32 sum lines: 2 x W x S x H/2 x 16 B]

Protocol by row count (``allreduce_add_rmsnorm``): up to ``ZSTEP_COLL_ONESHOT_ROWS``
rows one-shot (one NVLink hop), up to ``ZSTEP_COLL_LL_ROWS`` two-shot with LL lines
(data and epoch in one store, no barrier), above that two-shot with plain bf16 rows and
per-CTA release/acquire flags (full link bandwidth for prefill-sized reductions).  NCCL
is only used when ``ZSTEP_COLLECTIVES=nccl`` selects the baseline.

NVLS (``ZSTEP_COLL_NVLS_ROWS`` > 0, off by default): a second block from
``torch.distributed._symmetric_memory`` bound to an NVSwitch multicast object (the
allocation and handle exchange are the library's; the kernel is ours) holds
``[flags: 2 x FAR_CTAS u32][part: R x H bf16][out: R x H bf16]``.  All-reduces above the
one-shot size and up to that many rows then let the switch sum the ranks' copies
(``multimem.ld_reduce``) and broadcast each result (``multimem.st``).  Every rank must
see multicast support, or none uses it.

Epoch words and completion counters are rank-local device memory, one pair per protocol;
the kernels advance them themselves, so every call (eager or CUDA-graph replay) uses
fresh flag values and nothing needs resetting between steps.  The collectives are issued
by every rank in the same order (the model's layer order), which is what the epochs rely
on.  Waits are bounded: a peer that never arrives makes the kernel record
``kErrPeerTimeout`` (2) in ``err`` and return.

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


FAR_CTAS = 128          # csrc/kernels/zs_kernels.h
FAR_ONESHOT_ROWS = 64   # csrc/kernels/zs_kernels.h
ONESHOT, TWOSHOT, PLAIN, NVLS = 0, 1, 2, 3
# Epoch / completion-counter slots, one per kernel family.
_E_ONE, _E_TWO, _E_PLAIN, _E_ARGMAX, _E_SUM, _E_SUMP, _E_NVLS = range(7)


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
        self.epoch = torch.zeros(7, dtype=torch.int32, device=self.device)
        self.grid = torch.zeros(7, dtype=torch.int32, device=self.device)
        self.sum_rows = sum_rows
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        cfg = runtime_config()
        self.timeout_ms = cfg.coll_timeout_ms  # bound on every cross-rank wait
        self.oneshot_rows = min(cfg.coll_oneshot_rows, FAR_ONESHOT_ROWS)
        self.ll_rows = cfg.coll_ll_rows
        self.push = cfg.coll_push
        self.nvls_rows = cfg.coll_nvls_rows if self.world > 1 else 0
        self.nvls = None          # (local block tensor, part, out, flags, mc part, mc out, mc flags)
        self.nvls_error = ""      # why NVLS is not in use, when it was asked for
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
        R, H, W = max_rows, hidden, self.world
        Rl = min(R, self.ll_rows)
        self.ll_cap = Rl
        off = 0
        self.off_flags = off
        off += _up(2 * 8 * FAR_CTAS * 4)
        self.off_argmax = off
        off += _up(2 * W * R * 16)
        self.off_one = off
        off += _up(2 * W * FAR_ONESHOT_ROWS * H * 4)
        self.off_ll_part = off
        off += _up((Rl + W) * H * 4)
        self.off_ll_out = off
        off += _up(Rl * H * 4)
        self.off_plain_part = off
        off += _up((R + W) * H * 2)
        self.off_plain_out = off
        off += _up(R * H * 2)
        self.off_sum = off
        off += _up(2 * W * self.sum_rows * H * 8)
        # Plain two-shot fp32 sum (rows above sum_rows): its own flags, fp32 part and out.
        self.off_sum_flags = off
        off += _up(2 * 8 * FAR_CTAS * 4)
        self.off_sum_part = off
        off += _up((R + W) * H * 4)
        self.off_sum_out = off
        off += _up(R * H * 4)
        self.nbytes = off
        with torch.cuda.device(self.device):
            self._base = self.C.symm_alloc(self.nbytes)
            handle = self.C.ipc_handle(self._base)
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=self.group)
            self._peers = [self._base if r == self.rank else self.C.ipc_open(handles[r]) for r in range(self.world)]
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.max_rows, self.hidden = R, H
        at = lambda o: [p + o for p in self._peers]  # noqa: E731
        self.flag_ptrs = at(self.off_flags)
        self.argmax_ptrs = at(self.off_argmax)
        self.one_ptrs = at(self.off_one)
        self.ll_part_ptrs, self.ll_out_ptrs = at(self.off_ll_part), at(self.off_ll_out)
        self.plain_part_ptrs, self.plain_out_ptrs = at(self.off_plain_part), at(self.off_plain_out)
        self.sum_ptrs = at(self.off_sum)
        self.sum_flag_ptrs = at(self.off_sum_flags)
        self.sum_part_ptrs, self.sum_out_ptrs = at(self.off_sum_part), at(self.off_sum_out)
        if self.nvls_rows:
            self._nvls_setup(min(R, self.nvls_rows), H)

    def _nvls_setup(self, R: int, H: int) -> None:
        """Collective: the multicast-bound block of the NVLS protocol (see the module doc)."""
        ok, err = 1, ""
        blk = handle = None
        try:
            import torch.distributed._symmetric_memory as symm

            if (H // 8) % self.world:
                raise ValueError(f"hidden {H} does not split into {self.world} column slices of 16 bytes")
            nbytes = _up(2 * FAR_CTAS * 4) + 2 * _up(R * H * 2)
            blk = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
            handle = symm.rendezvous(blk, self.group if self.group is not None else dist.group.WORLD)
            if not handle.has_multicast_support or not handle.multicast_ptr:
                raise RuntimeError("no NVSwitch multicast support on this group")
        except Exception as e:  # any rank without multicast turns NVLS off for all
            ok, err = 0, f"{type(e).__name__}: {e}"
        agree = torch.tensor([ok], dtype=torch.int32, device=self.device)
        dist.all_reduce(agree, op=dist.ReduceOp.MIN, group=self.group)
        if not int(agree.item()):
            self.nvls, self.nvls_error = None, err or "a peer has no NVSwitch multicast support"
            return
        blk.zero_()
        base = blk.data_ptr()
        mc = handle.multicast_ptr + (base - handle.buffer_ptrs[handle.rank])
        o_part = _up(2 * FAR_CTAS * 4)
        o_out = o_part + _up(R * H * 2)
        self.nvls = {"block": blk, "handle": handle, "rows": R, "flags": base, "part": base + o_part,
                     "out": base + o_out, "mc": [mc + o_part, mc + o_out, mc]}
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        if not self._base:
            return
        self.nvls = None
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
    def protocol_for(self, rows: int) -> int:
        if rows <= self.oneshot_rows:
            return ONESHOT
        if self.nvls is not None and rows <= self.nvls["rows"]:
            return NVLS
        if rows <= self.ll_cap:
            return TWOSHOT
        return PLAIN

    def push_target(self, rows: int):
        """Where a row-parallel GEMM's epilogue pushes its partial sums for an all-reduce of
        `rows` rows: (protocol, receive buffers of every rank, epoch counter), or None when
        that row count takes the plain or NVLS protocol (the GEMM then writes its output
        locally)."""
        if rows > self.max_rows or not self.push:
            return None
        proto = self.protocol_for(rows)
        if proto == ONESHOT:
            return proto, self.one_ptrs, self.epoch[_E_ONE:_E_ONE + 1]
        if proto == TWOSHOT:
            return proto, self.ll_part_ptrs, self.epoch[_E_TWO:_E_TWO + 1]
        return None

    def allreduce_add_rmsnorm(self, delta, n_terms: int, row_stride: int, term_stride: int, hidden_buf,
                              norm_w, eps: float, rows: int, xq, xsf, term_index=None, term_scale=None,
                              protocol: int | None = None, pushed: bool = False) -> None:
        """hidden_buf[:rows] += sum over ranks of the local term sums; then RMSNorm(norm_w)
        -> MXFP8 (xq, xsf).  Every rank ends with the same bf16 residual stream.  With
        ``pushed`` the local sums were already delivered by a GEMM epilogue
        (``push_target``) and ``delta`` is not read."""
        H = hidden_buf.shape[-1]
        if rows > self.max_rows or H != self.hidden:
            raise ValueError(f"fused all-reduce reserved for {self.max_rows}x{self.hidden}, got {rows}x{H}")
        proto = self.protocol_for(rows) if protocol is None else protocol
        mc = []
        if proto == NVLS:
            nv = self.nvls
            if nv is None or rows > nv["rows"] or pushed:
                raise ValueError("NVLS all-reduce: no multicast block for these rows (or a pushed call)")
            here = lambda p: [p if r == self.rank else 0 for r in range(self.world)]  # noqa: E731
            part, out, flags, e, mc = here(nv["part"]), here(nv["out"]), here(nv["flags"]), _E_NVLS, nv["mc"]
        elif proto == ONESHOT:
            part, out, flags, e = self.one_ptrs, [], [], _E_ONE
        elif proto == TWOSHOT:
            if rows > self.ll_cap:
                raise ValueError(f"LL two-shot buffers hold {self.ll_cap} rows, got {rows}")
            part, out, flags, e = self.ll_part_ptrs, self.ll_out_ptrs, [], _E_TWO
        else:
            part, out, flags, e = self.plain_part_ptrs, self.plain_out_ptrs, self.flag_ptrs, _E_PLAIN
        self.C.fused_allreduce_norm(self.rank, self.world, proto, delta, n_terms, row_stride, term_stride, part, out,
                                    flags, self.epoch[e:e + 1], self.grid[e:e + 1], hidden_buf, norm_w, 1.0, eps,
                                    rows, None, xq, xsf, self.err, term_index, term_scale, self.timeout_ms,
                                    pushed=pushed, mc=mc)

    def allreduce_sum(self, t: torch.Tensor) -> None:
        """In-place fp32 sum over ranks of t [rows, hidden] (mHC sublayer outputs): one-shot
        LL lines over NVLink up to ``sum_rows`` rows, the plain two-shot above (prefill)."""
        ok = t.dim() == 2 and t.shape[1] == self.hidden and t.dtype == torch.float32 and t.is_contiguous()
        if ok and t.shape[0] <= self.sum_rows:
            self.C.allreduce_sum_f32(self.rank, self.world, t, t.shape[0], self.sum_rows, self.sum_ptrs,
                                     self.epoch[_E_SUM:_E_SUM + 1], self.grid[_E_SUM:_E_SUM + 1], self.err,
                                     self.timeout_ms)
            return
        if ok and t.shape[0] <= self.max_rows:
            self.C.allreduce_sum_f32(self.rank, self.world, t, t.shape[0], self.max_rows, self.sum_ptrs,
                                     self.epoch[_E_SUMP:_E_SUMP + 1], self.grid[_E_SUMP:_E_SUMP + 1], self.err,
                                     self.timeout_ms, part=self.sum_part_ptrs, out=self.sum_out_ptrs,
                                     flags=self.sum_flag_ptrs)
            return
        self.nccl.allreduce_sum(t)

    def argmax_allreduce(self, keys, rows: int, tiles: int, id_offset: int, out_ids, out_vals) -> None:
        """Global greedy token per row from per-tile packed keys of this rank's vocab shard
        (one kernel: tile reduction, id rebase, LL exchange, max over ranks)."""
        if rows > self.max_rows:
            raise ValueError(f"fused argmax reserved for {self.max_rows} rows, got {rows}")
        self.C.allreduce_argmax(self.rank, self.world, rows, self.max_rows, keys, tiles, id_offset, self.argmax_ptrs,
                                self.epoch[_E_ARGMAX:_E_ARGMAX + 1], self.grid[_E_ARGMAX:_E_ARGMAX + 1], out_ids,
                                out_vals, self.err, self.timeout_ms)

    def reset(self) -> None:
        """Collective: bring every rank's protocol state back to the start (after a call
        that timed out left the ranks' epochs apart).  Waits for all local work, clears
        the symmetric block, epochs, counters and the error word, then barriers so no rank
        pushes into a peer's block before that peer has cleared it."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        if self._base:
            self.C.symm_memset(self._base, self.nbytes)
        if self.nvls is not None:
            self.nvls["block"].zero_()
        self.epoch.zero_()
        self.grid.zero_()
        self.err.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
