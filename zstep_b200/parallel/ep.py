"""Expert-parallel MoE all-to-all over NVLink peer memory (dispatch + combine).

Rank ``r`` of ``W`` owns the routed experts ``[r * E / W, (r + 1) * E / W)``.  ``dispatch``
quantizes every local token row to MXFP8 once and stores it, with its scale atoms and a
metadata word, straight into the grouped receive buffer of each rank that owns one of
its top-k experts; on return the local buffer is the A operand of the grouped expert
GEMMs (segments per local expert, 128-row aligned, the format of the single-GPU router).
``combine`` sends each received row's expert output back to its source, which sums its
top-k outputs in k order with the routing weights (+ residual).  Both are single
cooperative sm_100a kernels (csrc/kernels/ep.cu) over a symmetric block shared through
CUDA IPC; every wait is bounded by ``coll_timeout_ms``.

``NcclEp`` is the library baseline of the same two operations (``all_to_all_single``
with per-rank splits).  ``reference_dispatch`` / ``reference_combine`` are the fp32
restatement the tests compare against.

Reference parity: the reference keeps experts tensor-parallel over host shared memory
and has no expert all-to-all; the routing format follows its moe_align step
(csrc/qwen35_ops_kernels.cu:26) and the EP=8 DeepSeek configuration it serves
(worker/zstep_worker/models/deepseek_v41.py).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import mx

_ALIGN = 256


def _up(x: int, a: int = _ALIGN) -> int:
    return (x + a - 1) // a * a


def ep_layout(world: int, num_experts: int, hidden: int, top_k: int, max_tokens: int,
              recv_cap: int) -> dict:
    """Byte offsets of the symmetric block (identical on every rank)."""
    off = {"flags": 0}
    off["counts"] = _up(64 * 4)
    off["q"] = off["counts"] + _up(world * num_experts * 8)
    off["sf"] = off["q"] + _up(recv_cap * hidden)
    off["meta"] = off["sf"] + _up(mx.atoms_bytes(recv_cap, hidden))
    off["comb"] = off["meta"] + _up(recv_cap * 8)
    off["nbytes"] = off["comb"] + _up(max_tokens * top_k * hidden * 2)
    return off


def default_recv_cap(world: int, num_experts: int, top_k: int, max_tokens: int) -> int:
    """Worst case: every pair of every rank lands on one rank, plus each local segment's
    128-row alignment."""
    local = num_experts // world
    return (world * max_tokens * top_k + local * 127 + 127) // 128 * 128


class EpAllToAll:
    def __init__(self, device, num_experts: int, hidden: int, top_k: int, max_tokens: int, group=None,
                 recv_cap: int | None = None, chunk_rows: int = 128, timeout_ms: int | None = None):
        from ..ops import _ext
        from ..utils.env import runtime_config

        self.C = _ext.load()
        self.device = torch.device(device)
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if self.world > 8:
            raise ValueError("expert all-to-all supports up to 8 ranks (one NVLink domain)")
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        if hidden % 512:
            raise ValueError("hidden must be a multiple of 512")
        self.E, self.H, self.K, self.T = num_experts, hidden, top_k, max_tokens
        self.local_experts = num_experts // self.world
        self.expert_begin = self.rank * self.local_experts
        self.recv_cap = recv_cap or default_recv_cap(self.world, num_experts, top_k, max_tokens)
        self.chunk_rows = chunk_rows
        self.timeout_ms = runtime_config().coll_timeout_ms if timeout_ms is None else timeout_ms
        self.off = ep_layout(self.world, num_experts, hidden, top_k, max_tokens, self.recv_cap)
        self.offs = [self.off[k] for k in ("flags", "counts", "q", "sf", "meta", "comb")]
        dev = self.device
        self.cnt = torch.zeros(num_experts, dtype=torch.int32, device=dev)
        self.pair_slot = torch.zeros(max_tokens * top_k, dtype=torch.int32, device=dev)
        self.bar = torch.zeros(1, dtype=torch.int64, device=dev)
        self.epoch = torch.zeros(2, dtype=torch.int32, device=dev)
        self.group_count = torch.zeros(self.local_experts, dtype=torch.int32, device=dev)
        self.group_offset = torch.zeros(self.local_experts, dtype=torch.int32, device=dev)
        self.chunk_prefix = torch.zeros(self.local_experts + 1, dtype=torch.int32, device=dev)
        self.recv_rows = torch.zeros(1, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            self._base = self.C.symm_alloc(self.off["nbytes"])
            if self.world > 1:
                handle = self.C.ipc_handle(self._base)
                handles = [None] * self.world
                dist.all_gather_object(handles, handle, group=group)
                self._peers = [self._base if r == self.rank else self.C.ipc_open(handles[r])
                               for r in range(self.world)]
            else:
                self._peers = [self._base]
        torch.cuda.synchronize(dev)
        if self.world > 1:
            dist.barrier(group=group)
        base, di = self._base, dev.index or 0
        # Views of the local receive side (the grouped GEMM's A operand) and return buffer.
        self.recv_q = self.C.tensor_from_ptr(base + self.off["q"], [self.recv_cap, hidden], torch.uint8, di)
        self.recv_sf = self.C.tensor_from_ptr(base + self.off["sf"], [mx.atoms_bytes(self.recv_cap, hidden)],
                                              torch.uint8, di)
        self.recv_meta = self.C.tensor_from_ptr(base + self.off["meta"], [self.recv_cap, 2], torch.int32, di)

    def close(self) -> None:
        if not getattr(self, "_base", 0):
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer may still write into our block
            for r, p in enumerate(self._peers):
                if r != self.rank:
                    self.C.ipc_close(p)
            dist.barrier(group=self.group)
        self.recv_q = self.recv_sf = self.recv_meta = None
        self.C.symm_free(self._base)
        self._base, self._peers = 0, []

    def check_error(self) -> int:
        return int(self.err.item())

    def _call(self, which: int, tokens: int, topk_ids, topk_w, x=None, y=None, residual=None, out=None):
        if tokens > self.T:
            raise ValueError(f"expert all-to-all reserved for {self.T} tokens, got {tokens}")
        self.C.ep_call(which, self.rank, self.world, tokens, self.T, self.H, self.K, self.E, self.recv_cap,
                       self.chunk_rows, topk_ids, topk_w, x, self._peers, self.offs, self.cnt, self.pair_slot,
                       self.bar, self.epoch, self.group_count, self.group_offset, self.chunk_prefix,
                       self.recv_rows, y, 0 if y is None else y.stride(0), residual, out, self.err,
                       self.timeout_ms)

    def dispatch(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor) -> None:
        """x bf16 [tokens, hidden]; topk_ids int32 / topk_w f32 [tokens, top_k] (global ids).
        Afterwards ``recv_q``/``recv_sf`` hold the local experts' rows and ``group_count``,
        ``group_offset``, ``chunk_prefix``, ``recv_rows`` describe them (collective)."""
        self._call(0, x.shape[0], topk_ids, topk_w, x=x)

    def combine(self, y: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, out: torch.Tensor,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        """y bf16 [recv rows, hidden] = expert outputs in receive order; out[t] = residual[t]
        + sum_k w[t, k] * y(row of (t, k)) in k order (collective).  Calls alternate
        dispatch, combine: a dispatch is what tells every rank that the previous combine's
        return buffers have been read."""
        self._call(1, out.shape[0], topk_ids, topk_w, y=y, residual=residual, out=out)
        return out


class NcclEp:
    """Library baseline: per-destination sort, ``all_to_all_single`` of the counts, then
    of the MXFP8 rows (+ scale codes), and back for the bf16 expert outputs."""

    def __init__(self, num_experts: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = num_experts
        self.local = num_experts // self.world

    def dispatch(self, xq: torch.Tensor, xcode: torch.Tensor, topk_ids: torch.Tensor):
        T, K = topk_ids.shape
        dest = (topk_ids.reshape(-1) // self.local).long()
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        tok = order // K
        payload = torch.cat([xq[tok], xcode[tok]], dim=1)
        recv = torch.empty(sum(rc), payload.shape[1], dtype=payload.dtype, device=payload.device)
        dist.all_to_all_single(recv, payload, rc, sc, group=self.group)
        return recv, order, sc, rc

    def combine(self, y: torch.Tensor, order, sc, rc, topk_w: torch.Tensor) -> torch.Tensor:
        T, K = topk_w.shape
        back = torch.empty(sum(sc), y.shape[1], dtype=y.dtype, device=y.device)
        dist.all_to_all_single(back, y, sc, rc, group=self.group)
        pair = torch.empty_like(back)
        pair[order] = back
        return (pair.view(T, K, -1).float() * topk_w.unsqueeze(-1)).sum(1).to(y.dtype)


# ----------------------------------------------------------------------- fp32 reference
def reference_dispatch(xs: list[torch.Tensor], ids: list[torch.Tensor], num_experts: int, world: int) -> list[dict]:
    """Per receiving rank: for each local expert, the (source, token, k) pairs it gets
    (sources in rank order; order inside one source is free) and the quantized rows."""
    local = num_experts // world
    out = []
    for d in range(world):
        experts = []
        for el in range(local):
            e = d * local + el
            pairs = []
            for s in range(world):
                hit = (ids[s] == e).nonzero().tolist()
                pairs.append([(s, t, k) for t, k in hit])
            experts.append(pairs)
        out.append({"experts": experts})
    return out


def reference_combine(y_of_pair, ids: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
    """out[t] = residual[t] + sum_k w[t, k] * y_of_pair(t, k) (fp32; skipped where ids < 0)."""
    T, K = ids.shape
    acc = residual.float().clone() if residual is not None else None
    rows = []
    for t in range(T):
        r = acc[t] if acc is not None else 0.0
        for k in range(K):
            if int(ids[t, k]) >= 0:
                r = r + float(w[t, k]) * y_of_pair(t, k)
        rows.append(r)
    return torch.stack(rows)
