"""Collective microbenchmark: fused NVLink all-reduce + residual + RMSNorm + MXFP8, the
cross-rank argmax, and the expert-parallel dispatch / combine all-to-all, against the NCCL
baseline over a range of row counts.

Run one rank per GPU::

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port 29555 -m zstep_b200.parallel.bench_collectives

Each case captures `calls` back-to-back calls in one CUDA graph, replays it `reps` times
between CUDA events and reports the median per call, max over ranks.  Roofline for the
all-reduce: a two-shot all-reduce moves 2 (W-1)/W * M * H * 2 bytes out of every GPU, so
the bound is that over the measured 770 GB/s per-direction peer bandwidth.  Every protocol
of the fused kernel (one-shot LL, two-shot LL, two-shot plain, and NVLS when
``ZSTEP_COLL_NVLS_ROWS`` enables it and the group has multicast support) is timed where it
applies; ``fused_us`` is the one the runner picks for that row count.  Expert
all-to-all (hidden 4096, top-8 of 256 experts, uniform random routing): every pair whose
expert lives on another rank moves one MXFP8 row (hidden + hidden/32 + 8 bytes) out on
dispatch and one bf16 row (2 * hidden bytes) back on combine; the NCCL baseline is
``all_to_all_single`` with per-rank splits (host-synchronised, timed eagerly).
"""

from __future__ import annotations

import datetime
import json
import statistics

import torch
import torch.distributed as dist

from ..ops import _ext, mx
from .collectives import NcclCollectives
from ..utils.env import dist_env
from .fused import FAR_ONESHOT_ROWS, NVLS, ONESHOT, PLAIN, TWOSHOT, FusedCollectives

LINK_GBS = 770.0  # measured peer copy bandwidth per direction per GPU on this pool


def _time_graph(body, calls: int, reps: int) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        body()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls):
            body()
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) / calls)
    torch.cuda.synchronize()
    dist.barrier()
    del g
    t = torch.tensor([statistics.median(ts)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    de = dist_env()
    rank, world, local = de.rank, de.world_size, de.local_rank
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    C = _ext.load()
    R = 4096
    fused = FusedCollectives(dev)
    nccl = NcclCollectives(None, dev)
    results = []
    if fused.nvls_rows and rank == 0:
        print(json.dumps({"nvls_requested_rows": fused.nvls_rows}), flush=True)
    names = {ONESHOT: "oneshot", TWOSHOT: "twoshot_ll", PLAIN: "twoshot_plain", NVLS: "nvls"}
    for H in (2048, 4096):
        fused.reserve(R, H)
        if fused.nvls_rows and fused.nvls is None and rank == 0:
            print(json.dumps({"nvls_unavailable": fused.nvls_error}), flush=True)
        w = torch.randn(H, device=dev).to(torch.bfloat16)
        hidden = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
        delta = (0.01 * torch.randn(R, H, device=dev)).to(torch.bfloat16)
        xq = torch.zeros(R, H, dtype=torch.uint8, device=dev)
        xsf = torch.zeros(mx.atoms_bytes(R, H), dtype=torch.uint8, device=dev)
        for m in (1, 8, 32, 64, 128, 256, 512, 1024, 4096):
            row = {"op": "allreduce_add_rmsnorm_mxfp8", "world": world, "rows": m, "hidden": H,
                   "auto_protocol": names[fused.protocol_for(m)]}
            calls = 50 if m <= 256 else 10
            for proto in (ONESHOT, TWOSHOT, PLAIN, NVLS):
                if (proto == ONESHOT and m > FAR_ONESHOT_ROWS) or (proto == TWOSHOT and m > fused.ll_cap):
                    continue
                if proto == NVLS and (fused.nvls is None or m > fused.nvls["rows"]):
                    continue
                row[f"{names[proto]}_us"] = round(1000 * _time_graph(
                    lambda: fused.allreduce_add_rmsnorm(delta, 1, H, 0, hidden, w, 1e-6, m, xq, xsf, protocol=proto),
                    calls, 10), 2)
            row["fused_us"] = row[f"{row['auto_protocol']}_us"]
            row["nccl_us"] = round(1000 * _time_graph(
                lambda: nccl.allreduce_add_rmsnorm(delta, 1, H, 0, hidden, w, 1e-6, m, xq, xsf), calls, 10), 2)
            link_bytes = 2 * (world - 1) / world * m * H * 2
            bound_us = link_bytes / (LINK_GBS * 1e3)
            row["nvlink_bytes_per_gpu"] = int(link_bytes)
            row["roofline_us"] = round(bound_us, 3)
            row["fused_frac_of_roofline"] = round(bound_us / row["fused_us"], 4)
            row["speedup_vs_nccl"] = round(row["nccl_us"] / row["fused_us"], 3)
            results.append(row)
    # Vocab-sharded lm_head argmax exchange (256 rows, 8 local tiles of 128 ids).
    for rows in (1, 256):
        tiles = 8
        keys = torch.randint(0, 2**62, (rows, tiles), dtype=torch.int64, device=dev)
        ids = torch.zeros(rows, dtype=torch.int32, device=dev)
        vals = torch.zeros(rows, dtype=torch.float32, device=dev)
        row = {"op": "argmax_allreduce", "world": world, "rows": rows}
        for name, coll in (("fused", fused), ("nccl", nccl)):
            row[f"{name}_us"] = round(1000 * _time_graph(
                lambda: coll.argmax_allreduce(keys, rows, tiles, rank * 1024, ids, vals), 50, 10), 2)
        row["speedup_vs_nccl"] = round(row["nccl_us"] / row["fused_us"], 3)
        results.append(row)
    assert fused.check_error() == 0, fused.check_error()
    results += bench_ep(rank, world, dev)
    if rank == 0:
        for r in results:
            print(json.dumps(r), flush=True)
    fused.close()
    dist.destroy_process_group()
    del C


def _time_eager(body, reps: int) -> float:
    body()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        body()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    t = torch.tensor([statistics.median(ts)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bench_ep(rank: int, world: int, dev, H: int = 4096, E: int = 256, K: int = 8,
             token_counts=(1, 8, 64, 256, 1024, 4096)) -> list[dict]:
    from .ep import EpAllToAll, NcclEp

    T_max = max(token_counts)
    # Receive capacity: twice the average load plus every segment's alignment (overflow is
    # reported, never written past); y covers all of it.
    ep = EpAllToAll(dev, num_experts=E, hidden=H, top_k=K, max_tokens=T_max, recv_cap=2 * T_max * K + E * 128)
    nccl = NcclEp(E)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    x_all = torch.randn(T_max, H, device=dev, generator=g).to(torch.bfloat16)
    ids_all = torch.rand(T_max, E, device=dev, generator=g).topk(K, dim=1).indices.to(torch.int32).contiguous()
    w_all = torch.rand(T_max, K, device=dev, generator=g).contiguous()
    y = torch.randn(ep.recv_cap, H, device=dev, dtype=torch.bfloat16)
    out = torch.empty(T_max, H, dtype=torch.bfloat16, device=dev)
    results = []
    for T in token_counts:
        x, ids, w = x_all[:T], ids_all[:T].contiguous(), w_all[:T].contiguous()
        remote = int(((ids // (E // world)) != rank).sum())
        pairs = torch.tensor([remote], device=dev)
        dist.all_reduce(pairs, op=dist.ReduceOp.MAX)  # the busiest rank bounds the step
        remote = int(pairs.item())
        row = {"op": "ep_dispatch_combine", "world": world, "tokens": T, "hidden": H, "experts": E, "top_k": K}
        calls = 20 if T <= 256 else 5
        row["fused_dispatch_us"] = round(1000 * _time_graph(lambda: ep.dispatch(x, ids, w), calls, 10), 2)
        ep.dispatch(x, ids, w)
        row["fused_combine_us"] = round(1000 * _time_graph(
            lambda: ep.combine(y, ids, w, out[:T]), calls, 10), 2)
        if world > 1:
            xq, xc = mx.quantize(x.float())
            state = {}

            def nd():
                state["r"] = nccl.dispatch(xq, xc, ids)

            row["nccl_dispatch_us"] = round(1000 * _time_eager(nd, 10), 2)
            recv, order, sc, rc = state["r"]
            yb = torch.randn(recv.shape[0], H, device=dev).to(torch.bfloat16)
            row["nccl_combine_us"] = round(1000 * _time_eager(lambda: nccl.combine(yb, order, sc, rc, w), 10), 2)
        d_bytes = remote * (H + H // 32 + 8)
        c_bytes = remote * 2 * H
        row["nvlink_bytes_dispatch"] = d_bytes
        row["nvlink_bytes_combine"] = c_bytes
        if d_bytes:
            row["dispatch_frac_of_roofline"] = round(d_bytes / (LINK_GBS * 1e3) / row["fused_dispatch_us"], 4)
            row["combine_frac_of_roofline"] = round(c_bytes / (LINK_GBS * 1e3) / row["fused_combine_us"], 4)
        results.append(row)
    torch.cuda.synchronize()
    assert ep.check_error() == 0, ep.check_error()
    ep.close()
    return results


if __name__ == "__main__":
    main()
