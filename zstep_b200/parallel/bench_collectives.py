"""Collective microbenchmark: fused NVLink all-reduce + residual + RMSNorm + MXFP8 and the
cross-rank argmax, against the NCCL baseline, at hidden 2048 over a range of row counts.

Run one rank per GPU::

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port 29555 -m zstep_b200.parallel.bench_collectives

Each case captures `calls` back-to-back calls in one CUDA graph, replays it `reps` times
between CUDA events and reports the median per call, max over ranks.  Roofline for the
all-reduce: a two-shot all-reduce moves 2 (W-1)/W * M * H * 2 bytes out of every GPU, so
the bound is that over the measured 770 GB/s per-direction peer bandwidth.
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
from .fused import FusedCollectives

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
    H, R = 2048, 4096
    fused = FusedCollectives(dev, max_rows=R, hidden=H)
    nccl = NcclCollectives(None, dev)
    w = torch.randn(H, device=dev).to(torch.bfloat16)
    hidden = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
    delta = (0.01 * torch.randn(R, H, device=dev)).to(torch.bfloat16)
    xq = torch.zeros(R, H, dtype=torch.uint8, device=dev)
    xsf = torch.zeros(mx.atoms_bytes(R, H), dtype=torch.uint8, device=dev)
    results = []
    for m in (1, 8, 32, 128, 256, 1024, 4096):
        row = {"op": "allreduce_add_rmsnorm_mxfp8", "world": world, "rows": m, "hidden": H}
        calls = 50 if m <= 256 else 10
        for name, coll in (("fused", fused), ("nccl", nccl)):
            row[f"{name}_us"] = round(1000 * _time_graph(
                lambda: coll.allreduce_add_rmsnorm(delta, 1, H, 0, hidden, w, 1e-6, m, xq, xsf), calls, 10), 2)
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
    if rank == 0:
        for r in results:
            print(json.dumps(r), flush=True)
    fused.close()
    dist.destroy_process_group()
    del C


if __name__ == "__main__":
    main()
