"""Expert-parallel dispatch/combine kernels (csrc/kernels/ep.cu) against an fp32 restatement.

The single-GPU case runs the full protocol with one rank (every expert local); the
two-rank case runs one process per GPU over NCCL for the handle exchange and the
kernels over NVLink peer memory (skipped with fewer than two GPUs).
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, T, H, E, K, rank):
    g = torch.Generator().manual_seed(seed * 100 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32) if T else \
        torch.zeros(0, K, dtype=torch.int32)
    if T > 3:
        ids[3, K - 1] = -1  # a pair with no expert
    w = torch.rand(T, K, generator=g)
    return x, ids, w


def _expert_scale(e):
    return 1.0 + 0.01 * e


def _check_and_combine(ep, xs, idss, ws, rank, world, E, K, H):
    """Checks this rank's receive buffer, runs the combine with y = dequant(row) *
    scale(expert) and compares with the fp32 restatement."""
    from zstep_b200.ops import mx

    dev = ep.device
    local = E // world
    # Expected counts per local expert over all sources.
    counts = torch.zeros(local, dtype=torch.int64)
    for s in range(world):
        ids = idss[s]
        for el in range(local):
            counts[el] += int((ids == rank * local + el).sum())
    torch.cuda.synchronize()
    assert ep.check_error() == 0
    assert ep.group_count.cpu().tolist() == counts.tolist()
    seg = ((counts + 127) // 128) * 128
    off = torch.cumsum(seg, 0) - seg
    assert ep.group_offset.cpu().tolist() == off.tolist()
    ch = (counts + ep.chunk_rows - 1) // ep.chunk_rows
    assert ep.chunk_prefix.cpu().tolist() == (torch.cumsum(ch, 0) - ch).tolist() + [int(ch.sum())]
    R = int(ep.recv_rows.item())
    assert R == int(seg.sum())
    meta = ep.recv_meta[:R].cpu()
    q = ep.recv_q[:R].cpu()
    codes = mx.codes_from_atoms(ep.recv_sf.cpu(), ep.recv_cap, H)[:R]
    quant = [mx.quantize(xs[s].float()) for s in range(world)]
    seen = set()
    row_expert = torch.full((R,), -1, dtype=torch.int64)
    for el in range(local):
        lo, n = int(off[el]), int(counts[el])
        row_expert[lo:lo + n] = rank * local + el
        assert (meta[lo + n: lo + int(seg[el]), 0] == -1).all()
        prev_src = -1
        for i in range(lo, lo + n):
            code = int(meta[i, 0])
            s, pair = code >> 24, code & 0xFFFFFF
            t, k = divmod(pair, K)
            assert s >= prev_src  # sources in rank order inside a segment
            prev_src = s
            assert int(idss[s][t, k]) == rank * local + el
            assert (s, t, k) not in seen
            seen.add((s, t, k))
            assert torch.equal(q[i], quant[s][0][t]), (i, s, t, k)
            assert torch.equal(codes[i], quant[s][1][t])
            assert abs(torch.tensor(int(meta[i, 1]), dtype=torch.int32).view(torch.float32).item()
                       - float(ws[s][t, k])) < 1e-7
    assert len(seen) == int(counts.sum())
    # Expert outputs: dequantized row times a per-expert scale.
    deq = mx.dequantize(ep.recv_q[:R], mx.codes_from_atoms(ep.recv_sf, ep.recv_cap, H)[:R])
    scale = torch.tensor([_expert_scale(int(e)) if e >= 0 else 0.0 for e in row_expert], device=dev)
    y = (deq * scale[:, None]).to(torch.bfloat16).contiguous()
    T = xs[rank].shape[0]
    res = (0.1 * torch.randn(T, H)).to(torch.bfloat16)
    out = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
    ids_d, w_d = idss[rank].to(dev), ws[rank].to(dev).contiguous()
    ep.combine(y, ids_d, w_d, out, residual=res.to(dev))
    torch.cuda.synchronize()
    assert ep.check_error() == 0
    qx, cx = quant[rank]
    xr = mx.dequantize(qx, cx)
    want = res.float().clone()
    for t in range(T):
        for k in range(K):
            e = int(idss[rank][t, k])
            if e >= 0:
                v = (xr[t] * _expert_scale(e)).to(torch.bfloat16).float()
                want[t] += float(ws[rank][t, k]) * v
    torch.testing.assert_close(out.float().cpu(), want, atol=3e-2, rtol=2e-2)


def _run(ep, rank, world, E, K, H, cases):
    dev = ep.device
    for seed, T in cases:
        print(f"ep case seed={seed} tokens={T} rank={rank}", flush=True)
        xs, idss, ws = zip(*[_inputs(seed, T, H, E, K, s) for s in range(world)])
        ep.dispatch(xs[rank].to(dev), idss[rank].to(dev), ws[rank].to(dev).contiguous())
        _check_and_combine(ep, xs, idss, ws, rank, world, E, K, H)


def test_ep_dispatch_combine_single_rank():
    from zstep_b200.parallel.ep import EpAllToAll

    E, K, H = 64, 4, 1024
    ep = EpAllToAll("cuda:0", num_experts=E, hidden=H, top_k=K, max_tokens=256)
    try:
        _run(ep, 0, 1, E, K, H, [(1, 200), (2, 7), (3, 0), (4, 256)])
    finally:
        ep.close()


def test_ep_overflow_is_reported_and_drops_rows():
    from zstep_b200.parallel.ep import EpAllToAll

    E, K, H = 8, 2, 512
    ep = EpAllToAll("cuda:0", num_experts=E, hidden=H, top_k=K, max_tokens=512, recv_cap=256)
    try:
        x = torch.randn(300, H, device="cuda").to(torch.bfloat16)
        ids = torch.zeros(300, K, dtype=torch.int32, device="cuda")
        ids[:, 1] = 1  # 300 rows for expert 0 and 300 for expert 1 > 256
        w = torch.ones(300, K, device="cuda")
        ep.dispatch(x, ids, w)
        torch.cuda.synchronize()
        assert ep.check_error() == 3
        assert int(ep.recv_rows.item()) == 0 and int(ep.chunk_prefix[-1].item()) == 0
        out = torch.full((300, H), 7.0, dtype=torch.bfloat16, device="cuda")
        ep.err.zero_()
        ep.combine(torch.zeros(1, H, dtype=torch.bfloat16, device="cuda"), ids, w, out)
        torch.cuda.synchronize()
        assert ep.check_error() == 0 and int(out.abs().max().item()) == 0  # every pair dropped
    finally:
        ep.close()


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=datetime.timedelta(seconds=60))
        from zstep_b200.parallel.ep import EpAllToAll

        E, K, H = 32, 4, 1024
        ep = EpAllToAll(f"cuda:{rank}", num_experts=E, hidden=H, top_k=K, max_tokens=128, timeout_ms=5000)
        _run(ep, rank, world, E, K, H, [(5, 100), (6, 1), (7, 128)])
        ep.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_dispatch_combine_two_ranks():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
