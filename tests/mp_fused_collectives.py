"""Worker for tests/test_multigpu.py: run under torch.distributed.run, one rank per GPU.

Checks the fused NVLink collectives (csrc/kernels/collective.cu) against plain PyTorch
fp32 math on the same data, eagerly and under CUDA-graph replay, then a tensor-parallel
Qwen3.5 runner against the single-GPU fp32 reference with the same MXFP8 quantization.
Exit code 0 = every check passed on this rank."""

import datetime
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from zstep_b200.ops import mx  # noqa: E402
from zstep_b200.parallel.fused import FusedCollectives  # noqa: E402


def _expected_residual(resid0, allp, rows, world, terms):
    """bf16(resid + sum_r bf16(sum_t part_r[t])) summed in rank order."""
    acc = resid0[:rows].float()
    for r in range(world):
        s = allp[r][0, :rows].clone()
        for t in range(1, terms):
            s = s + allp[r][t, :rows]
        acc = acc + s.to(torch.bfloat16).float()
    return acc.to(torch.bfloat16)


def check_allreduce(coll, C, rank, world, dev):
    """Every protocol (one-shot / two-shot LL / plain) at several row counts, against the
    rank-ordered sum; rows past `rows` must stay untouched."""
    from zstep_b200.parallel.fused import ONESHOT, PLAIN, TWOSHOT

    H, R = 2048, 96
    coll.reserve(R, H)
    g = torch.Generator(device=dev).manual_seed(100)
    resid0 = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.rand(H, generator=g, device=dev) + 0.5).to(torch.bfloat16)
    terms = 3
    # Each rank's split-K partials, [terms, R, H] f32 (rank-specific data).
    allp = [torch.randn(terms, R, H, generator=g, device=dev) for _ in range(world)]
    delta = allp[rank].contiguous()
    for rows in (R, 37, 1, 5, 8, 64):
        for proto in (ONESHOT, TWOSHOT, PLAIN):
            if proto == ONESHOT and rows > 64:
                continue
            for rep in range(2):  # the second call reuses the buffers with the next epoch
                hidden = resid0.clone()
                xq = torch.zeros(128 * ((R + 127) // 128), H, dtype=torch.uint8, device=dev)
                xsf = torch.zeros(mx.atoms_bytes(xq.shape[0], H), dtype=torch.uint8, device=dev)
                coll.allreduce_add_rmsnorm(delta, terms, H, R * H, hidden, w, 1e-6, rows, xq, xsf, protocol=proto)
                torch.cuda.synchronize()
                assert coll.check_error() == 0, (rows, proto)
                exp = _expected_residual(resid0, allp, rows, world, terms)
                assert torch.equal(hidden[:rows], exp), f"residual mismatch rows={rows} protocol={proto}"
                assert torch.equal(hidden[rows:], resid0[rows:]), "rows beyond `rows` were touched"
            # Normed + quantized output vs the single-GPU norm kernel on the expected residual.
            h2 = exp.clone()
            xq2, xsf2 = torch.zeros_like(xq), torch.zeros_like(xsf)
            C.add_rmsnorm_quant(h2, None, 0, H, H, w, 1.0, 1e-6, rows, None, xq2, xsf2)
            assert torch.equal(xq[:rows], xq2[:rows]), f"MXFP8 rows differ rows={rows} protocol={proto}"
            assert torch.equal(mx.codes_from_atoms(xsf, rows, H), mx.codes_from_atoms(xsf2, rows, H))


def check_gemm_push(coll, C, rank, world, dev):
    """Row-parallel GEMM whose epilogue pushes bf16 LL lines into the all-reduce's receive
    slots (one-shot and two-shot), then the all-reduce without its send phase: equal to
    residual + the rank-ordered sum of each rank's bf16 GEMM output."""
    from zstep_b200.models.qwen35 import EPI_BF16, EPI_PUSH, pack_linear

    H, K = 2048, 512
    coll.reserve(96, H)
    g = torch.Generator(device=dev).manual_seed(600)
    ws = [(0.02 * torch.randn(H, K, generator=g, device=dev)).to(torch.bfloat16) for _ in range(world)]
    xs = [torch.randn(96, K, generator=g, device=dev).to(torch.bfloat16) for _ in range(world)]
    resid0 = torch.randn(96, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.rand(H, generator=g, device=dev) + 0.5).to(torch.bfloat16)
    pw = pack_linear(ws[rank], C)
    xq = torch.zeros(128, K, dtype=torch.uint8, device=dev)
    xsf = torch.zeros(mx.atoms_bytes(128, K), dtype=torch.uint8, device=dev)
    C.quant_mxf8(xs[rank], xq[:96], xsf)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    # Each rank's plain bf16 GEMM output (same kernel, local store) for the expectation.
    mine = torch.zeros(96, H, dtype=torch.bfloat16, device=dev)
    C.gemm_mxf8(pw.q, pw.sf, xq, xsf, K, pw.n_pad, H, 1, 96, None, None, None, EPI_BF16, mine, H, None, None, None,
                err, 0, 32, 1, 0, 1)
    outs = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(outs, mine)
    for rows in (5, 37, 96):
        tgt = coll.push_target(rows)
        assert tgt is not None
        proto, parts, ep = tgt
        hidden = resid0.clone()
        oq = torch.zeros(128, H, dtype=torch.uint8, device=dev)
        osf = torch.zeros(mx.atoms_bytes(128, H), dtype=torch.uint8, device=dev)
        dummy = torch.zeros(1, dtype=torch.float32, device=dev)
        C.gemm_mxf8(pw.q, pw.sf, xq, xsf, K, pw.n_pad, H, 1, rows, None, None, None, EPI_PUSH, dummy, H, None, None,
                    None, err, 0, 32, 1, 0, 1, push_part=parts, push_epoch=ep, push_rank=rank, push_mode=proto)
        coll.allreduce_add_rmsnorm(dummy, 1, H, 0, hidden, w, 1e-6, rows, oq, osf, protocol=proto, pushed=True)
        torch.cuda.synchronize()
        assert int(err.item()) == 0 and coll.check_error() == 0, (rows, proto)
        acc = resid0[:rows].float()
        for r in range(world):
            acc = acc + outs[r][:rows].float()
        assert torch.equal(hidden[:rows], acc.to(torch.bfloat16)), f"pushed all-reduce rows={rows} protocol={proto}"
        assert torch.equal(hidden[rows:], resid0[rows:])


def check_prefill_sized(coll, rank, world, dev):
    """A prefill-sized reduction (2048 rows, hidden 4096 as in the DeepSeek shape) takes the
    plain two-shot protocol; gathered MoE-style terms with weights."""
    H, R = 4096, 2048
    coll.close()
    coll.reserve(R, H)
    g = torch.Generator(device=dev).manual_seed(500)
    resid0 = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.rand(H, generator=g, device=dev) + 0.5).to(torch.bfloat16)
    rows_y = 3 * R
    ally = [torch.randn(rows_y, H, generator=g, device=dev).to(torch.bfloat16) for _ in range(world)]
    idx = torch.randint(0, rows_y, (R, 2), generator=g, device=dev).to(torch.int32)
    idx[::7, 1] = -1  # terms this rank did not produce
    scale = torch.rand(R, 2, generator=g, device=dev)
    hidden = resid0.clone()
    xq = torch.zeros(R, H, dtype=torch.uint8, device=dev)
    xsf = torch.zeros(mx.atoms_bytes(R, H), dtype=torch.uint8, device=dev)
    assert coll.protocol_for(R) == 2
    coll.allreduce_add_rmsnorm(ally[rank], 2, H, 0, hidden, w, 1e-6, R, xq, xsf, term_index=idx, term_scale=scale)
    torch.cuda.synchronize()
    assert coll.check_error() == 0
    acc = resid0.float()
    for r in range(world):
        y = ally[r].float()
        s = torch.zeros(R, H, device=dev)
        for t in range(2):
            ok = (idx[:, t] >= 0).unsqueeze(1)
            s = s + torch.where(ok, y[idx[:, t].clamp(min=0).long()] * scale[:, t:t + 1], torch.zeros_like(s))
        acc = acc + s.to(torch.bfloat16).float()
    torch.testing.assert_close(hidden.float(), acc.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2)
    coll.close()


def check_graph_replay(coll, rank, world, dev):
    """The kernels advance their own epochs: several replays of one graph (one call of each
    protocol in it) stay correct."""
    H, R = 2048, 64
    coll.reserve(96, H)
    g = torch.Generator(device=dev).manual_seed(200 + rank)
    delta = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
    hidden = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
    w = torch.ones(H, dtype=torch.bfloat16, device=dev)
    xq = torch.zeros(128, H, dtype=torch.uint8, device=dev)
    xsf = torch.zeros(mx.atoms_bytes(128, H), dtype=torch.uint8, device=dev)
    all_d = [torch.empty_like(delta) for _ in range(world)]
    dist.all_gather(all_d, delta)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        coll.allreduce_add_rmsnorm(delta, 1, H, 0, hidden, w, 1e-6, R, xq, xsf)  # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for proto in (0, 1, 2):
            coll.allreduce_add_rmsnorm(delta, 1, H, 0, hidden, w, 1e-6, R, xq, xsf, protocol=proto)
    hidden.zero_()
    exp = torch.zeros(R, H, device=dev).to(torch.bfloat16)
    for _ in range(4):
        graph.replay()
        for _ in range(3):  # the graph holds three all-reduces
            acc = exp.float()
            for d in all_d:
                acc = acc + d.float()
            exp = acc.to(torch.bfloat16)
    torch.cuda.synchronize()
    assert coll.check_error() == 0
    assert torch.equal(hidden, exp), "graph replay mismatch"
    del graph


def check_allreduce_sum(coll, rank, world, dev):
    """fp32 in-place sum: the one-shot kernel (<= sum_rows rows, repeated and under graph
    replay) and the plain two-shot above, against the rank-ordered fp32 sum."""
    H = coll.hidden
    for rows in (1, 3, coll.sum_rows, coll.sum_rows + 5, min(coll.max_rows, 96)):  # > sum_rows: plain two-shot
        g = torch.Generator(device=dev).manual_seed(400 + rows)
        allx = [torch.randn(rows, H, generator=g, device=dev) for _ in range(world)]
        for _ in range(3):
            t = allx[rank].clone()
            coll.allreduce_sum(t)
            torch.cuda.synchronize()
            assert coll.check_error() == 0
            exp = allx[0].clone()
            for r in range(1, world):
                exp = exp + allx[r]
            torch.testing.assert_close(t, exp, rtol=1e-6, atol=1e-6)
    t = allx[rank][:3].clone()
    src = allx[rank][:3].clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        t.copy_(src)
        coll.allreduce_sum(t)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        t.copy_(src)
        coll.allreduce_sum(t)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    exp = sum(x[:3] for x in allx)
    torch.testing.assert_close(t, exp, rtol=1e-6, atol=1e-6)
    del graph


def check_argmax(coll, rank, world, dev):
    from zstep_b200.ops import _ext

    coll.reserve(96, 2048)
    rows, tiles, vloc = 50, 7, 7 * 128
    g = torch.Generator(device=dev).manual_seed(300)
    logits = [torch.randn(rows, vloc, generator=g, device=dev) for _ in range(world)]
    # Build per-tile keys of this rank's shard with the packing rule of the GEMM epilogue:
    # high word = orderable float bits, low word = ~local_id.
    lg = logits[rank].view(rows, tiles, 128)
    vals, idx = lg.max(-1)
    lid = idx + torch.arange(tiles, device=dev) * 128
    bits = vals.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    hi = torch.where(bits >= 0x80000000, (~bits) & 0xFFFFFFFF, bits | 0x80000000)
    keys = ((hi << 32) | ((~lid) & 0xFFFFFFFF)).contiguous()
    out_ids = torch.zeros(rows, dtype=torch.int32, device=dev)
    out_vals = torch.zeros(rows, dtype=torch.float32, device=dev)
    for _ in range(3):
        coll.argmax_allreduce(keys, rows, tiles, rank * vloc, out_ids, out_vals)
    torch.cuda.synchronize()
    assert coll.check_error() == 0
    full = torch.cat(logits, dim=1)
    v, i = full.max(-1)
    assert torch.equal(out_ids.long(), i), "argmax ids"
    assert torch.equal(out_vals, v), "argmax values"
    del _ext


TIE_MARGIN = 0.15  # the logit check allows 3e-2 + 3e-2|v| per logit (|v| ~ 1): two logits can swap across 0.15


def _same_or_near_tie(got, want, ref_logits):
    """Greedy tokens must equal the fp32 reference's, except where the reference itself
    nearly ties: the token chosen must then be within TIE_MARGIN of the reference's best."""
    for g_tok, w_tok, lg in zip(got, want, ref_logits):
        if g_tok == w_tok:
            continue
        gap = float(lg[w_tok] - lg[g_tok])
        assert gap < TIE_MARGIN, f"token {g_tok} != reference {w_tok} with reference margin {gap:.4f}"


def check_model(coll, rank, world, dev):
    from zstep_b200.config import qwen35_small_gpu
    from zstep_b200.models.qwen35 import Qwen35Runner
    from zstep_b200.models.qwen35_ref import Qwen35Reference
    from zstep_b200.models.weights import RandomWeights

    cfg = qwen35_small_gpu(num_layers=4, vocab=8192, experts=32)
    src = RandomWeights(cfg, seed=11)
    runner = Qwen35Runner(cfg, device=dev, weights=src, max_seqs=8, max_prefill_tokens=256, num_pages=64,
                          max_model_len=256, tp_rank=rank, tp_size=world, collectives=coll)
    ref = Qwen35Reference(cfg, src, device=dev, quant=True)
    g = torch.Generator().manual_seed(3)
    lens = [5, 17, 33]
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    for s in range(len(lens)):
        runner.set_pages(s, list(range(1 + 8 * s, 1 + 8 * (s + 1))))
    ids, pos, slots, starts = [], [], [], [0]
    for s, p in enumerate(prompts):
        ids += p
        pos += list(range(len(p)))
        slots += [s] * len(p)
        starts.append(starts[-1] + len(p))
    runner.stage(ids, pos, slots, seq_start=starts)
    first = runner.prefill_forward(len(ids), len(lens)).cpu().tolist()
    assert runner.check_error() == 0
    states = [ref.new_state() for _ in lens]
    ref_next, first_logits = [], []
    for s, p in enumerate(prompts):
        for t in p:
            lg = ref.step(states[s], t)
        ref_next.append(int(lg.argmax()))
        first_logits.append(lg)
    _same_or_near_tie(first, ref_next, first_logits)
    # Every rank must produce the same tokens (the fused reductions are rank-order fixed).
    gathered = [None] * world
    dist.all_gather_object(gathered, first)
    assert all(x == first for x in gathered), gathered
    toks = ref_next
    for step in range(4):
        p_now = [len(p) + step for p in prompts]
        runner.stage(toks, p_now, list(range(3)))
        out = runner.decode_step(3).cpu().tolist()
        assert runner.check_error() == 0
        ref_out, ref_l, ref_lg = [], [], []
        for s in range(3):
            lg = ref.step(states[s], toks[s])
            ref_out.append(int(lg.argmax()))
            ref_l.append(lg.max().item())
            ref_lg.append(lg)
        vals = runner.buf["out_vals"][:3].cpu()
        torch.testing.assert_close(vals, torch.tensor(ref_l), rtol=3e-2, atol=3e-2)
        _same_or_near_tie(out, ref_out, ref_lg)
        dist.all_gather_object(gathered, out)
        assert all(x == out for x in gathered), gathered
        toks = ref_out
    runner.graphs.clear()


def check_nvls(rank, world, dev):
    """NVLS protocol (NVSwitch multicast object; run when ZSTEP_TEST_NVLS=1): the residual
    is the rank-ordered sum up to the switch's bf16 rounding of the partial sum, identical
    bits on every rank, MXFP8 output equal to the norm kernel's on that residual, rows past
    `rows` untouched, and repeated calls (epochs) plus a CUDA-graph replay stay right."""
    from zstep_b200.ops import _ext
    from zstep_b200.parallel.fused import NVLS

    C = _ext.load()
    H, R = 2048, 256
    coll = FusedCollectives(dev)
    coll.nvls_rows = R
    coll.reserve(R, H)
    if coll.nvls is None:
        print(f"rank {rank}: NVLS unavailable: {coll.nvls_error}", flush=True)
        coll.close()
        return
    g = torch.Generator(device=dev).manual_seed(300)
    resid0 = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.rand(H, generator=g, device=dev) + 0.5).to(torch.bfloat16)
    terms = 2
    allp = [torch.randn(terms, R, H, generator=g, device=dev) for _ in range(world)]
    delta = allp[rank].contiguous()
    xq = torch.zeros(R, H, dtype=torch.uint8, device=dev)
    xsf = torch.zeros(mx.atoms_bytes(R, H), dtype=torch.uint8, device=dev)
    for rows in (17, 130, R):
        assert coll.protocol_for(rows) == NVLS
        exp = _expected_residual(resid0, allp, rows, world, terms)
        for rep in range(3):
            hidden = resid0.clone()
            coll.allreduce_add_rmsnorm(delta, terms, H, R * H, hidden, w, 1e-6, rows, xq, xsf, protocol=NVLS)
            torch.cuda.synchronize()
            assert coll.check_error() == 0, (rows, rep, coll.check_error())
            torch.testing.assert_close(hidden[:rows].float(), exp.float(), rtol=2e-2, atol=0.15)
            assert torch.equal(hidden[rows:], resid0[rows:]), "rows beyond `rows` were touched"
            everyone = [torch.empty_like(hidden) for _ in range(world)]
            dist.all_gather(everyone, hidden)
            assert all(torch.equal(x, hidden) for x in everyone), "ranks hold different residuals"
        h2 = hidden[:rows].clone()
        xq2, xsf2 = torch.zeros_like(xq), torch.zeros_like(xsf)
        C.add_rmsnorm_quant(h2, None, 0, H, H, w, 1.0, 1e-6, rows, None, xq2, xsf2)
        assert torch.equal(xq[:rows], xq2[:rows]), f"MXFP8 rows differ rows={rows}"
    hidden = resid0.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(4):
            coll.allreduce_add_rmsnorm(delta, terms, H, R * H, hidden, w, 1e-6, R, xq, xsf, protocol=NVLS)
    for _ in range(3):
        hidden.copy_(resid0)
        graph.replay()
        torch.cuda.synchronize()
        assert coll.check_error() == 0
        want = resid0.clone()
        for _ in range(4):
            coll.allreduce_add_rmsnorm(delta, terms, H, R * H, want, w, 1e-6, R, xq2, xsf2, protocol=NVLS)
        torch.cuda.synchronize()
        assert torch.equal(hidden, want), "graph replay differs from eager calls"
    del graph
    coll.close()


def check_peer_timeout(coll, rank, world, dev):
    """Bounded device waits: rank 1 skips one all-reduce between steps (its GPU runs
    nothing), so rank 0's kernel must give up after timeout_ms, report kErrPeerTimeout (2)
    and return.  After a collective reset every rank's next call succeeds again."""
    H, R = 2048, 32
    coll.reserve(R, H)
    coll.timeout_ms = 50
    delta = torch.ones(R, H, dtype=torch.bfloat16, device=dev)
    hidden = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
    w = torch.ones(H, dtype=torch.bfloat16, device=dev)
    xq = torch.zeros(128, H, dtype=torch.uint8, device=dev)
    xsf = torch.zeros(mx.atoms_bytes(128, H), dtype=torch.uint8, device=dev)
    for proto in (0, 1, 2):
        dist.barrier()
        if rank != 1:
            t0 = time.time()
            coll.allreduce_add_rmsnorm(delta, 1, H, 0, hidden, w, 1e-6, R, xq, xsf, protocol=proto)
            torch.cuda.synchronize()
            assert time.time() - t0 < 5.0
            assert coll.check_error() == 2, (proto, coll.check_error())
        dist.barrier()
        coll.reset()
        hidden.zero_()
        coll.allreduce_add_rmsnorm(delta, 1, H, 0, hidden, w, 1e-6, R, xq, xsf, protocol=proto)
        torch.cuda.synchronize()
        assert coll.check_error() == 0
        assert torch.equal(hidden, torch.full_like(hidden, float(world))), proto
    coll.close()


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    coll = FusedCollectives(dev)
    from zstep_b200.ops import _ext

    C = _ext.load()
    try:
        check_allreduce(coll, C, rank, world, dev)
        check_graph_replay(coll, rank, world, dev)
        check_argmax(coll, rank, world, dev)
        check_allreduce_sum(coll, rank, world, dev)
        check_gemm_push(coll, C, rank, world, dev)
        check_prefill_sized(coll, rank, world, dev)
        if world > 1 and os.environ.get("ZSTEP_TEST_NVLS") == "1":
            check_nvls(rank, world, dev)
        coll = FusedCollectives(dev)
        if world > 1:
            check_peer_timeout(coll, rank, world, dev)
        what = os.environ.get("ZSTEP_MP_CHECKS", "all")
        if what == "all":
            coll.close()
            coll = FusedCollectives(dev)
            check_model(coll, rank, world, dev)
        torch.cuda.synchronize()
        coll.close()
        print(f"rank {rank}: ok", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
