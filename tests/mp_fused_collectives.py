"""Worker for tests/test_multigpu.py: run under torch.distributed.run, one rank per GPU.

Checks the fused NVLink collectives (csrc/kernels/collective.cu) against plain PyTorch
fp32 math on the same data, eagerly and under CUDA-graph replay, then a tensor-parallel
Qwen3.5 runner against the single-GPU fp32 reference with the same MXFP8 quantization.
Exit code 0 = every check passed on this rank."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from zstep_b200.ops import mx  # noqa: E402
from zstep_b200.parallel.fused import FusedCollectives  # noqa: E402


def check_allreduce(coll, C, rank, world, dev):
    H, R = 2048, 96
    coll.reserve(R, H)
    g = torch.Generator(device=dev).manual_seed(100)
    resid0 = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.rand(H, generator=g, device=dev) + 0.5).to(torch.bfloat16)
    terms = 3
    # Each rank's split-K partials, [terms, R, H] f32 (rank-specific data).
    allp = [torch.randn(terms, R, H, generator=g, device=dev) for _ in range(world)]
    delta = allp[rank].contiguous()
    for rows in (R, 37, 1, 5, 8):  # <= 8 rows take the one-shot cluster kernel
        hidden = resid0.clone()
        xq = torch.zeros(128 * ((R + 127) // 128), H, dtype=torch.uint8, device=dev)
        xsf = torch.zeros(mx.atoms_bytes(xq.shape[0], H), dtype=torch.uint8, device=dev)
        coll.allreduce_add_rmsnorm(delta, terms, H, R * H, hidden, w, 1e-6, rows, xq, xsf)
        torch.cuda.synchronize()
        assert coll.check_error() == 0
        # Expected: bf16(resid + sum_r bf16(sum_t part_r[t])) in rank order.
        acc = resid0[:rows].float()
        for r in range(world):
            s = allp[r][0, :rows].clone()
            for t in range(1, terms):
                s = s + allp[r][t, :rows]
            acc = acc + s.to(torch.bfloat16).float()
        exp = acc.to(torch.bfloat16)
        assert torch.equal(hidden[:rows], exp), f"residual mismatch rows={rows}"
        assert torch.equal(hidden[rows:], resid0[rows:]), "rows beyond `rows` were touched"
        # Normed + quantized output vs the single-GPU norm kernel on the expected residual.
        h2 = exp.clone()
        xq2, xsf2 = torch.zeros_like(xq), torch.zeros_like(xsf)
        C.add_rmsnorm_quant(h2, None, 0, H, H, w, 1.0, 1e-6, rows, None, xq2, xsf2)
        d1 = mx.dequantize(xq[:rows], mx.codes_from_atoms(xsf, rows, H))
        d2 = mx.dequantize(xq2[:rows], mx.codes_from_atoms(xsf2, rows, H))
        torch.testing.assert_close(d1, d2, rtol=0.07, atol=1e-2)


def check_graph_replay(coll, rank, world, dev):
    """The kernels advance their own epochs: several replays of one graph stay correct."""
    H, R = 2048, 64
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
        coll.allreduce_add_rmsnorm(delta, 1, H, 0, hidden, w, 1e-6, R, xq, xsf)
    hidden.zero_()
    exp = torch.zeros(R, H, device=dev).to(torch.bfloat16)
    for _ in range(4):
        graph.replay()
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
    replay) and the NCCL path above, against the rank-ordered fp32 sum."""
    H = coll.hidden
    for rows in (1, 3, coll.sum_rows, coll.sum_rows + 5):
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
    ref_next = []
    for s, p in enumerate(prompts):
        for t in p:
            lg = ref.step(states[s], t)
        ref_next.append(int(lg.argmax()))
    assert sum(int(a == b) for a, b in zip(first, ref_next)) >= 2, (first, ref_next)
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
        ref_out, ref_l = [], []
        for s in range(3):
            lg = ref.step(states[s], toks[s])
            ref_out.append(int(lg.argmax()))
            ref_l.append(lg.max().item())
        vals = runner.buf["out_vals"][:3].cpu()
        torch.testing.assert_close(vals, torch.tensor(ref_l), rtol=3e-2, atol=3e-2)
        assert sum(int(a == b) for a, b in zip(out, ref_out)) >= 2, (step, out, ref_out)
        dist.all_gather_object(gathered, out)
        assert all(x == out for x in gathered), gathered
        toks = ref_out
    runner.graphs.clear()


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
