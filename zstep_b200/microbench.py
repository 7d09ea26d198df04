"""Kernel and step micro-benchmarks with roofline fractions.

    python -m zstep_b200.microbench breakdown [--layers 40] [--batch 256] [--ctx 1280]
    python -m zstep_b200.microbench step --model deepseek --layers 48 --batch 64 --ctx 8192 --tp 8
    python -m zstep_b200.microbench step --eager 1        (one eager decode step; for ncu)
    python -m zstep_b200.microbench gemm --m 256 --n 12352 --k 2048 [--groups 1]
    python -m zstep_b200.microbench moe --m 256
    python -m zstep_b200.microbench gdn --m 256
    python -m zstep_b200.microbench attn --m 256 --ctx 1280

Times are CUDA-event times on the launching stream after warm-up, with inputs larger
than L2 (or an L2 flush between iterations for small operands).  Peaks come from
MEASURED_PEAKS.json at the repository root when present (else 6.65 TB/s and 1.59
PFLOP/s bf16 dense, doubled for fp8).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
from collections import defaultdict

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def _flush(n_bytes=256 << 20):
    """Evict L2 by *reading* a buffer twice its size (a write flush would leave dirty
    lines that the timed kernel then has to write back)."""
    buf = _flush.__dict__.setdefault("buf", torch.ones(n_bytes, dtype=torch.uint8, device="cuda"))
    buf.max()


def time_fn(fn, iters=20, warmup=3, flush=False, reps=8) -> float:
    """Median device milliseconds per call.  `fn` is captured `reps` times into one CUDA
    graph so host launch overhead never sits between the timing events; with `flush`
    an L2-evicting read is captured before every call and its own time subtracted."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()

    def capture(body):
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            body()  # allocate any lazily created buffers outside the capture
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                body()
        torch.cuda.current_stream().wait_stream(s)
        return g

    def run_body(with_fn):
        def body():
            for _ in range(reps):
                if flush:
                    _flush()
                if with_fn:
                    fn()
        return body

    def med(g):
        ts = []
        for _ in range(iters):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    g = capture(run_body(True))
    total = med(g)
    base = med(capture(run_body(False))) if flush else 0.0
    return (total - base) / reps


def build_runner(layers: int, batch: int, ctx: int, experts: int = 256, vocab: int = 248320, tp: int = 1,
                 prefill_tokens: int = 0, num_spec: int = 0):
    """Runner on one GPU; with tp > 1 it holds rank 0's shard of a tp-way layout and its
    reductions stay local (LocalCollectives), so timings are one rank's compute only."""
    from .config import Qwen35Config
    from .models.qwen35 import Qwen35Runner
    from .parallel.collectives import LocalCollectives

    types = tuple("full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(layers))
    cfg = Qwen35Config(num_hidden_layers=layers, layer_types=types, num_experts=experts, vocab_size=vocab)
    page = 16
    pages_per_seq = (ctx + 64 + page - 1) // page
    r = Qwen35Runner(cfg, max_seqs=batch, max_prefill_tokens=max(batch, prefill_tokens),
                     num_pages=batch * pages_per_seq + 1,
                     page_size=page, max_model_len=ctx + 64, tp_rank=0, tp_size=tp,
                     collectives=LocalCollectives() if tp > 1 else None, num_spec_tokens=num_spec)
    for s in range(batch):
        r.set_pages(s, list(range(1 + s * pages_per_seq, 1 + (s + 1) * pages_per_seq)))
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (batch,), generator=g)
    r.stage(ids, [ctx] * batch, list(range(batch)))
    return r


def build_ds_runner(layers: int, batch: int, ctx: int, tp: int = 1, expert_format: str = "mxfp4"):
    """DeepSeek-style runner (full per-layer shapes, `layers` deep) holding rank 0's shard
    of a tp-way attention / expert-parallel layout; reductions stay local.  Every row
    decodes at position `ctx`, so the indexer scores `ctx + 1` keys and attention reads
    the top-k (cache contents are left as allocated: the timing does not depend on them)."""
    from .config import DeepSeekConfig
    from .models.deepseek import DeepSeekRunner
    from .parallel.collectives import LocalCollectives

    cfg = DeepSeekConfig(num_hidden_layers=layers, expert_format=expert_format)
    page = 16
    pages_per_seq = (ctx + 64 + page - 1) // page
    r = DeepSeekRunner(cfg, max_seqs=batch, max_prefill_tokens=batch, num_pages=batch * pages_per_seq + 1,
                       page_size=page, max_model_len=ctx + 64, tp_rank=0, tp_size=tp,
                       collectives=LocalCollectives() if tp > 1 else None)
    for s in range(batch):
        r.set_pages(s, list(range(1 + s * pages_per_seq, 1 + (s + 1) * pages_per_seq)))
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (batch,), generator=g)
    r.stage(ids, [ctx] * batch, list(range(batch)))
    return r


def _runner_for(a):
    if a.model == "deepseek":
        return build_ds_runner(a.layers, a.batch, a.ctx, tp=a.tp)
    return build_runner(a.layers, a.batch, a.ctx, tp=a.tp, prefill_tokens=a.prefill_seqs * a.ctx)


def cmd_breakdown(a):
    """Per-op device time of one eager decode step (events around every kernel call); with
    --prefill-seqs N, of one varlen prefill of N sequences of --ctx tokens instead."""
    r = _runner_for(a)
    if hasattr(r, "prefill_attn_impl"):
        r.prefill_attn_impl = a.impl
    if a.prefill_seqs:
        n, L = a.prefill_seqs, a.ctx
        g = torch.Generator().manual_seed(1)
        ids = torch.randint(0, r.cfg.vocab_size, (n * L,), generator=g).tolist()
        pos = [p for _ in range(n) for p in range(L)]
        slots = [s for s in range(n) for _ in range(L)]

        def step():
            r.stage(ids, pos, slots, seq_start=[s * L for s in range(n + 1)])
            r.prefill_forward(n * L, n)
    else:
        def step():
            r.decode_forward(a.batch)
    kind = f"prefill of {a.prefill_seqs} x {a.ctx} tokens" if a.prefill_seqs else f"decode step (batch {a.batch}, ctx {a.ctx})"
    _op_breakdown(r, step, f"eager {kind}", a.layers)


def _op_breakdown(r, step, label: str, layers: int) -> None:
    """Run `step` twice, then once more with CUDA events around every extension call
    (through a proxy of the runner's kernel module), and print the per-op device time."""
    real = r.C
    events = []

    class Proxy:
        def __getattr__(self, name):
            fn = getattr(real, name)

            def wrapped(*args, **kw):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                out = fn(*args, **kw)
                e.record()
                tag = name
                if name == "gemm_mxf8":
                    tag = f"gemm[n={args[5]},k={args[4]},g={args[7]},epi={args[12]}]"
                events.append((tag, s, e))
                return out
            return wrapped

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    r.C = Proxy()
    events.clear()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    step()
    en.record()
    torch.cuda.synchronize()
    r.C = real
    tot = defaultdict(float)
    cnt = defaultdict(int)
    for tag, s, e in events:
        tot[tag] += s.elapsed_time(e)
        cnt[tag] += 1
    step_ms = st.elapsed_time(en)
    rows = sorted(tot.items(), key=lambda kv: -kv[1])
    print(f"{label}: {step_ms:.3f} ms, layers {layers}")
    for tag, ms in rows:
        print(f"  {ms:8.3f} ms  {100 * ms / step_ms:5.1f}%  x{cnt[tag]:<4d} {tag}")


def _graph_ms(replay, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        replay()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    return statistics.median(ts)


def cmd_spec(a):
    """Device time of one steady-state speculative step (one CUDA graph: target forward over
    batch x (K+1) rows, lm_head argmax, on-device greedy verify, GDN replay of the accepted
    rows, MTP catch-up and the chained drafts) next to a plain decode step of the same batch.
    Random weights accept no drafts, so every replay is the acceptance-1 worst case.  With
    --eager 1: the per-op device time of one eager verify step instead."""
    K = a.spec_k
    r = build_runner(a.layers, a.batch, a.ctx, tp=a.tp, prefill_tokens=a.batch * (K + 1), num_spec=K)
    bk = r.bucket_for(a.batch)
    n, K1 = a.batch, K + 1
    nb = r.spec.graph_bucket(n)
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, r.cfg.vocab_size, (nb * K1,), generator=g).tolist()
    pos = [a.ctx + j for _ in range(nb) for j in range(K1)]
    slot = [i for i in range(nb) for _ in range(K1)]

    def stage_verify():
        r.stage(ids, pos, slot, seq_start=[i * K1 for i in range(nb + 1)])
        r.spec.out_slots[:nb].copy_(torch.arange(nb, dtype=torch.int32) + r.spec_slot_base)

    if a.eager:
        r.spec._graph_buffers()
        stage_verify()
        _op_breakdown(r, lambda: r.spec.verify_step(nb), f"eager verify step ({n} x {K1} rows, ctx {a.ctx})",
                      a.layers)
        return
    r.capture_decode_graph(bk)
    dec = _graph_ms(r.graphs[bk].replay, a.warmup, a.iters)
    stage_verify()
    r.spec.run_verify_graph(nb)
    ver = _graph_ms(lambda: r.spec.g_graphs[nb].replay(), a.warmup, a.iters)
    print(json.dumps({"op": "spec_step", "batch": n, "K": K, "ctx": a.ctx, "tp": a.tp, "decode_step_ms": round(dec, 4),
                      "verify_step_ms": round(ver, 4), "ratio": round(ver / dec, 3)}))


def cmd_step(a):
    r = _runner_for(a)
    if a.eager:
        for _ in range(a.warmup):
            r.decode_forward(a.batch)
        torch.cuda.synchronize()
        r.decode_forward(a.batch)
        torch.cuda.synchronize()
        return
    r.capture_decode_graph(r.bucket_for(a.batch))
    g = r.graphs[r.bucket_for(a.batch)]
    for _ in range(a.warmup):
        g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(a.iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    ms = statistics.median(ts)
    if a.profile_replay:
        # One replay bracketed for `ncu --profile-from-start off`.
        torch.cuda.cudart().cudaProfilerStart()
        g.replay()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"decode_step_ms": round(ms, 4), "tok_s": round(a.batch / ms * 1000, 1)}))


def _gemm_case(m, n, k, groups=1):
    from .ops import mx
    from .models.qwen35 import pack_linear, _pad128

    C = __import__("zstep_b200.ops._ext", fromlist=["load"]).load()
    w = (torch.randn(groups, n, k, device="cuda") * 0.02).to(torch.bfloat16)
    pw = pack_linear(w, C)
    rows = _pad128(m) if groups == 1 else _pad128(m) * groups
    x = torch.randn(rows, k, device="cuda").to(torch.bfloat16)
    xq = torch.empty(rows, k, dtype=torch.uint8, device="cuda")
    xsf = torch.empty(mx.atoms_bytes(rows, k), dtype=torch.uint8, device="cuda")
    C.quant_mxf8(x, xq, xsf)
    return C, pw, xq, xsf


def cmd_gemm(a):
    """Dense or uniform grouped MXFP8 GEMM; --epi 2 runs the SiLU(gate)*up + MXFP8 epilogue
    of the MoE gate/up projection (n = 2 x intermediate, output e4m3 + scale atoms), --epi 3
    the scaled scatter of the MoE down projection."""
    from .ops import mx

    C, pw, xq, xsf = _gemm_case(a.m, a.n, a.k, a.groups)
    rows_out = _pad128_(a.m) * a.groups
    out_sf = None
    if a.epi == 2:
        out = torch.empty(rows_out, a.n // 2, dtype=torch.uint8, device="cuda")
        out_sf = torch.empty(mx.atoms_bytes(rows_out, a.n // 2), dtype=torch.uint8, device="cuda")
    else:
        out = torch.empty(rows_out, a.n, dtype=torch.bfloat16, device="cuda")
    ldo = out.shape[1]
    if a.groups == 1:
        bn = a.bn or (32 if a.m <= 32 else 128)
        ws = torch.zeros(8 << 20, dtype=torch.float32, device="cuda")
        sem = torch.zeros(16384, dtype=torch.int32, device="cuda")
        fn = lambda: C.gemm_mxf8(pw.q, pw.sf, xq, xsf, a.k, pw.n_pad, a.n, 1, a.m, None, None, None, a.epi, out,  # noqa
                                 ldo, out_sf, None, None, None, 0, bn, 1, 0, 1, a.fix_splits, ws, sem)
    else:
        cnt = torch.full((a.groups,), a.m, dtype=torch.int32, device="cuda")
        off = torch.arange(a.groups, dtype=torch.int32, device="cuda") * _pad128_(a.m)
        bn = 32 if a.m <= 32 else 128
        pre = torch.arange(a.groups + 1, dtype=torch.int32, device="cuda") * ((a.m + bn - 1) // bn)
        ws = torch.zeros(8 << 20, dtype=torch.float32, device="cuda")
        sem = torch.zeros(16384, dtype=torch.int32, device="cuda")
        dst = scl = None
        if a.epi == 3:  # MoE down projection: rows scattered to (token, k) slots, times the routing weight
            dst = torch.randperm(rows_out, device="cuda").to(torch.int32)
            scl = torch.rand(rows_out, device="cuda")
        fn = lambda: C.gemm_mxf8(pw.q, pw.sf, xq, xsf, a.k, pw.n_pad, a.n, a.groups, 0, cnt, off, pre, a.epi,  # noqa
                                 out, ldo, out_sf, dst, scl, None, 0, bn, 1, 0, 1, a.fix_splits, ws, sem)
    ms = time_fn(fn, flush=bool(a.flush))
    pk = peaks()
    flops = 2.0 * a.m * a.n * a.k * a.groups
    bytes_ = a.n * a.k * a.groups * (1 + 1 / 32) + a.m * a.k * a.groups + a.m * a.n * 2 * a.groups
    res = {"op": "gemm_mxf8", "m": a.m, "n": a.n, "k": a.k, "groups": a.groups, "epi": a.epi,
           "fix_splits": a.fix_splits, "ms": round(ms, 4),
           "tflops": round(flops / ms / 1e9, 1), "gbs": round(bytes_ / ms / 1e6, 1),
           "frac_fp8_peak": round(flops / ms / 1e9 / (2 * pk["bf16_tflops"]), 3),
           "frac_hbm": round(bytes_ / ms / 1e6 / pk["hbm_gbs"], 3), "peaks": pk["src"]}
    print(json.dumps(res))


def _pad128_(n):
    return (n + 127) // 128 * 128


def cmd_gdn(a):
    if a.prefill_seqs:
        return _gdn_prefill(a)
    r = build_runner(4, a.m, 64, experts=32, vocab=8192)
    b = r.buf
    L = r.layers[0]
    proj = b["proj"][: a.m * r.gdn_w].view(a.m, r.gdn_w)
    proj.normal_()
    midq = r._mid(r.hv * 128)
    fn = lambda: r.C.gdn_decode(proj, r.hk, r.hv, L["conv_w"], r.conv_state[0], r.ssm_state[0], L["a_log"],  # noqa
                                L["dt_bias"], L["gnorm"], r.eps, b["in_slot"][:a.m], b["in_pos"][:a.m], a.m, None,
                                midq, b["midsf"], b["err"])
    ms = time_fn(fn, flush=True)
    state_bytes = a.m * r.hv * 128 * 128 * 4 * 2
    pk = peaks()
    print(json.dumps({"op": "gdn_decode", "rows": a.m, "ms": round(ms, 4), "gbs": round(state_bytes / ms / 1e6, 1),
                      "frac_hbm": round(state_bytes / ms / 1e6 / pk["hbm_gbs"], 3), "peaks": pk["src"]}))


def _gdn_prefill(a):
    """Varlen GDN prefill of --prefill-seqs fresh sequences sharing --m rows (--impl 0 auto,
    1 token-sequential, 2 chunked)."""
    n = a.prefill_seqs
    L = a.m // n
    rows = n * L
    r = build_runner(4, n, L, experts=32, vocab=8192, prefill_tokens=rows)
    b = r.buf
    lay = r.layers[0]
    r.stage([1] * rows, [p for _ in range(n) for p in range(L)], [s for s in range(n) for _ in range(L)],
            seq_start=[s * L for s in range(n + 1)])
    proj = b["proj"][: rows * r.gdn_w].view(rows, r.gdn_w)
    proj.normal_()
    midq = r._mid(r.hv * 128)
    fn = lambda: r.C.gdn_prefill(proj, r.hk, r.hv, lay["conv_w"], r.conv_state[0], r.ssm_state[0],  # noqa
                                 lay["a_log"], lay["dt_bias"], lay["gnorm"], r.eps, b["in_slot"][:rows],
                                 b["in_pos"][:rows], rows, None, midq, b["midsf"], b["seq_start"][:n + 1], n,
                                 None, None, 0, b["err"], None, impl=a.impl)
    ms = time_fn(fn, flush=True)
    flops = 2 * 4.2e6 * (rows / 64) * r.hv  # ~4.2M FMAs per 64-token chunk and value head
    print(json.dumps({"op": "gdn_prefill", "rows": rows, "seqs": n, "impl": a.impl, "ms": round(ms, 4),
                      "tflops_fp32": round(flops / ms / 1e9, 2)}))


def cmd_coll(a):
    """NVLink collective kernels as one rank on one GPU (peers = this GPU): the all-reduce +
    RMSNorm + MXFP8 (one-shot at 8 rows, two-shot LL and plain at 256 rows), the argmax
    exchange (256 rows x 243 vocab tiles), the fp32 sum (64 rows) and the expert all-to-all
    dispatch + combine (--m tokens, hidden 4096, top-8 of 256).  With --iters 1
    every kernel launches exactly once (for a profiler capture); otherwise CUDA-event medians."""
    import socket

    import torch.distributed as dist

    from .ops import mx
    from .parallel.ep import EpAllToAll
    from .parallel.fused import FusedCollectives

    if not dist.is_initialized():
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    dev = torch.device("cuda", 0)
    H = 2048
    coll = FusedCollectives(dev, max_rows=256, hidden=H)
    rows = 8
    delta = (0.01 * torch.randn(rows, H, device=dev)).to(torch.bfloat16)
    hid = torch.zeros(rows, H, dtype=torch.bfloat16, device=dev)
    w = torch.ones(H, dtype=torch.bfloat16, device=dev)
    xq = torch.zeros(128, H, dtype=torch.uint8, device=dev)
    xsf = torch.zeros(mx.atoms_bytes(128, H), dtype=torch.uint8, device=dev)
    t = torch.randn(64, H, device=dev)
    ep = EpAllToAll(dev, num_experts=256, hidden=4096, top_k=8, max_tokens=a.m, recv_cap=2 * a.m * 8 + 256 * 128)
    x = torch.randn(a.m, 4096, device=dev, dtype=torch.bfloat16)
    ids = torch.rand(a.m, 256, device=dev).topk(8, dim=1).indices.to(torch.int32).contiguous()
    wt = torch.rand(a.m, 8, device=dev)
    y = torch.randn(ep.recv_cap, 4096, device=dev, dtype=torch.bfloat16)
    out = torch.empty(a.m, 4096, dtype=torch.bfloat16, device=dev)
    big = 256
    delta_b = (0.01 * torch.randn(big, H, device=dev)).to(torch.bfloat16)
    hid_b = torch.zeros(big, H, dtype=torch.bfloat16, device=dev)
    xq_b = torch.zeros(big, H, dtype=torch.uint8, device=dev)
    xsf_b = torch.zeros(mx.atoms_bytes(big, H), dtype=torch.uint8, device=dev)
    keys = torch.randint(0, 2 ** 62, (big, 243), dtype=torch.int64, device=dev)
    ids_out = torch.zeros(big, dtype=torch.int32, device=dev)
    vals_out = torch.zeros(big, dtype=torch.float32, device=dev)
    ar = lambda proto, m: coll.allreduce_add_rmsnorm(delta_b, 1, H, 0, hid_b, w, 1e-6, m, xq_b, xsf_b,  # noqa: E731
                                                     protocol=proto)
    ops = {"allreduce_norm_small_8rows": lambda: coll.allreduce_add_rmsnorm(delta, 1, H, 0, hid, w, 1e-6, rows, xq, xsf),
           "allreduce_norm_twoshot_ll_256rows": lambda: ar(1, big),
           "allreduce_norm_twoshot_plain_256rows": lambda: ar(2, big),
           "argmax_exchange_256rows": lambda: coll.argmax_allreduce(keys, big, 243, 0, ids_out, vals_out),
           "allreduce_sum_f32_64rows": lambda: coll.allreduce_sum(t),
           "ep_dispatch": lambda: ep.dispatch(x, ids, wt),
           "ep_combine": lambda: ep.combine(y, ids, wt, out)}
    res = {"op": "coll_single_rank", "tokens": a.m}
    for name, fn in ops.items():
        if a.iters == 1:
            fn()
            continue
        ts = []
        for _ in range(a.iters):
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            fn()
            e_.record()
            e_.synchronize()
            ts.append(s_.elapsed_time(e_) * 1000)
        res[name + "_us"] = round(statistics.median(ts), 2)
    torch.cuda.synchronize()
    res["err"] = coll.check_error() | ep.check_error()
    print(json.dumps(res))
    ep.close()
    coll.close()
    dist.destroy_process_group()


def cmd_attn(a):
    r = build_runner(4, a.m, a.ctx, experts=32, vocab=8192, tp=a.tp)
    b = r.buf
    b["q_out"].normal_()
    b["gate_out"].normal_()
    r.k_cache.normal_()
    r.v_cache.normal_()
    ai = 0
    splits = a.splits or r._attn_splits(a.m, True)
    midq = r._mid(r.hq * 256)
    if b["partial"].numel() < a.m * r.hq * splits * 260:
        b["partial"] = torch.zeros(a.m * r.hq * splits * 260, device=r.dev)
    fn = lambda: r.C.attn_decode(b["q_out"], b["gate_out"], r.hq, r.hkv, r.k_cache[ai], r.v_cache[ai], r.page_size,  # noqa
                                 r.page_table, b["in_slot"][:a.m], b["in_len"][:a.m], a.m, b["partial"], splits,
                                 1 / 16.0, None, midq, b["midsf"], impl=a.impl)
    ms = time_fn(fn, flush=True)
    kv_bytes = a.m * (a.ctx + 1) * r.hkv * 256 * 2 * 2
    pk = peaks()
    print(json.dumps({"op": "attn_decode", "impl": a.impl, "tp": a.tp, "rows": a.m, "ctx": a.ctx, "splits": splits,
                      "ms": round(ms, 4),
                      "gbs": round(kv_bytes / ms / 1e6, 1), "frac_hbm": round(kv_bytes / ms / 1e6 / pk["hbm_gbs"], 3),
                      "peaks": pk["src"]}))


def cmd_moe(a):
    r = build_runner(4, a.m, 64, experts=256, vocab=8192)
    L = r.layers[0]
    # Realistic routing: quantize random activations into the MoE input buffer.
    x = torch.randn(a.m, r.cfg.hidden_size, device="cuda").to(torch.bfloat16)
    r.C.quant_mxf8(x, r.buf["xq"], r.buf["xsf"])
    fn = lambda: r._moe(L, a.m)  # noqa: E731
    ms = time_fn(fn, flush=True)
    w_bytes = (L["gate_up"].q.numel() + L["down"].q.numel()) * (1 + 1 / 32)
    pk = peaks()
    print(json.dumps({"op": "moe_decode(router+route+gate_up+down)", "rows": a.m, "ms": round(ms, 4),
                      "weight_gbs": round(w_bytes / ms / 1e6, 1),
                      "frac_hbm": round(w_bytes / ms / 1e6 / pk["hbm_gbs"], 3), "peaks": pk["src"]}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("cmd", choices=["breakdown", "step", "spec", "gemm", "gdn", "attn", "moe", "coll"])
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=1280)
    ap.add_argument("--prefill-seqs", type=int, default=0, help="breakdown: time a varlen prefill of this many sequences of --ctx tokens")
    ap.add_argument("--eager", type=int, default=0)
    ap.add_argument("--profile-replay", type=int, default=0)
    ap.add_argument("--spec-k", type=int, default=3, help="spec: draft tokens per verify step")
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--m", type=int, default=256)
    ap.add_argument("--n", type=int, default=2048)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--groups", type=int, default=1)
    ap.add_argument("--flush", type=int, default=1, help="evict L2 before every timed call")
    ap.add_argument("--tp", type=int, default=1, help="time rank 0 of a tp-way layout (no communication)")
    ap.add_argument("--model", default="qwen", choices=["qwen", "deepseek"])
    ap.add_argument("--splits", type=int, default=0, help="attn: split-KV factor (0 = the runner's choice)")
    ap.add_argument("--epi", type=int, default=0,
                    help="gemm: 0 bf16 store, 2 SiLU(gate)*up + MXFP8, 3 scaled scatter (grouped MoE down)")
    ap.add_argument("--fix-splits", type=int, default=1, help="gemm (dense): in-kernel split-K factor")
    ap.add_argument("--bn", type=int, default=0, help="gemm (dense): token tile 32 or 128 (0 = by rows)")
    ap.add_argument("--impl", type=int, default=0,
                    help="attn: 0 auto (tensor cores from 4 q heads per kv head), 1 SIMT, 2 tensor cores")
    a = ap.parse_args()
    torch.manual_seed(0)
    {"breakdown": cmd_breakdown, "step": cmd_step, "spec": cmd_spec, "gemm": cmd_gemm, "gdn": cmd_gdn, "attn": cmd_attn, "coll": cmd_coll,
     "moe": cmd_moe}[a.cmd](a)


if __name__ == "__main__":
    main()
