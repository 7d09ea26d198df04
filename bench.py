#!/usr/bin/env python
"""Headline benchmark: decode output tokens/s of the Qwen3.5-35B-A3B-shaped MXFP8 model.

Workload: 256 concurrent requests, uniform-random 1024-token prompts,
greedy decoding, paged KV with 16-token pages, random-init weights of the full
architecture (40 layers, 3:1 GatedDeltaNet:gated-GQA, 256 experts top-8 + shared,
vocab 248320), bf16 activations, MXFP8 weights and activations for every GEMM.

Run as ``python bench.py --gpus N --steps K --warmup W`` (N>1 under torchrun, one rank
per GPU, tensor parallel = N).  After the prefill of all prompts, W untimed decode steps
run, then K decode steps are timed with CUDA events between a barrier +
synchronize on each side; the value is the max over ranks.  Every step advances all 256
sequences by one token, so ``value = 256 * K / max_rank_seconds`` (whole-job tokens/s).

``e2e`` repeats K steps through the runner's public step API with the step's inputs
copied host->device from pinned memory (stage) and the sampled tokens read back
device->host every step.  Weights (~35 GB) and GDN state (~16 GB) exceed L2, so no
explicit flush is needed between steps.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

BASELINE_TOKS = 3128.09  # reference: Qwen3.5 in1024->256 c=128, docs/benchmark.md:139 (8x RTX 6000D)
METRIC = "decode out tok/s (8×B200, TP8, max over ranks) Qwen3.5-35B-A3B; p50 TTFT/TPOT"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="zstep", choices=["zstep", "reference"])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--gen", type=int, default=512)
    ap.add_argument("--layers", type=int, default=0, help="debug: reduced depth (0 = full 40 layers)")
    ap.add_argument("--prefill-chunk", type=int, default=8192)
    ap.add_argument("--mid-context", type=int, default=1,
                    help="prefill prompt + gen/2 tokens so timed steps sit at the mean decode context")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--engine-path", type=int, default=1,
                    help="also time decode through the native master (zstep run, SHM + eventfd) at N GPUs")
    ap.add_argument("--engine-gen", type=int, default=256, help="engine path: output tokens per request")
    ap.add_argument("--nccl-arm", type=int, default=1, help="N>1: also time the same decode step with NCCL collectives")
    return ap.parse_args()


def reference_unavailable(reason: str):
    print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        mhz, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                idx = int(f[0])
            except ValueError:
                continue
            if idx not in self.gpus:
                continue
            try:
                mhz.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                pass
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(mhz)}


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            reference_unavailable(
                "reference zstep cannot run on B200: its worker (installed into baseline/_ref with --no-deps) "
                "refuses any device but sm_120 (zstep_worker/runtime_loop.py:138) and builds its CUDA "
                "extensions for compute_120 only (kernels_sm120/qwen35_ops.py:75); its master and bench CLI "
                "are Rust and no Rust toolchain is installed")
        return

    import torch
    import torch.distributed as dist

    from zstep_b200.config import qwen35_35b_a3b, Qwen35Config
    from zstep_b200.models.qwen35 import Qwen35Runner

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    coll = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        from zstep_b200.parallel import make_collectives

        coll = make_collectives(dev)
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"

    cfg = qwen35_35b_a3b()
    if args.layers:
        types = tuple("full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(args.layers))
        cfg = Qwen35Config(num_hidden_layers=args.layers, layer_types=types)
    B, P, gen = args.batch, args.prompt, args.gen
    ctx0 = P + (gen // 2 if args.mid_context else 0)
    steps, warm = args.steps, args.warmup
    assert ctx0 + 2 * warm + 3 * steps + 4 <= P + gen + 64
    page = 16
    max_len = P + gen + 64
    pages_per_seq = (max_len + page - 1) // page
    num_pages = max(32768, B * pages_per_seq) + 1

    t_init = time.time()
    runner = Qwen35Runner(cfg, device=dev, max_seqs=B, max_prefill_tokens=args.prefill_chunk, num_pages=num_pages,
                          page_size=page, max_model_len=max_len, tp_rank=rank, tp_size=world, collectives=coll,
                          seed=args.seed)
    torch.cuda.synchronize()
    init_s = time.time() - t_init
    for s in range(B):
        runner.set_pages(s, list(range(1 + s * pages_per_seq, 1 + (s + 1) * pages_per_seq)))

    # ------------------------------------------------------------------ prefill
    g = torch.Generator().manual_seed(args.seed + 1)
    prompts = torch.randint(0, cfg.vocab_size, (B, ctx0), generator=g, dtype=torch.int32)
    per_chunk = max(1, args.prefill_chunk // ctx0)
    first_tok = torch.zeros(B, dtype=torch.int32)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    chunk_end_ms = []
    for c0 in range(0, B, per_chunk):
        seqs = list(range(c0, min(B, c0 + per_chunk)))
        ids = prompts[seqs].reshape(-1)
        pos = torch.arange(ctx0, dtype=torch.int32).repeat(len(seqs))
        slots = torch.tensor(seqs, dtype=torch.int32).repeat_interleave(ctx0)
        seq_start = [i * ctx0 for i in range(len(seqs) + 1)]
        runner.stage(ids, pos, slots, seq_start=seq_start)
        out = runner.prefill_forward(len(ids), len(seqs))
        first_tok[seqs] = out.cpu()
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        e.synchronize()
        chunk_end_ms.append((ev0.elapsed_time(e), len(seqs)))
    ttft = []
    for t, n in chunk_end_ms:
        ttft += [t] * n
    prefill_ms = chunk_end_ms[-1][0]
    err = runner.check_error()
    assert err == 0, f"kernel error word {err}"

    # ------------------------------------------------------------------ decode (device-timed)
    b = runner.buf
    runner.stage(first_tok, [ctx0] * B, list(range(B)))
    bucket = runner.bucket_for(B)
    runner.capture_decode_graph(bucket)
    runner.stage(first_tok, [ctx0] * B, list(range(B)))
    graph = runner.graphs[bucket]

    def advance():
        b["in_ids"][:B].copy_(b["out_ids"][:B])
        b["in_pos"][:B] += 1
        b["in_len"][:B] += 1

    for _ in range(warm):
        graph.replay()
        advance()
    sampler = ClockSampler(range(world) if rank == 0 else [])
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    # The barrier comes after the sampler's start-up so no rank enters the timed region
    # while another is still on the host (the fused collectives would time that wait).
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    start.record()
    step_ev[0].record()
    for i in range(steps):
        graph.replay()
        advance()
        step_ev[i + 1].record()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    dev_ms = start.elapsed_time(end)
    step_ms = [step_ev[i].elapsed_time(step_ev[i + 1]) for i in range(steps)]
    clocks = sampler.stop() if rank == 0 else None

    # ------------------------------------------------------------------ decode (end to end)
    host_tok = b["out_ids"][:B].cpu()
    pos_now = int(b["in_pos"][0].item())
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_start.record()
    h2d = d2h = 0
    for i in range(steps):
        runner.stage(host_tok, [pos_now + i] * B, list(range(B)))
        h2d = runner.staged_bytes()
        out = runner.decode_step(B)
        host_tok = out.cpu()
        d2h = host_tok.numel() * host_tok.element_size()
    e2e_end.record()
    torch.cuda.synchronize()
    e2e_ms = e2e_start.elapsed_time(e2e_end)
    err = runner.check_error()
    assert err == 0, f"kernel error word {err}"

    # Kernel launches per decode step: count our kernels in one eager step.
    launches = count_launches(runner, B)

    # ------------------------------------------------------------------ NCCL baseline arm
    # The same runner and CUDA-graph decode step with the tensor-parallel reductions and the
    # argmax exchange on NCCL (ZSTEP_COLLECTIVES=nccl): the fused NVLink kernels' end-to-end
    # gain on the same box.
    nccl_ms = None
    if world > 1 and args.nccl_arm:
        from zstep_b200.parallel.collectives import NcclCollectives

        del graph
        runner.graphs.clear()
        fused_coll = runner.coll
        runner.coll = NcclCollectives(None, dev)
        runner.stage(host_tok, [pos_now + steps] * B, list(range(B)))
        runner.capture_decode_graph(bucket)
        graph = runner.graphs[bucket]
        for _ in range(warm):
            graph.replay()
            advance()
        dist.barrier()
        torch.cuda.synchronize()
        n0, n1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0.record()
        for _ in range(steps):
            graph.replay()
            advance()
        n1.record()
        torch.cuda.synchronize()
        dist.barrier()
        t = torch.tensor([n0.elapsed_time(n1)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        nccl_ms = float(t.item())
        runner.coll = fused_coll

    if world > 1:
        t = torch.tensor([dev_ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, e2e_ms = t.tolist()
    if rank == 0:
        value = B * steps / (dev_ms / 1000.0)
        e2e = B * steps / (e2e_ms / 1000.0)
        res = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(dev_ms / steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": round(value / BASELINE_TOKS, 3), "dtype": "bf16",
            "data": "synthetic (uniform-random token prompts, random-init weights)",
            "config": {"model": "Qwen3.5-35B-A3B-shaped (40 layers, 256 experts top-8 + shared, vocab 248320)",
                       "weights": "MXFP8 (e4m3 + e8m0/32)", "global_batch": B, "seq_len": P,
                       "decode_context_start": ctx0, "gen_tokens": gen, "page_size": page,
                       "num_pages": num_pages - 1, "parallelism": f"tp{world}",
                       "l2": "inputs larger than L2 (weights ~35 GB + GDN state ~16 GB per step)",
                       "layers": cfg.num_hidden_layers},
            "p50_tpot_ms": round(statistics.median(step_ms), 4),
            "p50_ttft_ms": round(statistics.median(ttft), 2),
            "prefill_tok_s": round(B * ctx0 / (prefill_ms / 1000.0), 1),
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches * steps,
            "gpu_launches_per_step": launches,
            "clocks": clocks,
            "init_s": round(init_s, 1),
            "vs_baseline_note": "cross-hardware: divides by the reference's published 8x RTX 6000D number "
                                "(in1024->256, c=128); no same-box reference run exists",
        }
        if nccl_ms is not None:
            res["nccl_arm"] = {"value": round(B * steps / (nccl_ms / 1000.0), 2), "unit": "tok/s",
                               "ms_per_step": round(nccl_ms / steps, 4),
                               "what": "same decode graph, TP reductions + argmax exchange on NCCL"}
    del graph
    runner.graphs.clear()  # release graphs before the process group goes away
    if args.engine_path:
        # Free this process's model before the native engine's workers load theirs.
        runner.buf.clear()
        runner.layers.clear()
        del runner, b, advance, out
        import gc

        gc.collect()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        eng = None
        if world > 1:
            dist.barrier()
            store = dist.distributed_c10d._get_default_store()
            if rank == 0:
                eng = engine_path(args, world)
                store.set("zstep_bench_engine_done", "1")
            else:
                # Wait on the store (host only): a collective here would park a kernel on
                # every GPU while the engine's workers run on them.
                store.wait(["zstep_bench_engine_done"], datetime.timedelta(seconds=900))
        else:
            eng = engine_path(args, world)
        if rank == 0:
            res["engine_path"] = eng
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def engine_path(args, world: int) -> dict:
    """Decode through the product's serving path: the native master (`zstep run`) with
    `world` worker processes over shared memory + eventfds, the scheduler, the KV block
    pool and CUDA-graph decode steps, on the benchmark's shape (256 concurrent random
    1024-token prompts, greedy).  Reports the master's own p50 TPOT / TTFT and the decode
    throughput they imply (256 / p50 TPOT), wall-clock on the host (the master's clock)."""
    import tempfile

    root = os.path.dirname(os.path.abspath(__file__))
    binary = os.path.join(root, "zstep_b200", "bin", "zstep")
    if not os.path.exists(binary):
        return {"error": f"{binary} not built"}
    B, P, G = args.batch, args.prompt, args.engine_gen
    with tempfile.TemporaryDirectory() as d:
        cmd = [binary, "run", "--model-dir", d, "--model", "qwen3.5-35b-a3b", "--device", "cuda",
               "--world-size", str(world), "--max-seqs", str(B), "--max-model-len", str(P + G + 64),
               "--num-kv-pages", str(max(32768, B * ((P + G + 64 + 15) // 16) + 1)), "--max-step-tokens", "8192",
               "--max-prefill-chunk", "8192", "--no-enable-prefix-caching", "--python", sys.executable,
               "--worker-root", root, "--bench-tiers", f"engine:{B}:{B}:{P}:{G}", "--seed", str(args.seed)]
        # Drop the launcher's rendezvous variables (torchrun's RANK, MASTER_*, TORCHELASTIC_*,
        # ...): the master hosts its workers' own process group.
        launcher = ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "GROUP_RANK", "GROUP_WORLD_SIZE",
                    "MASTER_ADDR", "MASTER_PORT", "ROLE_RANK", "ROLE_WORLD_SIZE", "ROLE_NAME")
        env = {k: v for k, v in os.environ.items() if k not in launcher and not k.startswith("TORCHELASTIC_")}
        t0 = time.time()
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
        except subprocess.TimeoutExpired as e:
            tail = e.stderr.decode(errors="replace") if isinstance(e.stderr, bytes) else (e.stderr or "")
            return {"error": "zstep run timed out after 300 s", "stderr_tail": tail[-600:]}
        wall = time.time() - t0
    if r.returncode != 0:
        return {"error": f"zstep run exited {r.returncode}", "stderr_tail": r.stderr[-600:]}
    try:
        rep = json.loads(r.stdout.strip().splitlines()[-1])
        run0 = rep["tiers"][0]["runs"][0]
    except (ValueError, KeyError, IndexError) as e:
        return {"error": f"unparsable report: {e}", "stdout_tail": r.stdout[-600:]}
    tpot = float(run0["p50_tpot_ms"])
    return {"decode_tok_s": round(B / (tpot / 1000.0), 2) if tpot > 0 else None, "p50_tpot_ms": round(tpot, 4),
            "p50_ttft_ms": round(float(run0["p50_ttft_ms"]), 2),
            "output_tok_s_incl_prefill": round(float(run0["output_tok_s"]), 2), "requests": B, "input_len": P,
            "output_len": G, "n_gpus": world, "wall_s": round(wall, 1),
            "what": "zstep run --bench-tiers through the C++ master, SHM transport and worker processes"}


def count_launches(runner, rows: int) -> int:
    """Number of zstep_b200 kernels one decode step launches (counted on an eager step)."""
    per_call = {"gemm_mxf8": 1, "quant_mxf8": 1, "add_rmsnorm_quant": 1, "embed_rmsnorm_quant": 1,
                "argmax_reduce": 1, "gdn_decode": 1, "gdn_prefill": 2, "attn_prologue": 1, "attn_decode": 2,
                "moe_route": 3, "fused_allreduce_norm": 1, "allreduce_argmax": 1}
    counts = {"n": 0}
    real = runner.C

    class Proxy:
        def __getattr__(self, name):
            fn = getattr(real, name)

            def wrapped(*a, **k):
                counts["n"] += per_call.get(name, 1)
                return fn(*a, **k)
            return wrapped

    coll = runner.coll
    coll_real = getattr(coll, "C", None)
    runner.C = Proxy()
    if coll_real is not None:
        coll.C = Proxy()
    try:
        runner.pad_decode_inputs(0, runner.bucket_for(rows))
        runner.decode_forward(runner.bucket_for(rows))
    finally:
        runner.C = real
        if coll_real is not None:
            coll.C = coll_real
    return counts["n"]


if __name__ == "__main__":
    sys.exit(main())
