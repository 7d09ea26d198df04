"""the CPU plumbing model end to end.

C++ engine + shared-memory coordinator + 2 worker processes running the tiny
Qwen3.5-style hybrid (3 GatedDeltaNet + 1 gated GQA layer, hidden 256, 8 experts top-2
+ shared) in fp32, tensor-parallel over gloo.  8 requests with seeded random prompts of
16-64 tokens, 32 greedy tokens each, APC on; the tokens must equal a single-process fp32
reference forward exactly."""

import random

import pytest
import torch

from zstep_b200.config import qwen35_tiny
from zstep_b200.models.qwen35_ref import Qwen35Reference
from zstep_b200.models.weights import RandomWeights
from zstep_b200.runtime.launcher import launch, run_to_completion


def reference_generate(prompts, max_tokens, seed=0):
    cfg = qwen35_tiny()
    model = Qwen35Reference(cfg, RandomWeights(cfg, seed=seed))
    outs = []
    for p in prompts:
        st = model.new_state()
        for t in p:
            lg = model.step(st, t)
        gen = []
        for _ in range(max_tokens):
            nxt = int(torch.argmax(lg))
            gen.append(nxt)
            lg = model.step(st, nxt)
        outs.append(gen)
    return outs


def prompts(n=8, seed=7, shared=0):
    rng = random.Random(seed)
    base = [rng.randrange(4096) for _ in range(shared)]
    return [base + [rng.randrange(4096) for _ in range(rng.randint(16, 64))] for _ in range(n)]


@pytest.mark.timeout(600)
@pytest.mark.parametrize("apc,depth", [(False, 0), (True, 0), (True, 1)])
def test_tp2_shm_engine_matches_reference(apc, depth):
    """depth 1: decode steps are published one step ahead of result processing; workers
    continue each slot with the token they sampled (device tokens)."""
    import os

    shm0 = {f for f in os.listdir("/dev/shm") if f.startswith("zstep-")}
    ps = prompts(shared=48 if apc else 0)
    ref = reference_generate(ps, 32)
    eng, coord = launch(model="qwen3.5-tiny", world_size=2, device="cpu", max_seqs=4, max_step_tokens=96,
                        page_size=16, num_pages=256, max_model_len=512, num_ckpt_slots=32 if apc else 0,
                        engine={"max_prefill_chunk": 40, "prefix_caching": apc, "pages_per_node": 1,
                                "recurrent_state": True, "in_flight_depth": depth})
    try:
        for i, p in enumerate(ps):
            assert eng.submit(i, p, 32, True)
        out = run_to_completion(eng)
        for i in range(len(ps)):
            assert out[i] == ref[i], f"request {i} diverged"
        if apc:
            assert eng.stats().prefix_hit_tokens >= 48
        assert (eng.stats().run_ahead_steps > 0) == (depth == 1)
        # Every page is free or held by a cached prefix node (1 page per node here).
        assert eng.free_pages() + eng.cached_prefix_nodes() == 255 and eng.free_slots() == 4
        # The segment's name is unlinked once the workers hold its fd: nothing in /dev/shm.
        assert {f for f in os.listdir("/dev/shm") if f.startswith("zstep-")} == shm0
    finally:
        coord.shutdown()
    assert {f for f in os.listdir("/dev/shm") if f.startswith("zstep-")} == shm0


@pytest.mark.timeout(300)
def test_worker_crash_is_detected():
    """A worker that dies mid-run turns into an engine error, not a hang."""
    eng, coord = launch(model="qwen3.5-tiny", world_size=2, device="cpu", max_seqs=2, max_step_tokens=64,
                        num_pages=64, max_model_len=256, heartbeat_timeout_ms=5000, step_timeout_ms=60000)
    try:
        import os
        import signal

        eng.submit(1, list(range(20)), 50, True)
        eng.step()
        os.kill(coord.pids()[1], signal.SIGKILL)
        with pytest.raises(RuntimeError):
            run_to_completion(eng)
        assert eng.poisoned()
    finally:
        coord.shutdown()


@pytest.mark.timeout(300)
def test_stalled_worker_is_detected_by_its_heartbeat():
    """A worker that stays alive but stops making progress (SIGSTOP: its watchdog thread
    stops refreshing the heartbeat too) turns into an engine error after the heartbeat
    timeout, long before the step timeout."""
    import os
    import signal
    import time

    eng, coord = launch(model="qwen3.5-tiny", world_size=2, device="cpu", max_seqs=2, max_step_tokens=64,
                        num_pages=64, max_model_len=256, heartbeat_timeout_ms=1500, step_timeout_ms=120000)
    pid = coord.pids()[1]
    try:
        eng.submit(1, list(range(20)), 50, True)
        eng.step()
        os.kill(pid, signal.SIGSTOP)
        t0 = time.monotonic()
        with pytest.raises(RuntimeError, match="heartbeat"):
            run_to_completion(eng)
        assert time.monotonic() - t0 < 60  # the heartbeat, not the 120 s step timeout
        assert eng.poisoned()
    finally:
        try:
            os.kill(pid, signal.SIGCONT)
        except ProcessLookupError:
            pass
        coord.shutdown()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("apc,spec", [(False, "none"), (True, "none"), (False, "dspark")])
def test_deepseek_tp2_shm_engine_matches_reference(apc, spec):
    """The DeepSeek-style model (MLA + DSA indexer + mHC + expert-parallel MoE) through the
    same engine and transport: 2 CPU ranks split heads and place experts by rank.  With
    DSpark drafts the engine runs verify steps and the output is still plain greedy."""
    from zstep_b200.config import deepseek_tiny
    from zstep_b200.models.deepseek_ref import DeepSeekReference
    from zstep_b200.models.deepseek_weights import DeepSeekRandomWeights

    cfg = deepseek_tiny()
    rng = random.Random(11)
    base = [rng.randrange(cfg.vocab_size) for _ in range(32 if apc else 0)]
    ps = [base + [rng.randrange(cfg.vocab_size) for _ in range(rng.randint(8, 24))] for _ in range(6)]
    model = DeepSeekReference(cfg, DeepSeekRandomWeights(cfg, seed=0))
    ref = []
    for p in ps:
        st = model.new_state()
        for t in p:
            lg = model.step(st, t)
        gen = []
        for _ in range(12):
            gen.append(int(torch.argmax(lg)))
            lg = model.step(st, gen[-1])
        ref.append(gen)
    # The model keeps no recurrent state: a prefix hit reuses the shared pages through the
    # page table (the runner's paged caches), with no checkpoint slots.
    eng, coord = launch(model="deepseek-tiny", world_size=2, device="cpu", max_seqs=2, max_step_tokens=64,
                        page_size=16, num_pages=128, max_model_len=256,
                        engine={"max_prefill_chunk": 24, "prefix_caching": apc, "pages_per_node": 1,
                                "recurrent_state": False, "spec_method": spec,
                                "num_spec_tokens": 3 if spec != "none" else 0})
    try:
        for i, p in enumerate(ps):
            assert eng.submit(i, p, 12, True)
        out = run_to_completion(eng)
        for i in range(len(ps)):
            assert out[i] == ref[i], f"request {i} diverged"
        if apc:
            assert eng.stats().prefix_hit_tokens >= 16
        if spec != "none":
            assert eng.stats().spec_verify_steps > 0 and eng.stats().spec_drafts > 0
    finally:
        coord.shutdown()


@pytest.mark.timeout(300)
def test_tp2_workers_ignore_an_inherited_torchrun_agent_store(monkeypatch):
    """A master started inside a torchrun job inherits TORCHELASTIC_USE_AGENT_STORE=True.
    Its workers must still host their own process group (rank 0 runs the store); before
    the fix every worker became a store client and the group never formed."""
    monkeypatch.setenv("TORCHELASTIC_USE_AGENT_STORE", "True")
    ps = prompts(n=2)
    ref = reference_generate(ps, 4)
    eng, coord = launch(model="qwen3.5-tiny", world_size=2, device="cpu", max_seqs=2, max_step_tokens=96,
                        page_size=16, num_pages=64, max_model_len=256, ready_timeout_ms=120000)
    try:
        for i, p in enumerate(ps):
            assert eng.submit(i, p, 4, True)
        out = run_to_completion(eng)
        assert [out[i] for i in range(len(ps))] == ref
    finally:
        coord.shutdown()


@pytest.mark.timeout(600)
def test_tp2_mtp_speculation_matches_greedy_reference():
    """MTP drafting in the workers: every sampled step returns K drafts from the MTP layer,
    the engine schedules verify steps of width K+1 and the workers roll their state back to
    the last accepted row.  Drafts only change how many tokens a step yields, so the output
    must equal plain greedy decoding exactly."""
    ps = prompts(n=4)
    ref = reference_generate(ps, 24)
    eng, coord = launch(model="qwen3.5-tiny", world_size=2, device="cpu", max_seqs=4, max_step_tokens=96,
                        page_size=16, num_pages=256, max_model_len=512,
                        engine={"max_prefill_chunk": 40, "recurrent_state": True, "spec_method": "mtp",
                                "num_spec_tokens": 3})
    try:
        for i, p in enumerate(ps):
            assert eng.submit(i, p, 24, True)
        out = run_to_completion(eng)
        for i in range(len(ps)):
            assert out[i] == ref[i], f"request {i} diverged"
        st = eng.stats()
        assert st.spec_verify_steps > 0 and st.spec_drafts > 0
    finally:
        coord.shutdown()


@pytest.mark.timeout(600)
def test_tp2_ngram_speculation_matches_greedy_reference():
    """n-gram drafts (prompt lookup, windows 2..5) on prompts with repeated phrases: the
    engine proposes drafts from earlier occurrences, the workers verify and roll their
    recurrent state back, and the output is still plain greedy."""
    rng = random.Random(5)
    ps = []
    for _ in range(3):
        phrase = [rng.randrange(4096) for _ in range(6)]
        ps.append([rng.randrange(4096) for _ in range(5)] + phrase * 4 + phrase[:3])
    ref = reference_generate(ps, 16)
    eng, coord = launch(model="qwen3.5-tiny", world_size=2, device="cpu", max_seqs=4, max_step_tokens=96,
                        page_size=16, num_pages=256, max_model_len=512,
                        engine={"max_prefill_chunk": 40, "recurrent_state": True, "spec_method": "ngram",
                                "num_spec_tokens": 3})
    try:
        for i, p in enumerate(ps):
            assert eng.submit(i, p, 16, True)
        out = run_to_completion(eng)
        for i in range(len(ps)):
            assert out[i] == ref[i], f"request {i} diverged"
        st = eng.stats()
        assert st.spec_verify_steps > 0 and st.spec_drafts > 0
    finally:
        coord.shutdown()


@pytest.mark.timeout(600)
def test_deepseek_dram_tier_demotes_and_reloads_through_shm():
    """The host DRAM tier end to end: attention-only model, prefix caching with one page
    per node, HBM pages for about one request.  Alternating two prompt families evicts each
    family's prefix to the workers' host arenas (KvTransfer D2H) and reloads it for the next
    request of that family (H2D); the 2 CPU ranks keep paged caches, so the output equals the
    single-process reference only if every page comes back intact."""
    from zstep_b200.config import deepseek_tiny
    from zstep_b200.models.deepseek_ref import DeepSeekReference
    from zstep_b200.models.deepseek_weights import DeepSeekRandomWeights

    cfg = deepseek_tiny()
    V = cfg.vocab_size
    fam = [[(7 * i + 3) % V for i in range(40)], [(11 * i + 5) % V for i in range(40)]]
    ps = [fam[k % 2] + [(k * 13 + j) % V for j in range(5)] for k in range(6)]
    model = DeepSeekReference(cfg, DeepSeekRandomWeights(cfg, seed=0))
    ref = []
    for p in ps:
        st = model.new_state()
        for t in p:
            lg = model.step(st, t)
        gen = []
        for _ in range(6):
            gen.append(int(torch.argmax(lg)))
            lg = model.step(st, gen[-1])
        ref.append(gen)
    eng, coord = launch(model="deepseek-tiny", world_size=2, device="cpu", max_seqs=1, max_step_tokens=64,
                        page_size=4, num_pages=21, max_model_len=128, dram_kv_blocks=48,
                        engine={"max_prefill_chunk": 32, "prefix_caching": True, "pages_per_node": 1,
                                "recurrent_state": False, "dram_blocks": 48})
    try:
        for i, p in enumerate(ps):
            assert eng.submit(i, p, 6, True)
        out = run_to_completion(eng)
        for i in range(len(ps)):
            assert out[i] == ref[i], f"request {i} diverged"
        st = eng.stats()
        assert st.dram_offloads > 0 and st.dram_reloads > 0 and st.dram_hit_tokens > 0, \
            (st.dram_offloads, st.dram_reloads, st.dram_hit_tokens)
        assert st.prefix_hit_tokens > 0
    finally:
        coord.shutdown()
