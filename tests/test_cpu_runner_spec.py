"""The fp32 reference runner's speculative path, driven by hand-built step plans: MTP
drafts after a sampled step, a verify step whose drafts are all right (state advances by
K+1 rows), one whose drafts are all wrong (state rolls back to the first row), and greedy
output equal to plain decoding throughout."""

import argparse

import numpy as np
import torch

from zstep_b200.config import qwen35_tiny
from zstep_b200.models.qwen35_ref import Qwen35Reference
from zstep_b200.models.weights import RandomWeights
from zstep_b200.runtime import wire
from zstep_b200.runtime.runners import CpuReferenceRunner

K = 3


def plan(rows, positions, width=0, sample=True):
    n = len(rows)
    samp = np.zeros(1, dtype=wire.SAMPLING_DTYPE)
    samp["top_p"], samp["repetition"], samp["logprobs"] = 1.0, 1.0, -1
    return {"opcode": wire.OP_NORMAL, "num_seqs": 1, "query_start": np.array([0, n], np.int32),
            "token_ids": np.array(rows, np.int32), "positions": np.array(positions, np.int32),
            "ckpt_row": np.zeros(0, np.int32), "ckpt_slot": np.zeros(0, np.int32),
            "seq_slot": np.array([0], np.int32), "restore_slot": np.array([-1], np.int32),
            "spec_width": np.array([width], np.int32), "sample_row": np.array([n - 1 if sample else -1], np.int32),
            "sampling": samp,
            # slot 0's page table (attention-only models keep paged caches)
            "dirty_rows": np.array([0], np.int32), "dirty_pages": np.arange(1, 9, dtype=np.int32)[None]}


def greedy(prompt, n):
    cfg = qwen35_tiny()
    m = Qwen35Reference(cfg, RandomWeights(cfg, seed=0))
    st = m.new_state()
    for t in prompt:
        lg = m.step(st, t)
    out = []
    for _ in range(n):
        out.append(int(torch.argmax(lg)))
        lg = m.step(st, out[-1])
    return out


def test_mtp_drafts_verify_and_roll_back():
    args = argparse.Namespace(model="qwen3.5-tiny", seed=0, spec_method="mtp", num_spec_tokens=K)
    r = CpuReferenceRunner(args, 0, 1, wire.Geometry(max_seqs=1))
    prompt = [int(x) for x in torch.randint(0, 4096, (20,), generator=torch.Generator().manual_seed(3))]
    ref = greedy(prompt, 12)

    # Prefill in two chunks: the first samples nothing (MTP catch-up only).
    o = r.execute(plan(prompt[:8], range(8), sample=False))
    assert o[0]["num_tokens"] == 0 and o[0]["num_drafts"] == 0
    o = r.execute(plan(prompt[8:], range(8, 20)))
    assert o[0]["num_tokens"] == 1 and int(o[0]["tokens"][0]) == ref[0]
    assert o[0]["num_drafts"] == K
    assert r.states[0].mtp_keys.shape[0] == 20 + K - 1  # one MTP entry per row + chained drafts

    # All drafts right: K accepted + the bonus token; the state sits after the last row.
    o = r.execute(plan([ref[0]] + ref[1:1 + K], range(20, 21 + K), width=K + 1))
    assert o[0]["num_tokens"] == K + 1 and list(o[0]["tokens"][:K + 1]) == ref[1:2 + K]
    assert r.states[0].pos == 21 + K and o[0]["num_drafts"] == K
    last = ref[K + 1]

    # All drafts wrong: only the target's own token; the state rolls back to the first row.
    p0 = 21 + K
    wrong = [(t + 1) % 4096 for t in ref[K + 2:2 * K + 2]]
    o = r.execute(plan([last] + wrong, range(p0, p0 + K + 1), width=K + 1))
    assert o[0]["num_tokens"] == 1 and int(o[0]["tokens"][0]) == ref[K + 2]
    assert r.states[0].pos == p0 + 1

    # Plain decode continues from the rolled-back state.
    o = r.execute(plan([ref[K + 2]], [p0 + 1]))
    assert int(o[0]["tokens"][0]) == ref[K + 3]


def test_dspark_drafts_verify_and_roll_back():
    """The DeepSeek-style model with DSpark drafts: contexts stored for every row across
    prefill chunks (drafts equal a direct call sequence on a fresh reference), a verify step
    with right drafts advances K+1 rows, one with wrong drafts rolls the caches back."""
    from zstep_b200.config import deepseek_tiny
    from zstep_b200.models.deepseek_ref import DeepSeekReference
    from zstep_b200.models.deepseek_weights import DeepSeekRandomWeights

    cfg = deepseek_tiny()
    args = argparse.Namespace(model="deepseek-tiny", seed=0, spec_method="dspark", num_spec_tokens=K)
    r = CpuReferenceRunner(args, 0, 1, wire.Geometry(max_seqs=1))
    g = torch.Generator().manual_seed(5)
    prompt = [int(x) for x in torch.randint(0, cfg.vocab_size, (14,), generator=g)]

    m = DeepSeekReference(cfg, DeepSeekRandomWeights(cfg, seed=0))
    m.load_dspark(DeepSeekRandomWeights(cfg, seed=0))
    st = m.new_state()
    for p, t in enumerate(prompt):
        lg = m.step(st, t)
        m.dspark_context(st, m.last_aux, p)
    first = int(torch.argmax(lg))
    want = m.dspark_draft(m.clone_state(st), first, len(prompt), K)
    ref = []
    for _ in range(10):
        ref.append(int(torch.argmax(lg)))
        lg = m.step(st, ref[-1])

    o = r.execute(plan(prompt[:6], range(6), sample=False))
    assert o[0]["num_drafts"] == 0
    o = r.execute(plan(prompt[6:], range(6, 14)))
    assert int(o[0]["tokens"][0]) == ref[0] == first
    assert list(o[0]["next_drafts"][:K]) == want
    assert all(0 <= d < cfg.vocab_size for d in want)

    o = r.execute(plan([ref[0]] + ref[1:1 + K], range(14, 15 + K), width=K + 1))
    assert list(o[0]["tokens"][:K + 1]) == ref[1:2 + K] and r.states[0].pos == 15 + K
    p0 = 15 + K
    wrong = [(t + 1) % cfg.vocab_size for t in ref[K + 2:2 * K + 2]]
    o = r.execute(plan([ref[K + 1]] + wrong, range(p0, p0 + K + 1), width=K + 1))
    assert o[0]["num_tokens"] == 1 and int(o[0]["tokens"][0]) == ref[K + 2] and r.states[0].pos == p0 + 1
    o = r.execute(plan([ref[K + 2]], [p0 + 1]))
    assert int(o[0]["tokens"][0]) == ref[K + 3]


def test_new_request_past_position_zero_restarts_penalty_history():
    """Prefix hit: the new request's first plan starts at position 16 but carries the slot's
    page-table row, so the slot's generated-token history (penalties) restarts."""
    from zstep_b200.config import deepseek_tiny

    cfg = deepseek_tiny()
    args = argparse.Namespace(model="deepseek-tiny", seed=0, spec_method="none", num_spec_tokens=0)
    r = CpuReferenceRunner(args, 0, 1, wire.Geometry(max_seqs=1))
    prompt = [(7 * i + 1) % cfg.vocab_size for i in range(20)]
    r.execute(plan(prompt, range(20)))
    p = plan([prompt[-1]], [20])
    p["dirty_rows"], p["dirty_pages"] = np.zeros(0, np.int32), np.zeros((0, 8), np.int32)
    r.execute(p)  # the same request continues: history grows
    assert len(r.generated[0]) == 2
    r.execute(plan(prompt[16:], range(16, 20)))  # new request, prefix pages 0..15 reused
    assert len(r.generated[0]) == 1
