"""Speculative decoding on the B200 runner: verify steps with oracle drafts (full and
partial acceptance) must reproduce greedy decoding and leave the recurrent state exactly
as plain decoding would; the MTP head's first draft must match the fp32 reference head."""

import numpy as np
import pytest
import torch

from zstep_b200.config import qwen35_small_gpu
from zstep_b200.models.qwen35 import Qwen35Runner
from zstep_b200.models.qwen35_ref import Qwen35Reference
from zstep_b200.models.weights import RandomWeights
from zstep_b200.runtime import wire
from zstep_b200.runtime.runners import GpuRunner

pytestmark = pytest.mark.gpu
K = 3


@pytest.fixture(scope="module")
def setup():
    cfg = qwen35_small_gpu(num_layers=4, vocab=8192, experts=32)
    src = RandomWeights(cfg, seed=21)
    runner = Qwen35Runner(cfg, weights=src, max_seqs=8, max_prefill_tokens=256, num_pages=64, max_model_len=256,
                          num_spec_tokens=K)
    ref = Qwen35Reference(cfg, src, device="cuda", quant=True)
    g = GpuRunner.wrap(runner)
    return cfg, runner, ref, g


def make_plan(seqs):
    """seqs: list of (slot, row tokens, first position, spec_width, sample)."""
    ids, pos, rslot, qs, sw, sr, ss = [], [], [], [0], [], [], []
    for slot, toks, p0, w, sample in seqs:
        ids += toks
        pos += list(range(p0, p0 + len(toks)))
        rslot += [slot] * len(toks)
        qs.append(qs[-1] + len(toks))
        sw.append(w)
        sr.append(qs[-1] - 1 if sample else -1)
        ss.append(slot)
    i32 = lambda v: np.array(v, dtype=np.int32)  # noqa: E731
    return {"num_rows": len(ids), "query_start": i32(qs), "token_ids": i32(ids), "positions": i32(pos),
            "row_slot": i32(rslot), "spec_width": i32(sw), "sample_row": i32(sr), "seq_slot": i32(ss),
            "ckpt_row": i32([]), "ckpt_slot": i32([]), "flags": 0}


def greedy_ref(ref, prompt, n):
    st = ref.new_state()
    for t in prompt:
        lg = ref.step(st, t)
    out = []
    for _ in range(n):
        nxt = int(lg.argmax())
        out.append(nxt)
        lg = ref.step(st, nxt)
    return out


def runner_greedy(runner, prompts, slots, n):
    """Plain (non-speculative) greedy decoding with the runner's own decode path."""
    ids, pos, sl, starts = [], [], [], [0]
    for s, p in zip(slots, prompts):
        ids += p
        pos += list(range(len(p)))
        sl += [s] * len(p)
        starts.append(starts[-1] + len(p))
    runner.stage(ids, pos, sl, seq_start=starts)
    toks = runner.prefill_forward(len(ids), len(prompts)).cpu().tolist()
    out = [[t] for t in toks]
    for step in range(n - 1):
        runner.stage([o[-1] for o in out], [len(p) + step for p in prompts], slots)
        nxt = runner.decode_forward(len(prompts)).cpu().tolist()
        for o, t in zip(out, nxt):
            o.append(t)
    return out


@pytest.mark.parametrize("graphs", [True, False], ids=["graph", "eager"])
def test_verify_with_oracle_drafts_matches_greedy(setup, graphs, monkeypatch):
    """Verify steps fed the runner's own greedy continuation (corrupted at chosen places)
    accept exactly the uncorrupted prefix, reproduce greedy decoding, and leave the same
    recurrent state as plain decoding (the roll-back replay).  `graph`: the steady-state
    verify steps take the CUDA-graph path (on-device verify, roll-back and drafting);
    `eager`: the host-driven path."""
    import dataclasses

    from zstep_b200.runtime import runners
    from zstep_b200.utils.env import runtime_config

    monkeypatch.setattr(runners, "runtime_config",
                        lambda: dataclasses.replace(runtime_config(), decode_graphs=graphs))
    cfg, runner, ref, g = setup
    if graphs:
        calls = []
        real = g._execute_spec_graph
        monkeypatch.setattr(g, "_execute_spec_graph", lambda *a: calls.append(1) or real(*a))
    gen = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in (9, 23, 14)]
    for s in range(6):
        runner.set_pages(s, list(range(1 + 10 * s, 1 + 10 * (s + 1))))
    truth = runner_greedy(runner, prompts, [0, 1, 2], 14)
    spec_slots = [3, 4, 5]
    out = g._execute_spec(make_plan([(spec_slots[s], p, 0, 0, True) for s, p in enumerate(prompts)]), 3,
                          np.zeros(3, dtype=wire.SEQ_OUTPUT_DTYPE))
    produced = [[int(o["tokens"][0])] for o in out]
    assert all(int(o["num_drafts"]) == K for o in out)
    # Oracle drafts, corrupted per sequence so the steps exercise full acceptance, partial
    # acceptance and immediate rejection.
    corrupt = [None, 1, 0]
    ok = [p[0] == t[0] for p, t in zip(produced, truth)]
    for step in range(3):
        seqs = []
        for s in range(3):
            have = produced[s]
            drafts = list(truth[s][len(have):len(have) + K])
            if corrupt[s] is not None and step % 2 == 0:
                drafts[corrupt[s]] = (drafts[corrupt[s]] + 1) % cfg.vocab_size
            p0 = len(prompts[s]) + len(have) - 1
            seqs.append((spec_slots[s], [have[-1]] + drafts, p0, 1 + len(drafts), True))
        out = g._execute_spec(make_plan(seqs), 3, np.zeros(3, dtype=wire.SEQ_OUTPUT_DTYPE))
        assert runner.check_error() == 0
        for s in range(3):
            n = int(out[s]["num_tokens"])
            exp_n = K + 1 if (corrupt[s] is None or step % 2 == 1) else corrupt[s] + 1
            ok[s] = ok[s] and n == exp_n
            produced[s] += [int(t) for t in out[s]["tokens"][:n]]
            ok[s] = ok[s] and produced[s] == truth[s][:len(produced[s])]
    assert sum(ok) >= 2, (produced, truth)
    if graphs:
        assert len(calls) == 3  # every verify step took the graph path
    # Recurrent state after the accepted tokens equals plain decoding's state after the
    # same inputs (prompt plus every produced token but the newest).
    for s in range(3):
        if not ok[s]:
            continue
        plain = runner_greedy(runner, [prompts[s]], [s], len(produced[s]))[0]
        assert plain == produced[s]
        # The verify pass computes the replayed rows' GDN inputs through the grouped-row
        # kernels and the (K+1)-row GEMM tiles, plain decoding through one-row kernels: the
        # inputs agree to the last bits, not bit for bit.  A replay over wrong rows moves
        # whole state rows, which the mean difference catches.
        spec_st, plain_st = runner.ssm_state[:, spec_slots[s]], runner.ssm_state[:, s]
        torch.testing.assert_close(spec_st, plain_st, rtol=3e-2, atol=3e-2)
        assert (spec_st - plain_st).abs().mean().item() < 1e-3
        par = (len(prompts[s]) + len(produced[s]) - 1) & 1  # conv window buffer of the next position
        # The windows hold the last GDN inputs, which pass through MXFP8 re-quantization of
        # slightly different activations: a sequence whose window comes from verify-pass
        # rows can differ by up to ~0.1 where both paths differ from the fp32 reference by
        # ~0.16 (mean 0.03).  A window in the wrong buffer or from the wrong rows differs by
        # the values' own size (~1-4).
        spec_w = runner.conv_state[:, spec_slots[s], par].float()
        plain_w = runner.conv_state[:, s, par].float()
        assert (spec_w - plain_w).abs().max().item() < 0.25
        assert (spec_w - plain_w).abs().mean().item() < 0.02


def test_mtp_first_draft_matches_reference(setup):
    cfg, runner, ref, g = setup
    gen = torch.Generator().manual_seed(9)
    prompt = torch.randint(0, cfg.vocab_size, (12,), generator=gen).tolist()
    runner.set_pages(4, list(range(40, 48)))
    out = g._execute_spec(make_plan([(4, prompt, 0, 0, True)]), 1, np.zeros(1, dtype=wire.SEQ_OUTPUT_DTYPE))
    tok = int(out[0]["tokens"][0])
    st = ref.new_state()
    hidden = []
    for t in prompt:
        lg = ref.step(st, t)
        hidden.append(st.hidden)
    # Catch-up over the prompt: MTP input at position p is (token p+1, target hidden p).
    nxt = prompt[1:] + [tok]
    for p in range(len(prompt)):
        mlg, _ = ref.mtp_step(st, nxt[p], hidden[p], p)
    d1 = int(mlg.argmax())
    vals = runner.buf["out_vals"][:1]  # last lm_head call: the chained drafts (K-1th); check the first draft id
    assert int(out[0]["num_drafts"]) == K
    top2 = torch.topk(mlg, 2).values
    if float(top2[0] - top2[1]) > 0.05:  # skip near-ties
        assert int(out[0]["next_drafts"][0]) == d1
    del vals
