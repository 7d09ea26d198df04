"""The full-distribution sampling head inside the B200 runner: plans whose sequences ask
for top-k / top-p / penalties / logprobs go through the f32 lm_head + sampling kernel."""

import numpy as np
import pytest

from zstep_b200.config import qwen35_small_gpu
from zstep_b200.models.qwen35 import Qwen35Runner
from zstep_b200.models.weights import RandomWeights
from zstep_b200.runtime import wire
from zstep_b200.runtime.runners import GpuRunner

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    cfg = qwen35_small_gpu(num_layers=4, vocab=8192, experts=32)
    r = Qwen35Runner(cfg, weights=RandomWeights(cfg, seed=5), max_seqs=8, max_prefill_tokens=128, num_pages=64,
                     max_model_len=256)
    gr = GpuRunner.wrap(r)
    for s in range(4):
        r.set_pages(s, list(range(1 + 8 * s, 1 + 8 * (s + 1))))
    return gr


def plan(prompts, pos0, params, decode):
    ids, pos, slot, qs = [], [], [], [0]
    for s, p in enumerate(prompts):
        ids += p
        pos += list(range(pos0[s], pos0[s] + len(p)))
        slot += [s] * len(p)
        qs.append(qs[-1] + len(p))
    n = len(prompts)
    sp = np.zeros(n, dtype=wire.SAMPLING_DTYPE)
    for i, d in enumerate(params):
        sp[i]["temperature"], sp[i]["top_p"], sp[i]["top_k"] = d.get("t", 0.0), d.get("p", 1.0), d.get("k", 0)
        sp[i]["presence"], sp[i]["frequency"], sp[i]["repetition"] = d.get("pres", 0), d.get("freq", 0), d.get("rep", 1)
        sp[i]["seed"], sp[i]["logprobs"] = d.get("seed", i), d.get("lp", -1)
    i32 = lambda v: np.asarray(v, dtype=np.int32)  # noqa: E731
    flags = (wire.FLAG_DECODE_ONLY if decode else 0) | (wire.FLAG_SAMPLING if any(d.get("t", 0) > 0 for d in params)
                                                        else 0)
    return {"opcode": wire.OP_NORMAL, "flags": flags, "num_rows": len(ids), "num_seqs": n, "token_ids": i32(ids),
            "positions": i32(pos), "row_slot": i32(slot), "query_start": i32(qs), "seq_slot": i32(range(n)),
            "sample_row": i32([q - 1 for q in qs[1:]]), "sampling": sp, "dirty_rows": i32([]),
            "dirty_pages": np.zeros((0, 16), np.int32), "ckpt_row": i32([]), "ckpt_slot": i32([]),
            "restore_slot": i32([-1] * n), "spec_width": i32([0] * n)}


def run(g, params, steps=5):
    prompts = [[3, 77, 1500, 9], [4000, 12, 8], [600, 601, 602, 603, 604]]
    out = g.execute(plan(prompts, [0, 0, 0], params, False))
    toks = [[int(o["tokens"][0])] for o in out]
    lps = [[float(o["logprobs"][0])] for o in out]
    for st in range(steps - 1):
        cur = [[t[-1]] for t in toks]
        out = g.execute(plan(cur, [len(p) + st for p in prompts], params, True))
        for i, o in enumerate(out):
            toks[i].append(int(o["tokens"][0]))
            lps[i].append(float(o["logprobs"][0]))
    return toks, lps, out


def test_top_k_one_equals_greedy_and_logprobs(g):
    greedy, _, _ = run(g, [{}, {}, {}])
    topk1, lps, out = run(g, [{"t": 0.9, "k": 1, "lp": 3}] * 3)
    assert topk1 == greedy
    assert all(all(x <= 0.0 for x in row) for row in lps) and any(x < 0 for row in lps for x in row)
    assert all(int(o["top_ids"][0]) == int(o["tokens"][0]) for o in out)   # the greedy token is the top-1


def test_penalty_history_and_nucleus_reproducibility(g):
    """Penalised steps record each sequence's generated tokens in its slot ring (the
    prompt restarts it); the same seeds reproduce nucleus draws."""
    pen, _, _ = run(g, [{"rep": 1.3, "freq": 0.5, "pres": 0.5}] * 3, steps=6)
    h = g.head
    for s in range(3):
        n = int(h.hist_len[s])
        assert n == 6
        assert h.hist[s, :n].cpu().tolist() == pen[s]
    a, _, _ = run(g, [{"t": 1.0, "p": 0.9, "seed": 7}] * 3)
    b, _, _ = run(g, [{"t": 1.0, "p": 0.9, "seed": 7}] * 3)
    assert a == b
