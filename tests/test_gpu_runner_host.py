"""Host-side bookkeeping of the B200 runner's speculative path, on CPU: a fake model runner
records what `GpuRunner` asks of it (staging, target forward, state replay, draft-head
catch-up and drafting) for plans mixing a prefill chunk, a plain decode row and a verify
row.  Covers greedy acceptance, the replay of accepted rows, the catch-up rows an MTP head
(needs the following token) and a DSpark head (needs only the row) receive, and the
drafts written back for the engine."""

import numpy as np
import pytest
import torch

from zstep_b200.runtime import wire
from zstep_b200.runtime.runners import GpuRunner

K = 2


class FakeSpec:
    def __init__(self, context_only, targets):
        self.context_only = context_only
        self.targets = targets  # next token per lm row, in lm-row order
        self.calls = []

    def forward(self, rows, n, lm_t, verify_slots, ckpt=None):
        self.calls.append(("forward", lm_t.tolist(), list(verify_slots)))
        return torch.tensor(self.targets[:len(lm_t)])

    def replay(self, groups, slots, positions):
        self.calls.append(("replay", list(groups), list(slots), list(positions)))

    def draft(self, ids, positions, slots, rows_t, last_of_seq):
        self.calls.append(("draft", list(ids), list(positions), list(slots), rows_t.tolist(), list(last_of_seq)))
        return [[500 + 10 * i + k for k in range(K)] for i in range(len(last_of_seq))]

    def catch_up(self, ids, positions, slots, rows_t):
        self.calls.append(("catch_up", list(ids), list(positions), list(slots), rows_t.tolist()))


class FakeModel:
    def __init__(self, spec):
        self.spec = spec
        self.num_spec = K
        self.dev = torch.device("cpu")
        self.cfg = None
        self.page_table = torch.zeros(8, 4, dtype=torch.int32)
        self.max_pages = 4
        self.spec_slot_base = 100
        self.dummy_slot = 99
        self.staged = []

    def stage(self, ids, pos, slots, seq_start=None):
        self.staged.append((list(ids), list(pos), list(slots), seq_start))

    def copy_recurrent_state(self, src, dst):
        raise AssertionError("no restores in these plans")


def plan(seqs):
    """seqs: (slot, tokens, pos0, spec_width, sample)."""
    ids, pos, rslot, qs, srow, sw, slots = [], [], [], [0], [], [], []
    for slot, toks, p0, width, sample in seqs:
        ids += toks
        pos += list(range(p0, p0 + len(toks)))
        rslot += [slot] * len(toks)
        qs.append(len(ids))
        srow.append(len(ids) - 1 if sample else -1)
        sw.append(width)
        slots.append(slot)
    n = len(seqs)
    samp = np.zeros(n, dtype=wire.SAMPLING_DTYPE)  # greedy, no penalties, no logprobs
    samp["top_p"], samp["repetition"], samp["logprobs"] = 1.0, 1.0, -1
    return {"opcode": wire.OP_NORMAL, "num_seqs": n, "num_rows": len(ids), "flags": 0,
            "token_ids": np.array(ids, np.int32), "positions": np.array(pos, np.int32),
            "row_slot": np.array(rslot, np.int32), "query_start": np.array(qs, np.int32),
            "sample_row": np.array(srow, np.int32), "spec_width": np.array(sw, np.int32),
            "seq_slot": np.array(slots, np.int32), "restore_slot": np.full(n, -1, np.int32),
            "dirty_rows": np.zeros(0, np.int32), "dirty_pages": np.zeros((0, 4), np.int32),
            "ckpt_row": np.zeros(0, np.int32), "ckpt_slot": np.zeros(0, np.int32),
            "sampling": samp}


@pytest.mark.parametrize("context_only", [False, True])
def test_prefill_chunk_catch_up_rows(context_only):
    """A chunk that samples nothing: MTP catches up rows 0..L-2 (row j with token j+1);
    DSpark stores a context for every row, the last one included."""
    spec = FakeSpec(context_only, [])
    g = GpuRunner.wrap(FakeModel(spec))
    out = g.execute(plan([(3, [11, 12, 13], 0, 0, False)]))
    assert out[0]["num_tokens"] == 0 and out[0]["req_slot"] == 3
    (kind, ids, positions, slots, rows), = [c for c in spec.calls if c[0] == "catch_up"]
    assert not [c for c in spec.calls if c[0] == "draft"] and slots == [3] * len(ids)
    if context_only:
        assert positions == [0, 1, 2] and rows == [0, 1, 2]
    else:
        assert ids == [12, 13] and positions == [0, 1] and rows == [0, 1]


def test_decode_and_verify_rows():
    """Slot 1 decodes one row; slot 2 verifies [last, d1, d2] where the target accepts d1
    and then disagrees: 2 tokens, replay of the 2 accepted rows, drafts for both."""
    # lm rows: slot 1's row 0 -> 41; slot 2's rows 1..3 -> 7 (= d1), 9 (!= d2), 10
    spec = FakeSpec(False, [41, 7, 9, 10])
    g = GpuRunner.wrap(FakeModel(spec))
    out = g.execute(plan([(1, [5], 20, 0, True), (2, [6, 7, 8], 30, K + 1, True)]))
    assert out[0]["num_tokens"] == 1 and out[0]["tokens"][0] == 41
    assert out[1]["num_tokens"] == 2 and list(out[1]["tokens"][:2]) == [7, 9]
    fwd = spec.calls[0]
    assert fwd[0] == "forward" and fwd[1] == [0, 1, 2, 3] and fwd[2] == [None, 100 + 2]
    replay = [c for c in spec.calls if c[0] == "replay"][0]
    assert replay[1] == [(1, 2)] and replay[2] == [2] and replay[3] == [30]
    draft = [c for c in spec.calls if c[0] == "draft"][0]
    # MTP rows: slot 1 row 0 followed by its sampled token; slot 2 rows 1, 2 followed by
    # the accepted tokens 7 and 9.
    assert draft[1] == [41, 7, 9] and draft[2] == [20, 30, 31] and draft[4] == [0, 1, 2]
    assert draft[5] == [0, 2]  # newest row of each drafting sequence
    assert list(out[0]["next_drafts"][:K]) == [500, 501] and out[0]["num_drafts"] == K
    assert list(out[1]["next_drafts"][:K]) == [510, 511] and out[1]["num_drafts"] == K


class FakePlain(FakeModel):
    """No draft head: decode and prefill paths."""

    def __init__(self):
        super().__init__(None)
        self.calls = []
        self.buf = {"xq": None, "xsf": None, "xq_last": None}
        self.last_lm_sf = None

    def copy_recurrent_state(self, src, dst):
        self.calls.append(("restore", src, dst))

    def decode_step(self, rows):
        self.calls.append(("decode", rows))
        return torch.arange(rows, dtype=torch.int32) + 70

    def prefill_forward(self, rows, n, ckpt=None):
        self.calls.append(("prefill", rows, n, ckpt))
        return torch.arange(n, dtype=torch.int32) + 80

    def checkpoint_args(self, rows, slots, qs):
        return ("ck", list(rows), list(slots))


def test_decode_and_prefill_plans():
    m = FakePlain()
    g = GpuRunner.wrap(m)
    # Decode-only step: page-table rows refreshed, one graph step over the rows.
    p = plan([(1, [5], 20, 0, True), (4, [6], 9, 0, True)])
    p["flags"] = wire.FLAG_DECODE_ONLY
    p["dirty_rows"] = np.array([4], np.int32)
    p["dirty_pages"] = np.array([[7, 8, 9, 10]], np.int32)
    out = g.execute(p)
    assert m.calls == [("decode", 2)] and list(out["tokens"][:, 0]) == [70, 71]
    assert m.page_table[4].tolist() == [7, 8, 9, 10]
    assert m.staged[-1][:3] == ([5, 6], [20, 9], [1, 4])
    # Mixed step: a restored slot, a checkpoint row, one chunk that samples, one that does not.
    m.calls.clear()
    p = plan([(2, [1, 2, 3], 16, 0, True), (3, [4, 5], 0, 0, False)])
    p["restore_slot"] = np.array([40, -1], np.int32)
    p["ckpt_row"], p["ckpt_slot"] = np.array([2], np.int32), np.array([41], np.int32)
    out = g.execute(p)
    assert m.calls[0] == ("restore", 40, 2)
    assert m.calls[1] == ("prefill", 5, 2, ("ck", [2], [41]))
    assert m.staged[-1][3] == [0, 3, 5]
    assert out[0]["num_tokens"] == 1 and out[0]["tokens"][0] == 80 and out[1]["num_tokens"] == 0
    assert list(out["req_slot"]) == [2, 3]


def test_steady_state_verify_uses_the_graph_record():
    """Every sequence verifying K drafts, greedy, no checkpoints: the step replays the verify
    graph of the next bucket, with the padding rows on the dummy slot, and reads accepted
    tokens and next drafts from the device record [n, 2K + 2]."""

    class GraphSpec(FakeSpec):
        def __init__(self):
            super().__init__(False, [])
            self.out_slots = torch.zeros(8, dtype=torch.int32)
            self.g_record = torch.zeros(8, 2 * K + 2, dtype=torch.int32)

        def graph_bucket(self, n):
            return 4 if n <= 4 else None

        def run_verify_graph(self, nb):
            self.calls.append(("graph", nb, self.out_slots[:nb].tolist()))
            # sequence i accepts i + 1 tokens (tokens 60 + i ...), next drafts 90 + i, 91 + i
            for i in range(3):
                acc = i + 1
                self.g_record[i, 0] = acc
                self.g_record[i, 1:1 + acc] = torch.arange(acc, dtype=torch.int32) + 60 + i
                self.g_record[i, K + 2:2 * K + 2] = torch.tensor([90 + i, 91 + i], dtype=torch.int32)

    spec = GraphSpec()
    m = FakeModel(spec)
    g = GpuRunner.wrap(m)
    out = g.execute(plan([(s, [1, 2, 3], 10 * s, K + 1, True) for s in (1, 2, 5)]))
    (kind, nb, slots), = [c for c in spec.calls if c[0] == "graph"]
    assert nb == 4 and slots == [101, 102, 105, 99]  # spare state slots, dummy padding
    ids, pos, rslot, seq_start = m.staged[-1]
    assert len(ids) == 4 * (K + 1) and rslot[9:] == [99, 99, 99] and pos[9:] == [1, 1, 1]
    assert seq_start == [0, 3, 6, 9, 12]
    for i in range(3):
        assert out[i]["num_tokens"] == i + 1 and list(out[i]["tokens"][:i + 1]) == list(range(60 + i, 61 + 2 * i))
        assert list(out[i]["next_drafts"][:K]) == [90 + i, 91 + i]


def test_penalty_rings_restart_for_new_requests():
    """A request that starts past position 0 (prefix hit) in a reused slot is recognised by
    the page-table row its first plan carries; its penalty ring restarts like one starting
    at position 0, while a continuing request's ring is kept."""

    class FakeHead:
        def __init__(self):
            self.resets = []

        def reset(self, slots):
            self.resets.append(sorted(slots))

        def sample(self, n, xq, xsf, slots, params, top_n=0, record=None):
            return np.zeros(n, np.int64), None, None, None

    m = FakePlain()
    g = GpuRunner.wrap(m)
    g.head = FakeHead()
    p = plan([(1, [5], 40, 0, True), (2, [6, 7], 32, 0, True), (3, [8], 0, 0, True)])
    p["flags"] = 0
    p["sampling"]["presence"][:] = 0.5  # penalties: the full-distribution head runs
    p["dirty_rows"] = np.array([2], np.int32)  # slot 2's request is new (prefix hit at 32)
    p["dirty_pages"] = np.array([[3, 4, 5, 6]], np.int32)
    g.execute(p)
    assert g.head.resets == [[2, 3]]  # slot 1 continues; slot 3 starts at position 0
