"""Scheduler invariants of the C++ serving engine, driven through a fake backend.

The fake model's next token is a hash of the sequence's full token history, which the
backend reconstructs from the plans alone (positions, restores from checkpoint slots,
checkpoint snapshots, speculative rollback).  Any mistake in chunking, prefix reuse or
checkpoint bookkeeping therefore changes the generated tokens."""

import pytest

from zstep_b200 import _master as m

V = 1000


def f(history):
    h = 0
    for i, t in enumerate(history):
        h = (h * 1000003 + (i + 1) * (t + 7)) % 2147483647
    return h % V


def expected(prompt, max_tokens, eos=(), fn=None):
    fn = fn or f
    hist, out = list(prompt), []
    while len(out) < max_tokens:
        t = fn(hist)
        out.append(t)
        hist.append(t)
        if t in eos:
            break
    return out


class FakeBackend:
    def __init__(self, fn=None):
        self.hist = {}
        self.ckpt = {}
        self.plans = []
        self.f = fn or f

    def __call__(self, p):
        self.plans.append(p)
        outs = []
        qs = p["query_start"]
        ck = dict(zip(p["ckpt_row"], p["ckpt_slot"]))
        for i, slot in enumerate(p["seq_slot"]):
            r0, r1 = qs[i], qs[i + 1]
            if p["restore_slot"][i] >= 0:
                self.hist[slot] = list(self.ckpt[p["restore_slot"][i]])
            if p["positions"][r0] == 0:
                self.hist[slot] = []
            h = self.hist[slot]
            assert len(h) == p["positions"][r0], "plan position does not continue the slot's history"
            snaps = []
            for r in range(r0, r1):
                h.append(p["token_ids"][r])
                if r in ck:
                    self.ckpt[ck[r]] = list(h)
                snaps.append(list(h))
            if p["sample_row"][i] < 0:
                outs.append({"tokens": []})
                continue
            if p["spec_width"][i] > 0:
                drafts = p["token_ids"][r0 + 1:r1]
                targets = [self.f(s) for s in snaps]
                acc = []
                for j, d in enumerate(drafts):
                    if targets[j] != d:
                        acc.append(targets[j])
                        break
                    acc.append(d)
                else:
                    acc.append(targets[len(drafts)])
                self.hist[slot] = snaps[len(acc) - 1]
                outs.append({"tokens": acc})
            else:
                outs.append({"tokens": [self.f(h)]})
        return outs


def make(**kw):
    cfg = m.EngineConfig()
    cfg.max_seqs = kw.get("max_seqs", 8)
    cfg.max_step_tokens = kw.get("max_step_tokens", 64)
    cfg.max_prefill_chunk = kw.get("chunk", 32)
    cfg.page_size = 4
    cfg.num_pages = kw.get("num_pages", 256)
    cfg.max_model_len = 512
    cfg.prefix_caching = kw.get("apc", False)
    cfg.pages_per_node = kw.get("ppn", 2)
    cfg.recurrent_state = kw.get("recurrent", False)
    cfg.num_ckpt_slots = kw.get("ckpt", 0)
    cfg.prefill_policy = kw.get("policy", "fifo")
    cfg.spec_method = kw.get("spec", "none")
    cfg.num_spec_tokens = kw.get("k", 0)
    cfg.ngram_min = kw.get("ngram_min", 2)
    cfg.ngram_max = kw.get("ngram_max", 2)
    for k in ("starvation_steps", "starvation_ms", "max_mixed_step_tokens", "dynamic_prefill_budget",
              "backlog_low_tokens", "backlog_high_tokens"):
        if k in kw:
            setattr(cfg, k, kw[k])
    be = FakeBackend(kw.get("fn"))
    return m.Engine(cfg, be), be


def run(eng, limit=10000):
    out = {}
    done = set()
    for _ in range(limit):
        if not eng.has_work():
            break
        for ev in eng.step():
            out.setdefault(ev["request_id"], []).extend(ev["tokens"])
            if ev["finish"]:
                done.add(ev["request_id"])
    return out, done


def test_basic_generation_and_conservation():
    eng, be = make()
    reqs = {i: ([(i * 37 + j) % V for j in range(5 + 9 * i)], 3 + i) for i in range(6)}
    for rid, (p, mt) in reqs.items():
        assert eng.submit(rid, p, mt)
    out, done = run(eng)
    assert done == set(reqs)
    for rid, (p, mt) in reqs.items():
        assert out[rid] == expected(p, mt)
    assert eng.free_pages() == 255 and eng.free_slots() == 8


def test_chunked_prefill_and_decode_buckets():
    eng, be = make(chunk=8, max_step_tokens=20)
    p = list(range(50))
    eng.submit(1, p, 4)
    out, _ = run(eng)
    assert out[1] == expected(p, 4)
    prefill = [pl for pl in be.plans if not (pl["flags"] & 1)]
    assert all(len(pl["token_ids"]) <= 20 for pl in be.plans)
    assert len(prefill) >= 7  # 50 tokens in chunks of <= 8
    decode = [pl for pl in be.plans if pl["flags"] & 1]
    assert decode and all(pl["bucket"] >= len(pl["seq_slot"]) for pl in decode)


def test_eos_and_ignore_eos():
    p = [1, 2, 3]
    ref = expected(p, 20)
    eos = ref[2]
    eng, _ = make()
    eng.submit(1, p, 20, False, [eos])
    eng.submit(2, p, 20, True, [eos])
    out, _ = run(eng)
    assert out[1] == ref[:ref.index(eos) + 1]
    assert out[2] == ref


def test_cancel_releases_everything():
    eng, _ = make()
    for i in range(4):
        eng.submit(i, list(range(10 + i)), 50)
    eng.step()
    eng.step()
    assert eng.cancel(1) and eng.cancel(3)
    assert not eng.cancel(99)
    run(eng)
    assert eng.free_pages() == 255 and eng.free_slots() == 8


@pytest.mark.parametrize("seed", [1, 2, 3])
@pytest.mark.parametrize("mode", ["plain", "apc", "ngram"])
def test_random_cancellation_leaks_nothing(seed, mode):
    """Half of the requests are cancelled at random steps (while waiting, mid-prefill or
    mid-decode) among prompts that share prefixes.  Survivors must still produce exactly the
    model's tokens, and once idle every request slot, KV page and checkpoint slot is free
    or held by a cached prefix node."""
    import random

    rng = random.Random(seed)
    kw = dict(max_seqs=6, num_pages=160, chunk=16, max_step_tokens=48)
    if mode == "apc":
        kw.update(apc=True, ppn=1, recurrent=True, ckpt=24)
    if mode == "ngram":
        kw.update(spec="ngram", k=3)
    eng, _ = make(**kw)
    bases = [[rng.randrange(V) for _ in range(rng.randint(4, 20))] for _ in range(3)]
    prompts, maxt, live = {}, {}, set()
    pending = list(range(24))
    out, cancelled = {}, set()
    for step in range(4000):
        while pending and rng.random() < 0.5:
            rid = pending.pop(0)
            p = rng.choice(bases) + [rng.randrange(V) for _ in range(rng.randint(1, 24))]
            prompts[rid], maxt[rid] = p, rng.randint(1, 12)
            if eng.submit(rid, p, maxt[rid]):
                live.add(rid)
        if live and rng.random() < 0.15:
            rid = rng.choice(sorted(live))
            if rid % 2 == 0 and eng.cancel(rid):
                cancelled.add(rid)
                live.discard(rid)
        if not eng.has_work() and not pending:
            break
        for ev in eng.step():
            out.setdefault(ev["request_id"], []).extend(ev["tokens"])
            if ev["finish"]:
                live.discard(ev["request_id"])
    assert not eng.has_work() and not pending and not live
    assert cancelled, "the schedule cancelled nothing"
    for rid in prompts:
        if rid not in cancelled:
            assert out.get(rid) == expected(prompts[rid], maxt[rid]), rid
    assert eng.free_slots() == 6
    cached = eng.cached_prefix_nodes()
    assert eng.free_pages() + cached * (1 if mode == "apc" else 0) == 159
    if mode == "apc":
        assert eng.free_ckpt_slots() + cached == 24


def test_srpt_starvation_cap_admits_the_long_prompt():
    """SRPT with a steady stream of short prompts and one request slot: the long prompt
    that arrived first still gets in once it has waited the starvation cap."""
    eng, _ = make(max_seqs=1, policy="srpt", chunk=64, max_step_tokens=64)
    cap, slack = 64, 6  # the engine's default starvation cap (steps); steps to finish the short in the slot
    long_p = [(3 * j + 1) % V for j in range(40)]
    eng.submit(0, long_p, 2)
    first_token_step = {}
    rid = 1
    for step in range(200):
        if step < 60:  # a new short prompt every step
            eng.submit(rid, [rid % V, (rid * 7) % V], 1)
            rid += 1
        for ev in eng.step():
            first_token_step.setdefault(ev["request_id"], step)
        if not eng.has_work():
            break
    # Short prompts overtake it, but only until the cap (in steps) is reached.
    overtaken = [r for r, s in first_token_step.items() if r != 0 and s < first_token_step[0]]
    assert overtaken, "SRPT never preferred a short prompt"
    assert first_token_step[0] <= cap + slack, first_token_step[0]


def test_whole_request_reservation_never_overcommits_pages():
    """Admission reserves a request's whole KV (prompt + max_tokens): with pages for one
    such request plus a bit, the second waits until the first finishes instead of both
    starting and running out of pages mid-decode."""
    # 4-token pages: each request needs ceil((20 + 40) / 4) = 15 pages; 24 usable pages.
    eng, _ = make(max_seqs=4, num_pages=25, chunk=64, max_step_tokens=64)
    a = [(5 * j + 2) % V for j in range(20)]
    b = [(9 * j + 4) % V for j in range(20)]
    eng.submit(1, a, 40)
    eng.submit(2, b, 40)
    events = []
    for step in range(1000):
        if not eng.has_work():
            break
        for ev in eng.step():
            events.append((step, ev["request_id"], bool(ev["finish"])))
    finish_1 = min(s for s, r, f in events if r == 1 and f)
    first_2 = min(s for s, r, _ in events if r == 2)
    assert first_2 > finish_1  # request 2 was admitted only after request 1 released its pages
    assert eng.free_pages() == 24 and eng.free_slots() == 4


def test_prefix_cache_reuse_with_recurrent_checkpoints():
    eng, be = make(apc=True, ppn=2, recurrent=True, ckpt=16, chunk=16)
    shared = [(7 * j + 3) % V for j in range(40)]
    a = shared + [5, 6, 7]
    b = shared + [9, 9]
    eng.submit(1, a, 5)
    out, _ = run(eng)
    assert eng.cached_prefix_nodes() == 5  # 40 tokens / (2 pages x 4 tokens)
    eng.submit(2, b, 5)
    out2, _ = run(eng)
    assert out[1] == expected(a, 5)
    assert out2[2] == expected(b, 5)
    st = eng.stats()
    assert st.prefix_hit_tokens >= 40
    # The second request restored a checkpoint instead of recomputing the prefix.
    restores = [pl for pl in be.plans if any(r >= 0 for r in pl["restore_slot"])]
    assert restores


def test_prefix_cache_evicts_under_pressure():
    eng, _ = make(apc=True, ppn=1, num_pages=40, recurrent=True, ckpt=64, chunk=64)
    for i in range(12):
        p = [(i * 101 + j) % V for j in range(24)]
        eng.submit(i, p, 2)
        out, _ = run(eng)
        assert out[i] == expected(p, 2)
    assert eng.stats().prefix_evictions > 0


def test_ngram_speculative_matches_plain_decoding():
    def periodic(h):  # mostly repeats with period 3, deviating every 7th position
        return h[-3] if len(h) % 7 else (h[-1] + 1) % V

    p = [3, 4, 5, 3, 4, 5, 3, 4, 5, 3, 4]
    eng, be = make(spec="ngram", k=3, fn=periodic)
    eng.submit(1, p, 30, True)
    out, _ = run(eng)
    assert out[1] == expected(p, 30, fn=periodic)
    assert any(pl["flags"] & 32 for pl in be.plans)  # verify steps happened
    st = eng.stats()
    assert 0 < st.spec_accepted < st.spec_drafts  # some drafts accepted, some rejected
    assert st.decode_tokens < 30  # fewer steps than tokens


def test_srpt_admits_short_prompts_first():
    eng, be = make(max_seqs=1, policy="srpt")
    eng.submit(1, list(range(60)), 1)
    eng.submit(2, list(range(5)), 1)
    eng.submit(3, list(range(20)), 1)
    order = []
    for _ in range(100):
        if not eng.has_work():
            break
        for ev in eng.step():
            if ev["finish"]:
                order.append(ev["request_id"])
    assert order == [2, 3, 1]


def test_overload_rejects_submit():
    cfg = m.EngineConfig()
    cfg.max_waiting = 2
    eng = m.Engine(cfg, FakeBackend())
    assert eng.submit(1, [1], 1) and eng.submit(2, [1], 1)
    assert not eng.submit(3, [1], 1)


class PagedFakeBackend:
    """Fake model over a modelled paged KV: every row writes its token into the page the
    plan's page table names; the next token is f(tokens read back from the pages for
    positions 0..p).  Prefix reuse and DRAM demotion / reload are right only if the
    engine's page bookkeeping and the KvTransfer copies are."""

    def __init__(self, page_size):
        self.ps = page_size
        self.pages = {}
        self.dram = {}
        self.table = {}
        self.transfers = []

    def _history(self, slot, upto):
        h = []
        for pos in range(upto):
            page = self.table[slot][pos // self.ps]
            h.append(self.pages[page][pos % self.ps])
        return h

    def __call__(self, p):
        if p["opcode"] == 3:  # KvTransfer: token_ids = pages, positions = DRAM slots, row_slot = direction
            for page, slot, up in zip(p["token_ids"], p["positions"], p["row_slot"]):
                self.transfers.append((page, slot, up))
                if up:
                    self.pages[page] = list(self.dram[slot])
                else:
                    self.dram[slot] = list(self.pages[page])
            return []
        for row, pages in zip(p["dirty_rows"], p["dirty_pages"]):
            self.table[row] = list(pages)
        outs = []
        qs = p["query_start"]
        for i, slot in enumerate(p["seq_slot"]):
            r0, r1 = qs[i], qs[i + 1]
            for r in range(r0, r1):
                pos = p["positions"][r]
                page = self.table[slot][pos // self.ps]
                self.pages.setdefault(page, [None] * self.ps)[pos % self.ps] = p["token_ids"][r]
            if p["sample_row"][i] < 0:
                outs.append({"tokens": []})
                continue
            last = p["positions"][r1 - 1]
            outs.append({"tokens": [f(self._history(slot, last + 1))]})
        return outs


@pytest.mark.parametrize("dram", [0, 48])
def test_dram_tier_demotes_and_reloads_prefixes(dram):
    cfg = m.EngineConfig()
    cfg.max_seqs = 1
    cfg.max_step_tokens = 64
    cfg.max_prefill_chunk = 32
    cfg.page_size = 4
    cfg.num_pages = 21       # 20 usable pages: each request needs most of them
    cfg.max_model_len = 128
    cfg.prefix_caching = True
    cfg.pages_per_node = 1
    cfg.recurrent_state = False
    cfg.dram_blocks = dram
    be = PagedFakeBackend(4)
    eng = m.Engine(cfg, be)
    # Two families of prompts with long shared prefixes; alternating them evicts each
    # family's prefix from HBM before it is needed again.
    fam = [[(7 * i + 3) % V for i in range(40)], [(11 * i + 5) % V for i in range(40)]]
    prompts = [fam[k % 2] + [(k * 13 + j) % V for j in range(5)] for k in range(6)]
    for rid, pr in enumerate(prompts):
        assert eng.submit(rid, pr, 6)
    out, done = run(eng)
    assert done == set(range(6)) and not eng.poisoned(), eng.error()
    for rid, pr in enumerate(prompts):
        assert out[rid] == expected(pr, 6), rid
    st = eng.stats()
    if dram:
        assert st.dram_offloads > 0 and st.dram_reloads > 0 and st.dram_hit_tokens > 0
        assert any(up for _, _, up in be.transfers) and any(not up for _, _, up in be.transfers)
        assert st.prefix_hit_tokens > 0
    else:
        assert st.dram_capacity == 0 and not be.transfers


class DeviceTokenFake(FakeBackend):
    """FakeBackend that also serves run-ahead steps: rows flagged DEVICE_TOKENS continue
    their slot with the last token this backend produced for it."""

    def __init__(self):
        super().__init__()
        self.last = {}
        self.ahead = 0

    def __call__(self, p):
        if p["flags"] & 2:  # DEVICE_TOKENS
            self.ahead += 1
            p = dict(p)
            p["token_ids"] = [self.last[s] for s in p["row_slot"]]
        outs = super().__call__(p)
        for s, o in zip(p["seq_slot"], outs):
            if o["tokens"]:
                self.last[s] = o["tokens"][-1]
        return outs


@pytest.mark.parametrize("depth", [0, 1])
def test_in_flight_depth_one_matches_synchronous(depth):
    cfg = m.EngineConfig()
    cfg.max_seqs = 4
    cfg.max_step_tokens = 64
    cfg.max_prefill_chunk = 32
    cfg.page_size = 4
    cfg.num_pages = 256
    cfg.max_model_len = 512
    cfg.in_flight_depth = depth
    be = DeviceTokenFake()
    eng = m.Engine(cfg, be, async_backend=True)
    eos_tok = f(list(range(7)))  # some request will emit it mid-way
    reqs = {i: ([(i * 31 + j) % V for j in range(3 + 5 * i)], 4 + 3 * i) for i in range(7)}
    for rid, (p, mt) in reqs.items():
        assert eng.submit(rid, p, mt, False, [eos_tok])
    out, done = run(eng)
    assert done == set(reqs) and not eng.poisoned(), eng.error()
    for rid, (p, mt) in reqs.items():
        assert out[rid] == expected(p, mt, eos=(eos_tok,)), rid
    st = eng.stats()
    assert (st.run_ahead_steps > 0) == (depth == 1)
    assert eng.free_slots() == 4


def test_srpt_starvation_cap_in_milliseconds():
    """The wall-clock form of the cap: with the step cap out of reach, the long prompt that
    arrived first is admitted once it has waited `starvation_ms`, although shorter prompts
    keep arriving."""
    import time

    eng, _ = make(max_seqs=1, policy="srpt", chunk=64, max_step_tokens=64, starvation_steps=1 << 30,
                  starvation_ms=30)
    eng.submit(0, [(3 * j + 1) % V for j in range(40)], 2)
    first, rid, t0 = {}, 1, time.monotonic()
    for step in range(5000):
        if time.monotonic() - t0 < 0.5:  # a new short prompt every step for half a second
            eng.submit(rid, [rid % V, (rid * 7) % V], 1)
            rid += 1
        for ev in eng.step():
            first.setdefault(ev["request_id"], time.monotonic() - t0)
        if not eng.has_work():
            break
        time.sleep(0.001)
    assert any(r != 0 and t < first[0] for r, t in first.items()), "SRPT never preferred a short prompt"
    assert first[0] < 0.4, first[0]  # well before the stream of short prompts ends


def test_ngram_drafts_take_the_longest_matching_suffix():
    """Prompt-lookup windows: with lookup 2..5 the 3-token suffix [1, 2, 3] matches at the
    start and proposes what followed it there; with lookup 2..2 only [2, 3] is tried and its
    most recent earlier occurrence wins."""
    prompt = [1, 2, 3, 10, 11, 5, 2, 3, 20, 21, 7, 1, 2]
    for lo, hi, want in ((2, 5, [10, 11, 5]), (2, 2, [20, 21, 7])):
        eng, be = make(spec="ngram", k=3, ngram_min=lo, ngram_max=hi, fn=lambda h: 3)
        eng.submit(1, prompt, 8)
        run(eng)
        verify = [p for p in be.plans if any(w > 0 for w in p["spec_width"])]
        assert verify, "no verify step"
        assert list(verify[0]["token_ids"][1:4]) == want, (lo, hi, verify[0]["token_ids"])


def test_mixed_steps_respect_the_token_cap():
    """Steps that carry decode rows take prefill chunks only up to max(cap, decodes + 1)
    rows; steps without decode rows still use the full step budget.  Output unchanged."""
    eng, be = make(max_seqs=4, chunk=32, max_step_tokens=64, max_mixed_step_tokens=12)
    reqs = {0: [(5 * j) % V for j in range(8)], 1: [(7 * j + 1) % V for j in range(100)],
            2: [(3 * j + 2) % V for j in range(90)]}
    for rid, p in reqs.items():
        eng.submit(rid, p, 6)
    out, _ = run(eng)
    for rid, p in reqs.items():
        assert out[rid] == expected(p, 6)
    mixed = [p for p in be.plans if any(w == 1 for w in _rows(p)) and any(w > 1 for w in _rows(p))]
    assert mixed, "no step mixed decode rows with a prefill chunk"
    for p in mixed:
        decodes = sum(1 for w in _rows(p) if w == 1)
        assert len(p["token_ids"]) <= max(12, decodes + 1), (len(p["token_ids"]), decodes)
    assert max(len(p["token_ids"]) for p in be.plans) > 12  # pure prefill steps are not capped


def test_dynamic_prefill_budget_grows_with_the_backlog():
    """With the dynamic budget a large prefill backlog lifts the mixed-step cap toward
    max_step_tokens; without it the cap stays fixed."""
    sizes = {}
    for dyn in (False, True):
        eng, be = make(max_seqs=4, chunk=64, max_step_tokens=64, max_mixed_step_tokens=12,
                       dynamic_prefill_budget=dyn, backlog_low_tokens=16, backlog_high_tokens=64)
        eng.submit(0, [1, 2, 3], 20)
        for _ in range(3):  # request 0 is decoding before the long prompts arrive
            eng.step()
        for rid in (1, 2, 3):
            eng.submit(rid, [(11 * j + rid) % V for j in range(200)], 2)
        run(eng)
        sizes[dyn] = max(len(p["token_ids"]) for p in be.plans if any(w == 1 for w in _rows(p)))
    assert sizes[False] <= 12 and sizes[True] > 12, sizes


def _rows(p):
    qs = p["query_start"]
    return [qs[i + 1] - qs[i] for i in range(len(p["seq_slot"]))]
