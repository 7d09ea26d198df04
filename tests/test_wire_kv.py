"""Wire ABI parity (C++ <-> Python) and KV bookkeeping (pools, hashing, prefix tree)."""

import hashlib

import pytest

from zstep_b200 import _master as m
from zstep_b200.runtime import wire


@pytest.mark.parametrize("geo", [(1, 256, 8192, 256, 16), (2, 8, 256, 64, 16), (8, 512, 16384, 2048, 16)])
def test_layout_parity(geo):
    g = m.Geometry()
    g.world_size, g.max_seqs, g.max_step_tokens, g.max_pages_per_seq, g.page_size = geo
    d = m.layout(g)
    pg = wire.Geometry(*geo)
    py = wire.segment_layout(pg)
    for f in wire.PLAN_FIELDS:
        assert d[f] == py["plan"][f], f
    assert d["plan_bytes"] == py["plan"]["bytes"]
    assert d["total_bytes"] == py["total_bytes"]
    assert d["layout_hash"] == wire.layout_hash(pg)
    assert d["sizeof_superblock"] == wire.SIZEOF_SUPERBLOCK
    assert d["sizeof_seq_output"] == wire.SIZEOF_SEQ_OUTPUT
    assert d["sizeof_sampling"] == wire.SIZEOF_SAMPLING
    assert m.DECODE_BUCKETS == list(wire.DECODE_BUCKETS)


def test_layout_hash_detects_geometry_change():
    a = wire.layout_hash(wire.Geometry(1, 256, 8192, 256, 16))
    b = wire.layout_hash(wire.Geometry(1, 256, 8192, 257, 16))
    assert a != b


def test_sha256_matches_hashlib():
    for msg in [b"", b"abc", b"a" * 55, b"a" * 56, b"a" * 64, bytes(range(256)) * 5]:
        assert m.sha256(msg) == hashlib.sha256(msg).digest()


def test_block_hash_golden():
    # Golden vector shared with the reference's router-compatible hashing.
    toks = [37, 57610, 37611, 9934, 11, 7722, 1467, 1549, 11, 24132, 279, 4734, 1852, 15870, 17, 20]
    assert m.external_keys(toks, 16, "42") == [1015703622044383654]
    # Partial tail ignored; seed changes the chain.
    t = list(range(1, 21))
    assert len(m.external_keys(t, 16, "42")) == 1
    assert m.external_keys(t, 16, "42") != m.external_keys(t, 16, "99")


def test_block_pool_lease_conservation():
    pool = m.BlockPool(10, 1)
    a = pool.allocate(4)
    b = pool.allocate(6)
    assert pool.available() == 0
    assert pool.allocate(1) is None
    assert sorted(a.ids() + b.ids()) == list(range(1, 11))
    front = a.take_front(2)
    assert len(front) == 2 and len(a) == 2
    del front
    assert pool.available() == 2
    a.release()
    del b
    assert pool.available() == 10


def test_prefix_tree_match_insert_evict():
    pages = m.BlockPool(64, 1)
    tree = m.PrefixTree(4, 2)  # node = 8 tokens
    events = []
    tree.set_event_sink(lambda kind, keys, parent, toks: events.append((kind, len(keys))))
    toks = list(range(100, 124))
    n1, created = tree.insert(0, toks[0:8], pages.allocate(2))
    assert created and n1 > 0
    n2, created = tree.insert(n1, toks[8:16], pages.allocate(2))
    assert created
    # Duplicate insert keeps the caller's lease.
    dup = pages.allocate(2)
    n2b, created = tree.insert(n1, toks[8:16], dup)
    assert n2b == n2 and not created and len(dup) == 2
    lease = tree.match(toks)
    assert lease.matched_nodes() == 2 and lease.matched_tokens() == 16 and len(lease.pages()) == 4
    assert tree.peek(toks[:12]) == (1, 8)
    # Pinned nodes are not evictable.
    assert tree.evictable_pages() == 0
    assert tree.evict_lru(100) == []
    lease.release()
    assert tree.evictable_pages() == 4
    victims = tree.evict_lru(2)  # leaf first
    assert len(victims) == 1 and victims[0].tokens == toks[8:16]
    assert tree.cached_nodes() == 1
    before = pages.available()
    tree.evict_lru(100)
    assert pages.available() == before + 2
    assert [k for k, _ in events] == [0, 0, 1, 1]


def test_prefix_tree_lru_order_and_aux():
    pages = m.BlockPool(32, 1)
    aux = m.BlockPool(4, 100)
    tree = m.PrefixTree(4, 1)
    ids = []
    for base in (0, 10, 20):
        nid, _ = tree.insert(0, list(range(base, base + 4)), pages.allocate(1), aux.allocate(1))
        ids.append(nid)
    assert aux.available() == 1
    assert tree.aux_of(ids[0]) == 100
    tree.match(list(range(0, 4))).release()   # touch the first node
    victims = tree.evict_lru(1)
    assert victims[0].tokens == list(range(10, 14))  # least recently used
    assert aux.available() == 2


def test_hybrid_alias_and_subpages():
    t = m.HybridAliasTable()
    assert t.insert(5, 300, [5, 6])
    assert not t.insert(5, 301, [5])
    assert t.slot_for_anchor(5) == 300 and t.anchor_for_slot(300) == 5
    assert t.remove_by_anchor(5) and len(t) == 0
    sp = m.SubPageAllocator(128, 512, 2)  # 4 slices per page
    got = [sp.allocate() for _ in range(8)]
    assert all(g is not None for g in got) and sp.allocate() is None
    assert got[0][0] == got[3][0]  # best fit fills a page before opening the next
    sp.release(*got[0])
    assert sp.active() == 7
