"""The host page allocator of paged KV caches (b2a_pagepool_*), on the CPU.

A paged cache keeps the reference's per-sequence KVCache bound (capacity,
src/cpu/cache.js:24-26 and the overflow check of allocate, :53-58) but backs
each sequence's positions with fixed pages from one shared pool. These tests
pin the allocator's contract: pages are mapped as a prefix of the sequence's
table, a reservation is all or nothing, an exhausted pool reports who needed
how many, released pages come back in their old order, and the argument checks.
"""
import numpy as np
import pytest

import b2a


def test_pages_are_mapped_in_position_order_as_sequences_grow():
    p = b2a.PagePool(numPages=8, pageSize=128, batch=3, capacity=1024)
    assert p.freePages == 8
    p.reserve(0, 1)          # 1 position -> 1 page
    p.reserve(1, 128)        # exactly one page
    p.reserve(0, 129)        # a second page for sequence 0
    p.reserve(2, 300)        # three pages
    assert p.table(0).tolist() == [0, 2]
    assert p.table(1).tolist() == [1]
    assert p.table(2).tolist() == [3, 4, 5]
    assert p.freePages == 2
    p.reserve(2, 256)        # already backed: nothing changes
    p.reserve(0, 0)
    assert p.table(2).tolist() == [3, 4, 5] and p.freePages == 2


def test_exhausted_pool_changes_nothing_and_names_the_sequence():
    p = b2a.PagePool(numPages=4, pageSize=256, batch=2, capacity=4096)
    p.reserve(0, 600)        # 3 pages
    with pytest.raises(b2a.RangeError, match=r"page pool exhausted: 3 of 4 pages in use; sequence 1 needs 2 more"):
        p.reserve(1, 257)
    assert p.table(1).tolist() == [] and p.freePages == 1
    p.reserve(1, 256)
    assert p.table(1).tolist() == [3] and p.freePages == 0


def test_released_pages_are_reused_in_their_old_order():
    p = b2a.PagePool(numPages=6, pageSize=128, batch=3, capacity=2048)
    p.reserve(0, 128)
    p.reserve(1, 128)
    p.reserve(0, 384)
    assert p.table(0).tolist() == [0, 2, 3]
    p.release(0)
    assert p.table(0).tolist() == [] and p.freePages == 5
    p.reserve(2, 300)
    assert p.table(2).tolist() == [0, 2, 3]
    p.release()              # every sequence
    assert p.freePages == 6
    assert all(p.table(b).size == 0 for b in range(3))


def test_interleaved_growth_scatters_a_sequence_over_the_pool():
    rng = np.random.default_rng(7)
    batch, P = 5, 128
    p = b2a.PagePool(numPages=200, pageSize=P, batch=batch, capacity=4096)
    lens = np.zeros(batch, int)
    owner = {}
    for _ in range(300):
        b = int(rng.integers(batch))
        lens[b] = min(4096, lens[b] + int(rng.integers(1, 90)))
        p.reserve(b, int(lens[b]))
    for b in range(batch):
        t = p.table(b)
        assert t.size == -(-lens[b] // P)
        for page in t.tolist():
            assert page not in owner, "a page is mapped twice"
            owner[page] = b
    assert p.freePages == 200 - len(owner)


def test_argument_checks():
    with pytest.raises(b2a.B2AError, match="power of two of at least 128"):
        b2a.PagePool(numPages=4, pageSize=64, batch=1, capacity=512)
    with pytest.raises(b2a.B2AError, match="power of two of at least 128"):
        b2a.PagePool(numPages=4, pageSize=384, batch=1, capacity=512)
    with pytest.raises(b2a.RangeError, match="cache capacity must be a positive integer, got 0"):
        b2a.PagePool(numPages=4, pageSize=128, batch=1, capacity=0)
    with pytest.raises(b2a.B2AError, match="at least one page"):
        b2a.PagePool(numPages=0, pageSize=128, batch=1, capacity=512)
    p = b2a.PagePool(numPages=4, pageSize=128, batch=2, capacity=500)
    with pytest.raises(b2a.RangeError, match="cannot back 501 positions of a 500-position sequence"):
        p.reserve(0, 501)
    with pytest.raises(b2a.B2AError, match="sequence 2 out of range"):
        p.reserve(2, 1)
    with pytest.raises(b2a.B2AError, match="out of range"):
        p.release(5)


def test_random_reserve_release_keeps_the_pool_consistent():
    """Random reservations and releases: every page has at most one owner, owners'
    tables are exactly as long as their reservations need, free + held = pool, and
    a refused reservation changes nothing."""
    rng = np.random.default_rng(11)
    batch, P, pages, cap = 6, 128, 40, 3000
    p = b2a.PagePool(numPages=pages, pageSize=P, batch=batch, capacity=cap)
    want = [0] * batch          # pages each sequence must hold
    for step in range(2000):
        b = int(rng.integers(batch))
        if rng.random() < 0.15:
            p.release(b)
            want[b] = 0
        else:
            pos = int(rng.integers(0, cap + 1))
            need = -(-pos // P)
            before = [p.table(i).tolist() for i in range(batch)]
            extra = max(0, need - want[b])
            if extra > pages - sum(want):
                with pytest.raises(b2a.RangeError, match="page pool exhausted"):
                    p.reserve(b, pos)
                assert [p.table(i).tolist() for i in range(batch)] == before, step
            else:
                p.reserve(b, pos)
                want[b] = max(want[b], need)
        tables = [p.table(i).tolist() for i in range(batch)]
        assert [len(t) for t in tables] == want, step
        held = [x for t in tables for x in t]
        assert len(held) == len(set(held)) and all(0 <= x < pages for x in held), step
        assert p.freePages == pages - len(held), step
