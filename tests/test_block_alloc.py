"""Page bookkeeping of the multi-sequence KV pool (lc_block_alloc, host only):
sequence slots, per-sequence page lists, one LIFO free list. The single-
sequence case must hand out pages exactly as the reference's KVCache does
(src/layers/kv_cache.rs:73-76, 106-122: pages 0, 1, 2, ... in order)."""
import numpy as np
import pytest

import lucciola as L


def test_fresh_pool_hands_out_pages_in_order():
    a = L.BlockAlloc(64, 4, 32)
    s = a.add()
    assert s == 0
    for tokens in (1, 16, 17, 100, 512):
        a.reserve(s, tokens)
        assert a.pages(s) == list(range((tokens + 15) // 16))
    assert a.num_free == 64 - 32


def test_interleaved_sequences_get_distinct_pages():
    a = L.BlockAlloc(100, 3, 40)
    s0, s1, s2 = a.add(), a.add(), a.add()
    a.reserve(s0, 16)
    a.reserve(s1, 40)
    a.reserve(s0, 33)
    a.reserve(s2, 1)
    assert a.pages(s0) == [0, 4, 5]
    assert a.pages(s1) == [1, 2, 3]
    assert a.pages(s2) == [6]
    all_pages = a.pages(s0) + a.pages(s1) + a.pages(s2)
    assert len(set(all_pages)) == len(all_pages)
    assert a.num_free == 100 - 7


def test_release_returns_pages_in_the_same_order():
    a = L.BlockAlloc(16, 2, 16)
    s0 = a.add()
    a.reserve(s0, 5 * 16)
    first = a.pages(s0)
    a.release(s0)
    assert a.num_free == 16
    s1 = a.add()
    assert s1 == s0  # lowest free slot
    a.reserve(s1, 5 * 16)
    assert a.pages(s1) == first


def test_errors():
    a = L.BlockAlloc(4, 1, 8)
    s = a.add()
    with pytest.raises(L.LucciolaError) as e:
        a.add()
    assert e.value.status == 12  # every slot in use
    with pytest.raises(L.LucciolaError) as e:
        a.reserve(s, 9 * 16)
    assert e.value.status == 1  # beyond the table row
    a.reserve(s, 2 * 16)
    with pytest.raises(L.LucciolaError) as e:
        a.reserve(s, 5 * 16)
    assert e.value.status == 9  # free list exhausted
    assert a.pages(s) == [0, 1] and a.num_free == 2  # nothing taken by the failed call
    with pytest.raises(L.LucciolaError):
        a.release(5)


def test_random_walk_matches_a_model():
    rng = np.random.default_rng(7)
    nb, ns, mb = 200, 8, 64
    a = L.BlockAlloc(nb, ns, mb)
    free = list(range(nb - 1, -1, -1))
    pages = {}
    for _ in range(2000):
        op = rng.integers(0, 3)
        if op == 0 and len(pages) < ns:
            s = a.add()
            assert s == min(set(range(ns)) - set(pages))
            pages[s] = []
        elif op == 1 and pages:
            s = int(rng.choice(list(pages)))
            tokens = int(rng.integers(0, mb * 16 + 1))
            need = (tokens + 15) // 16
            grow = max(0, need - len(pages[s]))
            if grow > len(free):
                with pytest.raises(L.LucciolaError):
                    a.reserve(s, tokens)
            else:
                a.reserve(s, tokens)
                for _ in range(grow):
                    pages[s].append(free.pop())
        elif op == 2 and pages:
            s = int(rng.choice(list(pages)))
            a.release(s)
            free.extend(reversed(pages.pop(s)))
        for s, pg in pages.items():
            assert a.pages(s) == pg
        assert a.num_free == len(free)
