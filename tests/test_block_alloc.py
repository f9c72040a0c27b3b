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


def _reference_budget(L_, hkv, hd, free, total, fraction):
    """src/layers/kv_cache.rs:37-59, restated: budget in f32, K+V bytes per page."""
    used = total - free
    available_total = int(np.float32(total) * np.float32(fraction))
    if available_total <= used:
        return 0
    return (available_total - used) // (2 * L_ * hkv * 16 * hd * 2)


@pytest.mark.parametrize("L_,hkv,hd,free,total,fraction", [
    (24, 2, 64, 150 << 30, 183359 << 20, 0.9),     # 0.5B shape on an idle B200
    (28, 4, 128, 120 << 30, 183359 << 20, 0.85),   # 7B shape, 63 GB already used
    (80, 1, 128, 170 << 30, 183359 << 20, 0.95),   # 72B shape, one of 8 kv-head shards
    (24, 2, 64, 10 << 30, 80 << 30, 0.5),          # budget below what is used
])
def test_pool_budget_follows_the_reference_rule(L_, hkv, hd, free, total, fraction):
    got = L.pool_blocks_for_budget(L_, hkv, hd, free, total, fraction)
    assert got == _reference_budget(L_, hkv, hd, free, total, fraction)


def test_pool_budget_caps_at_int32_rows():
    # a tiny page (1 layer, 1 head, hd 64) and a huge budget: rows = blocks * 16 < 2^31
    got = L.pool_blocks_for_budget(1, 1, 64, 1 << 50, 1 << 50, 1.0)
    assert got == ((1 << 31) - 1) // 16
    assert L.pool_blocks_for_budget(0, 1, 64, 1 << 30, 1 << 30, 1.0) == 0


def test_fingerprint_tracks_every_decision():
    def run(extra):
        a = L.BlockAlloc(300, 6, 64)
        rng = np.random.default_rng(11)
        live = []
        for _ in range(400):
            op = rng.integers(0, 3)
            if op == 0 and len(live) < 6:
                live.append(a.add())
            elif op == 1 and live:
                try:
                    a.reserve(int(rng.choice(live)), int(rng.integers(0, 1024)))
                except L.LucciolaError:
                    pass
            elif op == 2 and live:
                s = int(rng.choice(live))
                a.release(s)
                live.remove(s)
        if extra:
            s = a.add() if not live else live[0]
            a.reserve(s, len(a.pages(s)) * 16 + 1)
        return a.fingerprint(), {s: a.pages(s) for s in live}
    f0, p0 = run(False)
    f1, p1 = run(False)
    f2, _ = run(True)
    assert f0 == f1 and p0 == p1  # the same calls give the same tables and state
    assert f2 != f0               # one more page taken changes it
