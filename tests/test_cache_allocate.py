"""CacheManager allocation / eviction with pages larger than one token
(the behaviours covered by the reference's tests/core/test_cache_allocate.py:
page alignment after eviction, no overlap, exact-need eviction, integrity)."""

import torch

from minisgl.scheduler.cache import CacheManager


def _cm(num_pages, page_size, kind="radix"):
    return CacheManager(num_pages, page_size, torch.zeros(4, 256, dtype=torch.int32), kind)


def _aligned(t, p):
    return bool((t % p == 0).all())


def _no_overlap(starts, p):
    seen = set()
    for s in starts.tolist():
        r = set(range(s, s + p))
        assert not (seen & r)
        seen |= r


def test_allocate_after_evict_is_page_aligned():
    cm = _cm(4, 4)
    cm._allocate(4)
    assert len(cm.free_slots) == 0
    ids = torch.arange(8, dtype=torch.int32)
    cm.prefix_cache.insert_prefix(ids, torch.arange(8, dtype=torch.int32))
    got = cm._allocate(1)
    assert _aligned(got, 4) and _aligned(cm.free_slots, 4)


def test_consecutive_allocations_do_not_overlap():
    cm = _cm(4, 4)
    cm._allocate(4)
    cm.prefix_cache.insert_prefix(torch.arange(8, dtype=torch.int32), torch.arange(8, dtype=torch.int32))
    a, b = cm._allocate(1), cm._allocate(1)
    both = torch.cat([a, b])
    assert _aligned(both, 4)
    _no_overlap(both, 4)


def test_eviction_frees_exactly_what_is_needed_and_integrity_holds():
    cm = _cm(8, 8)
    slots = cm._allocate(8)
    assert len(slots) == 8
    # three cached prefixes of 2, 3 and 3 pages, evictable
    base = 0
    for n_pages, first in ((2, 100), (3, 200), (3, 300)):
        ids = torch.arange(first, first + 8 * n_pages, dtype=torch.int32)
        idx = torch.arange(base, base + 8 * n_pages, dtype=torch.int32)
        cm.prefix_cache.insert_prefix(ids, idx)
        base += 8 * n_pages
    assert cm.prefix_cache.size_info.evictable_size == 64
    cm.check_integrity()
    got = cm._allocate(3)
    assert len(got) == 3 and _aligned(got, 8)
    _no_overlap(got, 8)
    # at least 3 pages were evicted; the rest of the evicted pages went to the free list
    assert cm.prefix_cache.size_info.evictable_size + 8 * (len(cm.free_slots) + 3) == 64


def test_expand_pages_to_token_slots():
    cm = _cm(4, 4)
    out = cm._expand(torch.tensor([0, 8], dtype=torch.int32))
    assert out.tolist() == [0, 1, 2, 3, 8, 9, 10, 11]


def test_naive_cache_never_shares():
    cm = _cm(4, 4, "naive")
    h = cm.prefix_cache.match_prefix(torch.arange(10, dtype=torch.int32)).cuda_handle
    assert h.cached_len == 0
    assert cm.available_size == 16
    cm.check_integrity()
