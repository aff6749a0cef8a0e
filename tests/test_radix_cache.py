"""Radix prefix cache: matching, splitting, locking and LRU eviction."""

import pytest
import torch

from minisgl import ops
from minisgl.kvcache.radix_cache import RadixPrefixCache


def t(xs):
    return torch.tensor(xs, dtype=torch.int32)


@pytest.mark.parametrize("page", [1, 2])
def test_match_insert_split(page):
    c = RadixPrefixCache(torch.device("cpu"), page)
    c.insert_prefix(t([1, 2, 3, 4, 5, 6]), t([10, 11, 12, 13, 14, 15]))
    h = c.match_prefix(t([1, 2, 3, 4, 9, 9])).cuda_handle
    assert h.cached_len == 4
    assert h.get_matched_indices().tolist() == [10, 11, 12, 13]
    c.insert_prefix(t([1, 2, 3, 4, 7, 8]), t([10, 11, 12, 13, 20, 21]))
    assert c.size_info.evictable_size == 8
    c.check_integrity()


def test_lock_protects_from_eviction():
    c = RadixPrefixCache(torch.device("cpu"), 1)
    c.insert_prefix(t([1, 2, 3]), t([0, 1, 2]))
    c.insert_prefix(t([5, 6]), t([3, 4]))
    h = c.match_prefix(t([1, 2, 3])).cuda_handle
    c.lock_handle(h)
    assert c.size_info == (2, 3)
    freed = c.evict(2)
    assert sorted(freed.tolist()) == [3, 4]
    with pytest.raises(RuntimeError):
        c.evict(1)
    c.lock_handle(h, unlock=True)
    assert c.size_info == (3, 0)
    c.check_integrity()


def test_lru_order():
    c = RadixPrefixCache(torch.device("cpu"), 1)
    c.insert_prefix(t([1, 2]), t([0, 1]))
    c.insert_prefix(t([3, 4]), t([2, 3]))
    c.match_prefix(t([1, 2]))  # touch the first prefix
    freed = c.evict(2)
    assert sorted(freed.tolist()) == [2, 3]


def test_partial_page_not_inserted():
    c = RadixPrefixCache(torch.device("cpu"), 4)
    res = c.insert_prefix(t(list(range(10))), t(list(range(10))))
    assert res.handle.cached_len == 8
    assert c.size_info.evictable_size == 8


def test_fast_compare_key():
    assert ops.fast_compare_key(t([1, 2, 3, 4]), t([1, 2, 9])) == 2
    assert ops.fast_compare_key(t([1, 2]), t([1, 2, 3])) == 2
    assert ops.fast_compare_key(t(list(range(100))), t(list(range(100)))) == 100
    a = torch.arange(50, dtype=torch.int64)
    b = a.clone()
    b[37] = -1
    assert ops.fast_compare_key(a, b) == 37
