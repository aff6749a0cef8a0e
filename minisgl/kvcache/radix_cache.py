"""Page-granular radix tree over token ids (prefix sharing across requests).

Each edge holds a run of token ids (host tensor) and the token slots that
store their KV (device tensor); edges always cover whole pages. Children are
keyed by their first page of ids. Nodes carry a reference count (requests
currently using the prefix) and a last-access time; unreferenced leaves are
evicted least-recently-used first. Sizes are tracked in tokens and split into
evictable (refcount 0) and protected parts, the accounting the scheduler's
admission check uses (behaviour of python/minisgl/kvcache/radix_cache.py).
"""

from __future__ import annotations

import heapq
import itertools
import time
from typing import Dict, Hashable, List, Optional, Tuple

import torch

from minisgl import ops
from minisgl.utils import align_down

from .base import BaseCacheHandle, BasePrefixCache, InsertResult, MatchResult, SizeInfo

_ids = itertools.count()


class _Node:
    __slots__ = ("key", "value", "children", "parent", "refs", "stamp", "uid")

    def __init__(self, key: torch.Tensor, value: torch.Tensor, parent: Optional["_Node"]) -> None:
        self.key = key
        self.value = value
        self.children: Dict[Hashable, _Node] = {}
        self.parent = parent
        self.refs = 0
        self.stamp = time.monotonic_ns()
        self.uid = next(_ids)

    @property
    def length(self) -> int:
        return len(self.key)

    def is_leaf(self) -> bool:
        return not self.children

    def __lt__(self, other: "_Node") -> bool:  # heap order: oldest first
        return (self.stamp, self.uid) < (other.stamp, other.uid)


class RadixCacheHandle(BaseCacheHandle):
    def __init__(self, cached_len: int, node: _Node) -> None:
        super().__init__(cached_len=cached_len)
        object.__setattr__(self, "node", node)

    def get_matched_indices(self) -> torch.Tensor:
        parts: List[torch.Tensor] = []
        node: Optional[_Node] = self.node  # type: ignore[attr-defined]
        while node is not None and node.parent is not None:
            parts.append(node.value)
            node = node.parent
        if not parts:
            return torch.empty(0, dtype=torch.int32)
        parts.reverse()
        return torch.cat(parts)


class RadixPrefixCache(BasePrefixCache):
    def __init__(self, device: torch.device, page_size: int = 1) -> None:
        self.device = device
        self.page_size = page_size
        self._empty = torch.empty(0, dtype=torch.int32, device=device)
        self.reset()

    # --------------------------------------------------------------- keys
    def _child_key(self, ids: torch.Tensor) -> Hashable:
        if self.page_size == 1:
            return int(ids[0])
        return tuple(ids[: self.page_size].tolist())

    # --------------------------------------------------------------- API
    def reset(self) -> None:
        self.root = _Node(torch.empty(0, dtype=torch.int32), self._empty, None)
        self.root.refs = 1  # never evicted
        self.evictable = 0
        self.protected = 0

    def lock_handle(self, handle: BaseCacheHandle, unlock: bool = False) -> None:
        assert isinstance(handle, RadixCacheHandle)
        node: _Node = handle.node  # type: ignore[attr-defined]
        while node.parent is not None:
            if unlock:
                node.refs -= 1
                assert node.refs >= 0, "unbalanced unlock"
                if node.refs == 0:
                    self.evictable += node.length
                    self.protected -= node.length
            else:
                if node.refs == 0:
                    self.evictable -= node.length
                    self.protected += node.length
                node.refs += 1
            node = node.parent

    def match_prefix(self, input_ids: torch.Tensor) -> MatchResult:
        node, n = self._walk(input_ids)
        return MatchResult(RadixCacheHandle(n, node))

    def insert_prefix(self, input_ids: torch.Tensor, indices: torch.Tensor) -> InsertResult:
        n = align_down(len(input_ids), self.page_size)
        ids, idx = input_ids[:n], indices[:n]
        node, matched = self._walk(ids)
        if matched < n:
            child = _Node(ids[matched:].clone(), idx[matched:].clone(), node)
            node.children[self._child_key(child.key)] = child
            self.evictable += child.length
            node = child
        return InsertResult(matched, RadixCacheHandle(n, node))

    def evict(self, size: int) -> torch.Tensor:
        if size <= 0:
            return self._empty
        if size > self.evictable:
            raise RuntimeError(f"cannot evict {size} tokens: only {self.evictable} are evictable")
        heap = [n for n in self._leaves() if n.refs == 0]
        heapq.heapify(heap)
        freed: List[torch.Tensor] = []
        total = 0
        while total < size:
            if not heap:
                raise RuntimeError(f"eviction stalled after {total} of {size} tokens")
            node = heapq.heappop(heap)
            parent = node.parent
            assert parent is not None and node.refs == 0 and node.is_leaf()
            del parent.children[self._child_key(node.key)]
            freed.append(node.value)
            total += node.length
            self.evictable -= node.length
            if parent.parent is not None and parent.is_leaf() and parent.refs == 0:
                heapq.heappush(heap, parent)
        return torch.cat(freed)

    @property
    def size_info(self) -> SizeInfo:
        return SizeInfo(self.evictable, self.protected)

    def check_integrity(self) -> None:
        ev = pr = 0
        stack = list(self.root.children.values())
        while stack:
            n = stack.pop()
            if n.length % self.page_size != 0 or len(n.value) != n.length:
                raise RuntimeError("radix node is not page aligned")
            if n.refs == 0:
                ev += n.length
            else:
                pr += n.length
            stack.extend(n.children.values())
        if (ev, pr) != (self.evictable, self.protected):
            raise RuntimeError(f"radix size accounting broken: tree ({ev}, {pr}) vs counters "
                               f"({self.evictable}, {self.protected})")

    # ---------------------------------------------------------- internals
    def _leaves(self) -> List[_Node]:
        out, stack = [], [self.root]
        while stack:
            n = stack.pop()
            if n.is_leaf():
                if n.parent is not None:
                    out.append(n)
            else:
                stack.extend(n.children.values())
        return out

    def _walk(self, ids: torch.Tensor) -> Tuple[_Node, int]:
        """Follow ``ids`` from the root; split an edge that matches only
        partially (at a page boundary). Returns (deepest node, matched len)."""
        node, pos, total = self.root, 0, len(ids)
        now = time.monotonic_ns()
        P = self.page_size
        while total - pos >= P:
            child = node.children.get(self._child_key(ids[pos:]))
            if child is None:
                break
            m = align_down(ops.fast_compare_key(child.key, ids[pos:]), P)
            child.stamp = now
            if m < child.length:
                if m == 0:
                    break
                child = self._split(child, m)
                child.stamp = now
                return child, pos + m
            node, pos = child, pos + m
        return node, pos

    def _split(self, node: _Node, at: int) -> _Node:
        parent = node.parent
        assert parent is not None and 0 < at < node.length
        head = _Node(node.key[:at], node.value[:at], parent)
        head.refs = node.refs
        head.stamp = node.stamp
        parent.children[self._child_key(head.key)] = head
        node.key, node.value = node.key[at:], node.value[at:]
        node.parent = head
        head.children[self._child_key(node.key)] = node
        return head
