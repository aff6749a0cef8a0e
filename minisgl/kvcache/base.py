"""Interfaces of the KV pool and of prefix caches.

The prefix-cache contract (match / lock / insert / evict with sizes split
into evictable and protected) is the one the scheduler relies on, as in the
reference (python/minisgl/kvcache/base.py:40-135).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import NamedTuple

import torch


class BaseKVCachePool(ABC):
    """Device storage of K and V for every layer."""

    @abstractmethod
    def k_cache(self, layer: int) -> torch.Tensor: ...

    @abstractmethod
    def v_cache(self, layer: int) -> torch.Tensor: ...

    @abstractmethod
    def store_kv(self, k: torch.Tensor, v: torch.Tensor, out_loc: torch.Tensor, layer: int) -> None: ...

    @property
    @abstractmethod
    def device(self) -> torch.device: ...

    @property
    @abstractmethod
    def dtype(self) -> torch.dtype: ...

    @property
    @abstractmethod
    def num_layers(self) -> int: ...


@dataclass(frozen=True)
class BaseCacheHandle(ABC):
    """A matched prefix: its length and (via get_matched_indices) the token
    slots that hold its KV. Only valid while locked."""

    cached_len: int

    @abstractmethod
    def get_matched_indices(self) -> torch.Tensor: ...


class SizeInfo(NamedTuple):
    evictable_size: int
    protected_size: int

    @property
    def total_size(self) -> int:
        return self.evictable_size + self.protected_size


class InsertResult(NamedTuple):
    cached_len: int  # prefix length that was already present (its new slots are duplicates)
    handle: BaseCacheHandle


class MatchResult(NamedTuple):
    cuda_handle: BaseCacheHandle


class BasePrefixCache(ABC):
    @abstractmethod
    def lock_handle(self, handle: BaseCacheHandle, unlock: bool = False) -> None:
        """Pin (or unpin) the nodes of a matched prefix against eviction."""

    @abstractmethod
    def match_prefix(self, input_ids: torch.Tensor) -> MatchResult:
        """Longest cached, page-aligned prefix of ``input_ids``."""

    @abstractmethod
    def insert_prefix(self, input_ids: torch.Tensor, indices: torch.Tensor) -> InsertResult:
        """Add ``input_ids`` (page-aligned part) with their token slots."""

    @abstractmethod
    def evict(self, size: int) -> torch.Tensor:
        """Free at least ``size`` tokens of unpinned entries (LRU first) and
        return their slots. ``evict(0)`` is a no-op."""

    @abstractmethod
    def reset(self) -> None: ...

    @property
    @abstractmethod
    def size_info(self) -> SizeInfo: ...

    @abstractmethod
    def check_integrity(self) -> None: ...
