"""Prefix cache that shares nothing (every request recomputes its prompt)."""

from __future__ import annotations

import torch

from .base import BaseCacheHandle, BasePrefixCache, InsertResult, MatchResult, SizeInfo


class NaiveCacheHandle(BaseCacheHandle):
    def __init__(self, empty: torch.Tensor) -> None:
        super().__init__(cached_len=0)
        object.__setattr__(self, "_empty", empty)

    def get_matched_indices(self) -> torch.Tensor:
        return self._empty  # type: ignore[attr-defined]


class NaivePrefixCache(BasePrefixCache):
    def __init__(self, device: torch.device, page_size: int = 1) -> None:
        self.device = device
        self._empty = torch.empty(0, dtype=torch.int32, device=device)

    def lock_handle(self, handle: BaseCacheHandle, unlock: bool = False) -> None:
        return None

    def match_prefix(self, input_ids: torch.Tensor) -> MatchResult:
        return MatchResult(NaiveCacheHandle(self._empty))

    def insert_prefix(self, input_ids: torch.Tensor, indices: torch.Tensor) -> InsertResult:
        return InsertResult(0, NaiveCacheHandle(self._empty))

    def evict(self, size: int) -> torch.Tensor:
        if size == 0:
            return self._empty
        raise RuntimeError("the naive prefix cache holds nothing to evict")

    def reset(self) -> None:
        return None

    @property
    def size_info(self) -> SizeInfo:
        return SizeInfo(0, 0)

    def check_integrity(self) -> None:
        return None
