"""Token-slot allocator on top of a prefix cache.

Free memory is a vector of page-aligned token slots (slot = page *
page_size). Pages are handed to requests as they grow and written into the
page table (which stores one token slot per position). When the free list
runs dry, unreferenced prefix-cache entries are evicted. The split between
"already cached by someone else" and "newly inserted" on ``cache_req`` is
the reference's accounting (python/minisgl/scheduler/cache.py:56-80).
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import TYPE_CHECKING, List, Tuple

import torch

from minisgl.core import Req
from minisgl.kvcache import BaseCacheHandle, MatchResult, create_prefix_cache
from minisgl.utils import div_ceil

if TYPE_CHECKING:
    from .prefill import PendingReq


class CacheManager:
    def __init__(self, num_pages: int, page_size: int, page_table: torch.Tensor, type: str,
                 page_classes: int = 1) -> None:
        self.device = page_table.device
        self.num_pages = num_pages
        self.page_size = page_size
        # context parallelism: page id g is stored on rank g % page_classes, and
        # page p of a sequence (its 64-key tile p) must live on rank p % classes
        self.page_classes = page_classes
        self.page_table = page_table
        self.free_slots = torch.arange(num_pages, dtype=torch.int32, device=self.device) * page_size
        self.prefix_cache = create_prefix_cache(self.device, type, page_size)
        self._pending_free: List[torch.Tensor] | None = None

    # ------------------------------------------------------------ queries
    @property
    def available_size(self) -> int:
        """Tokens obtainable right now: free pages plus evictable cache."""
        return len(self.free_slots) * self.page_size + self.prefix_cache.size_info.evictable_size

    def match_req(self, req: "PendingReq") -> MatchResult:
        # at least the last prompt token is always recomputed (it produces logits)
        assert req.input_len > 0
        return self.prefix_cache.match_prefix(req.input_ids[: req.input_len - 1])

    def lock(self, handle: BaseCacheHandle) -> None:
        self.prefix_cache.lock_handle(handle, unlock=False)

    def unlock(self, handle: BaseCacheHandle) -> None:
        self.prefix_cache.lock_handle(handle, unlock=True)

    # --------------------------------------------------------- allocation
    def allocate_paged(self, reqs: List[Req]) -> None:
        """Give every request the pages covering positions [cached_len,
        device_len) that it does not own yet, and record them in the page
        table."""
        plan: List[Tuple[int, int, int]] = []
        need = 0
        for r in reqs:
            first, last = div_ceil(r.cached_len, self.page_size), div_ceil(r.device_len, self.page_size)
            if last > first:
                plan.append((r.table_idx, first, last))
                need += last - first
        if need == 0:
            return
        if self.page_classes > 1:
            classes = torch.cat([torch.arange(first, last) % self.page_classes for _, first, last in plan])
            pages = self._allocate_classes(classes)
        else:
            pages = self._allocate(need)
        _write_page_table(self.page_table, self._expand(pages), plan, self.page_size)

    def cache_req(self, req: Req, *, finished: bool) -> None:
        """Insert the request's computed prefix into the prefix cache and
        release slots that became duplicates; on finish also release the
        tail that could not be cached (partial last page)."""
        ids = req.all_ids()[: req.cached_len]
        slots = self.page_table[req.table_idx, : req.cached_len]
        old = req.cache_handle
        already, new = self.prefix_cache.insert_prefix(ids, slots)
        self.unlock(old)
        # [old.cached_len, already): cached meanwhile by another request -> ours are duplicates
        self._free(slots[old.cached_len : already])
        if finished:
            self._free(slots[new.cached_len :])
        else:
            req.cache_handle = new
            self.lock(new)

    @contextmanager
    def lazy_free_region(self):
        """Batch all frees inside the block into one concatenation."""
        self._pending_free = []
        try:
            yield
        finally:
            pending, self._pending_free = self._pending_free, None
            if pending:
                self.free_slots = torch.cat([self.free_slots] + pending)

    def check_integrity(self) -> None:
        self.prefix_cache.check_integrity()
        cached_pages = self.prefix_cache.size_info.total_size // self.page_size
        if len(self.free_slots) + cached_pages != self.num_pages:
            raise RuntimeError(f"CacheManager integrity check failed: free pages {len(self.free_slots)} + "
                               f"cached pages {cached_pages} != {self.num_pages}")
        if self.page_size > 1 and bool((self.free_slots % self.page_size != 0).any()):
            raise RuntimeError("free slot list holds a slot that is not page aligned")

    # ------------------------------------------------------------ helpers
    def _allocate(self, pages: int) -> torch.Tensor:
        short = pages - len(self.free_slots)
        if short > 0:
            evicted = self.prefix_cache.evict(short * self.page_size)
            self.free_slots = torch.cat([self.free_slots, evicted[:: self.page_size]])
            if len(self.free_slots) < pages:
                raise RuntimeError("eviction did not free enough pages")
        out, self.free_slots = self.free_slots[:pages], self.free_slots[pages:]
        return out

    def _allocate_classes(self, classes: torch.Tensor) -> torch.Tensor:
        """Page-start slots whose page id class (id % page_classes) is
        classes[i], in that order; evicts cached pages until every class has
        enough."""
        K, P = self.page_classes, self.page_size
        need = torch.bincount(classes, minlength=K)
        for _ in range(8):
            have = torch.bincount(((self.free_slots // P) % K).long().cpu(), minlength=K)
            short = (need - have).clamp(min=0)
            if int(short.sum()) == 0:
                break
            # evicted pages may fall into any class: ask for K times the worst shortfall
            want = min(int(short.max()) * K * P, self.prefix_cache.size_info.evictable_size // P * P)
            if want <= 0:
                raise RuntimeError(f"no free or evictable pages of the classes needed ({short.tolist()} short)")
            evicted = self.prefix_cache.evict(want)
            self.free_slots = torch.cat([self.free_slots, evicted[::P]])
        else:
            raise RuntimeError("eviction did not free enough pages of the classes needed")
        cls_of_free = ((self.free_slots // P) % K).long()
        out = torch.empty(len(classes), dtype=self.free_slots.dtype, device=self.free_slots.device)
        keep = torch.ones(len(self.free_slots), dtype=torch.bool, device=self.free_slots.device)
        for c in range(K):
            n = int(need[c])
            if n == 0:
                continue
            idx = (cls_of_free == c).nonzero().flatten()[:n]
            out[(classes == c).nonzero().flatten().to(out.device)] = self.free_slots[idx]
            keep[idx] = False
        self.free_slots = self.free_slots[keep]
        return out

    def _free(self, slots: torch.Tensor) -> None:
        if len(slots) == 0:
            return
        firsts = slots[:: self.page_size]
        if self._pending_free is not None:
            self._pending_free.append(firsts)
        else:
            self.free_slots = torch.cat([self.free_slots, firsts])

    def _expand(self, pages: torch.Tensor) -> torch.Tensor:
        """Page-start slots -> every token slot of those pages."""
        if self.page_size == 1:
            return pages
        offs = torch.arange(self.page_size, dtype=torch.int32, device=pages.device)
        return (pages[:, None] + offs[None, :]).reshape(-1)


def _write_page_table(page_table: torch.Tensor, slots: torch.Tensor, plan: List[Tuple[int, int, int]],
                      page_size: int) -> None:
    rows, cols = [], []
    for row, first, last in plan:
        n = (last - first) * page_size
        rows.append(torch.full((n,), row, dtype=torch.int64))
        cols.append(torch.arange(first * page_size, last * page_size, dtype=torch.int64))
    r, c = torch.cat(rows), torch.cat(cols)
    assert len(r) == len(slots)
    if page_table.is_cuda:
        r, c = r.pin_memory().to(page_table.device, non_blocking=True), c.pin_memory().to(page_table.device, non_blocking=True)
    page_table[r, c] = slots
