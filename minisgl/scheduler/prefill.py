"""Prefill admission with a token budget and chunked prefill.

Pending requests are admitted first-come-first-served (chunked leftovers at
the head) while the batch's token budget lasts. A request is admitted only if
its remaining prompt plus all its output tokens fit next to what running
requests may still need (the reservation). A prompt longer than the
remaining budget is split: the admitted chunk runs as a ``ChunkedReq`` that
is never sampled and the rest is re-queued at the head (Sarathi-style
chunked prefill; behaviour of python/minisgl/scheduler/prefill.py).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import TYPE_CHECKING, List, Optional, Tuple

import torch

from minisgl.core import Batch, Req

if TYPE_CHECKING:
    from minisgl.core import SamplingParams
    from minisgl.kvcache import BaseCacheHandle
    from minisgl.message import UserMsg

    from .cache import CacheManager
    from .decode import DecodeManager
    from .table import TableManager


class ChunkedReq(Req):
    """A prompt chunk: computes KV only, never samples, never decodes."""

    def append_host(self, next_token: torch.Tensor) -> None:
        raise RuntimeError("a prompt chunk is never sampled")

    @property
    def can_decode(self) -> bool:
        return False


@dataclass(slots=True)
class PendingReq:
    """A request waiting for (more of) its prefill. Its prompt and output
    lengths are fixed when it arrives, so admission reads them as fields;
    ``chunked_req`` holds the part already admitted while the prompt is
    split over several steps."""

    uid: int
    input_ids: torch.Tensor
    sampling_params: "SamplingParams"
    input_len: int = field(init=False)
    output_len: int = field(init=False)
    chunked_req: Optional[ChunkedReq] = None

    def __post_init__(self) -> None:
        self.input_len = int(self.input_ids.shape[0])
        self.output_len = int(self.sampling_params.max_tokens)


def _copy_to_device(dst: torch.Tensor, src: torch.Tensor) -> None:
    if dst.is_cuda:
        dst.copy_(src.pin_memory(), non_blocking=True)
    else:
        dst.copy_(src)


@dataclass
class PrefillAdder:
    token_budget: int
    reserved_size: int
    cache_manager: "CacheManager"
    table_manager: "TableManager"

    def _reserve(self, pending: PendingReq) -> Optional[Tuple["BaseCacheHandle", int]]:
        if self.table_manager.available_size == 0:
            return None
        handle = self.cache_manager.match_req(pending).cuda_handle
        need = pending.input_len - handle.cached_len + pending.output_len
        if need + self.reserved_size > self.cache_manager.available_size:
            return None
        # locking turns the matched prefix from evictable into protected, so re-check
        self.cache_manager.lock(handle)
        if need + self.reserved_size > self.cache_manager.available_size:
            self.cache_manager.unlock(handle)
            return None
        row = self.table_manager.allocate()
        n = handle.cached_len
        if n > 0:
            _copy_to_device(self.table_manager.token_pool[row, :n], pending.input_ids[:n])
            self.table_manager.page_table[row, :n].copy_(handle.get_matched_indices())
        return handle, row

    def _admit(self, pending: PendingReq, handle: "BaseCacheHandle", row: int, cached_len: int) -> Req:
        remain = pending.input_len - cached_len
        chunk = min(self.token_budget, remain)
        self.token_budget -= chunk
        self.reserved_size += remain + pending.output_len
        end = cached_len + chunk
        _copy_to_device(self.table_manager.token_pool[row, cached_len:end], pending.input_ids[cached_len:end])
        cls = ChunkedReq if chunk < remain else Req
        return cls(input_ids=pending.input_ids[:end], table_idx=row, cached_len=cached_len,
                   output_len=pending.output_len, uid=pending.uid, cache_handle=handle,
                   sampling_params=pending.sampling_params)

    def try_add_one(self, pending: PendingReq) -> Optional[Req]:
        if self.token_budget <= 0:
            return None
        if (ch := pending.chunked_req) is not None:
            return self._admit(pending, ch.cache_handle, ch.table_idx, ch.cached_len)
        got = self._reserve(pending)
        if got is None:
            return None
        handle, row = got
        return self._admit(pending, handle, row, handle.cached_len)


@dataclass
class PrefillManager:
    cache_manager: "CacheManager"
    table_manager: "TableManager"
    decode_manager: "DecodeManager"
    pending_list: List[PendingReq] = field(default_factory=list)

    def add_one_req(self, msg: "UserMsg") -> None:
        self.pending_list.append(PendingReq(msg.uid, msg.input_ids, msg.sampling_params))

    def schedule_next_batch(self, prefill_budget: int) -> Optional[Batch]:
        if not self.pending_list:
            return None
        adder = PrefillAdder(prefill_budget, self.decode_manager.inflight_tokens, self.cache_manager,
                             self.table_manager)
        reqs: List[Req] = []
        chunked: List[PendingReq] = []
        for pending in self.pending_list:
            req = adder.try_add_one(pending)
            if req is None:
                break
            pending.chunked_req = req if isinstance(req, ChunkedReq) else None
            if pending.chunked_req is not None:
                chunked.append(pending)
            reqs.append(req)
        if not reqs:
            return None
        self.pending_list = chunked + self.pending_list[len(reqs):]
        return Batch(reqs=reqs, phase="prefill")

    def abort_req(self, uid: int) -> Optional[Req]:
        for i, p in enumerate(self.pending_list):
            if p.uid == uid:
                del self.pending_list[i]
                return p.chunked_req
        return None

    @property
    def runnable(self) -> bool:
        return bool(self.pending_list)
