"""The requests in their decode phase.

Kept as a dict keyed by uid, so aborts and removals are O(1) and the batch
order is decided only when a batch is formed. The reservation rule that
admission control reads (``inflight_tokens``: every running request's
remaining outputs plus at most one partly used page each) is the reference's
scheduling policy (python/minisgl/scheduler/decode.py:9-39), so both engines
admit the same prefill work.
"""

from __future__ import annotations

from typing import Dict, Iterable, List, Optional

from minisgl.core import Batch, Req


class DecodeManager:
    def __init__(self, page_size: int) -> None:
        self.page_size = page_size
        self._by_uid: Dict[int, Req] = {}

    @property
    def running_reqs(self) -> List[Req]:
        return list(self._by_uid.values())

    def filter_reqs(self, reqs: Iterable[Req]) -> None:
        """After a forward step: adopt the step's requests that now decode
        (finished prefills) and drop every request that can no longer decode
        (finished, or a prefill chunk that still has prompt left)."""
        merged = dict(self._by_uid)
        merged.update((r.uid, r) for r in reqs)
        self._by_uid = {uid: r for uid, r in merged.items() if r.can_decode}

    def remove_req(self, req: Req) -> None:
        self._by_uid.pop(req.uid, None)

    def abort_req(self, uid: int) -> Optional[Req]:
        return self._by_uid.pop(uid, None)

    @property
    def inflight_tokens(self) -> int:
        """KV slots running requests may still claim."""
        return sum(r.remain_len + self.page_size - 1 for r in self._by_uid.values())

    def schedule_next_batch(self) -> Optional[Batch]:
        if not self._by_uid:
            return None
        # longest first: the split-KV attention grid walks requests in batch
        # order, so the long ones start in the first waves and the last wave
        # holds only short ones (longest-processing-time order of the CTAs);
        # uid breaks ties, so the order is deterministic
        order = sorted(self._by_uid.values(), key=lambda r: (-r.device_len, r.uid))
        return Batch(reqs=order, phase="decode")

    @property
    def runnable(self) -> bool:
        return bool(self._by_uid)
