"""Set of running (decoding) requests."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Iterable, Optional, Set

from minisgl.core import Batch, Req


@dataclass
class DecodeManager:
    page_size: int
    running_reqs: Set[Req] = field(default_factory=set)

    def filter_reqs(self, reqs: Iterable[Req]) -> None:
        self.running_reqs = {r for r in self.running_reqs.union(reqs) if r.can_decode}

    def remove_req(self, req: Req) -> None:
        self.running_reqs.discard(req)

    def abort_req(self, uid: int) -> Optional[Req]:
        for r in self.running_reqs:
            if r.uid == uid:
                self.running_reqs.remove(r)
                return r
        return None

    @property
    def inflight_tokens(self) -> int:
        """Tokens running requests may still claim: their remaining outputs
        plus up to one partially used page each."""
        return sum(r.remain_len for r in self.running_reqs) + (self.page_size - 1) * len(self.running_reqs)

    def schedule_next_batch(self) -> Optional[Batch]:
        if not self.running_reqs:
            return None
        # longest first: the decode attention grid walks requests in batch
        # order, so long requests start in the first waves and the last wave
        # holds only short ones (longest-processing-time scheduling of the
        # split-KV CTAs); uid breaks ties, so the order is deterministic
        return Batch(reqs=sorted(self.running_reqs, key=lambda r: (-r.device_len, r.uid)), phase="decode")

    @property
    def runnable(self) -> bool:
        return bool(self.running_reqs)
