"""Core request / batch / context state shared by scheduler, engine and model.

Field names of ``SamplingParams`` are public API (the offline ``LLM`` and the
HTTP server build it) and match the reference (python/minisgl/core.py:15-26).
The per-request length bookkeeping follows the same model as the reference
(core.py:29-67): a request owns positions [0, device_len) of which
[0, cached_len) already have KV in the pool.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, List, Literal, Optional

import torch

if TYPE_CHECKING:
    from minisgl.attention import BaseAttnBackend, BaseAttnMetadata
    from minisgl.kvcache import BaseCacheHandle, BaseKVCachePool
    from minisgl.moe import BaseMoeBackend


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    ignore_eos: bool = False
    max_tokens: int = 1024

    @property
    def is_greedy(self) -> bool:
        return (self.temperature <= 0.0 or self.top_k == 1) and self.top_p == 1.0


@dataclass(eq=False)
class Req:
    """A request resident on the device.

    input_ids   host tokens known so far (prompt + generated)
    table_idx   row of the page table / token pool owned by this request
    cached_len  positions whose KV is already written
    device_len  positions whose token ids are on the device
    """

    input_ids: torch.Tensor
    table_idx: int
    cached_len: int
    output_len: int
    uid: int
    sampling_params: SamplingParams
    cache_handle: "BaseCacheHandle"

    def __post_init__(self) -> None:
        assert self.input_ids.device.type == "cpu"
        self._appended: List[int] = []  # sampled tokens not yet folded into input_ids
        self.device_len = len(self.input_ids)
        self.max_device_len = len(self.input_ids) + self.output_len
        assert 0 <= self.cached_len < self.device_len <= self.max_device_len, self

    @property
    def remain_len(self) -> int:
        return self.max_device_len - self.device_len

    @property
    def extend_len(self) -> int:
        return self.device_len - self.cached_len

    @property
    def can_decode(self) -> bool:
        return self.remain_len > 0

    def complete_one(self) -> None:
        """The forward pass wrote KV for every device token and produced one
        more token id on the device."""
        self.cached_len = self.device_len
        self.device_len += 1

    def append_host(self, next_token) -> None:
        """Record a sampled token on the host (an int or a 1-element tensor).
        Appends are buffered in a list; ``all_ids`` folds them in."""
        if isinstance(next_token, torch.Tensor):
            self._appended.extend(int(t) for t in next_token.reshape(-1).tolist())
        else:
            self._appended.append(int(next_token))

    def all_ids(self) -> torch.Tensor:
        """Every host-known token of the request (prompt + sampled)."""
        if self._appended:
            extra = torch.tensor(self._appended, dtype=self.input_ids.dtype)
            self.input_ids = torch.cat([self.input_ids, extra])
            self._appended = []
        return self.input_ids

    def __repr__(self) -> str:
        return (f"{type(self).__name__}(uid={self.uid}, table_idx={self.table_idx}, cached_len={self.cached_len}, "
                f"device_len={self.device_len}, max_device_len={self.max_device_len})")


@dataclass
class Batch:
    reqs: List[Req]
    phase: Literal["prefill", "decode"]
    # filled by the scheduler
    input_ids: torch.Tensor = field(init=False)
    positions: torch.Tensor = field(init=False)
    out_loc: torch.Tensor = field(init=False)
    padded_reqs: List[Req] = field(init=False)
    # filled by the attention backend
    attn_metadata: "BaseAttnMetadata" = field(init=False)

    @property
    def is_prefill(self) -> bool:
        return self.phase == "prefill"

    @property
    def is_decode(self) -> bool:
        return self.phase == "decode"

    @property
    def size(self) -> int:
        return len(self.reqs)

    @property
    def padded_size(self) -> int:
        return len(self.padded_reqs)


@dataclass
class FusedSample:
    """Sampling fused into the LM head: per-row temperatures (None: greedy),
    the sampler's seed and device step counter, and an optional output
    buffer for the tokens."""

    temperatures: Optional[torch.Tensor]
    seed: int
    step: torch.Tensor
    out: Optional[torch.Tensor] = None


@dataclass
class Context:
    """Per-process forward context: the page table (token slots per request
    row), the KV pool, the attention / MoE backends and the active batch."""

    page_size: int
    page_table: torch.Tensor = field(init=False)
    attn_backend: "BaseAttnBackend" = field(init=False)
    moe_backend: "BaseMoeBackend" = field(init=False)
    kv_cache: "BaseKVCachePool" = field(init=False)
    extras: dict = field(default_factory=dict)
    _batch: Optional[Batch] = field(default=None, init=False)
    # set around a forward whose LM head should return sampled tokens instead
    # of logits (engine / CUDA-graph capture; see FusedSample)
    fused_sample: Optional["FusedSample"] = field(default=None, init=False)

    @property
    def batch(self) -> Batch:
        if self._batch is None:
            raise RuntimeError("no active batch in the forward context")
        return self._batch

    @contextmanager
    def forward_batch(self, batch: Batch):
        if self._batch is not None:
            raise RuntimeError("nested forward_batch is not allowed")
        self._batch = batch
        try:
            yield
        finally:
            self._batch = None


_GLOBAL_CTX: Optional[Context] = None


def set_global_ctx(ctx: Context) -> None:
    global _GLOBAL_CTX
    if _GLOBAL_CTX is not None:
        raise RuntimeError("global context is already set")
    _GLOBAL_CTX = ctx


def get_global_ctx() -> Context:
    if _GLOBAL_CTX is None:
        raise RuntimeError("global context is not set")
    return _GLOBAL_CTX


def reset_global_ctx() -> None:
    global _GLOBAL_CTX
    _GLOBAL_CTX = None
