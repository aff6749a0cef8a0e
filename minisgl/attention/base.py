"""Attention backend interface (prefill / decode, CUDA-graph hooks).

Shaped like the reference's interface (python/minisgl/attention/base.py) so
the engine's graph runner drives any backend the same way, with one
difference: ``forward`` receives the fused qkv activation after the KV store
(the q heads are its first columns), because the store is fused into the
RoPE kernel of the attention layer.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import TYPE_CHECKING, List

if TYPE_CHECKING:
    import torch

    from minisgl.core import Batch


class BaseAttnMetadata(ABC):
    @abstractmethod
    def get_last_indices(self, bs: int) -> "torch.Tensor":
        """Row of the last token of each of the first ``bs`` requests."""


class BaseAttnBackend(ABC):
    @abstractmethod
    def forward(self, qkv: "torch.Tensor", layer_id: int, batch: "Batch") -> "torch.Tensor": ...

    @abstractmethod
    def prepare_metadata(self, batch: "Batch") -> None: ...

    @abstractmethod
    def init_capture_graph(self, max_seq_len: int, bs_list: List[int]) -> None: ...

    @abstractmethod
    def prepare_for_capture(self, batch: "Batch") -> None: ...

    @abstractmethod
    def prepare_for_replay(self, batch: "Batch") -> None: ...


class HybridBackend(BaseAttnBackend):
    """Different backends for prefill and decode (``--attn p,d``)."""

    def __init__(self, prefill_backend: BaseAttnBackend, decode_backend: BaseAttnBackend) -> None:
        self.prefill_backend = prefill_backend
        self.decode_backend = decode_backend

    def _pick(self, batch: "Batch") -> BaseAttnBackend:
        return self.prefill_backend if batch.is_prefill else self.decode_backend

    def forward(self, qkv, layer_id, batch):
        return self._pick(batch).forward(qkv, layer_id, batch)

    def prepare_metadata(self, batch) -> None:
        self._pick(batch).prepare_metadata(batch)

    def init_capture_graph(self, max_seq_len: int, bs_list: List[int]) -> None:
        self.decode_backend.init_capture_graph(max_seq_len, bs_list)

    def prepare_for_capture(self, batch) -> None:
        self.decode_backend.prepare_for_capture(batch)

    def prepare_for_replay(self, batch) -> None:
        self.decode_backend.prepare_for_replay(batch)
