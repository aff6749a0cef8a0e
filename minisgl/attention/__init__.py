"""Attention backends.

There is one implementation, the sm_100a kernels (``native``). The names the
reference accepts for ``--attention-backend`` (``trtllm``, ``fi``, ``fa``)
are kept as aliases so existing command lines still parse; they select the
same native backend.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

from minisgl.utils import Registry, init_logger

from .base import BaseAttnBackend, BaseAttnMetadata, HybridBackend

if TYPE_CHECKING:
    from minisgl.models import ModelConfig

logger = init_logger(__name__)
SUPPORTED_ATTENTION_BACKENDS = Registry("Attention Backend")


def _native(config: "ModelConfig", max_batch: int = 256) -> BaseAttnBackend:
    if config.is_mla:
        from .mla import MLAAttnBackend

        return MLAAttnBackend(config, max_batch)
    from .native import NativeAttnBackend

    return NativeAttnBackend(config, max_batch)


for _name in ("native", "trtllm", "fi", "fa"):
    SUPPORTED_ATTENTION_BACKENDS.register(_name)(_native)


def validate_attn_backend(backend: str, allow_auto: bool = True) -> str:
    if backend == "auto":
        if not allow_auto:
            raise ValueError("'auto' must be resolved before creating a backend")
        return backend
    SUPPORTED_ATTENTION_BACKENDS.assert_supported(backend.split(","))
    return backend


def create_attention_backend(backend: str, config: "ModelConfig", max_batch: int = 256) -> BaseAttnBackend:
    if backend == "auto":
        backend = "native"
    validate_attn_backend(backend, allow_auto=False)
    if "," in backend:
        p, d = backend.split(",", 1)
        if p != d:
            pb = SUPPORTED_ATTENTION_BACKENDS[p](config, max_batch)
            db = SUPPORTED_ATTENTION_BACKENDS[d](config, max_batch)
            if type(pb) is type(db):
                return db  # all names map to the same implementation
            return HybridBackend(pb, db)
        backend = p
    return SUPPORTED_ATTENTION_BACKENDS[backend](config, max_batch)


__all__ = ["BaseAttnMetadata", "BaseAttnBackend", "HybridBackend", "create_attention_backend",
           "SUPPORTED_ATTENTION_BACKENDS", "validate_attn_backend"]
