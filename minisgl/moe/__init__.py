"""MoE compute backends (``fused``: router + grouped tcgen05 GEMMs)."""

from __future__ import annotations

from minisgl.utils import Registry

from .base import BaseMoeBackend

SUPPORTED_MOE_BACKENDS = Registry("MoE Backend")


@SUPPORTED_MOE_BACKENDS.register("fused")
def _fused() -> BaseMoeBackend:
    from .fused import FusedMoe

    return FusedMoe()


def create_moe_backend(backend: str) -> BaseMoeBackend:
    return SUPPORTED_MOE_BACKENDS["fused" if backend == "auto" else backend]()


__all__ = ["BaseMoeBackend", "create_moe_backend", "SUPPORTED_MOE_BACKENDS"]
