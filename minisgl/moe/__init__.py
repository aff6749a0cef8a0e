"""MoE compute backends (``fused``: router + grouped tcgen05 GEMMs)."""

from __future__ import annotations

from minisgl.utils import Registry

from .base import BaseMoeBackend

SUPPORTED_MOE_BACKENDS = Registry("MoE Backend")


@SUPPORTED_MOE_BACKENDS.register("fused")
def _fused() -> BaseMoeBackend:
    from .fused import FusedMoe

    return FusedMoe()


def create_moe_backend(backend: str, ep_dispatch: bool = False, ep_size: int = 1, ep_rank: int = 0,
                       group=None, heap=None, context_parallel: bool = False) -> BaseMoeBackend:
    """``ep_dispatch``: experts split over the ranks and tokens dispatched to
    their owners (DP attention); ``context_parallel``: experts split over the
    context-parallel ranks (dispatch for token-sharded prefill, local experts
    + all-reduce for replicated decode); otherwise the named local backend."""
    if context_parallel:
        from .ep_a2a import ContextParallelMoe

        return ContextParallelMoe(ep_size, ep_rank, group)
    if ep_dispatch:
        from .ep_a2a import AllToAllMoe

        return AllToAllMoe(ep_size, ep_rank, group, heap)
    return SUPPORTED_MOE_BACKENDS["fused" if backend == "auto" else backend]()


__all__ = ["BaseMoeBackend", "create_moe_backend", "SUPPORTED_MOE_BACKENDS"]
