"""Kernel timing helpers: CUDA events on the launching stream after warm-up,
with a synchronize on both sides; optional L2 flush between iterations."""

from __future__ import annotations

from typing import Callable, Optional

import torch

_FLUSH: Optional[torch.Tensor] = None


def flush_l2() -> None:
    """Overwrite a buffer larger than the 126 MB L2 of a B200."""
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.zero_()


def time_kernel(fn: Callable[[], object], iters: int = 20, warmup: int = 5, flush: bool = True) -> float:
    """Mean milliseconds per call. With ``flush`` the L2 is flushed before
    every timed call and only the call itself sits between the events."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        if flush:
            flush_l2()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
    torch.cuda.synchronize()
    return total / iters


def time_graph(fn: Callable[[], object], iters: int = 100) -> float:
    """Mean ms per call with launches captured in a CUDA graph (launch
    overhead excluded); no L2 flush (back-to-back calls)."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    g.replay()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / iters
