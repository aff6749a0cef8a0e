"""Optional step profiler (MINISGL_PROFILE_STEPS=1) and CUDA profiler
window (MINISGL_CUDA_PROFILER_STEPS=a:b).

Records, per scheduler step, the phase, batch size, the host time spent in
the loop iteration and the device time of the forward pass (CUDA events on
the engine stream). ``summary()`` aggregates by phase and batch-size bucket
so one can see whether a workload is host-bound (host ms > device ms) or
device-bound.
"""

from __future__ import annotations

import time
from collections import defaultdict
from typing import Callable, Dict, List, Optional, Tuple

import torch


def parse_step_window(spec: str) -> Optional[Tuple[int, int]]:
    """``"a:b"`` -> (a, b): scheduler steps a .. b - 1 (0-based, counting
    every forward). Empty -> None; anything else malformed raises."""
    spec = spec.strip()
    if not spec:
        return None
    parts = spec.split(":")
    if len(parts) != 2:
        raise ValueError(f"profiler step window must look like 'a:b', got {spec!r}")
    a, b = int(parts[0]), int(parts[1])
    if a < 0 or b <= a:
        raise ValueError(f"profiler step window needs 0 <= a < b, got {spec!r}")
    return a, b


class CudaProfilerWindow:
    """Brackets scheduler steps [a, b) with cudaProfilerStart / Stop, so
    ``nsys profile --capture-range=cudaProfilerApi`` or ``ncu
    --profile-from-start off`` records only those steps. ``on_step(step)``
    runs before the forward of `step`; the stop synchronizes first so the
    window's kernels are finished."""

    def __init__(self, window: Tuple[int, int], start: Optional[Callable[[], None]] = None,
                 stop: Optional[Callable[[], None]] = None, sync: Optional[Callable[[], None]] = None) -> None:
        self.first, self.end = window
        self._start = start or torch.cuda.profiler.start
        self._stop = stop or torch.cuda.profiler.stop
        self._sync = sync or torch.cuda.synchronize
        self.active = False

    def on_step(self, step: int) -> None:
        if step == self.first and not self.active:
            self._start()
            self.active = True
        elif step >= self.end and self.active:
            self._sync()
            self._stop()
            self.active = False


class StepProfiler:
    def __init__(self) -> None:
        self.records: List[Tuple[str, int, float, "torch.cuda.Event", "torch.cuda.Event"]] = []
        self._t = time.perf_counter()

    def begin(self) -> Tuple[float, "torch.cuda.Event"]:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return time.perf_counter(), ev

    def end(self, phase: str, bs: int, started: Tuple[float, "torch.cuda.Event"]) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        now = time.perf_counter()
        host_ms = (now - self._t) * 1e3  # whole loop iteration on the host
        self._t = now
        self.records.append((phase, bs, host_ms, started[1], ev))

    def summary(self) -> Dict[str, Dict[str, float]]:
        torch.cuda.synchronize()
        agg: Dict[str, List[float]] = defaultdict(lambda: [0, 0.0, 0.0])
        for phase, bs, host_ms, s, e in self.records:
            key = phase if phase == "prefill" else f"decode bs<={1 << (max(bs, 1) - 1).bit_length()}"
            a = agg[key]
            a[0] += 1
            a[1] += host_ms
            a[2] += s.elapsed_time(e)
        return {k: {"steps": v[0], "host_ms_per_step": round(v[1] / v[0], 3), "gpu_ms_per_step": round(v[2] / v[0], 3)}
                for k, v in sorted(agg.items())}

    def reset(self) -> None:
        self.records.clear()
        self._t = time.perf_counter()
