"""Optional step profiler (MINISGL_PROFILE_STEPS=1).

Records, per scheduler step, the phase, batch size, the host time spent in
the loop iteration and the device time of the forward pass (CUDA events on
the engine stream). ``summary()`` aggregates by phase and batch-size bucket
so one can see whether a workload is host-bound (host ms > device ms) or
device-bound.
"""

from __future__ import annotations

import time
from collections import defaultdict
from typing import Dict, List, Tuple

import torch


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
