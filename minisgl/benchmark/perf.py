"""Kernel timing helpers: CUDA events on the launching stream after warm-up,
with a synchronize on both sides; optional L2 flush between iterations; and
SM clock sampling (nvidia-smi) to report beside kernel timings."""

from __future__ import annotations

import statistics
import subprocess
from typing import Callable, Dict, Optional

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


class SmClockLog:
    """SM clock and throttle reasons of one GPU, sampled by nvidia-smi every
    200 ms while a benchmark runs: kernel times taken power-capped or with a
    lowered clock are not comparable across runs, so the summary goes beside
    them. Unavailable (no nvidia-smi) gives an empty summary."""

    _FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
               "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
               "clocks_event_reasons.sw_power_cap")
    _REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu: int) -> None:
        self.gpu = gpu
        self.proc: Optional[subprocess.Popen] = None

    def start(self) -> "SmClockLog":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self._FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def stop(self) -> Dict[str, object]:
        if self.proc is None:
            return {"clocks": "nvidia-smi unavailable"}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        return self.summarize(out, self.gpu)

    @classmethod
    def summarize(cls, text: str, gpu: int) -> Dict[str, object]:
        """Median SM MHz of the samples under load (above 200 W), the largest
        clocks.max.sm and the throttle reasons seen active."""
        clocks, maxes, reasons = [], [], set()
        for line in text.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8 or not parts[0].isdigit() or int(parts[0]) != gpu:
                continue
            try:
                clk, mx, pw = float(parts[1]), float(parts[2]), float(parts[3])
            except ValueError:
                continue
            maxes.append(mx)
            if pw > 200:
                clocks.append(clk)
            reasons.update(n for n, v in zip(cls._REASONS, parts[4:8]) if v.lower() == "active")
        return {"clocks": {"sm_mhz_median_under_load": statistics.median(clocks) if clocks else None,
                           "sm_max_mhz": max(maxes) if maxes else None, "reasons": sorted(reasons),
                           "samples_under_load": len(clocks)}}
