"""Autotuned tile plans for the decode-shaped GEMMs.

Decode GEMMs are latency bound and the best tile plan (weight-major or
token-major tiles, N tile, cluster split-K factor) depends on (M, N, K) in
ways a closed-form heuristic gets wrong by up to 4x. Before CUDA-graph
capture the engine times every candidate plan for each (batch size, weight
shape) it will replay, with each candidate captured in a CUDA graph of
back-to-back launches (so launch overhead does not hide kernel time) that
cycle through copies of the weight larger than L2 in total (so weights
come from HBM, as in a real step), and records the fastest. ``minisgl.ops.gemm`` then uses the recorded plan for
exactly that shape and the built-in heuristic for everything else.

Plans can be saved to / loaded from a JSON file keyed by the device name.
"""

from __future__ import annotations

import json
import os
from typing import Dict, Iterable, List, Optional, Tuple

import torch

Plan = Tuple[int, int, int]  # (mode: 1 token-major / 2 weight-major, n tile, splits)
PLANS: Dict[Tuple[int, int, int], Plan] = {}
# best weight-major plan per shape: the fused-epilogue GEMMs need those tiles
SWAP_PLANS: Dict[Tuple[int, int, int], Plan] = {}


# batch sizes that are tuned; other sizes use the plan of the next tuned size
TUNED_SIZES = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256)


def candidates(M: int, K: int, full: bool = True) -> List[Plan]:
    """Plans worth timing for M tokens and reduction size K (``full`` adds
    plans that are rarely the best, for exhaustive tests)."""
    num_kb = (K + 63) // 64
    out: List[Plan] = []
    top = 16
    while top < M and top < 256:
        top *= 2
    for bn in (16, 32, 64, 128, 256):
        if bn > top or (not full and bn < top // 8):
            continue
        for s in (1, 2, 4, 8, 16):
            if s <= num_kb and bn % s == 0 and (full or s * 2 <= num_kb):
                out.append((2, bn, s))
    if M >= (32 if full else 128):
        for bn in (32, 64, 128, 256) if full else (64, 128, 256):
            for s in (1, 2, 4, 8):
                if s <= num_kb:
                    out.append((1, bn, s))
    return out


# bytes of weight copies cycled through while timing: above the 126 MB L2, so
# every launch streams its weights from HBM as in a real decode step
_COLD_BYTES = 192 << 20


def _time_plan(native, out, x, ws: List[torch.Tensor], plan: Plan, reps: int = 8) -> float:
    mode, bn, s = plan
    reps = max(reps, len(ws))

    def run(w):
        native.gemm(out, x, w, None, None, s, mode, None, bn)

    run(ws[0])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            run(ws[i % len(ws)])
    g.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(3):
        start.record()
        g.replay()
        end.record()
        end.synchronize()
        best = min(best, start.elapsed_time(end) / reps)
    del g
    return best


def tune(shapes: Iterable[Tuple[int, int]], batch_sizes: Iterable[int], device: torch.device,
         cache_file: Optional[str] = None) -> Dict[Tuple[int, int, int], Plan]:
    """Find the fastest plan for every (M, N, K); M from ``batch_sizes``,
    (N, K) from ``shapes``. Returns (and installs) the plan table."""
    from minisgl import ops

    native = ops.native()
    key_dev = torch.cuda.get_device_name(device) + "|cold-weights"
    cached = _load(cache_file, key_dev)
    shapes = sorted(set(shapes))
    wanted = sorted(set(int(m) for m in batch_sizes if m > 0))
    # tune representative sizes only; every wanted size maps to the next one
    sizes = sorted({next((t for t in TUNED_SIZES if t >= m), m) for m in wanted})
    with torch.cuda.device(device):
        for N, K in shapes:
            w = torch.randn(N, K, device=device, dtype=torch.bfloat16) * 0.02
            copies = max(1, min(24, -(-_COLD_BYTES // w.nbytes)))
            ws = [w] + [w.clone() for _ in range(copies - 1)]
            xmax = torch.randn(max(sizes), K, device=device, dtype=torch.bfloat16)
            omax = torch.empty(max(sizes), N, device=device, dtype=torch.bfloat16)
            for M in sizes:
                key = (M, N, K)
                skey = (-M, N, K)  # weight-major entry of the cache
                if key in cached and skey in cached:
                    PLANS[key] = cached[key]
                    SWAP_PLANS[key] = cached[skey]
                    continue
                x, out = xmax[:M], omax[:M]
                timed = []
                for plan in candidates(M, K, full=False):
                    try:
                        timed.append((_time_plan(native, out, x, ws, plan), plan))
                    except RuntimeError:
                        continue
                if timed:
                    PLANS[key] = min(timed)[1]
                    cached[key] = PLANS[key]
                    swap = [t for t in timed if t[1][0] == 2]
                    if swap:
                        SWAP_PLANS[key] = min(swap)[1]
                        cached[skey] = SWAP_PLANS[key]
            del w, ws, xmax, omax
    torch.cuda.synchronize(device)
    _save(cache_file, key_dev, cached)
    # wanted sizes that were not tuned themselves borrow the next tuned plan
    for N, K in shapes:
        for m in wanted:
            t = next((s for s in sizes if s >= m), None)
            if t is not None and (t, N, K) in PLANS:
                PLANS.setdefault((m, N, K), PLANS[(t, N, K)])
            if t is not None and (t, N, K) in SWAP_PLANS:
                SWAP_PLANS.setdefault((m, N, K), SWAP_PLANS[(t, N, K)])
    return dict(PLANS)


def lookup(M: int, N: int, K: int) -> Optional[Plan]:
    return PLANS.get((M, N, K))


def clear() -> None:
    PLANS.clear()
    SWAP_PLANS.clear()


def _load(path: Optional[str], dev: str) -> Dict[Tuple[int, int, int], Plan]:
    if not path or not os.path.isfile(path):
        return {}
    try:
        with open(path) as f:
            data = json.load(f).get(dev, {})
        return {tuple(int(v) for v in k.split(",")): tuple(p) for k, p in data.items()}  # type: ignore[misc]
    except (OSError, ValueError):
        return {}


def _save(path: Optional[str], dev: str, plans: Dict[Tuple[int, int, int], Plan]) -> None:
    if not path:
        return
    try:
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        data = {}
        if os.path.isfile(path):
            with open(path) as f:
                data = json.load(f)
        data[dev] = {",".join(map(str, k)): list(v) for k, v in plans.items()}
        with open(path, "w") as f:
            json.dump(data, f)
    except (OSError, ValueError):
        pass
