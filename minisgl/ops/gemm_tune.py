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

Plan = Tuple[int, int, int]  # (mode: 1 token-major / 2 weight-major / 3 persistent, n tile, splits)
PLANS: Dict[Tuple[int, int, int], Plan] = {}
# best plan per shape among those the fused epilogues accept (weight-major
# tiles, or token-major tiles with an N tile of 128 / 256)
FUSED_PLANS: Dict[Tuple[int, int, int], Plan] = {}


# batch sizes that are tuned; other sizes use the plan of the next tuned size
TUNED_SIZES = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256)
# prefill chunk sizes that are tuned; longer chunks use the plan of the next
# one (or of the largest)
PREFILL_SIZES = (512, 2048, 8192)



def candidates(M: int, K: int, full: bool = True) -> List[Plan]:
    """Plans worth timing for M tokens and reduction size K (``full`` adds
    plans that are rarely the best, for exhaustive tests)."""
    num_kb = (K + 63) // 64
    out: List[Plan] = []
    top = 16
    while top < M and top < 256:
        top *= 2
    # split counts: powers of two, and 3 / 6 so that a few dozen tiles can
    # fill the 148 SMs (40 tiles x 3 = 120 CTAs where x 4 would spill over a
    # second wave); the cluster reduction gives ragged row shares
    for bn in (16, 32, 64, 128, 256):
        if bn > top or (not full and bn < top // 8):
            continue
        for s in (1, 2, 3, 4, 6, 8, 16):
            if s <= num_kb and s <= bn and (full or s * 2 <= num_kb):
                out.append((2, bn, s))
    if M >= (32 if full else 128):
        for bn in (32, 64, 128, 256) if full else (64, 128, 256):
            for s in (1, 2, 3, 4, 6, 8):
                if s <= num_kb:
                    out.append((1, bn, s))
    if M >= 64 and K % 64 == 0:
        # persistent 128 x N-tile CTAs: win on wide outputs such as the LM
        # head (151936 features at 256 rows: 0.106 vs 0.138 ms)
        out += [(3, 256, 1), (3, 128, 1)]
    if M >= 128 and K % 64 == 0:
        # persistent 256 x 256 tiles on CTA pairs (cta_group::2): half the
        # operand traffic per SM; wins some Qwen3-32B shapes (TP1 gate_up at
        # 256 rows 0.122 vs 0.136 ms, TP2 o_proj at 8192 rows 0.256 vs 0.265)
        out.append((5, 256, 1))
    if M <= 256 and K % 64 == 0:
        # stream-K weight streaming over every SM, 128 or 256 weight rows per
        # work tile (mode 4: (4, R, k-blocks per stage; 0 = automatic))
        out += [(4, 1, 0), (4, 2, 0)]
    return out


def run_plan(out: torch.Tensor, x: torch.Tensor, w: torch.Tensor, plan: Plan) -> None:
    """One plain GEMM launch with a forced plan (the stream-K mode takes its
    per-stream workspace)."""
    from minisgl import ops

    mode, bn, s = plan
    if mode == ops.GEMM_STREAMK:
        ops.native().gemm(out, x, w, None, ops.streamk_workspace(x.device), 0, mode, None, bn, None, s)
    else:
        ops.native().gemm(out, x, w, None, None, s, mode, None, bn)


# bytes of weight copies cycled through while timing: above the 126 MB L2, so
# every launch streams its weights from HBM as in a real decode step
_COLD_BYTES = 192 << 20


def _time_runs(run, ws: List[torch.Tensor], reps: int = 8) -> float:
    """Mean ms of ``run(w)`` over back-to-back launches in a CUDA graph that
    cycles through the weight copies ``ws``; best of three replays."""
    reps = max(reps, len(ws))
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


def _fused_candidates(M: int, K: int, kind: int) -> List[Plan]:
    """Plans a fused-epilogue GEMM of this kind accepts: weight-major tiles,
    token-major tiles (with whole 128-feature heads / gate|up blocks when the
    epilogue needs them)."""
    from minisgl import ops

    num_kb = (K + 63) // 64
    out = [p for p in candidates(M, K, full=False) if p[0] == 2]
    if kind == ops.EPI_SAMPLE:  # the sampling epilogue needs weight-major tiles
        return out
    if M >= 64:
        whole = (kind & (ops.EPI_ROPE | ops.EPI_SILU)) != 0
        for bn in (128, 256) if whole else (64, 128, 256):
            for s in (1, 2, 4, 8):
                if s <= num_kb:
                    out.append((1, bn, s))
    return out


class _FusedBench:
    """Dummy epilogue operands for timing a fused GEMM of one kind."""

    def __init__(self, kind: int, hq: int, hk: int, M: int, N: int, device: torch.device) -> None:
        from minisgl import ops

        self.kw: dict = {}
        self.out = torch.empty(M, N // 2 if kind & ops.EPI_SILU else N, dtype=torch.bfloat16, device=device)
        if kind & ops.EPI_NORM:
            self.kw["norm_eps"] = 1e-6
        if kind & ops.EPI_SILU:
            self.kw["silu"] = True
        if kind & ops.EPI_RESIDUAL:
            self.kw["residual"] = self.out
        if kind & ops.EPI_ROPE:
            page = 64
            pages = (M + page - 1) // page + 1
            cache = torch.zeros(pages, hk, page, 128, dtype=torch.bfloat16, device=device)
            ang = torch.rand(64, 64, device=device)
            self.kw["rope"] = dict(
                positions=torch.zeros(M, dtype=torch.int32, device=device),
                cos_sin=torch.cat([ang.cos(), ang.sin()], 1).contiguous(),
                out_loc=torch.arange(M, dtype=torch.int32, device=device), q_norm_w=None, k_norm_w=None,
                head_eps=1e-6, k_cache=cache, v_cache=torch.zeros_like(cache), hq=hq, hk=hk, page_size=page)


def tune(shapes: Iterable[Tuple[int, int]], batch_sizes: Iterable[int], device: torch.device,
         cache_file: Optional[str] = None,
         fused: Optional[Dict[Tuple[int, int], Tuple[int, int, int]]] = None,
         prefill: bool = False) -> Dict[Tuple[int, int, int], Plan]:
    """Find the fastest plan for every (M, N, K); M from ``batch_sizes``,
    (N, K) from ``shapes``. ``fused`` maps (N, K) to (epilogue kind, q heads,
    kv heads) for the projections the fused decode layers run: those get a
    plan of their own (FUSED_PLANS), timed with that epilogue. ``prefill``
    also tunes the chunk sizes of PREFILL_SIZES. Returns (and installs) the
    plain plan table."""
    from minisgl import ops

    native = ops.native()
    fused = dict(fused or {})
    key_dev = torch.cuda.get_device_name(device) + "|cold-weights|fused-kinds|tcgen05-only|sample|streamk|pairs|splits3"
    cached = _load(cache_file, key_dev)
    shapes = sorted(set(shapes) | set(fused))
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
                skey = (-M, N, K)  # fused-epilogue entry of the cache
                x, out = xmax[:M], omax[:M]
                if key in cached:
                    PLANS[key] = cached[key]
                else:
                    timed = []
                    for plan in candidates(M, K, full=False):
                        try:
                            timed.append((_time_runs(lambda w_, p_=plan: run_plan(out, x, w_, p_), ws), plan))
                        except RuntimeError:
                            continue
                    if timed:
                        PLANS[key] = cached[key] = min(timed)[1]
                if (N, K) not in fused:
                    continue
                if skey in cached:
                    FUSED_PLANS[key] = cached[skey]
                    continue
                kind, hq, hk = fused[(N, K)]
                timed = []
                if kind == ops.EPI_SAMPLE:
                    temps = torch.full((M,), 0.7, device=device)
                    step = torch.zeros((), dtype=torch.int64, device=device)
                    toks = torch.empty(M, dtype=torch.int32, device=device)
                    for plan in _fused_candidates(M, K, kind):
                        try:
                            timed.append((_time_runs(lambda w_, p_=plan: ops.lm_head_sample(
                                x, w_, None, temps, 0, step, out=toks, plan=(p_[1], p_[2])), ws), plan))
                        except RuntimeError:
                            continue
                else:
                    fb = _FusedBench(kind, hq, hk, M, N, device)
                    for plan in _fused_candidates(M, K, kind):
                        try:
                            timed.append((_time_runs(lambda w_, p_=plan: ops.gemm_fused(
                                x, w_, out=fb.out, plan=p_, **fb.kw), ws), plan))
                        except RuntimeError:
                            continue
                if timed:
                    FUSED_PLANS[key] = cached[skey] = min(timed)[1]
            del w, ws, xmax, omax
    if prefill:
        _tune_prefill(native, shapes, device, cached)
    torch.cuda.synchronize(device)
    _save(cache_file, key_dev, cached)
    # wanted sizes that were not tuned themselves borrow the next tuned plan
    for N, K in shapes:
        for m in wanted:
            t = next((s for s in sizes if s >= m), None)
            if t is not None and (t, N, K) in PLANS:
                PLANS.setdefault((m, N, K), PLANS[(t, N, K)])
            if t is not None and (t, N, K) in FUSED_PLANS:
                FUSED_PLANS.setdefault((m, N, K), FUSED_PLANS[(t, N, K)])
    return dict(PLANS)


def _tune_prefill(native, shapes, device: torch.device, cached: Dict[Tuple[int, int, int], Plan]) -> None:
    """Plain plans for long prefill chunks: persistent or one-tile-per-CTA
    token-major tiles of 128 or 256 features (the weight-major and split-K
    plans only pay off for short batches)."""
    for N, K in shapes:
        for M in PREFILL_SIZES:
            key = (M, N, K)
            if M * N * 2 > (256 << 20):  # e.g. the LM head: prefill computes only last-token logits
                continue
            if key in cached:
                PLANS[key] = cached[key]
                continue
            x = torch.randn(M, K, device=device, dtype=torch.bfloat16)
            out = torch.empty(M, N, device=device, dtype=torch.bfloat16)
            w = torch.randn(N, K, device=device, dtype=torch.bfloat16) * 0.02
            timed = []
            for plan in ((3, 256, 1), (3, 128, 1), (1, 256, 1), (1, 128, 1)):
                mode, bn, s = plan
                timed.append((_time_runs(lambda w_, m=mode, b=bn, sp=s: native.gemm(
                    out, x, w_, None, None, sp, m, None, b), [w], reps=4), plan))
            PLANS[key] = cached[key] = min(timed)[1]
            del x, out, w


def lookup(M: int, N: int, K: int) -> Optional[Plan]:
    """The plan for (M, N, K): tuned for M itself, or for the next tuned
    prefill size (the largest one beyond it)."""
    plan = PLANS.get((M, N, K))
    if plan is not None or M <= TUNED_SIZES[-1]:
        return plan
    size = next((p for p in PREFILL_SIZES if p >= M), PREFILL_SIZES[-1])
    return PLANS.get((size, N, K))


def clear() -> None:
    PLANS.clear()
    FUSED_PLANS.clear()


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
