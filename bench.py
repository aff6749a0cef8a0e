"""Serving throughput benchmark: output tok/s of the whole box.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl minisgl|reference] [--shape qwen3-32b]

Default workload: the Qwen3-32B-shape dense decoder (64 layers, hidden 5120,
64 q / 8 kv heads, head_dim 128, SwiGLU 25600, vocabulary 151936), bf16,
random-init weights, tensor parallel over the N GPUs (TP = N, one rank per
GPU, launched by torchrun for N > 1). A pool of 1000 synthetic requests is
served continuously (all submitted at the start: the box runs saturated,
up to 256 requests at a time): prompt lengths lognormal with median 1024
(clipped to [32, 16384]), output lengths lognormal with median 256 (clipped
to [16, 2048]), random token ids, ignore_eos, temperature 0.6; 30% of the
requests start with one of 50 seeded shared prefixes of 512-2048 tokens
(the radix prefix cache serves them).

A *step* is ``--step-tokens`` output tokens (default 8192) of that run: the
run is cut at the scheduler iterations where the running output count
crosses each multiple; W untimed warm-up steps (the initial prefill burst
among them), then K timed steps, after which the run stops. Strong scaling:
the same request pool at every N.

Reported ``value``: output tokens of the K timed steps / device time between
the CUDA events recorded on the engine stream at the step boundaries, the
max over ranks (every rank runs the same schedule). ``e2e``: the same tokens
over the host wall clock between the boundaries, through the offline ``LLM``
API (tokenised prompts go host->device from pinned buffers and every sampled
token comes back each iteration; the byte counts are the engine's). The
latencies are per request in the timed window, from submission: p50 TTFT is
queueing + prefill under saturation; p50 TPOT is the inter-token time.

``--impl reference`` runs the unmodified reference (installed under
baseline/_ref) on the same pool through its own ``LLM`` class; see
baseline/run_reference.py. ``--shape qwen3-0.6b`` selects the reference's
offline-benchmark shape (prompts and outputs uniform in [100, 1024]).

``--shape kimi-k2`` serves the Kimi-K2-shape MLA + MoE decoder (61 layers,
384 routed experts top-8 with MXFP4 weights, a bf16 shared expert) with
attention data-parallel and the routed experts split over the N ranks
(EP = N, tokens dispatched to their experts' ranks): 512 requests, prompts
uniform in [512, 4096], outputs uniform in [128, 1024]. Each rank serves its
own requests; a step is ``--step-tokens`` output tokens summed over the
ranks (the count is all-reduced every lockstep iteration, so all ranks cut
the run at the same iteration). The full shape needs 8 GPUs (about 67 GB of
MXFP4 experts and 23 GB of replicated bf16 weights per rank); ``--layers``
runs a slice on fewer. The reference has no MLA, expert parallelism, DP
attention or MXFP4, so its arm reports itself unavailable for this shape.

``--shape kimi-k2-cp`` is the long-context config: an 8-layer slice of the
Kimi-K2 shape (MXFP4 experts) with context parallelism over the N ranks
(CP = EP = N: prefill tokens sharded, KV pages spread over the ranks) on a
batch of 4 requests of 131072 prompt tokens, then 256 greedy output tokens
each (``--prompt-len`` / ``--num-reqs`` scale it down). A step is one whole
batch; the line reports output tok/s over the device time of the K timed
batches, with the prefill part (until every request has its first token)
and the decode part beside it.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import time
from typing import Dict, List, Optional, Tuple

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "output tok/s (whole box, device-timed, max over ranks)"
MODEL_NAMES = {"qwen3-32b": "Qwen3-32B-shape", "qwen3-0.6b": "Qwen3-0.6B-shape", "qwen3-8b": "Qwen3-8B-shape",
               "kimi-k2": "Kimi-K2-shape", "kimi-k2-cp": "Kimi-K2-shape 8-layer slice"}
PAGE_SIZE = 64


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["minisgl", "reference"], default="minisgl")
    p.add_argument("--shape", default="qwen3-32b")
    p.add_argument("--layers", type=int, default=None, help="kimi-k2: decoder layers (default: all 61)")
    p.add_argument("--moe-quant", default="mxfp4", choices=["mxfp4", "mxfp4-a8", "none"],
                   help="kimi-k2: routed expert weights")
    p.add_argument("--num-reqs", type=int, default=None,
                   help="request pool (default 1000; kimi-k2: 512; kimi-k2-cp: 4 per batch)")
    p.add_argument("--prompt-len", type=int, default=131072, help="kimi-k2-cp: prompt tokens per request")
    p.add_argument("--output-len", type=int, default=256, help="kimi-k2-cp: output tokens per request")
    p.add_argument("--step-tokens", type=int, default=8192)
    p.add_argument("--temperature", type=float, default=0.6)
    p.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--json-out", default="")
    args = p.parse_args(argv)
    if args.num_reqs is None:
        args.num_reqs = {"kimi-k2": 512, "kimi-k2-cp": 4}.get(args.shape, 1000)
    return args


def dist_env() -> Tuple[int, int, int]:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ------------------------------------------------------------------ workload
def _workload():
    """minisgl/benchmark/workload.py, loaded by path: the reference arm's
    process imports this file while its ``minisgl`` is the reference's."""
    import importlib.util

    mod = sys.modules.get("_minisgl_bench_workload")
    if mod is None:
        spec = importlib.util.spec_from_file_location(
            "_minisgl_bench_workload", os.path.join(ROOT, "minisgl", "benchmark", "workload.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules["_minisgl_bench_workload"] = mod
    return mod


def make_pool(shape: str, num_reqs: int, seed: int, vocab_limit: int = 10000) -> Tuple[List[List[int]], List[int]]:
    """The request pool (same on every rank and in both arms): prompt token
    ids and output lengths (minisgl.benchmark.workload)."""
    return _workload().make_pool(shape, num_reqs, seed, vocab_limit)


class StopRun(Exception):
    """Raised from the result hook once the last timed step has ended."""


class StepMeter:
    """Cuts a continuous serving run into steps of ``step_tokens`` output
    tokens. ``on_reply`` is called with each iteration's replies (from the
    engine's offline result hook); at every boundary it records a CUDA event
    on the engine stream and the host clock."""

    def __init__(self, stream, step_tokens: int, warmup: int, steps: int, counters=None, group=None) -> None:
        import torch

        self.torch = torch
        self.group = group  # DP attention: count output tokens over all ranks (lockstep iterations)
        self.stream = stream
        self.step_tokens = step_tokens
        self.warmup, self.steps = warmup, steps
        self.counters = counters  # callable -> (h2d bytes, d2h bytes) so far, or None
        self.tokens = 0
        self.marks: List[Tuple[object, int, float, Tuple[int, int]]] = []
        self.t_submit = time.perf_counter()
        self.first: Dict[int, float] = {}
        self.last: Dict[int, float] = {}
        self.count: Dict[int, int] = {}
        self._mark()

    def _mark(self) -> None:
        ev = self.torch.cuda.Event(enable_timing=True)
        ev.record(self.stream)
        self.marks.append((ev, self.tokens, time.perf_counter(), self.counters() if self.counters else (0, 0)))

    def on_reply(self, replies) -> None:
        now = time.perf_counter()
        if self.group is not None:
            import torch.distributed as dist

            n = self.torch.tensor([len(replies)], dtype=self.torch.int64)
            dist.all_reduce(n, group=self.group)
            self.tokens += int(n) - len(replies)  # the other ranks' tokens; this rank's follow
        for m in replies:
            self.tokens += 1
            uid = m.uid
            if uid not in self.first:
                self.first[uid] = now
                self.count[uid] = 0
            self.last[uid] = now
            self.count[uid] += 1
        while self.tokens >= len(self.marks) * self.step_tokens and len(self.marks) <= self.warmup + self.steps:
            self._mark()
        if len(self.marks) > self.warmup + self.steps:
            raise StopRun()

    def result(self) -> Dict[str, float]:
        self.torch.cuda.synchronize()
        a, b = self.marks[self.warmup], self.marks[self.warmup + self.steps]
        t0, t1 = a[2], b[2]
        ttft = [self.first[u] - self.t_submit for u in self.first if t0 <= self.first[u] <= t1]
        tpot = [(self.last[u] - self.first[u]) / (self.count[u] - 1) for u in self.first
                if self.count[u] > 1 and t0 <= self.last[u] <= t1]
        return {"dev_ms": a[0].elapsed_time(b[0]), "wall_s": t1 - t0, "tokens": b[1] - a[1],
                "h2d": b[3][0] - a[3][0], "d2h": b[3][1] - a[3][1],
                "ttft_p50_ms": 1000 * statistics.median(ttft) if ttft else None,
                "tpot_p50_ms": 1000 * statistics.median(tpot) if tpot else None}


def metered_llm_class(base):
    """A subclass of an offline ``LLM`` class (ours or the reference's) whose
    per-iteration result hook feeds a StepMeter; everything else is the
    class's own code path."""

    class Metered(base):
        meter: Optional[StepMeter] = None
        h2d_counted = 0  # int32 prompt ids handed to the engine
        d2h_counted = 0  # int32 sampled tokens handed back

        def offline_receive_msg(self, blocking: bool = False):
            msgs = super().offline_receive_msg(blocking)
            for m in msgs:
                ids = getattr(m, "input_ids", None)
                if ids is not None:
                    self.h2d_counted += 4 * len(ids)
            return msgs

        def offline_send_result(self, reply):
            super().offline_send_result(reply)
            self.d2h_counted += 4 * len(reply)
            if self.meter is not None:
                self.meter.on_reply(reply)

    return Metered


def run_metered(llm, prompts, outs, temperature, stream, args, sampling_params_cls,
                counters=None, group=None) -> Dict[str, float]:
    """Serve the pool until W + K steps have passed; returns the meter's result."""
    params = [sampling_params_cls(temperature=temperature, ignore_eos=True, max_tokens=o) for o in outs]
    llm.meter = StepMeter(stream, args.step_tokens, args.warmup, args.steps, counters, group)
    try:
        llm.generate(prompts, params)
    except StopRun:
        pass
    meter, llm.meter = llm.meter, None
    if len(meter.marks) <= args.warmup + args.steps:
        raise RuntimeError(f"request pool exhausted after {len(meter.marks) - 1} steps; "
                           f"raise --num-reqs or lower --step-tokens")
    return meter.result()


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices: List[int]) -> None:
        self.gpus = set(gpu_indices)
        self.proc: Optional[subprocess.Popen] = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> Dict[str, object]:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        clocks, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                continue
            try:
                clk, mx, pw = float(parts[1]), float(parts[2]), float(parts[3])
            except ValueError:
                continue
            maxes.append(mx)
            if pw > 200:  # under load
                clocks.append(clk)
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(clocks) if clocks else None,
                "sm_max_mhz": max(maxes) if maxes else None, "reasons": sorted(reasons),
                "samples_under_load": len(clocks)}


def reduce_over_ranks(vals: List[float], op: str) -> List[float]:
    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        return vals
    t = torch.tensor([float(v) for v in vals], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.tolist()


def config_of(args, world: int) -> Dict[str, object]:
    cfg = {"model": MODEL_NAMES.get(args.shape, args.shape), "global_batch": 256, "parallelism": f"tp{world}",
           "requests": args.num_reqs, "step_tokens": args.step_tokens, "page_size": PAGE_SIZE,
           "temperature": args.temperature,
           "l2": "inputs larger than L2 (tens of GB of weights and KV cache streamed per step)"}
    if args.shape == "qwen3-0.6b":
        cfg["seq_len"] = "prompt U[100,1024] + output U[100,1024]"
    elif args.shape == "kimi-k2-cp":
        cfg.update(seq_len=f"{args.num_reqs} x {args.prompt_len} prompt tokens + {args.output_len} greedy outputs",
                   model=f"Kimi-K2-shape {args.layers or 8}-layer slice", global_batch=args.num_reqs,
                   parallelism=f"cp{world}+ep{world}", routed_experts=f"384 top-8, {args.moe_quant}",
                   step="one whole batch of fresh prompts", temperature=0.0)
        cfg.pop("step_tokens")
    elif args.shape == "kimi-k2":
        cfg.update(seq_len="prompt U[512,4096] + output U[128,1024]", global_batch=args.num_reqs,
                   parallelism=f"dp-attention{world}+ep{world}" if world > 1 else "single GPU",
                   layers=args.layers or 61, routed_experts=f"384 top-8, {args.moe_quant}",
                   latency_note="TTFT / TPOT of rank 0's requests")
    else:
        cfg["seq_len"] = ("prompt lognormal(median 1024) in [32,16384] + output lognormal(median 256) in [16,2048]; "
                          "30% share one of 50 prefixes of 512-2048 tokens")
    return cfg


def emit(line: Dict[str, object], args) -> None:
    print(json.dumps(line), flush=True)
    if args.json_out:
        with open(args.json_out, "w") as f:
            json.dump(line, f)


# ------------------------------------------------------------------ our arm
def run_minisgl(args) -> None:
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    sys.path.insert(0, ROOT)
    from minisgl import ops
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo
    from minisgl.utils.synthetic import make_model_dir

    if world > 1:  # the engine joins this group (NCCL for tensors, gloo for the host side)
        dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    prompts, outs = make_pool(args.shape, args.num_reqs, args.seed)
    moe = args.shape == "kimi-k2"
    if moe:  # attention data-parallel, routed experts split over the ranks (EP = N), MXFP4 experts
        overrides = {"num_hidden_layers": args.layers} if args.layers else None
        model_dir = make_model_dir(args.shape, overrides=overrides)
        # 2048-token prefill chunks: the DP token dispatch sizes its peer slots
        # and expert buffers for chunk x top-k pairs from every rank (about
        # 6 GB per rank at 2048; 25 GB at 8192), held beside the KV cache
        extra = dict(enable_dp_attention=world > 1, moe_quant=args.moe_quant, max_seq_len_override=5120,
                     max_extend_tokens=2048, memory_ratio=0.85)
    else:
        model_dir = make_model_dir(args.shape)
        extra = dict(max_seq_len_override=20480, max_extend_tokens=16384)
    llm = metered_llm_class(LLM)(
        model_dir, dtype=torch.bfloat16, use_dummy_weight=True, device=f"cuda:{local}",
        tp_info=DistributedInfo(rank, world), comm=args.comm, cuda_graph_max_bs=256, max_running_req=256,
        page_size=PAGE_SIZE, **extra)
    dp_group = llm.tp_cpu_group if moe and world > 1 else None
    launches0 = ops.LAUNCHES[0]
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler is not None:
        sampler.start()
    res = run_metered(llm, prompts, outs, args.temperature, llm.engine.stream, args, SamplingParams,
                      counters=lambda: (llm.h2d_bytes, llm.d2h_bytes), group=dp_group)
    clocks = sampler.stop() if sampler is not None else {}
    launches = ops.LAUNCHES[0] - launches0
    if getattr(llm, "profiler", None) is not None and rank == 0:  # MINISGL_PROFILE_STEPS=1: time per phase
        print(json.dumps({"step_profile": llm.profiler.summary()}), file=sys.stderr, flush=True)
    max_dev_ms, max_wall = reduce_over_ranks([res["dev_ms"], res["wall_s"]], "max")
    tot_launches, = reduce_over_ranks([launches], "sum")
    if dp_group is not None:  # each rank moved its own requests' bytes
        res["h2d"], res["d2h"] = reduce_over_ranks([res["h2d"], res["d2h"]], "sum")
    if rank == 0:
        # tensor parallel: every rank serves the same requests; DP attention:
        # the meter already summed the ranks' tokens
        tokens = res["tokens"]
        value = tokens / (max_dev_ms / 1000.0)
        emit({
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(max_dev_ms / args.steps, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if not moe else f"bf16 (routed experts {args.moe_quant})",
            "data": "synthetic (random token ids, random-init N(0,0.02) weights)",
            "config": dict(config_of(args, world), comm=args.comm),
            "clocks": clocks,
            "e2e": {"value": round(tokens / max_wall, 1), "unit": "tok/s (LLM.generate wall clock)",
                    "h2d_bytes_per_step": int(res["h2d"] / args.steps),
                    "d2h_bytes_per_step": int(res["d2h"] / args.steps)},
            "latency": {"ttft_p50_ms": res["ttft_p50_ms"], "tpot_p50_ms": res["tpot_p50_ms"],
                        "note": "saturated run, all requests submitted at t=0"},
            "gpu_launches": int(tot_launches), "impl": "minisgl",
        }, args)
    llm.shutdown()
    if world > 1 and dist.is_initialized():
        dist.destroy_process_group()


def run_minisgl_cp(args) -> None:
    """The long-context context-parallel config: W untimed and K timed
    batches of ``num_reqs`` fresh random prompts of ``prompt_len`` tokens
    (fresh, so the prefix cache serves none of them), ``output_len`` greedy
    tokens each, on an 8-layer Kimi-K2-shape slice with CP = EP = N. Every
    rank serves the whole batch (token-sharded prefill, replicated decode),
    so the device times are taken per rank and the max is reported."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    sys.path.insert(0, ROOT)
    from minisgl import ops
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo
    from minisgl.utils.synthetic import make_model_dir

    if world > 1:
        dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=900),
                                device_id=torch.device(f"cuda:{local}"))
    n, L, out_len = args.num_reqs, args.prompt_len, args.output_len
    model_dir = make_model_dir("kimi-k2", overrides={"num_hidden_layers": args.layers or 8})
    llm = metered_llm_class(LLM)(
        model_dir, dtype=torch.bfloat16, use_dummy_weight=True, device=f"cuda:{local}",
        tp_info=DistributedInfo(rank, world), cp_size=world, ep_size=world, moe_quant=args.moe_quant,
        comm=args.comm, page_size=PAGE_SIZE, max_running_req=max(8, n), cuda_graph_max_bs=max(8, n),
        max_seq_len_override=L + out_len + PAGE_SIZE, max_extend_tokens=16384)
    stream = llm.engine.stream

    def event():
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        return ev

    class BatchMeter:
        """Events at the start, once every request has its first token, and
        at the end of one batch."""

        def __init__(self) -> None:
            self.first: set = set()
            self.tokens = 0
            self.start, self.prefilled = event(), None

        def on_reply(self, replies) -> None:
            for m in replies:
                self.tokens += 1
                self.first.add(m.uid)
            if self.prefilled is None and len(self.first) == n:
                self.prefilled = event()

    launches0 = ops.LAUNCHES[0]
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    timed = {"total": 0.0, "prefill": 0.0, "decode": 0.0, "wall": 0.0, "tokens": 0, "h2d": 0, "d2h": 0}
    params = SamplingParams(temperature=0.0, ignore_eos=True, max_tokens=out_len)
    for b in range(args.warmup + args.steps):
        rng = random.Random(args.seed * 7919 + b)
        prompts = [[rng.randrange(10000) for _ in range(L)] for _ in range(n)]
        if b == args.warmup:
            launches0 = ops.LAUNCHES[0]
            if sampler is not None:
                sampler.start()
        h2d0, d2h0 = llm.h2d_bytes, llm.d2h_bytes
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        llm.meter = m = BatchMeter()
        llm.generate(prompts, params)
        end = event()
        end.synchronize()
        wall = time.perf_counter() - t0
        llm.meter = None
        if b >= args.warmup:
            timed["total"] += m.start.elapsed_time(end)
            timed["prefill"] += m.start.elapsed_time(m.prefilled)
            timed["decode"] += m.prefilled.elapsed_time(end)
            timed["wall"] += wall
            timed["tokens"] += m.tokens
            timed["h2d"] += llm.h2d_bytes - h2d0
            timed["d2h"] += llm.d2h_bytes - d2h0
    clocks = sampler.stop() if sampler is not None else {}
    launches = ops.LAUNCHES[0] - launches0
    tot, pre, dec, wall = reduce_over_ranks([timed["total"], timed["prefill"], timed["decode"], timed["wall"]], "max")
    tot_launches, = reduce_over_ranks([launches], "sum")
    if rank == 0:
        K, tokens = args.steps, timed["tokens"]  # every rank serves the same batch
        emit({
            "metric": METRIC, "value": round(tokens / (tot / 1000.0), 1), "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": round(tot / K, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"bf16 (routed experts {args.moe_quant})",
            "data": "synthetic (random token ids, random-init N(0,0.02) weights)",
            "config": dict(config_of(args, world), comm=args.comm),
            "clocks": clocks,
            "phases": {"prefill_ms_per_batch": round(pre / K, 2), "decode_ms_per_batch": round(dec / K, 2),
                       "prefill_tok_s": round(n * L * K / (pre / 1000.0), 1),
                       "decode_tpot_ms": round(dec / K / max(1, out_len - 1), 3),
                       "note": "prefill: until every request has its first token (max over ranks)"},
            "e2e": {"value": round(tokens / wall, 1), "unit": "tok/s (LLM.generate wall clock)",
                    "h2d_bytes_per_step": int(timed["h2d"] / K), "d2h_bytes_per_step": int(timed["d2h"] / K)},
            "gpu_launches": int(tot_launches), "impl": "minisgl",
        }, args)
    llm.shutdown()
    if world > 1 and dist.is_initialized():
        dist.destroy_process_group()


# ------------------------------------------------------------ reference arm
def run_reference(args) -> None:
    """Run the unmodified reference (baseline/_ref) on the same pool: one
    subprocess per rank whose import path holds only the reference package."""
    rank, world, local = dist_env()
    if args.shape in ("kimi-k2", "kimi-k2-cp"):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no MLA / DeepSeek-V3 "
                              "architecture, expert parallelism, DP attention or MXFP4 experts"}))
        return
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "minisgl")):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return
    import torch.distributed as dist

    if world > 1:
        dist.init_process_group("gloo")
    sys.path.insert(0, ROOT)
    from minisgl.utils.synthetic import make_model_dir

    model_dir = make_model_dir(args.shape)
    # the reference sets up its own process group: drop torchrun's rendezvous
    # variables (TORCHELASTIC_USE_AGENT_STORE would make its rank 0 a client)
    launcher = ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT", "LOCAL_WORLD_SIZE", "GROUP_RANK",
                "ROLE_RANK", "ROLE_NAME", "GROUP_WORLD_SIZE", "ROLE_WORLD_SIZE", "OMP_NUM_THREADS")
    env = {k: v for k, v in os.environ.items() if k not in launcher and not k.startswith("TORCHELASTIC_")}
    port = 29700 + (int(os.environ.get("MASTER_PORT", "29500")) % 97) * 3
    cmd = [sys.executable, os.path.join(ROOT, "baseline", "run_reference.py"), "--rank", str(rank),
           "--world", str(world), "--port", str(port), "--model-dir", model_dir] + \
          [f"--{k.replace('_', '-')}={v}" for k, v in vars(args).items()
           if k in ("steps", "warmup", "shape", "num_reqs", "step_tokens", "temperature", "seed")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=3000)
    result = None
    for line in proc.stdout.splitlines():
        if line.startswith("{") and "ref_result" in line:
            result = json.loads(line)
    (all_ok,) = reduce_over_ranks([1.0 if result is not None else 0.0], "sum")
    if all_ok < world:
        if rank == 0:
            tail = (proc.stderr or proc.stdout).strip().splitlines()[-3:]
            print(json.dumps({"impl": "reference", "unavailable": "reference run failed: " + " | ".join(tail)[:400]}))
        if world > 1:
            dist.destroy_process_group()
        return
    max_dev_ms, max_wall = reduce_over_ranks([result["dev_ms"], result["wall_s"]], "max")
    if rank == 0:
        tokens = result["tokens"]
        cfg = dict(config_of(args, world), page_size=result.get("page_size"),
                   attention_backend=result.get("attn"))
        emit({
            "metric": METRIC, "value": round(tokens / (max_dev_ms / 1000.0), 1), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(max_dev_ms / args.steps, 2), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random token ids, reference --dummy-weight)",
            "config": cfg,
            "e2e": {"value": round(tokens / max_wall, 1), "unit": "tok/s (LLM.generate wall clock)",
                    "h2d_bytes_per_step": int(result["h2d"] / args.steps),
                    "d2h_bytes_per_step": int(result["d2h"] / args.steps),
                    "bytes": "int32 prompt ids admitted + int32 sampled tokens, counted from the requests"},
            "latency": {"ttft_p50_ms": result["ttft_p50_ms"], "tpot_p50_ms": result["tpot_p50_ms"],
                        "note": "saturated run, all requests submitted at t=0"},
            "impl": "reference",
        }, args)
    if world > 1:
        dist.destroy_process_group()


def main(argv=None) -> None:
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.shape == "kimi-k2-cp":
        run_minisgl_cp(args)
    else:
        run_minisgl(args)


if __name__ == "__main__":
    main()
