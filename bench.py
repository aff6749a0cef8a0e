"""Offline serving throughput benchmark (the reference's headline workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl minisgl|reference]

Workload (the reference's benchmark/offline/bench.py):
Qwen3-0.6B-shape decoder with random bf16 weights, 256 requests per GPU,
prompt lengths U[100, 1024] of random token ids, output lengths U[100, 1024],
temperature 0.6, ignore_eos. One *step* is one ``LLM.generate`` call over a
fresh set of 256 requests (new prompts every step, so the prefix cache never
serves a previous step). For N > 1 (launched by torchrun) every GPU runs its
own engine on its own requests: data-parallel replicas, weak scaling.

Reported ``value``: output tokens of all ranks / max-over-ranks device time
(CUDA events around each generate call, synchronised on both sides).
``e2e``: the same through the public API with host wall-clock time (includes
tokenised inputs going host->device and every sampled token coming back).
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
from typing import Dict, List, Optional

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "output tok/s (whole box, device-timed, max over ranks)"
MODEL_NAME = "Qwen3-0.6B-shape"


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["minisgl", "reference"], default="minisgl")
    p.add_argument("--shape", default="qwen3-0.6b")
    p.add_argument("--num-reqs", type=int, default=256)
    p.add_argument("--min-len", type=int, default=100)
    p.add_argument("--max-input", type=int, default=1024)
    p.add_argument("--max-output", type=int, default=1024)
    p.add_argument("--temperature", type=float, default=0.6)
    p.add_argument("--page-size", type=int, default=64)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--json-out", default="")
    return p.parse_args(argv)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def make_workload(args, step: int, rank: int, vocab_limit: int = 10000):
    """Fresh prompts every step (token ids in [0, 10000) like the reference)."""
    rng = random.Random(args.seed * 1_000_003 + rank * 10_007 + step)
    prompts = [[rng.randint(0, vocab_limit - 1) for _ in range(rng.randint(args.min_len, args.max_input))]
               for _ in range(args.num_reqs)]
    outs = [rng.randint(args.min_len, args.max_output) for _ in range(args.num_reqs)]
    return prompts, outs


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


def allreduce(vals: List[float], op: str) -> List[float]:
    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        return vals
    t = torch.tensor(vals, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.tolist()


def run_minisgl(args) -> None:
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    if world > 1:
        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)
    sys.path.insert(0, ROOT)
    from minisgl import ops
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.utils.synthetic import make_model_dir

    model_dir = make_model_dir(args.shape)
    llm = LLM(model_dir, dtype=torch.bfloat16, use_dummy_weight=True, device=f"cuda:{local}",
              max_seq_len_override=4096, max_extend_tokens=16384, cuda_graph_max_bs=256,
              max_running_req=256, page_size=args.page_size)
    engine_stream = llm.engine.stream

    def one_step(step: int):
        prompts, outs = make_workload(args, step, rank)
        params = [SamplingParams(temperature=args.temperature, ignore_eos=True, max_tokens=o) for o in outs]
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h2d0, d2h0 = llm.h2d_bytes, llm.d2h_bytes
        launches0 = ops.LAUNCHES[0]
        start.record(engine_stream)
        t0 = time.perf_counter()
        res = llm.generate(prompts, params)
        t_api = time.perf_counter() - t0
        torch.cuda.synchronize()
        end.record(engine_stream)
        end.synchronize()
        dev_ms = start.elapsed_time(end)
        got = sum(len(r["token_ids"]) for r in res)
        assert got == sum(outs), f"generated {got} tokens, expected {sum(outs)}"
        prompt_bytes = 4 * sum(len(p) for p in prompts)
        return dict(dev_ms=dev_ms, wall_s=t_api, tokens=sum(outs), h2d=llm.h2d_bytes - h2d0 + prompt_bytes,
                    d2h=llm.d2h_bytes - d2h0, launches=ops.LAUNCHES[0] - launches0)

    for w in range(args.warmup):
        one_step(w)
    sampler = ClockSampler([local]) if local == 0 else None
    gpu_ids = list(range(world))
    if sampler is not None:
        sampler.gpus = set(gpu_ids)
        sampler.start()
    stats = [one_step(args.warmup + k) for k in range(args.steps)]
    clocks = sampler.stop() if sampler is not None else {}
    dev_ms = sum(s["dev_ms"] for s in stats)
    wall_s = sum(s["wall_s"] for s in stats)
    tokens = sum(s["tokens"] for s in stats)
    h2d = sum(s["h2d"] for s in stats) / args.steps
    d2h = sum(s["d2h"] for s in stats) / args.steps
    launches = sum(s["launches"] for s in stats)
    max_dev_ms, max_wall = allreduce([dev_ms, wall_s], "max")
    tot_tokens, tot_h2d, tot_d2h, tot_launches = allreduce([tokens, h2d, d2h, launches], "sum")
    if rank == 0:
        value = tot_tokens / (max_dev_ms / 1000.0)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(max_dev_ms / args.steps, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random token ids, random-init N(0,0.02) weights)",
            "config": {"model": MODEL_NAME, "global_batch": args.num_reqs * world,
                       "seq_len": f"prompt U[{args.min_len},{args.max_input}] + output U[{args.min_len},{args.max_output}]",
                       "parallelism": f"dp{world}" if world > 1 else "tp1", "page_size": args.page_size,
                       "temperature": args.temperature, "requests_per_gpu": args.num_reqs,
                       "l2": "inputs larger than L2 (multi-GB KV cache and 1.2 GB of weights per step)"},
            "clocks": clocks,
            "e2e": {"value": round(tot_tokens / max_wall, 1), "unit": "tok/s (LLM.generate wall clock)",
                    "h2d_bytes_per_step": int(tot_h2d), "d2h_bytes_per_step": int(tot_d2h)},
            "gpu_launches": int(tot_launches),
            "impl": "minisgl",
        }
        print(json.dumps(line), flush=True)
        if args.json_out:
            with open(args.json_out, "w") as f:
                json.dump(line, f)
    llm.shutdown()
    if world > 1:
        dist.destroy_process_group()


def run_reference(args) -> None:
    """Run the unmodified reference (baseline/_ref) on the same workload."""
    rank, world, local = dist_env()
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "minisgl")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return
    import torch.distributed as dist

    if world > 1:
        dist.init_process_group("gloo")
    sys.path.insert(0, ROOT)
    from minisgl.utils.synthetic import make_model_dir

    model_dir = make_model_dir(args.shape)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(local) if "CUDA_VISIBLE_DEVICES" not in os.environ
               else os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT", "LOCAL_WORLD_SIZE",
              "GROUP_RANK", "ROLE_RANK", "TORCHELASTIC_RUN_ID"):
        env.pop(k, None)
    cmd = [sys.executable, os.path.join(ROOT, "baseline", "run_reference.py"), "--rank", str(rank),
           "--port", str(29700 + local), "--model-dir", model_dir] + [f"--{k.replace('_', '-')}={v}" for k, v in vars(args).items()
                                             if k in ("steps", "warmup", "shape", "num_reqs", "min_len", "max_input",
                                                      "max_output", "temperature", "seed")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=3000)
    result = None
    for line in proc.stdout.splitlines():
        if line.startswith("{") and "ref_result" in line:
            result = json.loads(line)
    ok = 1.0 if result is not None else 0.0
    (all_ok,) = allreduce([ok], "sum")
    if all_ok < world:
        if rank == 0:
            tail = (proc.stderr or proc.stdout).strip().splitlines()[-3:]
            print(json.dumps({"impl": "reference", "unavailable": "reference run failed: " + " | ".join(tail)[:400]}))
        return
    max_dev_ms, max_wall = allreduce([result["dev_ms"], result["wall_s"]], "max")
    (tot_tokens,) = allreduce([result["tokens"]], "sum")
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(tot_tokens / (max_dev_ms / 1000.0), 1), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(max_dev_ms / args.steps, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random token ids, reference --dummy-weight)",
            "config": {"model": MODEL_NAME, "global_batch": args.num_reqs * world,
                       "parallelism": f"dp{world}" if world > 1 else "tp1", "page_size": 256,
                       "attention_backend": result.get("attn"), "l2": "inputs larger than L2"},
            "e2e": {"value": round(tot_tokens / max_wall, 1), "unit": "tok/s (LLM.generate wall clock)"},
            "impl": "reference",
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main(argv=None) -> None:
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_minisgl(args)


if __name__ == "__main__":
    main()
