"""Run the unmodified reference engine (installed in baseline/_ref) on the
bench.py workload and print one JSON result line.

Only the reference's public offline API is used (``minisgl.llm.LLM`` and
``SamplingParams`` of the reference package) with the settings of the
reference's own offline benchmark (benchmark/offline/bench.py: page 256,
max_extend_tokens 16384, CUDA graphs up to batch 256, seq len 4096). The one
setting changed from outside is the TCP port of its single-rank gloo
rendezvous, so that several replicas can start on one machine.
"""

import argparse
import importlib.util
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")
sys.path = [REF] + [p for p in sys.path if os.path.abspath(p or ".") not in (ROOT, HERE)]


def _load_bench():
    spec = importlib.util.spec_from_file_location("_bench_workload", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--rank", type=int, default=0)
    p.add_argument("--port", type=int, default=29700)
    p.add_argument("--model-dir", required=True)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--shape", default="qwen3-0.6b")
    p.add_argument("--num-reqs", type=int, default=256)
    p.add_argument("--min-len", type=int, default=100)
    p.add_argument("--max-input", type=int, default=1024)
    p.add_argument("--max-output", type=int, default=1024)
    p.add_argument("--temperature", type=float, default=0.6)
    p.add_argument("--seed", type=int, default=0)
    args = p.parse_args()
    bench = _load_bench()

    import minisgl  # the reference package from baseline/_ref

    where = os.path.abspath(list(minisgl.__path__)[0])
    assert where.startswith(REF), where
    import minisgl.engine.config as ref_cfg
    import torch
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM

    ref_cfg.EngineConfig.distributed_addr = property(lambda self: f"tcp://127.0.0.1:{args.port}")
    llm = LLM(args.model_dir, use_dummy_weight=True, max_seq_len_override=4096, max_extend_tokens=16384,
              cuda_graph_max_bs=256, page_size=256)
    llm.generate(["Benchmark: "], SamplingParams(temperature=0.1))

    def step(i):
        prompts, outs = bench.make_workload(args, i, args.rank)
        params = [SamplingParams(temperature=args.temperature, ignore_eos=True, max_tokens=o) for o in outs]
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        t0 = time.perf_counter()
        llm.generate(prompts, params)
        wall = time.perf_counter() - t0
        torch.cuda.synchronize()
        end.record()
        end.synchronize()
        return start.elapsed_time(end), wall, sum(outs)

    for i in range(args.warmup):
        step(i)
    res = [step(args.warmup + k) for k in range(args.steps)]
    print(json.dumps({"ref_result": True, "dev_ms": sum(r[0] for r in res), "wall_s": sum(r[1] for r in res),
                      "tokens": sum(r[2] for r in res), "attn": llm.engine.attn_backend.__class__.__name__}),
          flush=True)
    os._exit(0)  # the reference's scheduler holds process groups / graphs; skip teardown


if __name__ == "__main__":
    main()
