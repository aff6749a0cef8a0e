"""Kimi-K2-shape slice on one GPU: MLA attention, MXFP4 routed experts and
the shared expert at the real dimensions, through the offline API.

    python -m minisgl.benchmark.kimi_slice [--layers 4] [--experts 48] [--reqs 64]

The model is the Kimi-K2 shape (hidden 7168, 64 heads, q_lora 1536,
kv_lora 512, rope 64, expert intermediate 2048, top-8 sigmoid routing with
a shared expert, vocab 163840) cut to ``--layers`` layers (layer 0 dense)
and to ``--experts`` routed experts — 48 is one rank's share of 384 under
8-way expert parallelism — with random N(0, 0.02) weights quantised to
MXFP4. ``--reqs`` requests with prompts U[512, 1024] and outputs U[64, 128]
run through ``LLM.generate``; the step is timed on the device (CUDA events
on the engine stream) after one warm-up batch. One JSON line: output tokens
per second of the slice, its per-decode-token time, and the prefill / decode
split.
"""

from __future__ import annotations

import argparse
import json
import random
import time

import torch


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--layers", type=int, default=4)
    p.add_argument("--experts", type=int, default=48)
    p.add_argument("--reqs", type=int, default=64)
    p.add_argument("--quant", default="mxfp4", choices=["mxfp4", "mxfp4-a8", "none"])
    args = p.parse_args()
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.utils.synthetic import make_model_dir

    d = make_model_dir("kimi-k2", overrides=dict(num_hidden_layers=args.layers, n_routed_experts=args.experts))
    llm = LLM(d, dtype=torch.bfloat16, device="cuda:0", use_dummy_weight=True, page_size=64,
              max_running_req=max(64, args.reqs), max_seq_len_override=2048, max_extend_tokens=8192,
              cuda_graph_max_bs=max(64, args.reqs), moe_quant=args.quant, num_page_override=4096)
    stream = llm.engine.stream

    def batch(seed: int):
        g = random.Random(seed)
        prompts = [[g.randrange(163840) for _ in range(g.randint(512, 1024))] for _ in range(args.reqs)]
        outs = [g.randint(64, 128) for _ in range(args.reqs)]
        return prompts, [SamplingParams(temperature=0.0, max_tokens=o, ignore_eos=True) for o in outs], outs

    def run(seed: int):
        prompts, params, outs = batch(seed)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        t0 = time.perf_counter()
        res = llm.generate(prompts, params)
        wall = time.perf_counter() - t0
        b.record(stream)
        b.synchronize()
        assert sum(len(r["token_ids"]) for r in res) == sum(outs)
        return a.elapsed_time(b), wall, sum(outs), sum(len(x) for x in prompts)

    run(0)  # warm-up (tuning and graph paths)
    ms, wall, out_tokens, prompt_tokens = run(1)
    print(json.dumps({"bench": "kimi_k2_slice", "layers": args.layers, "routed_experts": args.experts,
                      "quant": args.quant, "requests": args.reqs, "prompt_tokens": prompt_tokens,
                      "output_tokens": out_tokens, "device_ms": round(ms, 1), "wall_s": round(wall, 3),
                      "output_tok_per_s": round(out_tokens / (ms / 1000.0), 1)}), flush=True)
    llm.shutdown()


if __name__ == "__main__":
    main()
