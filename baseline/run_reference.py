"""Run the unmodified reference engine (installed in baseline/_ref) on the
bench.py request pool and print one JSON result line (one process per rank).

Only the reference's own offline code path is used: its ``LLM`` class (the
offline scheduler loop, its ``generate`` and result hooks), ``SamplingParams``
and, under it, its engine (pynccl collectives, flashinfer / TRT-LLM attention,
cuBLAS GEMMs, CUDA-graph decode). Settings are those of the reference's own
offline benchmark (benchmark/offline/bench.py: max_extend_tokens 16384, CUDA
graphs up to batch 256, ``--dummy-weight``) with the bench's page size (64,
the size the reference itself picks on sm100) and sequence-length cap.

Two things are set from outside, because the reference's ``LLM`` is built for
one rank (python/minisgl/llm/llm.py:28-39 fixes ``DistributedInfo(0, 1)``):

* the TCP port of its gloo rendezvous (a property on its ``EngineConfig``);
* for tensor parallelism over N ranks, the ``LLM`` subclass below builds the
  same ``SchedulerConfig`` with ``tp_info = DistributedInfo(rank, N)``; the
  offline hooks, scheduler and engine are the reference's code unchanged.
"""

import argparse
import importlib.util
import json
import os
import sys

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
    p.add_argument("--world", type=int, default=1)
    p.add_argument("--port", type=int, default=29700)
    p.add_argument("--model-dir", required=True)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--shape", default="qwen3-32b")
    p.add_argument("--num-reqs", type=int, default=1000)
    p.add_argument("--step-tokens", type=int, default=8192)
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
    from minisgl.distributed import DistributedInfo
    from minisgl.llm import LLM
    from minisgl.scheduler import Scheduler, SchedulerConfig

    ref_cfg.EngineConfig.distributed_addr = property(lambda self: f"tcp://127.0.0.1:{args.port}")

    class TensorParallelLLM(LLM):
        """The reference's offline LLM on rank ``rank`` of ``world``."""

        def __init__(self, model_path, dtype=torch.bfloat16, *, rank, world, **kwargs):
            config = SchedulerConfig(model_path=model_path, tp_info=DistributedInfo(rank, world), dtype=dtype,
                                     offline_mode=True, **kwargs)
            Scheduler.__init__(self, config)
            self.pending_requests, self.status_map, self.counter = [], {}, 0

    base = TensorParallelLLM if args.world > 1 else LLM
    extra = dict(rank=args.rank, world=args.world) if args.world > 1 else {}
    llm = bench.metered_llm_class(base)(args.model_dir, use_dummy_weight=True, max_seq_len_override=20480,
                                        max_extend_tokens=16384, cuda_graph_max_bs=256, max_running_req=256,
                                        page_size=bench.PAGE_SIZE, **extra)
    llm.generate([[1, 2, 3, 4]], SamplingParams(temperature=0.1, max_tokens=4))
    prompts, outs = bench.make_pool(args.shape, args.num_reqs, args.seed)
    res = bench.run_metered(llm, prompts, outs, args.temperature, llm.engine.stream, args, SamplingParams,
                            counters=lambda: (llm.h2d_counted, llm.d2h_counted))
    ctx = getattr(llm.engine, "ctx", None)
    page = getattr(ctx, "page_size", None) or getattr(llm.engine.config, "page_size", None)
    print(json.dumps(dict(res, ref_result=True, page_size=page,
                          attn=llm.engine.attn_backend.__class__.__name__)), flush=True)
    os._exit(0)  # the reference's scheduler holds process groups / graphs; skip teardown


if __name__ == "__main__":
    main()
