"""Row-parallel projection with its tensor-parallel all-reduce, per rank count.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m minisgl.benchmark.tp_comm [--layers 64]

For each decode batch size and each Qwen3-32B row-parallel shape (o_proj:
K = 8192 / N, down_proj: K = 25600 / N, output 5120) three paths are timed
on the device inside a CUDA graph with autotuned tile plans (rank 0's plans on
every rank, as the engine does), cycling over ``--layers`` weight copies
(weights stream from HBM), max over ranks:

* ``nccl``: tcgen05 GEMM, NCCL all-reduce, residual add (the baseline);
* ``fused``: one kernel (GEMM tiles exchanged over NVLink and summed with the
  residual in the epilogue; falls back to GEMM + collective kernel when the
  grid does not fit on the GPU);
* ``gemm_then_nvlink``: the tuned plain GEMM writing into the symmetric heap,
  then the NVLink all-reduce kernel with the residual add;
* ``sp_nccl``: the sequence-parallel step as library collectives: GEMM,
  NCCL all-reduce, fused residual add + RMSNorm (the reference's o_proj /
  down_proj followed by its next fused_add_rmsnorm);
* ``sp``: the same step on the token-sharded residual stream: the tuned
  GEMM into the symmetric heap, then one NVLink kernel that reduce-scatters
  into this rank's residual rows, RMS-normalises them and all-gathers the
  normalised rows (``SymmMemImpl.rs_norm_ag``); ``sp_frac_roofline`` is its
  fraction of the roofline below;
* ``roofline``: the slowest of the GEMM at the measured bf16 peak, the
  weight bytes at the measured HBM copy bandwidth, and the bytes an
  all-reduce must move per GPU over NVLink (2 (N - 1) / N of the output) at
  770 GB/s per direction; the fused path is reported as a fraction of it.

Rank 0 prints one JSON line per case.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

from minisgl import ops

LINK_GBS = 770.0  # measured peer copy bandwidth per direction per GPU on this pool


def _peaks():
    """(bf16 TFLOP/s, HBM GB/s) measured on this pool, else the fallback figures."""
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d.get("bf16_tflops", 1590.0)), float(d.get("hbm_gbs", 6650.0))
    except (OSError, ValueError):
        return 1590.0, 6650.0


def _time(fn, iters: int) -> float:
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=s):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b) / iters
    del g
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--batches", default="1,16,64,128,256")
    args = p.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from minisgl.parallel.symm import SymmMemImpl

    impl = SymmMemImpl(dev, (256 + world) * 5120 * 2)
    tflops, hbm = _peaks()
    H = 5120
    from minisgl.ops import gemm_tune

    batches = [int(b) for b in args.batches.split(",")]
    shapes = [(H, 64 * 128 // world), (H, 25600 // world)]
    gemm_tune.tune(shapes, batches, dev, fused={sh: (ops.EPI_RESIDUAL, 0, 0) for sh in shapes})
    tables = [dict(gemm_tune.PLANS), dict(gemm_tune.FUSED_PLANS)]
    dist.broadcast_object_list(tables, src=0)
    gemm_tune.PLANS.clear()
    gemm_tune.PLANS.update(tables[0])
    gemm_tune.FUSED_PLANS.clear()
    gemm_tune.FUSED_PLANS.update(tables[1])
    for label, K_full in (("o_proj", 64 * 128), ("down_proj", 25600)):
        K = K_full // world
        ws = [torch.randn(H, K, device=dev, dtype=torch.bfloat16) * 0.02 for _ in range(args.layers)]
        for M in batches:
            x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
            res = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
            out = torch.empty(M, H, device=dev, dtype=torch.bfloat16)

            def nccl(i=0):
                ops.gemm(x, ws[i % len(ws)], out=out)
                dist.all_reduce(out)
                res.add_(out)

            def fused(i=0):
                impl.gemm_reduce_into(x, ws[i % len(ws)], None, res)

            part = impl.partial_buffer(M, H)

            def two_kernel(i=0):
                ops.gemm(x, ws[i % len(ws)], out=part)
                impl.reduce_into(part, res)

            rows = -(-M // world)
            sp_part = impl.sp_partial(rows * world, H, torch.bfloat16, dev)
            r_slice = torch.randn(rows, H, device=dev, dtype=torch.bfloat16)
            norm_w = torch.ones(H, device=dev, dtype=torch.bfloat16)
            h = torch.empty(M, H, device=dev, dtype=torch.bfloat16)

            def sp(i=0):
                ops.gemm(x, ws[i % len(ws)], out=sp_part[:M])
                impl.rs_norm_ag(sp_part, r_slice, True, norm_w, 1e-6)

            def sp_nccl(i=0):
                ops.gemm(x, ws[i % len(ws)], out=h)
                dist.all_reduce(h)
                ops.fused_add_rmsnorm(h, res, norm_w, 1e-6)

            t_nccl = _time(nccl, args.layers)
            t_fused = _time(fused, args.layers)
            t_two = _time(two_kernel, args.layers)
            t_sp = _time(sp, args.layers)
            t_sp_nccl = _time(sp_nccl, args.layers)
            flops = 2.0 * M * K * H
            link_bytes = (world - 1) / max(world, 1) * M * H * 2 * (2 if world > 1 else 0)
            bound = max(flops / (tflops * 1e9), link_bytes / (LINK_GBS * 1e6), H * K * 2 / (hbm * 1e6))
            if rank == 0:
                print(json.dumps({"shape": label, "tp": world, "M": M, "K": K, "N": H,
                                  "plan": gemm_tune.FUSED_PLANS.get((M, H, K)),
                                  "nccl_us": round(t_nccl * 1000, 2), "fused_us": round(t_fused * 1000, 2),
                                  "gemm_then_nvlink_us": round(t_two * 1000, 2),
                                  "sp_nccl_us": round(t_sp_nccl * 1000, 2), "sp_us": round(t_sp * 1000, 2),
                                  "roofline_us": round(bound * 1000, 2),
                                  "fused_frac_roofline": round(bound / t_fused, 3),
                                  "sp_frac_roofline": round(bound / t_sp, 3)}), flush=True)
    impl.shutdown()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
