"""Time one GEMM tile plan, optionally with per-CTA phase stamps.

    python -m minisgl.benchmark.gemm_probe --M 256 --N 4096 --K 1024 --mode 2 --bn 64 --splits 1 [--kps 4] [--trace]

Runs ``--iters`` back-to-back launches cycling over 8 weight copies and
prints the mean microseconds per launch. ``--trace`` then runs one more
launch that records %globaltimer stamps in every CTA (entry, set-up done,
producer past griddepcontrol.wait, first stage consumed, accumulator ready,
exit) and prints min / median / max of each phase.
"""

from __future__ import annotations

import argparse
import json

import torch

from minisgl import ops


def _q(v: torch.Tensor) -> str:
    v = v.sort().values
    n = len(v)
    return f"min {v[0]:.2f} med {v[n // 2]:.2f} max {v[-1]:.2f}"


def main() -> None:
    p = argparse.ArgumentParser()
    for name, d in (("M", 256), ("N", 4096), ("K", 1024), ("mode", 0), ("bn", 0), ("splits", 0), ("kps", 0),
                    ("iters", 40)):
        p.add_argument(f"--{name}", type=int, default=d)
    p.add_argument("--trace", action="store_true")
    a = p.parse_args()
    x = torch.randn(a.M, a.K, device="cuda", dtype=torch.bfloat16)
    ws = [torch.randn(a.N, a.K, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(8)]
    out = torch.empty(a.M, a.N, device="cuda", dtype=torch.bfloat16)
    nat = ops.native()

    def run(w, trace=None):
        nat.gemm(out, x, w, None, None, a.splits, a.mode, None, a.bn, trace, a.kps)

    for i in range(8):
        run(ws[i % 8])
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(a.iters):
        run(ws[i % 8])
    e.record()
    torch.cuda.synchronize()
    print(json.dumps({"M": a.M, "N": a.N, "K": a.K, "plan": [a.mode, a.bn, a.splits], "kps": a.kps,
                      "us_per_launch": round(s.elapsed_time(e) / a.iters * 1000, 2)}))
    if not a.trace:
        return
    tr = torch.zeros(1 << 16, dtype=torch.int64, device="cuda")
    run(ws[3], tr)
    torch.cuda.synchronize()
    t = tr.view(-1, 8).cpu()
    t = t[t[:, 0] > 0].double()
    rel = (t - t[:, 0].min()) / 1000.0
    print("ctas", len(t))
    print(" entry", _q(rel[:, 0]))
    print(" set-up", _q(rel[:, 1] - rel[:, 0]))
    print(" producer past wait", _q(rel[:, 2]))
    print(" first stage after wait", _q(rel[:, 3] - rel[:, 2]))
    print(" mainloop (accumulator ready after first stage)", _q(rel[:, 4] - rel[:, 3]))
    print(" epilogue (exit after accumulator ready)", _q(rel[:, 5] - rel[:, 4]))
    print(" exit", _q(rel[:, 5]))


if __name__ == "__main__":
    main()
