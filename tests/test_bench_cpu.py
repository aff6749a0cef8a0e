"""bench.py host logic on the CPU: the request pools of the named shapes and
the step meter, including its DP-attention form (two gloo ranks with
different token counts per iteration cut the run at the same iteration and
agree on the summed count). CUDA events are replaced by a host clock."""

import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


class _Event:
    def __init__(self, enable_timing: bool = True) -> None:
        self.t = 0.0

    def record(self, stream=None) -> None:
        import time

        self.t = time.perf_counter()

    def elapsed_time(self, other: "_Event") -> float:
        return 1000.0 * (other.t - self.t)


class _Reply:
    def __init__(self, uid: int) -> None:
        self.uid = uid


def test_request_pools():
    p, o = bench.make_pool("kimi-k2", 512, 0)
    assert len(p) == len(o) == 512
    assert all(512 <= len(x) <= 4096 for x in p) and all(128 <= n <= 1024 for n in o)
    p2, o2 = bench.make_pool("qwen3-32b", 100, 0)
    assert all(32 <= len(x) <= 16384 for x in p2) and all(16 <= n <= 2048 for n in o2)
    assert bench.make_pool("kimi-k2", 8, 1) == bench.make_pool("kimi-k2", 8, 1)  # same pool on every rank
    assert bench.parse_args(["--shape", "kimi-k2"]).num_reqs == 512
    assert bench.parse_args([]).num_reqs == 1000


def test_step_meter_single_rank(monkeypatch):
    monkeypatch.setattr(torch.cuda, "Event", _Event)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: None)
    m = bench.StepMeter(None, step_tokens=10, warmup=1, steps=2)
    uid = 0
    with pytest.raises(bench.StopRun):
        for _ in range(100):
            m.on_reply([_Reply(uid), _Reply(uid + 1), _Reply(uid + 2)])
            uid += 3
    # boundaries at 10, 20, 30 tokens (crossed at 12, 21, 30): 3 steps after the start mark
    assert [mk[1] for mk in m.marks] == [0, 12, 21, 30]
    assert m.result()["tokens"] == 30 - 12


def _dp_rank(rank, world, port, q):
    import torch.distributed as dist

    torch.cuda.Event = _Event
    torch.cuda.synchronize = lambda *a: None
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        m = bench.StepMeter(None, step_tokens=16, warmup=1, steps=3, group=dist.group.WORLD)
        it = 0
        try:
            while it < 1000:
                # rank 0 returns 3 tokens an iteration, rank 1 one (or none: a filler step)
                n = 3 if rank == 0 else it % 2
                m.on_reply([_Reply(1000 * rank + it * 4 + j) for j in range(n)])
                it += 1
        except bench.StopRun:
            pass
        q.put((rank, it, [mk[1] for mk in m.marks], m.result()["tokens"]))
    finally:
        dist.destroy_process_group()


def test_step_meter_dp_ranks_stop_together():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (it, marks, tok)) for r, it, marks, tok in (q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]  # same stopping iteration, same marks, same summed count
    it, marks, tokens = res[0]
    assert len(marks) == 5 and marks[-1] >= 4 * 16
    assert tokens == marks[-1] - marks[1]
