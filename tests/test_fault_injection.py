"""Failure detection, exercised with faults made on the host (CPU ranks,
gloo): a rank that raises, stalls or dies mid-generation must make its peer
fail with an error within the process-group timeout instead of hanging, and
the fault-injection rules parse as documented. No GPU is involved."""

import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from minisgl.utils import fault

PROMPTS = [[5, 6, 7, 8, 9, 10, 11, 12, 13], [100, 200, 300, 400, 500, 600, 700, 800, 900, 1000, 11, 12]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, spec, q):
    os.environ[fault.ENV] = spec
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo
    from minisgl.utils.synthetic import make_model_dir

    t0 = time.time()
    try:
        llm = LLM(make_model_dir("tiny-qwen3"), dtype=torch.float32, device="cpu", use_dummy_weight=True,
                  tp_info=DistributedInfo(rank, world), page_size=16, num_page_override=64, max_running_req=4,
                  max_seq_len_override=256, max_extend_tokens=64, distributed_port=port, distributed_timeout=15)
        outs = llm.generate(PROMPTS, SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
        q.put((rank, "ok", [o["token_ids"] for o in outs], time.time() - t0))
        llm.shutdown()
    except BaseException as e:  # reported to the parent
        q.put((rank, "error", f"{type(e).__name__}: {e}"[:300], time.time() - t0))


def _spawn(spec, expect_reports):
    """Runs two ranks; waits for the reports of ranks 0 .. expect_reports - 1
    (a rank outside that set may report too, e.g. when a loaded machine
    makes it fail before its injected fault; such a report is kept)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, spec, q)) for r in range(2)]
    for p in procs:
        p.start()
    reports = {}
    deadline = time.time() + 240
    try:
        while any(r not in reports for r in range(expect_reports)):
            rank, status, payload, secs = q.get(timeout=max(1.0, deadline - time.time()))
            reports[rank] = (status, payload, secs)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():  # a stalled rank: end exactly the child we started
                p.kill()
                p.join(timeout=30)
    return reports, procs


def test_rules_parse():
    r = fault.parse("raise:rank=1:step=3; stall:rank=0:seconds=2.5;skip_collective:rank=1")
    assert [x.action for x in r] == ["raise", "stall", "skip_collective"]
    assert r[0].step == 3 and r[1].seconds == 2.5 and r[2].step == 0
    with pytest.raises(ValueError):
        fault.parse("explode:rank=0")
    with pytest.raises(ValueError):
        fault.parse("raise:step=1")
    assert fault.skip_collective(0, 5) is False


def test_raising_rank_fails_its_peer():
    reports, _ = _spawn("raise:rank=1:step=3", 2)
    assert reports[1][0] == "error" and "InjectedFault" in reports[1][1]
    assert reports[0][0] == "error", reports[0]  # the peer's collective fails instead of hanging


def test_dead_rank_fails_its_peer():
    reports, procs = _spawn("exit:rank=1:step=2", 1)
    assert reports[0][0] == "error", reports[0]
    assert procs[1].exitcode == 17


def test_stalled_rank_times_out_its_peer():
    # rank 1 sleeps far beyond the 15 s process-group timeout at step 2
    reports, _ = _spawn("stall:rank=1:step=2:seconds=120", 1)
    status, payload, secs = reports[0]
    assert status == "error", payload
    assert secs < 90, secs
