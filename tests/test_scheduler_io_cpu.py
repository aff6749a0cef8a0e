"""Scheduler processes driven over their sockets, on CPU ranks (gloo).

The test stands in for the tokenizer:

- It pushes UserMsgs into rank 0's backend socket and reads DetokenizeMsgs
  from the detokenizer socket.
- With 2 TP ranks, rank 0 re-publishes every message to rank 1 and both
  ranks step together.
- Greedy tokens must equal the offline engine's on the same checkpoint.
- An AbortBackendMsg sent mid-generation stops that request: no token for it
  arrives after the scheduler has processed the abort, and a request sent
  afterwards still completes.
- ExitMsg shuts every rank down cleanly.

This is the counterpart of the reference's scheduler integration test, on
CPU ranks instead of a GPU.
"""

import shutil
import socket
import tempfile
import time
from dataclasses import replace

import pytest
import torch
import torch.multiprocessing as mp

PROMPTS = [[5, 6, 7, 8, 9, 10, 11, 12, 13], [100, 200, 300, 400, 500, 600, 700, 800, 900, 1000, 11, 12],
           [42] * 20]
LENS = [6, 4, 8]
ENGINE = dict(dtype=torch.float32, device="cpu", page_size=16, num_page_override=64, max_running_req=4,
              max_seq_len_override=256, max_extend_tokens=64)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def checkpoint():
    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_sched_io_")
    shutil.rmtree(folder)
    make_model_dir("tiny-qwen3", folder=folder)
    write_random_checkpoint(folder, seed=5, std=0.05)
    yield folder
    shutil.rmtree(folder, ignore_errors=True)


def _offline(folder, port, q):
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM

    llm = LLM(folder, distributed_port=port, **ENGINE)
    sps = [SamplingParams(temperature=0.0, max_tokens=m, ignore_eos=True) for m in LENS]
    q.put([o["token_ids"] for o in llm.generate(PROMPTS, sps)])
    llm.shutdown()


def _scheduler_rank(cfg, rank, world, q):
    from minisgl.parallel import DistributedInfo
    from minisgl.scheduler import Scheduler

    with torch.inference_mode():
        sched = Scheduler(replace(cfg, tp_info=DistributedInfo(rank, world)))
        sched.sync_all_ranks()
        q.put(("ready", rank))
        try:
            sched.run_forever()
        except KeyboardInterrupt:
            sched.shutdown()
        except Exception as e:  # reported to the test, then the rank dies with it
            q.put(("error", rank, type(e).__name__, str(e)))
            raise
    q.put(("done", rank))


class _Client:
    def __init__(self, cfg):
        from minisgl.message import BaseBackendMsg, BaseTokenizerMsg
        from minisgl.utils import ZmqPullQueue, ZmqPushQueue

        self.push = ZmqPushQueue(cfg.zmq_backend_addr, create=False, encoder=BaseBackendMsg.encoder)
        self.pull = ZmqPullQueue(cfg.zmq_detokenizer_addr, create=False, decoder=BaseTokenizerMsg.decoder)
        self.tokens, self.finished = {}, set()

    def send(self, uid, prompt, max_tokens):
        from minisgl.core import SamplingParams
        from minisgl.message import UserMsg

        sp = SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True)
        self.tokens[uid] = []
        self.push.put(UserMsg(uid=uid, input_ids=torch.tensor(prompt, dtype=torch.int32), sampling_params=sp))

    def _take(self):
        from minisgl.message import BatchTokenizerMsg

        msg = self.pull.get()
        for m in (msg.data if isinstance(msg, BatchTokenizerMsg) else [msg]):
            assert m.uid not in self.finished, f"token for uid {m.uid} after it finished"
            self.tokens[m.uid].append(m.next_token)
            if m.finished:
                self.finished.add(m.uid)

    def drain(self, until, timeout=300.0):
        """Collect replies until `until()` holds (bounded wait)."""
        deadline = time.monotonic() + timeout
        while not until():
            assert time.monotonic() < deadline, f"replies stalled: finished {sorted(self.finished)}"
            if self.pull.poll(50):
                self._take()

    def drain_pending(self, quiet_ms=500):
        """Collect whatever arrives until the socket stays quiet for `quiet_ms`."""
        while self.pull.poll(quiet_ms):
            self._take()


def _start(checkpoint, world, **overrides):
    from minisgl.parallel import DistributedInfo
    from minisgl.scheduler import SchedulerConfig

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    cfg = SchedulerConfig(model_path=checkpoint, tp_info=DistributedInfo(0, world), offline_mode=False,
                          distributed_port=_free_port(), **dict(ENGINE, **overrides))
    procs = [ctx.Process(target=_scheduler_rank, args=(cfg, r, world, q)) for r in range(world)]
    for p in procs:
        p.start()
    assert sorted(q.get(timeout=300) for _ in range(world)) == [("ready", r) for r in range(world)]
    client = _Client(cfg)
    time.sleep(0.5)  # let the rank-0 -> other-rank subscription settle before the first message
    return procs, q, client


def _stop(procs, q, client):
    from minisgl.message import ExitMsg

    try:
        client.push.put(ExitMsg())
        assert sorted(q.get(timeout=120) for _ in procs) == [("done", r) for r in range(len(procs))]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)


@pytest.fixture(scope="module")
def expect(checkpoint):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_offline, args=(checkpoint, _free_port(), q))
    p.start()
    out = q.get(timeout=300)
    p.join(timeout=120)
    assert p.exitcode == 0
    return out


@pytest.mark.parametrize("world", [1, 2])
def test_scheduler_over_sockets_matches_offline(checkpoint, expect, world):
    procs, q, client = _start(checkpoint, world)
    try:
        for uid, (prompt, m) in enumerate(zip(PROMPTS, LENS)):
            client.send(uid, prompt, m)
        client.drain(lambda: len(client.finished) == len(PROMPTS))
        assert [client.tokens[uid] for uid in range(len(PROMPTS))] == expect
    finally:
        _stop(procs, q, client)


def test_abort_stops_a_request(checkpoint):
    from minisgl.message import AbortBackendMsg

    procs, q, client = _start(checkpoint, 2)
    try:
        client.send(0, PROMPTS[0], 200)  # long: still running when the abort arrives
        client.drain(lambda: len(client.tokens[0]) >= 3)
        client.push.put(AbortBackendMsg(uid=0))
        # a later request completes, so the scheduler processed the abort before it
        client.send(1, PROMPTS[1], 4)
        client.drain(lambda: 1 in client.finished)
        n_at_done = len(client.tokens[0])
        client.drain_pending()  # the abort was handled before uid 1 started: nothing more for uid 0
        assert 0 not in client.finished
        assert len(client.tokens[0]) == n_at_done < 200
        assert len(client.tokens[1]) == 4
    finally:
        _stop(procs, q, client)


def test_lost_broadcast_message_is_detected(checkpoint, monkeypatch):
    """Rank 0 drops the first message it announces to rank 1 (host fault
    injection): rank 1's bounded wait runs out and it raises MessageLostError
    instead of waiting forever. Rank 0 learns of it through the CPU process
    group: its next count broadcast fails (the peer is gone, or the group's
    short timeout runs out) and it exits with an error too."""
    monkeypatch.setenv("MINISGL_FAULT_INJECT", "drop_broadcast:rank=0:step=0")
    monkeypatch.setenv("MINISGL_BROADCAST_TIMEOUT_S", "3")
    procs, q, client = _start(checkpoint, 2, distributed_timeout=10.0)
    try:
        client.send(0, PROMPTS[0], 100)  # taken while idle: published before any count, never dropped
        client.drain(lambda: len(client.tokens[0]) >= 2)  # both ranks are stepping now
        client.send(1, PROMPTS[1], 4)  # announced in a count broadcast: the dropped one
        t0 = time.monotonic()
        events = {}
        while len(events) < 2:
            event = q.get(timeout=120)
            assert event[0] == "error", event
            events[event[1]] = event
        assert events[1][2] == "MessageLostError", events[1]
        assert "did not arrive within 3.0 s" in events[1][3]
        # rank 0 fails in its collective within the group's 10 s timeout (plus slack), not later
        assert time.monotonic() - t0 < 60.0
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode not in (0, None)
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
            p.join(timeout=60)
