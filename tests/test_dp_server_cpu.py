"""DP attention behind the server's message path, on CPU ranks (gloo, world
size 2). Two scheduler processes run exactly as the launcher starts them:
rank 0 pulls requests from the backend socket and re-publishes them, and the
detokenizer socket gets every reply. The test stands in for the tokenizer:
it pushes UserMsgs and collects DetokenizeMsgs. Each rank serves the requests
with uid % 2 == rank; the tokens must equal the single-rank offline engine's
(same checkpoint, greedy)."""

import shutil
import socket
import tempfile
import time
from dataclasses import replace

import pytest
import torch
import torch.multiprocessing as mp

PROMPTS = [[5, 6, 7, 8, 9, 10, 11, 12, 13], [100, 200, 300, 400, 500, 600, 700, 800, 900, 1000, 11, 12],
           [42] * 20, [7, 7, 9], [3, 1, 4, 1, 5]]
LENS = [6, 3, 9, 5, 4]  # uneven: ranks finish at different steps and keep stepping with filler batches
ENGINE = dict(dtype=torch.float32, device="cpu", page_size=16, num_page_override=64, max_running_req=4,
              max_seq_len_override=256, max_extend_tokens=64)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def checkpoint():
    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_dp_server_")
    shutil.rmtree(folder)
    make_model_dir("tiny-qwen3-moe", folder=folder)
    write_random_checkpoint(folder, seed=21, std=0.05)
    yield folder
    shutil.rmtree(folder, ignore_errors=True)


def _offline_single(folder, port, q):
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
    q.put(("done", rank))


def test_dp2_server_path_matches_single_rank(checkpoint):
    from minisgl.core import SamplingParams
    from minisgl.message import BaseBackendMsg, BaseTokenizerMsg, BatchTokenizerMsg, ExitMsg, UserMsg
    from minisgl.parallel import DistributedInfo
    from minisgl.scheduler import SchedulerConfig
    from minisgl.utils import ZmqPullQueue, ZmqPushQueue

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_offline_single, args=(checkpoint, _free_port(), q))
    p.start()
    expect = q.get(timeout=300)
    p.join(timeout=120)
    assert p.exitcode == 0

    cfg = SchedulerConfig(model_path=checkpoint, tp_info=DistributedInfo(0, 2), offline_mode=False,
                          distributed_port=_free_port(), enable_dp_attention=True, **ENGINE)
    procs = [ctx.Process(target=_scheduler_rank, args=(cfg, r, 2, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    try:
        assert sorted(q.get(timeout=300) for _ in range(2)) == [("ready", 0), ("ready", 1)]
        push = ZmqPushQueue(cfg.zmq_backend_addr, create=False, encoder=BaseBackendMsg.encoder)
        pull = ZmqPullQueue(cfg.zmq_detokenizer_addr, create=False, decoder=BaseTokenizerMsg.decoder)
        time.sleep(0.5)  # let the rank-0 -> rank-1 subscription settle before the first message
        for uid, (prompt, m) in enumerate(zip(PROMPTS, LENS)):
            sp = SamplingParams(temperature=0.0, max_tokens=m, ignore_eos=True)
            push.put(UserMsg(uid=uid, input_ids=torch.tensor(prompt, dtype=torch.int32), sampling_params=sp))
        got = {uid: [] for uid in range(len(PROMPTS))}
        finished = set()
        deadline = time.monotonic() + 300
        while len(finished) < len(PROMPTS):
            assert time.monotonic() < deadline, f"replies stalled: finished {sorted(finished)}"
            if not pull.poll(100):
                continue
            msg = pull.get()
            for m in (msg.data if isinstance(msg, BatchTokenizerMsg) else [msg]):
                assert m.uid not in finished, f"token for uid {m.uid} after it finished"
                got[m.uid].append(m.next_token)
                if m.finished:
                    finished.add(m.uid)
        push.put(ExitMsg())
        assert sorted(q.get(timeout=120) for _ in range(2)) == [("done", 0), ("done", 1)]
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.exitcode is None:
                pr.kill()
    assert [got[uid] for uid in range(len(PROMPTS))] == expect
    assert all(pr.exitcode == 0 for pr in procs)
