"""Tensor parallelism on CPU ranks (gloo, world size 2): the sharded engine
loading the same HF checkpoint must generate what the single-rank engine
generates. Exercises the weight loader's shard/merge rules, vocab-parallel
embedding and LM head, row-parallel all-reduce and the rank-0 message
fan-out path of the engine. The sequence-parallel form of the decoder
(token-sharded residual stream; reduce-scatter + residual + RMSNorm +
all-gather after each row-parallel projection, token counts padded to a
multiple of the rank count) runs here through the library collectives and
must generate the same tokens."""

import os
import shutil
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

PROMPTS = [[5, 6, 7, 8, 9, 10, 11, 12, 13], [100, 200, 300, 400, 500, 600, 700, 800, 900, 1000, 11, 12]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, folder, port, out_q, sp=False):
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedCommunicator, DistributedInfo

    llm = LLM(folder, dtype=torch.float32, device="cpu", tp_info=DistributedInfo(rank, world), page_size=16,
              num_page_override=64, max_running_req=4, max_seq_len_override=256, max_extend_tokens=64,
              distributed_port=port)
    if sp:
        DistributedCommunicator.plugins[-1].sequence_parallel = True
        assert llm.engine.model.model.sp_comm() is not None
    # 21 prompt tokens (odd: the sequence-parallel form pads), then decode
    # batches of 2 and, after the second request ends, of 1
    sps = [SamplingParams(temperature=0.0, max_tokens=m, ignore_eos=True) for m in (8, 5)]
    outs = llm.generate(PROMPTS, sps)
    out_q.put((rank, [o["token_ids"] for o in outs]))
    llm.shutdown()


@pytest.fixture(scope="module")
def checkpoint():
    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_tp_ckpt_")
    shutil.rmtree(folder)
    make_model_dir("tiny-qwen3", folder=folder, overrides={"tie_word_embeddings": False})
    write_random_checkpoint(folder, seed=3, std=0.05)
    yield folder
    shutil.rmtree(folder, ignore_errors=True)


def _generate(world, folder, sp=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, folder, port, q, sp)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


@pytest.fixture(scope="module")
def single(checkpoint):
    return _generate(1, checkpoint)[0]


def test_tp2_matches_tp1(checkpoint, single):
    tp = _generate(2, checkpoint)
    assert tp[0] == tp[1] == single


def test_tp2_sequence_parallel_matches_tp1(checkpoint, single):
    tp = _generate(2, checkpoint, sp=True)
    assert tp[0] == tp[1] == single


def test_tp4_sequence_parallel_matches_tp1(checkpoint, single):
    """Four ranks: more ranks than kv heads (the kv heads are replicated), and
    token counts padded up to a multiple of 4 (21 prompt tokens, then decode
    batches of 2 and 1)."""
    tp = _generate(4, checkpoint, sp=True)
    assert tp[0] == tp[1] == tp[2] == tp[3] == single
