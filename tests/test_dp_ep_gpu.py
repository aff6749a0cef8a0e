"""DP attention with expert-parallel token dispatch on 2 GPUs (NCCL
all-to-all; NVLS off): a Qwen3-MoE-shape model served by two DP ranks, each
holding half of the experts, generates what one GPU generates."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, dp, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo
    from minisgl.utils.synthetic import make_model_dir

    torch.cuda.set_device(rank)
    llm = LLM(make_model_dir("tiny-qwen3-moe", overrides=dict(head_dim=128, num_attention_heads=2,
                                                               num_key_value_heads=1)),
              dtype=torch.bfloat16, device=f"cuda:{rank}", use_dummy_weight=True, dummy_weight_device="cpu",
              tp_info=DistributedInfo(rank, world), page_size=64, num_page_override=64, max_running_req=8,
              max_seq_len_override=1024, distributed_port=port, enable_dp_attention=dp)
    prompts = [[(7 * i + 3 * j) % 1000 for j in range(20 + 9 * i)] for i in range(5)]
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    q.put((rank, [o["token_ids"] for o in outs]))
    llm.shutdown()


def _spawn(world, dp):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, dp, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=400) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


def test_dp2_ep2_matches_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    one = _spawn(1, False)[0]
    two = _spawn(2, True)
    assert two[0] == two[1]
    same = sum(a == b for x, y in zip(one, two[0]) for a, b in zip(x, y))
    assert same >= 0.8 * sum(len(x) for x in one), (one, two[0])
