"""DP attention with expert-parallel token dispatch on CPU ranks (gloo,
world size 2): each rank serves half of the prompts with a replicated model
except the routed experts (split in halves), the MoE layers send every
(token, expert) row to the expert's owner and back (all-to-all), ranks step
together (a rank without work runs a one-token filler step), and the
gathered results equal the single-rank engine's. An odd prompt count leaves
one rank idle at the end."""

import shutil
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

PROMPTS = [[5, 6, 7, 8, 9, 10, 11, 12, 13], [100, 200, 300, 400, 500, 600, 700, 800, 900, 1000, 11, 12],
           [42] * 20, [7, 7, 9]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, folder, port, dp, prompts, max_tokens, q, quant="none"):
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo

    llm = LLM(folder, dtype=torch.float32, device="cpu", tp_info=DistributedInfo(rank, world), page_size=16,
              num_page_override=64, max_running_req=4, max_seq_len_override=256, max_extend_tokens=64,
              distributed_port=port, enable_dp_attention=dp, moe_quant=quant)
    sps = [SamplingParams(temperature=0.0, max_tokens=m, ignore_eos=True) for m in max_tokens]
    outs = llm.generate(prompts, sps)
    q.put((rank, [o["token_ids"] for o in outs]))
    llm.shutdown()


@pytest.fixture(scope="module")
def checkpoint():
    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_dp_ckpt_")
    shutil.rmtree(folder)
    make_model_dir("tiny-qwen3-moe", folder=folder)
    write_random_checkpoint(folder, seed=11, std=0.05)
    yield folder
    shutil.rmtree(folder, ignore_errors=True)


def _generate(world, folder, dp, prompts, max_tokens, quant="none"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, folder, port, dp, prompts, max_tokens, q, quant))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


def test_dp2_ep2_matches_single_rank(checkpoint):
    lens = [8, 3, 12, 5]  # uneven: one rank finishes first and keeps stepping with filler batches
    single = _generate(1, checkpoint, False, PROMPTS, lens)[0]
    dp = _generate(2, checkpoint, True, PROMPTS, lens)
    assert dp[0] == dp[1] == single


def test_dp2_mx_a8_matches_single_rank(checkpoint):
    """Block-scaled MX experts (``--moe-quant mxfp4-a8``) behind the token
    dispatch: the received rows go through the same MXFP8 statement."""
    lens = [6, 4, 7, 5]
    single = _generate(1, checkpoint, False, PROMPTS, lens, quant="mxfp4-a8")[0]
    dp = _generate(2, checkpoint, True, PROMPTS, lens, quant="mxfp4-a8")
    assert dp[0] == dp[1] == single


def test_dp2_odd_prompt_count(checkpoint):
    prompts, lens = PROMPTS[:3], [4, 4, 6]
    single = _generate(1, checkpoint, False, prompts, lens)[0]
    dp = _generate(2, checkpoint, True, prompts, lens)
    assert dp[0] == dp[1] == single


@pytest.fixture(scope="module")
def kimi_checkpoint():
    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_dp_kimi_")
    shutil.rmtree(folder)
    make_model_dir("tiny-kimi", folder=folder)
    write_random_checkpoint(folder, seed=13, std=0.05)
    yield folder
    shutil.rmtree(folder, ignore_errors=True)


def test_dp2_kimi_mla_moe_matches_single_rank(kimi_checkpoint):
    """DeepSeek-V3 shape: MLA attention replicated per DP rank, routed experts
    dispatched, the shared expert computed locally."""
    lens = [5, 7, 3, 6]
    single = _generate(1, kimi_checkpoint, False, PROMPTS, lens)[0]
    dp = _generate(2, kimi_checkpoint, True, PROMPTS, lens)
    assert dp[0] == dp[1] == single


def test_tp2_kimi_checkpoint_matches_single_rank(kimi_checkpoint):
    """The HF DeepSeek-V3 layout loaded with TP=2: q_b / kv_b split by heads,
    experts and the shared expert split on the intermediate dimension."""
    lens = [4, 4, 4, 4]
    single = _generate(1, kimi_checkpoint, False, PROMPTS, lens)[0]
    tp = _generate(2, kimi_checkpoint, False, PROMPTS, lens)
    assert tp[0] == tp[1] == single


def test_random_init_experts_are_per_global_expert():
    """--random-init under expert parallelism: rank r's local expert j has
    the values the single-rank model gives global expert r * E / R + j."""
    from minisgl.models.weight import random_weights

    full = {"model.layers.1.mlp.experts.gate_up_proj": torch.empty(8, 16, 32, device="meta")}
    half = {"model.layers.1.mlp.experts.gate_up_proj": torch.empty(4, 16, 32, device="meta")}
    w = random_weights(full, torch.device("cpu"))["model.layers.1.mlp.experts.gate_up_proj"]
    r1 = random_weights(half, torch.device("cpu"), first_expert=4)["model.layers.1.mlp.experts.gate_up_proj"]
    r0 = random_weights(half, torch.device("cpu"), first_expert=0)["model.layers.1.mlp.experts.gate_up_proj"]
    assert torch.equal(r0, w[:4]) and torch.equal(r1, w[4:])
