"""DP attention with expert-parallel token dispatch on GPUs (NVLS off): a
Qwen3-MoE-shape model served by two DP ranks, each holding half of the
experts, generates what one GPU generates, with the rows moved by NCCL or by
our peer-store kernels (``--comm fused``); and the peer-store dispatch on a
one-rank heap equals the local expert pipeline."""

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


def _run(rank, world, port, dp, q, comm, folder):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo

    torch.cuda.set_device(rank)
    # weights from a written checkpoint: each EP rank must load its own
    # experts (per-name random init would give every rank the same ones)
    llm = LLM(folder, dtype=torch.bfloat16, device=f"cuda:{rank}", tp_info=DistributedInfo(rank, world),
              page_size=64, num_page_override=64, max_running_req=8, max_seq_len_override=1024,
              distributed_port=port, enable_dp_attention=dp, comm=comm)
    prompts = [[(7 * i + 3 * j) % 1000 for j in range(20 + 9 * i)] for i in range(5)]
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    q.put((rank, [o["token_ids"] for o in outs]))
    llm.shutdown()


@pytest.fixture(scope="module")
def checkpoint():
    import shutil
    import tempfile

    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_dp_gpu_ckpt_")
    shutil.rmtree(folder)
    make_model_dir("tiny-qwen3-moe", folder=folder, overrides=dict(head_dim=128, num_attention_heads=2,
                                                                    num_key_value_heads=1))
    write_random_checkpoint(folder, seed=17, std=0.05)
    yield folder
    shutil.rmtree(folder, ignore_errors=True)


def _spawn(world, dp, folder, comm="nccl"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, dp, q, comm, folder)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=400) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


@pytest.mark.parametrize("comm", ["nccl", "fused"])
def test_dp2_ep2_matches_one_gpu(comm, checkpoint):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    one = _spawn(1, False, checkpoint)[0]
    two = _spawn(2, True, checkpoint, comm)
    assert two[0] == two[1]
    same = sum(a == b for x, y in zip(one, two[0]) for a, b in zip(x, y))
    assert same >= 0.8 * sum(len(x) for x in one), (one, two[0])


def test_nvlink_dispatch_one_rank_matches_local_experts():
    """The peer-store dispatch / return kernels on a one-rank heap (rows
    stored into this GPU's own heap) give what the local expert pipeline
    gives."""
    import torch.distributed as dist

    from minisgl import ops
    from minisgl.moe.ep_a2a import AllToAllMoe
    from minisgl.moe.fused import FusedMoe
    from minisgl.parallel.ep_comm import EpHeap

    port = _free_port()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    heap = None
    try:
        dev = torch.device("cuda", 0)
        g = torch.Generator(device="cpu").manual_seed(4)
        T, H, I, E, k = 37, 256, 128, 8, 2
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
        w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16).to(dev)
        w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16).to(dev)
        logits = torch.randn(T, E, generator=g).to(dev)
        heap = EpHeap(dev, 64 * k, H)
        a2a = AllToAllMoe(1, 0, None, heap)
        got = a2a.forward(x, w1, w2, logits, k, True, interleaved=True)
        got2 = a2a.forward(x, w1, w2, logits, k, True, interleaved=True)  # the barriers reset for a second step
        want = FusedMoe().forward(x, w1, w2, logits, k, True, interleaved=True)
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        assert torch.allclose(got.float(), want.float(), atol=2e-2, rtol=1e-2)
        assert torch.equal(got, got2)
    finally:
        if heap is not None:
            heap.shutdown()
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def tp_checkpoint():
    import shutil
    import tempfile

    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_tp_moe_gpu_ckpt_")
    shutil.rmtree(folder)
    make_model_dir("tiny-qwen3-moe", folder=folder, overrides=dict(head_dim=128, num_attention_heads=4,
                                                                    num_key_value_heads=2))
    write_random_checkpoint(folder, seed=19, std=0.05)
    yield folder
    shutil.rmtree(folder, ignore_errors=True)


def test_tp2_moe_fused_comm_matches_nccl(tp_checkpoint):
    """Plain tensor parallelism over a MoE model (experts sharded over the
    ranks; MoE decoders keep the all-reduce form, not the sequence-parallel
    one): the NVLink collectives, the default, generate what NCCL generates
    (the two reduce in different orders, so a near-tie may flip a token)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    fused = _spawn(2, False, tp_checkpoint, "fused")
    nccl = _spawn(2, False, tp_checkpoint, "nccl")
    assert fused[0] == fused[1] and nccl[0] == nccl[1]
    same = sum(a == b for x, y in zip(fused[0], nccl[0]) for a, b in zip(x, y))
    assert same >= 0.8 * sum(len(x) for x in fused[0]), (fused[0], nccl[0])
