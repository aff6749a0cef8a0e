"""Routed experts on the B200: expert-sorted grouped tcgen05 GEMMs against the
fp32 reference, and a Qwen3-MoE-shaped model through the engine."""

import random

import pytest
import torch

from minisgl import ops
from minisgl.core import SamplingParams
from minisgl.moe.fused import moe_reference

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _interleave(w1: torch.Tensor) -> torch.Tensor:
    E, n2, H = w1.shape
    n = n2 // 2
    return w1.view(E, 2, n // 64, 64, H).transpose(1, 2).reshape(E, n2, H).contiguous()


@pytest.mark.parametrize("T", [1, 5, 64, 300])
@pytest.mark.parametrize("tile", [0, 16, 32, 128])
def test_moe_experts_match_reference(T, tile):
    E, k, H, I = 8, 2, 256, 128
    g = torch.Generator().manual_seed(T * 7 + tile)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1 = _interleave((torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16))
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    topk_w, topk_ids = ops.moe_route(logits, k, "softmax", True)
    expect = moe_reference(x, w1, w2, topk_w, topk_ids, "silu", interleaved=True)
    out = ops.moe_experts(x.to(DEV), w1.to(DEV), w2.to(DEV), topk_w.to(DEV), topk_ids.to(DEV), tile=tile)
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device(DEV))
    err = (out.float().cpu() - expect.float()).abs()
    tol = 2e-2 + 2e-2 * expect.float().abs()
    assert (err <= tol).all(), f"max err {err.max().item():.4g}"


def test_moe_model_graph_equals_eager():
    from minisgl.llm import LLM
    from minisgl.utils.synthetic import make_model_dir

    d = make_model_dir("tiny-qwen3-moe", overrides=dict(head_dim=128, num_attention_heads=2, num_key_value_heads=1))
    rng = random.Random(3)
    prompts = [[rng.randrange(1024) for _ in range(rng.randint(20, 90))] for _ in range(4)]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    outs = []
    for graph_bs in (8, 0):
        llm = LLM(d, dtype=torch.bfloat16, device="cuda:0", use_dummy_weight=True, page_size=64, max_running_req=8,
                  max_seq_len_override=512, num_page_override=64, cuda_graph_max_bs=graph_bs, max_extend_tokens=256)
        try:
            outs.append([o["token_ids"] for o in llm.generate(prompts, sp)])
            ops.check_device_errors(torch.device("cuda:0"))
        finally:
            llm.shutdown()
    assert all(len(t) == 8 for t in outs[0])
    assert outs[0] == outs[1]
