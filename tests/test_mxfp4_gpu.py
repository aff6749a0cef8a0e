"""MXFP4 experts on the GPU: the quantiser kernel is bit-exact with the
PyTorch statement of the OCP MX rules, the W4A16 grouped tcgen05 expert
pipeline matches fp32 experts on the dequantised weights, and a MoE model
with MXFP4 experts runs through the engine with CUDA graphs."""

import pytest
import torch

from minisgl import ops
from minisgl.moe.fused import moe_reference
from minisgl.ops import reference as ref
from minisgl.quant import dequantize_mxfp4, quantize_mxfp4, quantize_mxfp4_reference

pytestmark = pytest.mark.gpu


def test_quantiser_bit_exact():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(3, 256, 512, generator=g) * 0.02
    w[0, 0, :32] = 0.0                     # an all-zero block
    w[0, 1, :32] = 1e-39                   # a subnormal block (scale byte 0)
    w[1, 2, :8] = torch.tensor([6.0, 3.0, 1.75, 0.75, -0.25, 5.0, -5.5, 2.5])  # ties and saturation
    w = w.to(torch.bfloat16)
    p_ref, s_ref = quantize_mxfp4_reference(w)
    p, s = quantize_mxfp4(w.cuda())
    torch.cuda.synchronize()
    assert torch.equal(p.cpu(), p_ref)
    assert torch.equal(s.cpu(), s_ref)


@pytest.mark.parametrize("T,E,k", [(1, 8, 2), (37, 8, 2), (300, 16, 4)])
def test_moe_experts_mxfp4_matches_dequantised(T, E, k):
    g = torch.Generator().manual_seed(T + E)
    H, I = 256, 256
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    tw, ti = ref.moe_route(logits, k, "softmax", True)
    # gate|up rows interleaved in 64-row blocks, as the layer stores them
    w1i = w1.view(E, 2, I // 64, 64, H).transpose(1, 2).reshape(E, 2 * I, H).contiguous()
    q1 = quantize_mxfp4(w1i.cuda())
    q2 = quantize_mxfp4(w2.cuda())
    got = ops.moe_experts_mxfp4(x.cuda(), *q1, *q2, tw.cuda(), ti.cuda())
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device("cuda"))
    d1 = dequantize_mxfp4(q1[0].cpu(), q1[1].cpu()).to(torch.bfloat16)
    d2 = dequantize_mxfp4(q2[0].cpu(), q2[1].cpu()).to(torch.bfloat16)
    want = moe_reference(x, d1, d2, tw, ti, "silu", interleaved=True)
    err = (got.cpu().float() - want.float()).abs().max().item()
    assert err <= 3e-2 * max(1.0, want.float().abs().max().item()), err


def test_mxfp4_moe_model_graphs():
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.utils.synthetic import make_model_dir

    kw = dict(dtype=torch.bfloat16, device="cuda:0", use_dummy_weight=True, page_size=64, num_page_override=64,
              max_running_req=8, max_seq_len_override=1024, moe_quant="mxfp4")
    prompts = [[(11 * i + 5 * j) % 4000 for j in range(30 + 7 * i)] for i in range(4)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    outs = {}
    for graphs in (0, 8):
        llm = LLM(make_model_dir("tiny-qwen3-moe", overrides=dict(head_dim=128, num_attention_heads=2,
                                                                num_key_value_heads=1)),
                  cuda_graph_max_bs=graphs, **kw)
        outs[graphs] = [o["token_ids"] for o in llm.generate(prompts, sp)]
        torch.cuda.synchronize()
        ops.check_device_errors(torch.device("cuda:0"))
        llm.shutdown()
    assert all(len(o) == 6 for o in outs[0])
    assert outs[0] == outs[8]
