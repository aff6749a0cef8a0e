"""The engine on a B200: native kernels end to end, checked against the
dense fp32 oracle with teacher forcing (bf16 vs fp32 may flip near-ties, so
each generated token must be the oracle's argmax or within a small logit
margin of it) - both on the engine's own folded weights and on the original
checkpoint before the norm weights are folded into the projections - and
CUDA-graph decode identical to eager decode."""

import random

import pytest
import torch

from minisgl import ops
from minisgl.core import SamplingParams
from minisgl.llm import LLM
from minisgl.models.oracle import dense_logits
from minisgl.utils.synthetic import make_model_dir

pytestmark = pytest.mark.gpu


def _make(graph_bs, **kw):
    d = make_model_dir("small-qwen3")
    args = dict(dtype=torch.bfloat16, device="cuda:0", use_dummy_weight=True, dummy_weight_device="cpu",
                page_size=64, max_running_req=16, max_seq_len_override=2048, num_page_override=256,
                cuda_graph_max_bs=graph_bs, max_extend_tokens=256)
    args.update(kw)
    return LLM(d, **args)


def _prompts(n, seed=0):
    rng = random.Random(seed)
    return [[rng.randrange(4096) for _ in range(rng.randint(20, 300))] for _ in range(n)]


def test_gpu_engine_tracks_oracle():
    llm = _make(16)
    try:
        prompts = _prompts(6)
        outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
        ops.check_device_errors(torch.device("cuda:0"))
        state = llm.engine.model.state_dict()
        cfg = llm.engine.model_config
        for p, o in zip(prompts, outs):
            toks = o["token_ids"]
            assert len(toks) == 12
            logits = dense_logits(state, cfg, p + toks[:-1],
                                  fused_layout=llm.engine.model.fused_layout)[len(p) - 1 :]
            for t, row in zip(toks, logits):
                assert row[t] >= row.max() - 0.03 * row.abs().max(), (t, int(row.argmax()))
    finally:
        llm.shutdown()


def test_gpu_engine_tracks_unfolded_checkpoint(tmp_path):
    """A bf16 checkpoint with non-unit norm weights, loaded from disk: the
    engine folds the norm weights into the qkv / gate_up projections (in
    bf16); its tokens are checked against the fp32 oracle run on the
    checkpoint as written, so the error of the folding is inside the check."""
    import os

    from minisgl.models.weight import load_weight
    from minisgl.utils.synthetic import write_random_checkpoint

    folder = os.path.join(str(tmp_path), "m")
    make_model_dir("small-qwen3", folder=folder)
    write_random_checkpoint(folder, seed=11, std=0.05, norm_std=0.3)
    llm = LLM(folder, dtype=torch.bfloat16, device="cuda:0", use_dummy_weight=False, page_size=64,
              max_running_req=16, max_seq_len_override=2048, num_page_override=256, cuda_graph_max_bs=16,
              max_extend_tokens=256)
    try:
        assert llm.engine.model.fused_layout
        prompts = _prompts(6, seed=2)
        outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
        ops.check_device_errors(torch.device("cuda:0"))
        state = {k: v.float() for k, v in load_weight(folder, torch.device("cpu"))}
        cfg = llm.engine.model_config
        exact = total = 0
        for p, o in zip(prompts, outs):
            toks = o["token_ids"]
            logits = dense_logits(state, cfg, p + toks[:-1], fused_layout=False)[len(p) - 1 :]
            for t, row in zip(toks, logits):
                assert row[t] >= row.max() - 0.03 * row.abs().max(), (t, int(row.argmax()))
                exact += int(t == int(row.argmax()))
                total += 1
        assert exact >= 0.8 * total, (exact, total)
    finally:
        llm.shutdown()


def test_graph_decode_equals_eager():
    # 4 requests: a captured batch size, so the graph runs the same kernels
    # (same split-KV count and tile plans) as eager decode, bit for bit
    prompts = _prompts(4, seed=3)
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    llm = _make(8)
    try:
        with_graph = [o["token_ids"] for o in llm.generate(prompts, sp)]
    finally:
        llm.shutdown()
    llm = _make(0)
    try:
        eager = [o["token_ids"] for o in llm.generate(prompts, sp)]
    finally:
        llm.shutdown()
    assert with_graph == eager


def test_chunked_prefill_and_sampling():
    llm = _make(16, max_extend_tokens=64)
    try:
        prompts = _prompts(4, seed=5)
        outs = llm.generate(prompts, SamplingParams(temperature=0.8, top_k=50, top_p=0.9, max_tokens=20,
                                                    ignore_eos=True))
        assert all(len(o["token_ids"]) == 20 for o in outs)
        assert all(0 <= t < 4096 for o in outs for t in o["token_ids"])
        llm.cache_manager.check_integrity()
    finally:
        llm.shutdown()


def test_fused_sampling_matches_logits_path():
    """Sampling inside the LM-head GEMM (CUDA graphs and eager) against
    sampling from materialised logits: identical greedy tokens, and the same
    random stream for temperature sampling (the two paths' LM-head tile plans
    may differ in the last fp32 bits, so a rare near-tie may diverge)."""
    from minisgl.env import ENV

    prompts = _prompts(4, seed=7)
    outs = {}
    for fused in (True, False):
        ENV.NO_FUSED_SAMPLING.value = not fused
        llm = _make(8)
        try:
            greedy = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8,
                                                                                   ignore_eos=True))]
            hot = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(temperature=0.8, max_tokens=8,
                                                                                ignore_eos=True))]
            ops.check_device_errors(torch.device("cuda:0"))
        finally:
            llm.shutdown()
            ENV.NO_FUSED_SAMPLING.value = False
        outs[fused] = (greedy, hot)
    assert outs[True][0] == outs[False][0]
    a, b = outs[True][1], outs[False][1]
    assert [x[0] for x in a] == [y[0] for y in b]
    same = sum(p == q for x, y in zip(a, b) for p, q in zip(x, y))
    assert same >= 0.9 * sum(len(x) for x in a)
