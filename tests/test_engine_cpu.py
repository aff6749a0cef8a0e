"""End-to-end engine on the CPU (tiny Qwen3, fp32): the paged, chunked,
radix-cached scheduler must reproduce the dense fp32 oracle token for token."""

import random

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.llm import LLM
from minisgl.models.oracle import greedy_generate
from minisgl.utils.synthetic import make_model_dir


@pytest.fixture(scope="module")
def llm():
    d = make_model_dir("tiny-qwen3", overrides={"tie_word_embeddings": False})
    engine = LLM(d, dtype=torch.float32, device="cpu", use_dummy_weight=True, page_size=16, max_extend_tokens=32,
                 num_page_override=256, max_running_req=16, max_seq_len_override=512, cache_type="radix")
    yield engine
    engine.shutdown()


def _oracle(llm, prompt, n):
    model = llm.engine.model
    return greedy_generate(model.state_dict(), llm.engine.model_config, prompt, n,
                           fused_layout=getattr(model, "fused_layout", False))


def test_tiny_qwen3_matches_dense_oracle(llm):
    rng = random.Random(0)
    prompts = [[rng.randrange(1024) for _ in range(rng.randint(16, 64))] for _ in range(8)]
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert len(o["token_ids"]) == 16
        assert o["token_ids"] == _oracle(llm, p, 16)
    llm.cache_manager.check_integrity()


def test_shared_prefixes_hit_radix_cache(llm):
    rng = random.Random(1)
    prefix = [rng.randrange(1024) for _ in range(48)]
    prompts = [prefix + [rng.randrange(1024) for _ in range(rng.randint(1, 20))] for _ in range(6)]
    first = llm.generate(prompts[:1], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    before = llm.cache_manager.prefix_cache.size_info.total_size
    assert before >= 48
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    assert outs[0]["token_ids"] == first[0]["token_ids"]
    for p, o in zip(prompts, outs):
        assert o["token_ids"] == _oracle(llm, p, 8)
    llm.cache_manager.check_integrity()


def test_sampling_params_respected(llm):
    outs = llm.generate([[5, 6, 7, 8, 9]] * 3, [SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True)
                                                 for n in (1, 3, 7)])
    assert [len(o["token_ids"]) for o in outs] == [1, 3, 7]
    sampled = llm.generate([[5, 6, 7, 8, 9]], SamplingParams(temperature=1.0, top_k=5, top_p=0.9, max_tokens=6,
                                                             ignore_eos=True))
    assert len(sampled[0]["token_ids"]) == 6
