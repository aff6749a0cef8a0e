"""DeepSeek-V3 / Kimi-K2 architecture on the CPU: the engine's absorbed MLA
over the paged latent cache, with routed + shared experts, must reproduce a
dense fp32 oracle that decompresses K / V for every head."""

import random

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.llm import LLM
from minisgl.models.oracle import greedy_generate
from minisgl.utils.synthetic import make_model_dir


@pytest.fixture(scope="module")
def llm():
    d = make_model_dir("tiny-kimi")
    engine = LLM(d, dtype=torch.float32, device="cpu", use_dummy_weight=True, page_size=16, max_extend_tokens=32,
                 num_page_override=128, max_running_req=8, max_seq_len_override=512, cache_type="radix")
    yield engine
    engine.shutdown()


def test_tiny_kimi_matches_dense_mla_oracle(llm):
    rng = random.Random(3)
    prompts = [[rng.randrange(1024) for _ in range(rng.randint(8, 48))] for _ in range(4)]
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True))
    model = llm.engine.model
    for p, o in zip(prompts, outs):
        assert o["token_ids"] == greedy_generate(model.state_dict(), llm.engine.model_config, p, 10)
    llm.cache_manager.check_integrity()


def test_latent_cache_is_one_row_per_token(llm):
    pool = llm.engine.kv_cache
    cfg = llm.engine.model_config
    assert pool.latent(0).shape[-1] == cfg.kv_lora_rank + cfg.qk_rope_head_dim
    assert pool.v_cache(0).shape[-1] == cfg.kv_lora_rank

