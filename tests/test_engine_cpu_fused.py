"""The fused-epilogue decoder path on the CPU: head_dim 128 (so the qkv /
o / gate_up / down GEMMs carry the norms, RoPE + KV store, SiLU and residual
adds) and non-unit norm weights (so folding them into the projections is
exercised), checked token for token against the dense fp32 oracle run on the
original, unfolded checkpoint. Long prompts take the unfused path over the
same folded weights."""

import os
import random
import tempfile

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.llm import LLM
from minisgl.models.oracle import greedy_generate
from minisgl.models.weight import load_weight
from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

SHAPE = dict(head_dim=128, num_attention_heads=2, num_key_value_heads=1, hidden_size=256,
             intermediate_size=512, tie_word_embeddings=False)


@pytest.fixture(scope="module")
def model_dir():
    folder = os.path.join(tempfile.mkdtemp(prefix="minisgl_fused_"), "m")
    make_model_dir("tiny-qwen3", folder=folder, overrides=SHAPE)
    write_random_checkpoint(folder, seed=7, std=0.05, norm_std=0.3)
    return folder


@pytest.fixture(scope="module")
def llm(model_dir):
    engine = LLM(model_dir, dtype=torch.float32, device="cpu", use_dummy_weight=False, page_size=16,
                 max_extend_tokens=512, num_page_override=256, max_running_req=8, max_seq_len_override=1024,
                 cache_type="radix")
    yield engine
    engine.shutdown()


def _oracle(llm, model_dir, prompt, n):
    state = dict(load_weight(model_dir, torch.device("cpu")))
    return greedy_generate(state, llm.engine.model_config, prompt, n)


def test_fused_layout_is_active(llm):
    assert llm.engine.model.fused_layout
    assert llm.engine.model.model.fusable


@pytest.mark.parametrize("length", [24, 300])
def test_fused_path_matches_unfolded_oracle(llm, model_dir, length):
    rng = random.Random(length)
    prompts = [[rng.randrange(1024) for _ in range(length + i)] for i in range(3)]
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert o["token_ids"] == _oracle(llm, model_dir, p, 8)
    llm.cache_manager.check_integrity()
