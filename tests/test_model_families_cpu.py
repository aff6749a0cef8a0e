"""The dense decoder families the reference serves besides Qwen3 (its
python/minisgl/models/register.py:5-12): Llama (llama3 RoPE scaling),
Qwen2 (q/k/v biases, no q/k norm) and Mistral, each through the CPU engine
(paged, chunked, radix-cached) against the dense fp32 oracle, token for
token, from a checkpoint whose biases and norm weights are not trivial."""

import random
import shutil
import tempfile

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.llm import LLM
from minisgl.models.oracle import greedy_generate
from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint


@pytest.mark.parametrize("shape,arch", [("tiny-llama", "LlamaForCausalLM"), ("tiny-qwen2", "Qwen2ForCausalLM"),
                                        ("tiny-mistral", "MistralForCausalLM")])
def test_family_matches_dense_oracle(shape, arch):
    folder = tempfile.mkdtemp(prefix=f"minisgl_{shape}_")
    shutil.rmtree(folder)
    make_model_dir(shape, folder=folder)
    write_random_checkpoint(folder, seed=3, std=0.05, norm_std=0.3)
    llm = LLM(folder, dtype=torch.float32, device="cpu", page_size=16, max_extend_tokens=32, num_page_override=128,
              max_running_req=8, max_seq_len_override=512, cache_type="radix")
    try:
        model = llm.engine.model
        assert type(model).__name__ == arch
        state = model.state_dict()
        has_bias = any(k.endswith("qkv_proj.bias") for k in state)
        assert has_bias == (shape == "tiny-qwen2")
        if has_bias:  # the biases are drawn, not zero: they take part in the comparison
            assert any(v.abs().sum() > 0 for k, v in state.items() if k.endswith("qkv_proj.bias"))
        rng = random.Random(1)
        prompts = [[rng.randrange(1024) for _ in range(rng.randint(20, 60))] for _ in range(4)]
        outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True))
        for p, o in zip(prompts, outs):
            want = greedy_generate(state, llm.engine.model_config, p, 10,
                                   fused_layout=getattr(model, "fused_layout", False))
            assert o["token_ids"] == want, (shape, p)
        llm.cache_manager.check_integrity()
    finally:
        llm.shutdown()
        shutil.rmtree(folder, ignore_errors=True)
