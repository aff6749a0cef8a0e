"""The Llama, Qwen2 (q/k/v biases, no q/k norm) and Mistral families on a
B200: bf16 engine from a checkpoint with non-unit norm weights and drawn
biases, each generated token checked against the dense fp32 oracle of the
checkpoint as written (teacher forcing: the oracle's argmax or within a
small logit margin of it, as for Qwen3 in test_engine_gpu)."""

import os
import random

import pytest
import torch

from minisgl import ops
from minisgl.core import SamplingParams
from minisgl.llm import LLM
from minisgl.models.oracle import dense_logits
from minisgl.models.weight import load_weight
from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

pytestmark = pytest.mark.gpu

# the tiny CPU shapes at the sizes the sm_100a kernels take (head_dim 128)
_GPU_SIZE = dict(hidden_size=1024, num_attention_heads=8, num_key_value_heads=4, head_dim=128,
                 intermediate_size=3072, vocab_size=4096, max_position_embeddings=8192, torch_dtype="bfloat16")


@pytest.mark.parametrize("shape", ["tiny-llama", "tiny-qwen2", "tiny-mistral"])
def test_family_tracks_oracle(shape, tmp_path):
    folder = os.path.join(str(tmp_path), shape)
    make_model_dir(shape, folder=folder, overrides=_GPU_SIZE)
    write_random_checkpoint(folder, seed=5, std=0.05, norm_std=0.3)
    llm = LLM(folder, dtype=torch.bfloat16, device="cuda:0", page_size=64, max_running_req=16,
              max_seq_len_override=2048, num_page_override=256, cuda_graph_max_bs=16, max_extend_tokens=256)
    try:
        rng = random.Random(3)
        prompts = [[rng.randrange(4096) for _ in range(rng.randint(20, 300))] for _ in range(6)]
        outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
        ops.check_device_errors(torch.device("cuda:0"))
        state = {k: v.float() for k, v in load_weight(folder, torch.device("cpu"))}
        assert any(k.endswith("qkv_proj.bias") for k in state) == (shape == "tiny-qwen2")
        cfg = llm.engine.model_config
        exact = total = 0
        for p, o in zip(prompts, outs):
            toks = o["token_ids"]
            assert len(toks) == 12
            logits = dense_logits(state, cfg, p + toks[:-1], fused_layout=False)[len(p) - 1:]
            for t, row in zip(toks, logits):
                assert row[t] >= row.max() - 0.03 * row.abs().max(), (shape, t, int(row.argmax()))
                exact += int(t == int(row.argmax()))
                total += 1
        assert exact >= 0.8 * total, (shape, exact, total)
    finally:
        llm.shutdown()
