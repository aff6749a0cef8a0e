"""Synthetic model folders for benchmarks and tests (no network needed).

``make_model_dir("qwen3-0.6b")`` writes a Hugging Face style folder with a
``config.json`` of the named shape and a word-level tokenizer covering the
whole vocabulary (token ``i`` is the word ``t{i}``). Engines started on it
with ``use_dummy_weight=True`` (``--dummy-weight``) draw random weights, so
the shapes, kernels and scheduling are real while no checkpoint is read.
"""

from __future__ import annotations

import copy
import hashlib
import json
import os
import shutil
import tempfile
from typing import Any, Dict, Optional

_QWEN3_BASE: Dict[str, Any] = {
    "model_type": "qwen3",
    "architectures": ["Qwen3ForCausalLM"],
    "hidden_act": "silu",
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "max_position_embeddings": 40960,
    "torch_dtype": "bfloat16",
    "bos_token_id": 0,
    "eos_token_id": 1,
    "attention_bias": False,
}

SHAPES: Dict[str, Dict[str, Any]] = {
    # tiny Qwen3-style decoder for CPU tests (fp32)
    "tiny-qwen3": dict(_QWEN3_BASE, num_hidden_layers=2, hidden_size=256, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=64, intermediate_size=512, vocab_size=1024,
                       tie_word_embeddings=True, max_position_embeddings=4096, torch_dtype="float32"),
    # Qwen3-0.6B: the reference's offline-benchmark model
    "qwen3-0.6b": dict(_QWEN3_BASE, num_hidden_layers=28, hidden_size=1024, num_attention_heads=16,
                       num_key_value_heads=8, head_dim=128, intermediate_size=3072, vocab_size=151936,
                       tie_word_embeddings=True),
    # small GPU smoke / numerics shape (head_dim 128 like the real models)
    "small-qwen3": dict(_QWEN3_BASE, num_hidden_layers=2, hidden_size=1024, num_attention_heads=16,
                        num_key_value_heads=8, head_dim=128, intermediate_size=3072, vocab_size=4096,
                        tie_word_embeddings=False, max_position_embeddings=8192),
    # Qwen3-32B: the tensor-parallel serving benchmark model
    "qwen3-32b": dict(_QWEN3_BASE, num_hidden_layers=64, hidden_size=5120, num_attention_heads=64,
                      num_key_value_heads=8, head_dim=128, intermediate_size=25600, vocab_size=151936,
                      tie_word_embeddings=False),
    "qwen3-8b": dict(_QWEN3_BASE, num_hidden_layers=36, hidden_size=4096, num_attention_heads=32,
                     num_key_value_heads=8, head_dim=128, intermediate_size=12288, vocab_size=151936,
                     tie_word_embeddings=False),
    "qwen3-30b-a3b": dict(_QWEN3_BASE, model_type="qwen3_moe", architectures=["Qwen3MoeForCausalLM"],
                          num_hidden_layers=48, hidden_size=2048, num_attention_heads=32, num_key_value_heads=4,
                          head_dim=128, intermediate_size=6144, moe_intermediate_size=768, num_experts=128,
                          num_experts_per_tok=8, norm_topk_prob=True, vocab_size=151936,
                          tie_word_embeddings=False),
    "tiny-qwen3-moe": dict(_QWEN3_BASE, model_type="qwen3_moe", architectures=["Qwen3MoeForCausalLM"],
                           num_hidden_layers=2, hidden_size=256, num_attention_heads=4, num_key_value_heads=2,
                           head_dim=64, intermediate_size=512, moe_intermediate_size=128, num_experts=8,
                           num_experts_per_tok=2, norm_topk_prob=True, vocab_size=1024,
                           tie_word_embeddings=False, max_position_embeddings=4096, torch_dtype="float32"),
    "tiny-llama": {
        "model_type": "llama", "architectures": ["LlamaForCausalLM"], "hidden_act": "silu", "rms_norm_eps": 1e-5,
        "rope_theta": 500000.0, "max_position_embeddings": 4096, "num_hidden_layers": 2, "hidden_size": 256,
        "num_attention_heads": 4, "num_key_value_heads": 2, "intermediate_size": 512, "vocab_size": 1024,
        "tie_word_embeddings": False, "torch_dtype": "float32", "bos_token_id": 0, "eos_token_id": 1,
        "rope_scaling": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                         "original_max_position_embeddings": 1024},
    },
    # Qwen2 (q/k/v biases, no q/k norm) and Mistral (Llama-style, plain RoPE)
    "tiny-qwen2": {
        "model_type": "qwen2", "architectures": ["Qwen2ForCausalLM"], "hidden_act": "silu", "rms_norm_eps": 1e-6,
        "rope_theta": 1000000.0, "max_position_embeddings": 4096, "num_hidden_layers": 2, "hidden_size": 256,
        "num_attention_heads": 4, "num_key_value_heads": 2, "intermediate_size": 512, "vocab_size": 1024,
        "tie_word_embeddings": False, "torch_dtype": "float32", "bos_token_id": 0, "eos_token_id": 1,
    },
    "tiny-mistral": {
        "model_type": "mistral", "architectures": ["MistralForCausalLM"], "hidden_act": "silu",
        "rms_norm_eps": 1e-5, "rope_theta": 10000.0, "max_position_embeddings": 4096, "num_hidden_layers": 2,
        "hidden_size": 256, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
        "intermediate_size": 512, "vocab_size": 1024, "tie_word_embeddings": False, "torch_dtype": "float32",
        "bos_token_id": 0, "eos_token_id": 1, "sliding_window": None,
    },
    # Kimi-K2 shape (DeepSeek-V3 architecture): expert / context parallel benchmarks
    "kimi-k2": {
        "model_type": "kimi_k2", "architectures": ["DeepseekV3ForCausalLM"], "hidden_act": "silu",
        "rms_norm_eps": 1e-6, "rope_theta": 50000.0, "max_position_embeddings": 262144,
        "num_hidden_layers": 61, "hidden_size": 7168, "num_attention_heads": 64, "num_key_value_heads": 64,
        "intermediate_size": 18432, "moe_intermediate_size": 2048, "n_routed_experts": 384, "n_shared_experts": 1,
        "num_experts_per_tok": 8, "first_k_dense_replace": 1, "n_group": 1, "topk_group": 1,
        "norm_topk_prob": True, "routed_scaling_factor": 2.827, "scoring_func": "sigmoid",
        "q_lora_rank": 1536, "kv_lora_rank": 512, "qk_nope_head_dim": 128, "qk_rope_head_dim": 64,
        "v_head_dim": 128, "vocab_size": 163840, "tie_word_embeddings": False, "torch_dtype": "bfloat16",
        "bos_token_id": 0, "eos_token_id": 1,
        "rope_scaling": {"type": "yarn", "factor": 32.0, "beta_fast": 1.0, "beta_slow": 1.0, "mscale": 1.0,
                         "mscale_all_dim": 1.0, "original_max_position_embeddings": 4096},
    },
}
SHAPES["tiny-kimi"] = dict(copy.deepcopy(SHAPES["kimi-k2"]), num_hidden_layers=2, hidden_size=256,
                           num_attention_heads=4, num_key_value_heads=4, intermediate_size=512,
                           moe_intermediate_size=128, n_routed_experts=8, num_experts_per_tok=2,
                           q_lora_rank=96, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=16,
                           v_head_dim=32, vocab_size=1024, torch_dtype="float32", max_position_embeddings=4096)

# GPU tests: the Kimi-K2 latent dims (kv_lora 512, rope 64) that the sm_100a
# MLA kernels take, on a 2-layer model (layer 0 dense, layer 1 MoE)
SHAPES["small-kimi"] = dict(copy.deepcopy(SHAPES["kimi-k2"]), num_hidden_layers=2, hidden_size=1024,
                            num_attention_heads=16, num_key_value_heads=16, intermediate_size=2048,
                            moe_intermediate_size=256, n_routed_experts=8, num_experts_per_tok=2,
                            q_lora_rank=384, vocab_size=4096, max_position_embeddings=8192)

_CHAT_TEMPLATE = (
    "{% for m in messages %}<|{{ m['role'] }}|>{{ m['content'] }}<|end|>{% endfor %}"
    "{% if add_generation_prompt %}<|assistant|>{% endif %}"
)


def _write_tokenizer(folder: str, vocab_size: int) -> None:
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {f"t{i}": i for i in range(vocab_size)}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="t2"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, bos_token="t0", eos_token="t1", unk_token="t2",
                                   pad_token="t3")
    fast.chat_template = _CHAT_TEMPLATE
    fast.save_pretrained(folder)


def make_model_dir(shape: str, folder: Optional[str] = None, overrides: Optional[Dict[str, Any]] = None) -> str:
    """Create (or reuse) a synthetic model folder of a named shape."""
    if shape not in SHAPES:
        raise KeyError(f"unknown synthetic shape {shape!r}; have {sorted(SHAPES)}")
    cfg = dict(copy.deepcopy(SHAPES[shape]), **(overrides or {}))
    if folder is None:
        key = hashlib.sha1(json.dumps(cfg, sort_keys=True).encode()).hexdigest()[:12]
        folder = os.path.join(tempfile.gettempdir(), f"minisgl_synthetic_{shape}_{key}")
    if os.path.isfile(os.path.join(folder, "config.json")):
        return folder
    # build in a private folder, then publish it with one rename (several
    # ranks may race to create the same folder)
    parent = os.path.dirname(os.path.abspath(folder))
    os.makedirs(parent, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix=".tmp_minisgl_", dir=parent)
    _write_tokenizer(tmp, cfg["vocab_size"])
    with open(os.path.join(tmp, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    try:
        os.rename(tmp, folder)
    except OSError:  # another process won the race (or the folder exists)
        shutil.rmtree(tmp, ignore_errors=True)
        if not os.path.isfile(os.path.join(folder, "config.json")):
            os.makedirs(folder, exist_ok=True)
            _write_tokenizer(folder, cfg["vocab_size"])
            with open(os.path.join(folder, "config.json"), "w") as f:
                json.dump(cfg, f, indent=1)
    return folder


def write_random_checkpoint(folder: str, seed: int = 0, std: float = 0.02, norm_std: float = 0.0) -> str:
    """Write HF-named random weights (``model.safetensors``) for the config
    in ``folder``: separate q/k/v and gate/up projections, per-expert tensors,
    exactly as a downloaded checkpoint is laid out. Norm weights are
    1 + N(0, norm_std) (exactly one with the default 0)."""
    import torch
    from safetensors.torch import save_file

    with open(os.path.join(folder, "config.json")) as f:
        c = json.load(f)
    g = torch.Generator().manual_seed(seed)
    dt = {"bfloat16": torch.bfloat16, "float16": torch.float16}.get(c.get("torch_dtype"), torch.float32)

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * std).to(dt)

    def norm_w(n):
        return (1.0 + torch.randn(n, generator=g) * norm_std).to(dt) if norm_std > 0 else torch.ones(n, dtype=dt)

    H, V = c["hidden_size"], c["vocab_size"]
    hq, hk = c["num_attention_heads"], c.get("num_key_value_heads", c["num_attention_heads"])
    d = c.get("head_dim") or H // hq
    W = {"model.embed_tokens.weight": rnd(V, H), "model.norm.weight": torch.ones(H, dtype=dt)}
    if not c.get("tie_word_embeddings", False):
        W["lm_head.weight"] = rnd(V, H)
    moe = c.get("num_experts", 0) > 0
    if c.get("kv_lora_rank"):
        return _write_deepseek(folder, c, W, rnd, norm_w, dt)
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}."
        W[p + "input_layernorm.weight"] = norm_w(H)
        W[p + "post_attention_layernorm.weight"] = norm_w(H)
        W[p + "self_attn.q_proj.weight"] = rnd(hq * d, H)
        W[p + "self_attn.k_proj.weight"] = rnd(hk * d, H)
        W[p + "self_attn.v_proj.weight"] = rnd(hk * d, H)
        W[p + "self_attn.o_proj.weight"] = rnd(H, hq * d)
        if c.get("model_type", "").startswith("qwen3"):
            W[p + "self_attn.q_norm.weight"] = norm_w(d)
            W[p + "self_attn.k_norm.weight"] = norm_w(d)
        if c.get("model_type") == "qwen2":
            for n, size in (("q", hq * d), ("k", hk * d), ("v", hk * d)):
                W[p + f"self_attn.{n}_proj.bias"] = rnd(size)
        if moe:
            I = c["moe_intermediate_size"]
            W[p + "mlp.gate.weight"] = rnd(c["num_experts"], H)
            for e in range(c["num_experts"]):
                q = p + f"mlp.experts.{e}."
                W[q + "gate_proj.weight"] = rnd(I, H)
                W[q + "up_proj.weight"] = rnd(I, H)
                W[q + "down_proj.weight"] = rnd(H, I)
        else:
            I = c["intermediate_size"]
            W[p + "mlp.gate_proj.weight"] = rnd(I, H)
            W[p + "mlp.up_proj.weight"] = rnd(I, H)
            W[p + "mlp.down_proj.weight"] = rnd(H, I)
    save_file({k: v.contiguous() for k, v in W.items()}, os.path.join(folder, "model.safetensors"))
    return folder


def _write_deepseek(folder: str, c: dict, W: dict, rnd, norm_w, dt) -> str:
    """DeepSeek-V3 / Kimi-K2 HF layout: MLA projections (q LoRA, compressed
    KV with the shared positional key, kv_b up-projection), dense MLP for
    the first ``first_k_dense_replace`` layers, then the router (weight and
    fp32 score-correction bias), per-expert routed MLPs and the shared
    expert."""
    import torch
    from safetensors.torch import save_file

    H, hq = c["hidden_size"], c["num_attention_heads"]
    nope, rope, vd = c["qk_nope_head_dim"], c["qk_rope_head_dim"], c["v_head_dim"]
    qlr, kvl = c.get("q_lora_rank") or 0, c["kv_lora_rank"]
    E, I, Id = c["n_routed_experts"], c["moe_intermediate_size"], c["intermediate_size"]
    shared = c.get("n_shared_experts", 0) or 0
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        W[p + "input_layernorm.weight"] = norm_w(H)
        W[p + "post_attention_layernorm.weight"] = norm_w(H)
        if qlr:
            W[a + "q_a_proj.weight"] = rnd(qlr, H)
            W[a + "q_a_layernorm.weight"] = norm_w(qlr)
            W[a + "q_b_proj.weight"] = rnd(hq * (nope + rope), qlr)
        else:
            W[a + "q_proj.weight"] = rnd(hq * (nope + rope), H)
        W[a + "kv_a_proj_with_mqa.weight"] = rnd(kvl + rope, H)
        W[a + "kv_a_layernorm.weight"] = norm_w(kvl)
        W[a + "kv_b_proj.weight"] = rnd(hq * (nope + vd), kvl)
        W[a + "o_proj.weight"] = rnd(H, hq * vd)
        m = p + "mlp."
        if i < c.get("first_k_dense_replace", 0) or E == 0:
            W[m + "gate_proj.weight"] = rnd(Id, H)
            W[m + "up_proj.weight"] = rnd(Id, H)
            W[m + "down_proj.weight"] = rnd(H, Id)
            continue
        W[m + "gate.weight"] = rnd(E, H)
        if c.get("scoring_func") == "sigmoid":
            W[m + "gate.e_score_correction_bias"] = (torch.randn(E) * 0.01).float()
        for e in range(E):
            q = m + f"experts.{e}."
            W[q + "gate_proj.weight"] = rnd(I, H)
            W[q + "up_proj.weight"] = rnd(I, H)
            W[q + "down_proj.weight"] = rnd(H, I)
        if shared:
            W[m + "shared_experts.gate_proj.weight"] = rnd(I * shared, H)
            W[m + "shared_experts.up_proj.weight"] = rnd(I * shared, H)
            W[m + "shared_experts.down_proj.weight"] = rnd(H, I * shared)
    save_file({k: v.contiguous() for k, v in W.items()}, os.path.join(folder, "model.safetensors"))
    return folder
