"""HF ``architectures`` name -> model class."""

from __future__ import annotations

import importlib

from .config import ModelConfig

_MODELS = {
    "LlamaForCausalLM": (".llama", "LlamaForCausalLM"),
    "Qwen2ForCausalLM": (".qwen2", "Qwen2ForCausalLM"),
    "Qwen3ForCausalLM": (".qwen3", "Qwen3ForCausalLM"),
    "Qwen3MoeForCausalLM": (".qwen3_moe", "Qwen3MoeForCausalLM"),
    "MistralForCausalLM": (".mistral", "MistralForCausalLM"),
    "Mistral3ForConditionalGeneration": (".mistral", "MistralForCausalLM"),
    "DeepseekV3ForCausalLM": (".deepseek_v3", "DeepseekV3ForCausalLM"),
    "KimiK2ForCausalLM": (".deepseek_v3", "DeepseekV3ForCausalLM"),
}


def supported_architectures():
    return list(_MODELS)


def get_model_class(architecture: str, config: ModelConfig):
    if architecture not in _MODELS:
        raise ValueError(f"model architecture {architecture} is not supported")
    module, name = _MODELS[architecture]
    cls = getattr(importlib.import_module(module, package=__package__), name)
    return cls(config)
