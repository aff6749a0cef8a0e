"""Qwen2ForCausalLM: the shared decoder with qk_norm=False, qkv bias=True, MoE MLP=False."""

from .decoder import DecoderForCausalLM


class Qwen2ForCausalLM(DecoderForCausalLM):
    QK_NORM = False
    ATTN_BIAS = True
    MOE = False


__all__ = ["Qwen2ForCausalLM"]
