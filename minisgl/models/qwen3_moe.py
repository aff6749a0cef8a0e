"""Qwen3MoeForCausalLM: the shared decoder with qk_norm=True, qkv bias=False, MoE MLP=True."""

from .decoder import DecoderForCausalLM


class Qwen3MoeForCausalLM(DecoderForCausalLM):
    QK_NORM = True
    ATTN_BIAS = False
    MOE = True


__all__ = ["Qwen3MoeForCausalLM"]
