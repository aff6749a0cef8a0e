"""Qwen3ForCausalLM: the shared decoder with qk_norm=True, qkv bias=False, MoE MLP=False."""

from .decoder import DecoderForCausalLM


class Qwen3ForCausalLM(DecoderForCausalLM):
    QK_NORM = True
    ATTN_BIAS = False
    MOE = False


__all__ = ["Qwen3ForCausalLM"]
