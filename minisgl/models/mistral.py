"""MistralForCausalLM: the shared decoder with qk_norm=False, qkv bias=False, MoE MLP=False."""

from .decoder import DecoderForCausalLM


class MistralForCausalLM(DecoderForCausalLM):
    QK_NORM = False
    ATTN_BIAS = False
    MOE = False


__all__ = ["MistralForCausalLM"]
