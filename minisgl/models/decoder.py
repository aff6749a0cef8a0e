"""The decoder skeleton shared by Llama, Qwen2, Qwen3, Qwen3-MoE and
Mistral: embed -> N x (add+norm, attention, add+norm, MLP) -> norm -> LM
head. Family differences are constructor flags (qkv bias, q/k norm, MoE)."""

from __future__ import annotations

from typing import TYPE_CHECKING, Optional, Tuple

import torch

from minisgl.core import get_global_ctx
from minisgl.layers import BaseOP, OPList, ParallelLMHead, RMSNormFused, VocabParallelEmbedding
from minisgl.utils import nvtx_annotate

from .base import BaseLLMModel
from .utils import GatedMLP, MoEMLP, RopeAttn

if TYPE_CHECKING:
    from .config import ModelConfig


class DecoderLayer(BaseOP):
    def __init__(self, config: "ModelConfig", layer_id: int, *, qk_norm: bool, attn_bias: bool, moe: bool) -> None:
        self.self_attn = RopeAttn(config, layer_id, has_attn_bias=attn_bias, has_qk_norm=qk_norm)
        self.mlp = MoEMLP(config) if moe else GatedMLP(config)
        self.input_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self._layer_id = layer_id

    @nvtx_annotate("Layer_{}", layer_id_field="_layer_id")
    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor]) -> Tuple[torch.Tensor, torch.Tensor]:
        x, residual = self.input_layernorm.forward(x, residual)
        x = self.self_attn.forward(x)
        x, residual = self.post_attention_layernorm.forward(x, residual)
        return self.mlp.forward(x), residual


class DecoderModel(BaseOP):
    def __init__(self, config: "ModelConfig", **flags: bool) -> None:
        self.embed_tokens = VocabParallelEmbedding(config.vocab_size, config.hidden_size)
        self.layers = OPList([DecoderLayer(config, i, **flags) for i in range(config.num_layers)])
        self.norm = RMSNormFused(config.hidden_size, config.rms_norm_eps)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        x = self.embed_tokens.forward(input_ids)
        residual: Optional[torch.Tensor] = None
        for layer in self.layers.op_list:
            x, residual = layer.forward(x, residual)
        return self.norm.forward(x, residual)[0]


class DecoderForCausalLM(BaseLLMModel):
    QK_NORM = False
    ATTN_BIAS = False
    MOE = False

    def __init__(self, config: "ModelConfig") -> None:
        self.model = DecoderModel(config, qk_norm=self.QK_NORM, attn_bias=self.ATTN_BIAS, moe=self.MOE)
        tied = config.tie_word_embeddings
        self.lm_head = ParallelLMHead(config.vocab_size, config.hidden_size, tie_word_embeddings=tied,
                                      tied_embedding=self.model.embed_tokens if tied else None)

    def forward(self) -> torch.Tensor:
        hidden = self.model.forward(get_global_ctx().batch.input_ids)
        return self.lm_head.forward(hidden)
