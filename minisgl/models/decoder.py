"""The decoder skeleton shared by Llama, Qwen2, Qwen3, Qwen3-MoE and
Mistral: embed -> N x (add+norm, attention, add+norm, MLP) -> norm -> LM
head. Family differences are constructor flags (qkv bias, q/k norm, MoE)."""

from __future__ import annotations

from typing import TYPE_CHECKING, Dict, Optional, Tuple

import torch

from minisgl import ops
from minisgl.core import get_global_ctx
from minisgl.layers import BaseOP, OPList, ParallelLMHead, RMSNormFused, VocabParallelEmbedding
from minisgl.utils import nvtx_annotate

from .base import BaseLLMModel
from .utils import GatedMLP, MoEMLP, RopeAttn

if TYPE_CHECKING:
    from .config import ModelConfig

# batches of up to this many tokens (every CUDA-graph decode batch) take the
# fused-epilogue path: 4 GEMMs per layer instead of 4 GEMMs + 4 row kernels
# (per-layer chain on a B200: 14-22% faster at 1-128 tokens, even at 256);
# longer prefill chunks take the token-major GEMMs plus separate kernels
FUSED_MAX_TOKENS = 256


class DecoderLayer(BaseOP):
    """One block. Two equivalent forward paths over the same weights:

    * ``forward`` (long prefill chunks): norm, projections, RoPE / KV store,
      attention and activation as separate kernels (GEMMs with the best
      token-major tiles);
    * ``forward_fused`` (decode and short chunks): four GEMMs per layer whose
      epilogues carry the RMSNorms, q/k-norm + RoPE + KV store, SiLU x up and
      both residual adds; the residual stream is updated in place.

    After loading, the input / post-attention RMSNorm weights are folded into
    the columns of the qkv / gate_up weights (norm(x) @ W^T = rstd(x) *
    (x @ (W diag(g))^T)), and gate|up rows are interleaved in 64-row blocks;
    the unfused path then runs weightless norms and the interleaved
    activation, so both paths compute the same function.
    """

    def __init__(self, config: "ModelConfig", layer_id: int, *, qk_norm: bool, attn_bias: bool, moe: bool) -> None:
        self.self_attn = RopeAttn(config, layer_id, has_attn_bias=attn_bias, has_qk_norm=qk_norm)
        self.mlp = MoEMLP(config) if moe else GatedMLP(config)
        self.input_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self._layer_id = layer_id
        self._fused_attn = self.self_attn.attn.fusable
        # the MLP is only refolded when the whole layer takes the fused path
        self._fused_mlp = self._fused_attn and isinstance(self.mlp, GatedMLP) and self.mlp.fusable

    @property
    def fusable(self) -> bool:
        return self._fused_attn

    def post_load(self) -> None:
        super().post_load()
        if self._fused_attn and not self.input_layernorm.folded:
            qkv = self.self_attn.qkv_proj
            g = self.input_layernorm.weight
            qkv.weight = (qkv.weight.float() * g.float()[None, :]).to(qkv.weight.dtype).contiguous()
            self.input_layernorm.fold()
        if self._fused_mlp and not self.post_attention_layernorm.folded:
            gu = self.mlp.gate_up_proj
            g = self.post_attention_layernorm.weight
            gu.weight = (gu.weight.float() * g.float()[None, :]).to(gu.weight.dtype)
            self.mlp.interleave()
            self.post_attention_layernorm.fold()

    @nvtx_annotate("Layer_{}", layer_id_field="_layer_id")
    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor]) -> Tuple[torch.Tensor, torch.Tensor]:
        x, residual = self.input_layernorm.forward(x, residual)
        x = self.self_attn.forward(x)
        x, residual = self.post_attention_layernorm.forward(x, residual)
        return self.mlp.forward(x), residual

    @nvtx_annotate("Layer_{}", layer_id_field="_layer_id")
    def forward_fused(self, r: torch.Tensor) -> torch.Tensor:
        """The residual stream after this layer (``r`` is updated in place on
        one rank)."""
        r = self.self_attn.forward_fused(r, self.input_layernorm.eps)
        if self._fused_mlp:
            return self.mlp.forward_fused(r, self.post_attention_layernorm.eps)
        h = ops.rmsnorm(r, self.post_attention_layernorm.weight, self.post_attention_layernorm.eps)
        return r.add_(self.mlp.forward(h))


class DecoderModel(BaseOP):
    def __init__(self, config: "ModelConfig", **flags: bool) -> None:
        self.embed_tokens = VocabParallelEmbedding(config.vocab_size, config.hidden_size)
        self.layers = OPList([DecoderLayer(config, i, **flags) for i in range(config.num_layers)])
        self.norm = RMSNormFused(config.hidden_size, config.rms_norm_eps)

    @property
    def fusable(self) -> bool:
        return all(layer.fusable for layer in self.layers.op_list)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        x = self.embed_tokens.forward(input_ids)
        if self.fusable and x.shape[0] <= FUSED_MAX_TOKENS:
            r = x  # a fresh buffer: the residual stream is updated in place
            for layer in self.layers.op_list:
                r = layer.forward_fused(r)
            return self.norm.forward(r, None)[0]
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

    @property
    def samples_in_lm_head(self) -> bool:
        """The LM head can return sampled tokens (one rank holds the whole vocabulary)."""
        return self.lm_head.tp_size == 1

    @property
    def fused_layout(self) -> bool:
        """True when norm weights are folded into qkv / gate_up and gate|up
        rows are interleaved (what ``state_dict`` then returns)."""
        return any(l.input_layernorm.folded for l in self.model.layers.op_list)

    def fused_gemm_kinds(self) -> Dict[Tuple[int, int], Tuple[int, int, int]]:
        """(N, K) of each projection the fused decode path runs -> (epilogue
        kind, local q heads, local kv heads), for the GEMM autotuner."""
        out: Dict[Tuple[int, int], Tuple[int, int, int]] = {}
        if not self.model.fusable:
            return out
        for layer in self.model.layers.op_list:
            attn = layer.self_attn
            hq, hk = attn.attn.num_qo_heads, attn.attn.num_kv_heads
            out[tuple(attn.qkv_proj.weight.shape)] = (ops.EPI_NORM | ops.EPI_ROPE, hq, hk)
            out[tuple(attn.o_proj.weight.shape)] = (ops.EPI_RESIDUAL, hq, hk)
            if layer._fused_mlp:
                out[tuple(layer.mlp.gate_up_proj.weight.shape)] = (ops.EPI_NORM | ops.EPI_SILU, hq, hk)
                out[tuple(layer.mlp.down_proj.weight.shape)] = (ops.EPI_RESIDUAL, hq, hk)
        if self.samples_in_lm_head:
            head = self.lm_head._tied.weight if self.lm_head._tied is not None else self.lm_head.weight
            out[tuple(head.shape)] = (ops.EPI_SAMPLE, 0, 0)
        return out

    def forward(self) -> torch.Tensor:
        hidden = self.model.forward(get_global_ctx().batch.input_ids)
        return self.lm_head.forward(hidden)
