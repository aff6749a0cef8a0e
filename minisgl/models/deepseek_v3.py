"""DeepSeek-V3 / Kimi-K2: multi-head latent attention (MLA) + routed experts
with a shared expert (not in the reference, whose registry stops at
Qwen3-MoE / Mistral; python/minisgl/models/register.py:5-12).

Per layer (HF names kept, so DeepSeek-V3 / Kimi-K2 checkpoints load):

* attention: q = q_b_proj(q_a_layernorm(q_a_proj(x))) (or q_proj without a
  q LoRA), [T, heads, qk_nope + qk_rope]; kv_a_proj_with_mqa(x) gives the
  compressed KV (kv_lora_rank, normalised by kv_a_layernorm) and one shared
  positional key (qk_rope). The latent row [c_kv | rope(k_pe)] is cached.
  Prefill batches whose keys are long enough run the non-absorbed form
  (every key's c_kv expanded through kv_b_proj into per-head k_nope / v,
  then 192 / 128-dim attention: ``ops.mla_prefill_attention``); decode and
  short prefills run the absorbed form: q_nope goes into the latent space
  through W_UK (the first qk_nope rows of each head of kv_b_proj), scores are
  q_lat . c_kv + q_pe . k_pe, the latent output comes back through W_UV (the
  last v_head_dim rows) and o_proj. RoPE is DeepSeek's interleaved (GPT-J)
  form: element pairs (2i, 2i + 1) rotate by frequency i.
* MLP: dense SwiGLU for the first ``first_k_dense_replace`` layers, then the
  router (sigmoid scores + e_score_correction_bias, group-limited top-k,
  ``routed_scaling_factor``) over the routed experts plus the shared expert;
  both partial sums meet in one tensor-parallel reduction.
"""

from __future__ import annotations

from typing import TYPE_CHECKING, Optional, Tuple

import torch

from minisgl import ops
from minisgl.core import get_global_ctx
from minisgl.layers import (
    BaseOP,
    LinearColParallelMerged,
    LinearOProj,
    LinearReplicated,
    OPList,
    ParallelLMHead,
    RMSNorm,
    RMSNormFused,
    VocabParallelEmbedding,
)
from minisgl.layers.moe import MoELayer
from minisgl.layers.rotary import get_rope
from minisgl.parallel import DistributedCommunicator, get_tp_info
from minisgl.utils import div_even

from .base import BaseLLMModel
from .utils import GatedMLP

if TYPE_CHECKING:
    from .config import ModelConfig


class _CPComm:
    """All-reduce over the context-parallel ranks (the whole world: layers
    see a single tensor-parallel rank under context parallelism)."""

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        dist.all_reduce(x)
        return x


class MLAAttention(BaseOP):
    def __init__(self, config: "ModelConfig", layer_id: int) -> None:
        tp = get_tp_info().size
        self.heads = div_even(config.num_qo_heads, tp)
        self.nope = config.qk_nope_head_dim
        self.rope_dim = config.qk_rope_head_dim
        self.v_dim = config.v_head_dim
        self.kv_lora = config.kv_lora_rank
        self.eps = config.rms_norm_eps
        qk = self.nope + self.rope_dim
        H, heads_full = config.hidden_size, config.num_qo_heads
        if config.q_lora_rank > 0:
            self.q_a_proj = LinearReplicated(H, config.q_lora_rank, has_bias=False)
            self.q_a_layernorm = RMSNorm(config.q_lora_rank, config.rms_norm_eps)
            self.q_b_proj = LinearColParallelMerged(config.q_lora_rank, [heads_full * qk], has_bias=False)
        else:
            self.q_proj = LinearColParallelMerged(H, [heads_full * qk], has_bias=False)
        self.kv_a_proj_with_mqa = LinearReplicated(H, self.kv_lora + self.rope_dim, has_bias=False)
        self.kv_a_layernorm = RMSNorm(self.kv_lora, config.rms_norm_eps)
        self.kv_b_proj = LinearColParallelMerged(self.kv_lora, [heads_full * (self.nope + self.v_dim)],
                                                 has_bias=False)
        self.o_proj = LinearOProj(heads_full * self.v_dim, H, has_bias=False)
        rc = config.rotary_config
        scaling = tuple(rc.scaling.items()) if rc.scaling else None
        self._rotary = get_rope(self.rope_dim, self.rope_dim, rc.max_position, rc.base, scaling)
        self._layer_id = layer_id
        self._q_lora = config.q_lora_rank > 0
        self._comm = _CPComm()

    def post_load(self) -> None:
        super().post_load()
        # per-head W_UK^T [H, kv_lora, nope] and W_UV [H, v, kv_lora], each
        # contiguous: the weights of the two head-grouped GEMMs
        kv_b = self.kv_b_proj.weight.view(self.heads, self.nope + self.v_dim, self.kv_lora)
        self._w_uk_t = kv_b[:, : self.nope, :].transpose(1, 2).contiguous()
        self._w_uv = kv_b[:, self.nope :, :].contiguous()

    def _q(self, x: torch.Tensor) -> torch.Tensor:
        if self._q_lora:
            return self.q_b_proj.forward(self.q_a_layernorm.forward(self.q_a_proj.forward(x)))
        return self.q_proj.forward(x)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        ctx = get_global_ctx()
        backend = ctx.attn_backend
        if getattr(backend, "cp_size", 1) > 1:
            return self._forward_cp(x, ctx, backend)
        batch = ctx.batch
        T = x.shape[0]
        q = self._q(x)
        kv_a = self.kv_a_proj_with_mqa.forward(x)
        md = batch.attn_metadata
        if getattr(md, "expanded", False):
            # non-absorbed prefill: the new latent rows into the cache, then
            # attention over every key expanded through kv_b_proj
            ops.mla_store_latent(kv_a, self.kv_a_layernorm.weight, self.eps, batch.positions,
                                 self._rotary.cos_sin_cache, ctx.kv_cache.latent(self._layer_id), batch.out_loc,
                                 ctx.page_size)
            qh = q.view(T, self.heads, self.nope + self.rope_dim)
            q_rope = ops.mla_rope_q(qh, self.rope_dim, batch.positions, self._rotary.cos_sin_cache)
            o = ops.mla_prefill_attention(qh, q_rope, ctx.kv_cache.latent(self._layer_id), ctx.page_table,
                                          md.req_rows, md.seq_lens, md.cu_q, md.max_q, self.kv_b_proj.weight,
                                          self.nope, self.v_dim, ctx.page_size, backend.scale, md.prefill_plan)
            return self.o_proj.forward(o)
        q_lat, q_pe = ops.mla_prepare(q.view(T, self.heads, self.nope + self.rope_dim), kv_a, self._w_uk_t,
                                      self.kv_a_layernorm.weight, self.eps, batch.positions,
                                      self._rotary.cos_sin_cache, ctx.kv_cache.latent(self._layer_id),
                                      batch.out_loc, ctx.page_size)
        o_lat = backend.forward_mla(q_lat, q_pe, self._layer_id, batch)
        return self.o_proj.forward(ops.mla_output(o_lat, self._w_uv, T))

    def _forward_cp(self, x: torch.Tensor, ctx, backend) -> torch.Tensor:
        """Context parallelism. x holds this rank's rows: the tokens of its
        own 64-key tiles (plus padding) for a sharded prefill, every token
        for a decode batch. The rank stores the latent rows of its tiles,
        builds the queries of every token (for a sharded prefill from the
        all-gathered query input: q_lora_rank values a token, the narrowest
        tensor before the heads fan out), attends them over its tiles and
        maps its share of the output through W_UV; the shares meet in one
        reduce-scatter back to the owners' rows (one all-reduce when decode
        rows are replicated), and o_proj runs on the rank's own rows."""
        batch = ctx.batch
        plan = batch.attn_metadata.cp_plan
        kv_a = self.kv_a_proj_with_mqa.forward(x)
        ops.mla_store_latent(kv_a, self.kv_a_layernorm.weight, self.eps,
                             plan.positions if plan is not None else batch.positions, self._rotary.cos_sin_cache,
                             ctx.kv_cache.latent(self._layer_id), plan.out_loc if plan is not None else batch.out_loc,
                             ctx.page_size, backend.cp_size, backend.cp_rank)
        if self._q_lora:
            q_in = self.q_a_layernorm.forward(self.q_a_proj.forward(x))
            q_up = self.q_b_proj
        else:
            q_in, q_up = x, self.q_proj
        if plan is not None:
            q_in = plan.gather(q_in)
        T = q_in.shape[0]
        q = q_up.forward(q_in).view(T, self.heads, self.nope + self.rope_dim)
        q_lat, q_pe = ops.mla_prepare_q(q, self._w_uk_t, batch.positions, self._rotary.cos_sin_cache)
        share = backend.forward_mla(q_lat, q_pe, self._layer_id, batch)
        if plan is not None:
            y = plan.reduce_scatter(ops.mla_output(share, self._w_uv, T, plan.row_map, plan.cp * plan.T_max))
        else:
            y = self._comm.all_reduce(ops.mla_output(share, self._w_uv, T))
        return self.o_proj.forward(y)


class DeepseekGate(BaseOP):
    """Router weight and the per-expert score correction bias (fp32)."""

    def __init__(self, num_experts: int, hidden: int, has_bias: bool) -> None:
        self.weight = torch.empty(num_experts, hidden)
        self.e_score_correction_bias = torch.empty(num_experts, dtype=torch.float32) if has_bias else None


class DeepseekMoE(BaseOP):
    def __init__(self, config: "ModelConfig") -> None:
        self.gate = DeepseekGate(config.num_experts, config.hidden_size, config.scoring_func == "sigmoid")
        self.experts = MoELayer(config.num_experts, config.num_experts_per_tok, config.hidden_size,
                                config.moe_intermediate_size, renormalize=config.norm_topk_prob,
                                scoring=config.scoring_func, n_group=config.n_group, topk_group=config.topk_group,
                                routed_scale=config.routed_scaling_factor, reduce_results=False,
                                quant=config.moe_quant, ep_size=config.ep_size, ep_rank=config.ep_rank)
        self.shared_experts = (GatedMLP(config, config.moe_intermediate_size * config.n_shared_experts)
                               if config.n_shared_experts > 0 else None)
        self._tp = get_tp_info().size
        self._comm = DistributedCommunicator()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        logits = ops.gemm(x, self.gate.weight, out_dtype=torch.float32)
        e = self.experts
        out = get_global_ctx().moe_backend.forward(
            hidden_states=x, w1=e.gate_up_proj, w2=e.down_proj, gating_output=logits,
            correction_bias=self.gate.e_score_correction_bias, **e.backend_kwargs())
        if self.shared_experts is not None:
            s = self.shared_experts
            h = ops.silu_and_mul(s.gate_up_proj.forward(x))
            out = out + ops.gemm(h, s.down_proj.weight)  # partial over TP, reduced once below
        if self._tp > 1:
            out = self._comm.all_reduce(out)
        return out


class DeepseekLayer(BaseOP):
    def __init__(self, config: "ModelConfig", layer_id: int) -> None:
        self.self_attn = MLAAttention(config, layer_id)
        dense = layer_id < config.first_k_dense_replace or config.num_experts == 0
        self.mlp = GatedMLP(config) if dense else DeepseekMoE(config)
        self.input_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor]) -> Tuple[torch.Tensor, torch.Tensor]:
        x, residual = self.input_layernorm.forward(x, residual)
        x = self.self_attn.forward(x)
        x, residual = self.post_attention_layernorm.forward(x, residual)
        return self.mlp.forward(x), residual


class DeepseekModel(BaseOP):
    def __init__(self, config: "ModelConfig") -> None:
        self.embed_tokens = VocabParallelEmbedding(config.vocab_size, config.hidden_size)
        self.layers = OPList([DeepseekLayer(config, i) for i in range(config.num_layers)])
        self.norm = RMSNormFused(config.hidden_size, config.rms_norm_eps)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        batch = get_global_ctx().batch
        plan = getattr(batch.attn_metadata, "cp_plan", None)
        if plan is not None:  # token-sharded prefill: this rank's rows only
            input_ids = input_ids.index_select(0, plan.local)
        x = self.embed_tokens.forward(input_ids)
        residual: Optional[torch.Tensor] = None
        for layer in self.layers.op_list:
            x, residual = layer.forward(x, residual)
        h = self.norm.forward(x, residual)[0]
        if plan is not None:  # one row per request for the LM head
            h = plan.last_rows(h, batch.size)
        return h


class DeepseekV3ForCausalLM(BaseLLMModel):
    def __init__(self, config: "ModelConfig") -> None:
        self.model = DeepseekModel(config)
        tied = config.tie_word_embeddings
        self.lm_head = ParallelLMHead(config.vocab_size, config.hidden_size, tie_word_embeddings=tied,
                                      tied_embedding=self.model.embed_tokens if tied else None)

    def forward(self) -> torch.Tensor:
        hidden = self.model.forward(get_global_ctx().batch.input_ids)
        return self.lm_head.forward(hidden)


__all__ = ["DeepseekV3ForCausalLM"]
