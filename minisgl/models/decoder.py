"""The decoder skeleton shared by Llama, Qwen2, Qwen3, Qwen3-MoE and
Mistral: embed -> N x (add+norm, attention, add+norm, MLP) -> norm -> LM
head. Family differences are constructor flags (qkv bias, q/k norm, MoE)."""

from __future__ import annotations

from typing import TYPE_CHECKING, Dict, Optional, Tuple

import torch

from minisgl import ops
from minisgl.core import get_global_ctx
from minisgl.layers import BaseOP, OPList, ParallelLMHead, RMSNormFused, VocabParallelEmbedding
from minisgl.parallel import DistributedImpl, get_tp_info, sequence_parallel_comm
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

    Under tensor parallelism with a sequence-parallel communicator
    (``forward_sp``) the residual stream is token-sharded and the collectives
    after o_proj / down_proj carry the residual adds and the RMSNorms.

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

    @nvtx_annotate("Layer_{}", layer_id_field="_layer_id")
    def forward_sp(self, x: torch.Tensor, r: torch.Tensor, comm: DistributedImpl, T: int,
                   next_norm: RMSNormFused, fused: bool) -> torch.Tensor:
        """Sequence-parallel block over tensor-parallel ranks. ``x`` [T_pad, H]
        holds every rank's normalised input rows (gathered by the previous
        collective), ``r`` this rank's slice of the residual stream (updated in
        place). Each row-parallel projection writes its partial product where
        ``comm.rs_norm_ag`` reduce-scatters it into ``r``, normalises the new
        rows and gathers them for the next column-parallel GEMM; the last
        collective applies ``next_norm`` (the next layer's input norm or the
        final norm). Returns the gathered rows after this block."""
        Tp, H = x.shape
        first = get_tp_info().rank == 0
        attn = self.self_attn
        fused = fused and self._fused_attn
        xt = x[:T]
        if fused:  # q/k norm, RoPE and the KV store in the qkv GEMM's epilogue
            q = torch.empty(T, attn.attn.qo_attn_dim, dtype=x.dtype, device=x.device)
            ops.gemm_fused(xt, attn.qkv_proj.weight, bias=attn.qkv_proj.bias, rope=attn.attn.rope_args(), out=q)
            o = attn.attn.attend(q)
        else:
            o = attn.attn.forward(attn.qkv_proj.forward(xt))
        part = comm.sp_partial(Tp, H, x.dtype, x.device)
        ops.gemm(o, attn.o_proj.weight, attn.o_proj.bias if first else None, out=part[:T])
        norm = self.post_attention_layernorm
        x = comm.rs_norm_ag(part, r, True, norm.active_weight, norm.eps)
        xt = x[:T]
        mlp = self.mlp
        if fused and self._fused_mlp:
            h = ops.gemm_fused(xt, mlp.gate_up_proj.weight, silu=True)
        else:
            g = mlp.gate_up_proj.forward(xt)
            h = ops.silu_and_mul(g, interleaved=True) if mlp._interleaved else mlp._act(g)
        part = comm.sp_partial(Tp, H, x.dtype, x.device)
        ops.gemm(h, mlp.down_proj.weight, mlp.down_proj.bias if first else None, out=part[:T])
        return comm.rs_norm_ag(part, r, True, next_norm.active_weight, next_norm.eps)


class DecoderModel(BaseOP):
    def __init__(self, config: "ModelConfig", **flags: bool) -> None:
        self.embed_tokens = VocabParallelEmbedding(config.vocab_size, config.hidden_size)
        self.layers = OPList([DecoderLayer(config, i, **flags) for i in range(config.num_layers)])
        self.norm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        # batch size -> whether the fused-epilogue layer form runs at that size;
        # measured per CUDA-graph batch size when the graphs are captured (the
        # fused form wins on narrow models, the plain-GEMM form with separate
        # row kernels can win on wide ones at large batches)
        self._fused_choice: Dict[int, bool] = {}

    def fused_for(self, T: int) -> bool:
        """Whether a batch of T tokens takes the fused-epilogue form: the
        measured choice of the smallest captured size >= T (fused when none
        was measured), never beyond FUSED_MAX_TOKENS."""
        if T > FUSED_MAX_TOKENS or not self.fusable:
            return False
        size = min((b for b in self._fused_choice if b >= T), default=None)
        return self._fused_choice[size] if size is not None else True

    @property
    def fusable(self) -> bool:
        return all(layer.fusable for layer in self.layers.op_list)

    @property
    def sp_capable(self) -> bool:
        """Dense blocks only: the sequence-parallel form needs every MLP to be a
        row-parallel GatedMLP (MoE layers keep the all-reduce form)."""
        return all(isinstance(layer.mlp, GatedMLP) for layer in self.layers.op_list)

    def sp_comm(self) -> Optional[DistributedImpl]:
        comm = sequence_parallel_comm()
        return comm if comm is not None and self.sp_capable else None

    def forward_sp(self, input_ids: torch.Tensor, comm: DistributedImpl) -> torch.Tensor:
        """Tensor parallelism with a token-sharded residual stream: T tokens
        are padded to a multiple of the rank count R and rank r keeps residual
        rows [r * T_pad / R, (r + 1) * T_pad / R). The vocabulary-sharded
        embedding's partial rows are reduce-scattered like a projection's;
        every collective also applies the following RMSNorm and gathers the
        normalised rows. Returns the final-normed hidden rows [T, H]."""
        T = input_ids.shape[0]
        R = get_tp_info().size
        rows = -(-T // R)
        Tp = rows * R
        emb = self.embed_tokens
        H = emb.weight.shape[1]
        part = comm.sp_partial(Tp, H, emb.weight.dtype, emb.weight.device)
        ops.embedding(input_ids, emb.weight, emb.vocab_range, out=part[:T])
        if Tp > T:
            part[T:].zero_()
        r = torch.empty(rows, H, dtype=emb.weight.dtype, device=emb.weight.device)
        layers = self.layers.op_list
        norm0 = layers[0].input_layernorm if layers else self.norm
        x = comm.rs_norm_ag(part, r, False, norm0.active_weight, norm0.eps)
        fused = self.fused_for(T)
        for i, layer in enumerate(layers):
            x = layer.forward_sp(x, r, comm, T, layers[i + 1].input_layernorm if i + 1 < len(layers) else self.norm,
                                 fused)
        return x[:T]

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        comm = self.sp_comm()
        if comm is not None:
            return self.forward_sp(input_ids, comm)
        x = self.embed_tokens.forward(input_ids)
        if self.fused_for(x.shape[0]):
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

    def forward_variants(self) -> Tuple[Optional[bool], ...]:
        """Layer forms the graph runner measures per batch size (fused
        epilogues, plain GEMMs + row kernels); (None,) when only one exists."""
        return (True, False) if self.model.fusable else (None,)

    def set_forward_variant(self, batch_size: int, fused: Optional[bool]) -> None:
        if fused is not None:
            self.model._fused_choice[batch_size] = fused

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
        # sequence parallel: the collectives apply the norms and the residual
        # adds, so the GEMMs carry only RoPE / SiLU epilogues
        sp = self.model.sp_comm() is not None
        norm = 0 if sp else ops.EPI_NORM
        for layer in self.model.layers.op_list:
            attn = layer.self_attn
            hq, hk = attn.attn.num_qo_heads, attn.attn.num_kv_heads
            out[tuple(attn.qkv_proj.weight.shape)] = (norm | ops.EPI_ROPE, hq, hk)
            if not sp:
                out[tuple(attn.o_proj.weight.shape)] = (ops.EPI_RESIDUAL, hq, hk)
            if layer._fused_mlp:
                out[tuple(layer.mlp.gate_up_proj.weight.shape)] = (norm | ops.EPI_SILU, hq, hk)
                if not sp:
                    out[tuple(layer.mlp.down_proj.weight.shape)] = (ops.EPI_RESIDUAL, hq, hk)
        if self.samples_in_lm_head:
            head = self.lm_head._tied.weight if self.lm_head._tied is not None else self.lm_head.weight
            out[tuple(head.shape)] = (ops.EPI_SAMPLE, 0, 0)
        return out

    def forward(self) -> torch.Tensor:
        hidden = self.model.forward(get_global_ctx().batch.input_ids)
        return self.lm_head.forward(hidden)
