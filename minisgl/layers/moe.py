"""Routed-expert MLP layer (experts sharded over TP on the intermediate dim,
or distributed over ranks with expert parallelism), bf16 or MXFP4.

Expert parallelism over the tensor-parallel ranks: every rank routes all
tokens over all experts, runs only the experts it holds (the others are
dropped by the align kernel) and the partial sums meet in the same
all-reduce tensor parallelism needs. With DP attention the tokens differ per
rank and are dispatched to the experts' owners instead
(minisgl/moe/ep_a2a.py)."""

from __future__ import annotations

import torch

from minisgl.core import get_global_ctx
from minisgl.parallel import DistributedCommunicator, get_tp_info
from minisgl.utils import div_even

from .base import BaseOP


class MoELayer(BaseOP):
    """Packed expert weights: gate_up_proj [E, 2 * I_local, H] and
    down_proj [E, H, I_local] (checkpoint experts are stacked by the loader,
    python/minisgl/models/weight.py:55-66 in the reference)."""

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 renormalize: bool = True, activation: str = "silu", scoring: str = "softmax",
                 n_group: int = 1, topk_group: int = 1, routed_scale: float = 1.0,
                 has_correction_bias: bool = False, reduce_results: bool = True, quant: str = "none",
                 ep_size: int = 1, ep_rank: int = 0) -> None:
        tp = get_tp_info().size
        if quant not in ("none", "mxfp4", "mxfp4-a8"):
            raise ValueError(f"unknown expert quantisation {quant!r}")
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.renormalize = renormalize
        self.activation = activation
        self.scoring = scoring
        self.n_group = n_group
        self.topk_group = topk_group
        self.routed_scale = routed_scale
        self._tp = tp
        self._reduce = reduce_results
        self._comm = DistributedCommunicator()
        # expert parallelism: this rank holds experts [first, first + E / ep)
        # whole; tensor parallelism: every rank holds a slice of every expert
        local_e = div_even(num_experts, ep_size) if ep_size > 1 else num_experts
        local_i = intermediate_size if ep_size > 1 else div_even(intermediate_size, tp)
        self._first_expert = ep_rank * local_e if ep_size > 1 else 0
        self.gate_up_proj = torch.empty(local_e, 2 * local_i, hidden_size)
        self.down_proj = torch.empty(local_e, hidden_size, local_i)
        self.e_score_correction_bias = torch.empty(num_experts, dtype=torch.float32) if has_correction_bias else None
        self._interleaved = False
        self._quant = quant
        self._mxfp4 = None  # (w1 packed, w1 scales, w2 packed, w2 scales) after post_load

    def post_load(self) -> None:
        """Interleave each expert's gate|up rows in 64-row blocks (64 gate rows,
        then the matching 64 up rows): the layout whose grouped GEMM applies
        SiLU x up in its epilogue."""
        super().post_load()
        if self._interleaved:  # already done when the weights were loaded
            return
        n = self.gate_up_proj.shape[1] // 2
        if self.activation != "silu" or n % 64 != 0:
            return
        E, _, H = self.gate_up_proj.shape
        w = self.gate_up_proj.view(E, 2, n // 64, 64, H).transpose(1, 2)
        self.gate_up_proj = w.reshape(E, 2 * n, H).contiguous()
        self._interleaved = True
        if self._quant in ("mxfp4", "mxfp4-a8"):
            self.quantize()

    def load_state_dict(self, state_dict, *, prefix: str = "", _internal: bool = False) -> None:
        super().load_state_dict(state_dict, prefix=prefix, _internal=_internal)
        if self._quant != "none":
            # interleave and quantise now rather than after the whole model is
            # in place: with weights drawn or read as they are taken, only this
            # layer's bf16 experts are alive
            self.post_load()

    def quantize(self) -> None:
        """Replace the bf16 expert weights by MXFP4 (E2M1 + E8M0 per 32; see
        minisgl.quant.mxfp4). On the GPU the bf16 copies are released; on
        the CPU they are kept for inspection."""
        from minisgl.quant import MxfpExperts, block_scales, quantize_mxfp4

        w1q, w1s = quantize_mxfp4(self.gate_up_proj.to(torch.bfloat16).contiguous())
        w2q, w2s = quantize_mxfp4(self.down_proj.to(torch.bfloat16).contiguous())
        self._mxfp4 = MxfpExperts((w1q, w1s, w2q, w2s))
        if self._quant == "mxfp4-a8":
            # the block-scaled GEMM reads the scales in 512-byte scale blocks
            self._mxfp4.blocked = (block_scales(w1s), block_scales(w2s))
        if self.gate_up_proj.is_cuda:
            self.gate_up_proj = self.gate_up_proj.new_empty(0)
            self.down_proj = self.down_proj.new_empty(0)

    def backend_kwargs(self) -> dict:
        """Arguments of the MoE backend that describe this layer's experts."""
        return dict(topk=self.top_k, renormalize=self.renormalize, activation=self.activation,
                    scoring=self.scoring, n_group=self.n_group, topk_group=self.topk_group,
                    routed_scale=self.routed_scale, interleaved=self._interleaved,
                    expert_offset=self._first_expert, mxfp4=self._mxfp4)

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        ctx = get_global_ctx()
        out = ctx.moe_backend.forward(
            hidden_states=hidden_states, w1=self.gate_up_proj, w2=self.down_proj, gating_output=router_logits,
            correction_bias=self.e_score_correction_bias, **self.backend_kwargs())
        if self._tp > 1 and self._reduce:
            out = self._comm.all_reduce(out)
        return out
