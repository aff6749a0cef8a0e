"""Routed-expert MLP layer (experts sharded over TP on the intermediate dim,
or distributed over ranks with expert parallelism)."""

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
                 has_correction_bias: bool = False, reduce_results: bool = True) -> None:
        tp = get_tp_info().size
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
        local_i = div_even(intermediate_size, tp)
        self.gate_up_proj = torch.empty(num_experts, 2 * local_i, hidden_size)
        self.down_proj = torch.empty(num_experts, hidden_size, local_i)
        self.e_score_correction_bias = torch.empty(num_experts, dtype=torch.float32) if has_correction_bias else None
        self._interleaved = False

    def post_load(self) -> None:
        """Interleave each expert's gate|up rows in 64-row blocks (64 gate rows,
        then the matching 64 up rows): the layout whose grouped GEMM applies
        SiLU x up in its epilogue."""
        super().post_load()
        n = self.gate_up_proj.shape[1] // 2
        if self._interleaved or self.activation != "silu" or n % 64 != 0:
            return
        E, _, H = self.gate_up_proj.shape
        w = self.gate_up_proj.view(E, 2, n // 64, 64, H).transpose(1, 2)
        self.gate_up_proj = w.reshape(E, 2 * n, H).contiguous()
        self._interleaved = True

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        ctx = get_global_ctx()
        out = ctx.moe_backend.forward(
            hidden_states=hidden_states, w1=self.gate_up_proj, w2=self.down_proj, gating_output=router_logits,
            topk=self.top_k, renormalize=self.renormalize, activation=self.activation, scoring=self.scoring,
            correction_bias=self.e_score_correction_bias, n_group=self.n_group, topk_group=self.topk_group,
            routed_scale=self.routed_scale, interleaved=self._interleaved,
        )
        if self._tp > 1 and self._reduce:
            out = self._comm.all_reduce(out)
        return out
