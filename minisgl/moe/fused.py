"""Routed experts: top-k routing, grouped expert GEMMs, weighted combine.

CUDA path: the router kernel, a device-side sort of (token, slot) pairs by
expert into tiles, two grouped tcgen05 GEMMs over the expert-sorted rows
(gate_up, then down) and a combine kernel that sums the k weighted expert
outputs per token. CPU path: the same math in fp32 PyTorch.
Replaces the reference's Triton fused-MoE pipeline
(python/minisgl/moe/fused.py:9-256, kernel/triton/fused_moe.py).
"""

from __future__ import annotations

from typing import Optional

import torch

from minisgl import ops
from minisgl.ops import reference as ref

from .base import BaseMoeBackend


def moe_reference(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor,
                  activation: str, interleaved: bool = False) -> torch.Tensor:
    out = torch.zeros(x.shape[0], w2.shape[1], dtype=torch.float32, device=x.device)
    xf = x.float()
    for e in torch.unique(topk_ids).tolist():
        tok, slot = (topk_ids == e).nonzero(as_tuple=True)
        h = xf[tok] @ w1[e].float().t()
        a = (ref.silu_mul_interleaved(h) if interleaved else ref.act_and_mul(h, activation)).float()
        y = a @ w2[e].float().t()
        out.index_add_(0, tok, y * topk_w[tok, slot, None])
    return out.to(x.dtype)


class FusedMoe(BaseMoeBackend):
    def forward(self, hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, gating_output: torch.Tensor,
                topk: int, renormalize: bool, activation: str = "silu", scoring: str = "softmax",
                correction_bias: Optional[torch.Tensor] = None, n_group: int = 1, topk_group: int = 1,
                routed_scale: float = 1.0, interleaved: bool = False) -> torch.Tensor:
        topk_w, topk_ids = ops.moe_route(gating_output, topk, scoring, renormalize, correction_bias, n_group,
                                         topk_group, routed_scale)
        if not hidden_states.is_cuda:
            return moe_reference(hidden_states, w1, w2, topk_w, topk_ids, activation, interleaved)
        if not interleaved:
            raise RuntimeError("minisgl: the CUDA MoE path needs SiLU experts with gate|up rows interleaved "
                               "in 64-row blocks (MoELayer does this after loading)")
        return ops.moe_experts(hidden_states, w1, w2, topk_w, topk_ids)
