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
    """fp32 routed experts; ids outside [0, E) (another rank's experts) are skipped."""
    out = torch.zeros(x.shape[0], w2.shape[1], dtype=torch.float32, device=x.device)
    xf = x.float()
    for e in torch.unique(topk_ids).tolist():
        if e < 0 or e >= w1.shape[0]:
            continue
        tok, slot = (topk_ids == e).nonzero(as_tuple=True)
        h = xf[tok] @ w1[e].float().t()
        a = (ref.silu_mul_interleaved(h) if interleaved else ref.act_and_mul(h, activation)).float()
        y = a @ w2[e].float().t()
        out.index_add_(0, tok, y * topk_w[tok, slot, None])
    return out.to(x.dtype)


class FusedMoe(BaseMoeBackend):
    def __init__(self) -> None:
        self._dequant: dict = {}  # CPU path: dequantised MXFP4 weights, per tensor

    def _cpu_weights(self, mxfp4: tuple):
        from minisgl.quant import dequantize_mxfp4

        key = id(mxfp4[0])
        w = self._dequant.get(key)
        if w is None:
            w = (dequantize_mxfp4(mxfp4[0], mxfp4[1]), dequantize_mxfp4(mxfp4[2], mxfp4[3]))
            self._dequant[key] = w
        return w

    def forward(self, hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, gating_output: torch.Tensor,
                topk: int, renormalize: bool, activation: str = "silu", scoring: str = "softmax",
                correction_bias: Optional[torch.Tensor] = None, n_group: int = 1, topk_group: int = 1,
                routed_scale: float = 1.0, interleaved: bool = False, expert_offset: int = 0,
                mxfp4: Optional[tuple] = None) -> torch.Tensor:
        topk_w, topk_ids = ops.moe_route(gating_output, topk, scoring, renormalize, correction_bias, n_group,
                                         topk_group, routed_scale)
        if expert_offset:
            topk_ids = topk_ids - expert_offset  # global -> local ids; others fall outside [0, E_local)
        if not hidden_states.is_cuda:
            if getattr(mxfp4, "blocked", None) is not None and interleaved:
                from minisgl.quant import moe_experts_mx_reference

                # the block-scaled path's statement: MXFP8 token and SiLU rows
                return moe_experts_mx_reference(hidden_states, *mxfp4, topk_w, topk_ids).to(hidden_states.dtype)
            if mxfp4 is not None:
                w1, w2 = self._cpu_weights(mxfp4)
            return moe_reference(hidden_states, w1, w2, topk_w, topk_ids, activation, interleaved)
        if not interleaved:
            raise RuntimeError("minisgl: the CUDA MoE path needs SiLU experts with gate|up rows interleaved "
                               "in 64-row blocks (MoELayer does this after loading)")
        if mxfp4 is not None:  # W4A16, or MXFP8 activations on the block-scaled tensor cores
            return ops.moe_experts_quantised(hidden_states, mxfp4, topk_w, topk_ids)
        return ops.moe_experts(hidden_states, w1, w2, topk_w, topk_ids)
