"""Building blocks shared by the decoder families."""

from __future__ import annotations

from typing import TYPE_CHECKING

import torch

from minisgl import ops
from minisgl.layers import (
    AttentionLayer,
    BaseOP,
    LinearColParallelMerged,
    LinearOProj,
    LinearQKVMerged,
    LinearReplicated,
    LinearRowParallel,
    MoELayer,
    RMSNorm,
    gelu_and_mul,
    silu_and_mul,
)
from minisgl.utils import nvtx_annotate

if TYPE_CHECKING:
    from .config import ModelConfig

_ACT = {"silu": silu_and_mul, "gelu": gelu_and_mul, "gelu_pytorch_tanh": gelu_and_mul}


class GatedMLP(BaseOP):
    """down(act(gate(x)) * up(x)) with gate|up fused into one GEMM."""

    def __init__(self, config: "ModelConfig", intermediate_size: int | None = None) -> None:
        inter = intermediate_size or config.intermediate_size
        self.gate_up_proj = LinearColParallelMerged(config.hidden_size, [inter, inter], has_bias=False)
        if config.hidden_act not in _ACT:
            raise ValueError(f"unsupported activation {config.hidden_act}")
        self._act = _ACT[config.hidden_act]
        self._silu = config.hidden_act == "silu"
        self._interleaved = False
        self.down_proj = LinearRowParallel(inter, config.hidden_size, has_bias=False)

    @property
    def fusable(self) -> bool:
        """SiLU MLPs whose local gate / up halves split into 64-row blocks can
        run the gate_up GEMM with the activation in its epilogue."""
        return self._silu and self.gate_up_proj.local_output_size % 128 == 0

    def interleave(self) -> None:
        """Reorder gate|up rows into alternating blocks of 64 (64 gate rows,
        then the matching 64 up rows), the layout of the fused epilogue."""
        w = self.gate_up_proj.weight
        n = w.shape[0] // 2
        self.gate_up_proj.weight = w.view(2, n // 64, 64, -1).transpose(0, 1).reshape(2 * n, -1).contiguous()
        self._interleaved = True

    @nvtx_annotate("MLP")
    def forward(self, x: "torch.Tensor") -> "torch.Tensor":
        h = self.gate_up_proj.forward(x)
        a = ops.silu_and_mul(h, interleaved=True) if self._interleaved else self._act(h)
        return self.down_proj.forward(a)

    def forward_fused(self, r: "torch.Tensor", norm_eps: float) -> "torch.Tensor":
        """r + down(silu(gate) * up) of rmsnorm(r): two GEMMs, the norm and the
        activation in the first one's epilogue, the add in the second's."""
        h = ops.gemm_fused(r, self.gate_up_proj.weight, norm_eps=norm_eps, silu=True)
        return self.down_proj.forward_residual(h, r)


class MoEMLP(BaseOP):
    """Replicated router + routed experts (Qwen3-MoE style)."""

    def __init__(self, config: "ModelConfig") -> None:
        self.experts = MoELayer(config.num_experts, config.num_experts_per_tok, config.hidden_size,
                                config.moe_intermediate_size, renormalize=config.norm_topk_prob,
                                quant=config.moe_quant, ep_size=config.ep_size, ep_rank=config.ep_rank)
        self.gate = LinearReplicated(config.hidden_size, config.num_experts, has_bias=False)

    @nvtx_annotate("MoE")
    def forward(self, x: "torch.Tensor") -> "torch.Tensor":
        return self.experts.forward(x, self.gate.forward(x))


class RopeAttn(BaseOP):
    """qkv projection -> fused norm/RoPE/KV-store + paged attention -> o_proj."""

    def __init__(self, config: "ModelConfig", layer_id: int, *, has_attn_bias: bool = False,
                 has_qk_norm: bool = False) -> None:
        d = config.head_dim
        self.qkv_proj = LinearQKVMerged(config.hidden_size, d, config.num_qo_heads, config.num_kv_heads, has_attn_bias)
        self.q_norm = RMSNorm(d, config.rms_norm_eps) if has_qk_norm else None
        self.k_norm = RMSNorm(d, config.rms_norm_eps) if has_qk_norm else None
        self.attn = AttentionLayer(layer_id, config.num_qo_heads, config.num_kv_heads, d, config.rotary_config,
                                   self.q_norm, self.k_norm, eps=config.rms_norm_eps)
        self.o_proj = LinearOProj(d * config.num_qo_heads, config.hidden_size, has_bias=False)

    @nvtx_annotate("MHA")
    def forward(self, x: "torch.Tensor") -> "torch.Tensor":
        return self.o_proj.forward(self.attn.forward(self.qkv_proj.forward(x)))

    def forward_fused(self, r: "torch.Tensor", norm_eps: float) -> "torch.Tensor":
        """r + o_proj(attention(rmsnorm(r))): the norm, q/k-norm, RoPE and
        KV store in the qkv GEMM epilogue, the add in the o_proj epilogue."""
        q = torch.empty(r.shape[0], self.attn.qo_attn_dim, dtype=r.dtype, device=r.device)
        ops.gemm_fused(r, self.qkv_proj.weight, bias=self.qkv_proj.bias, norm_eps=norm_eps,
                       rope=self.attn.rope_args(), out=q)
        return self.o_proj.forward_residual(self.attn.attend(q), r)


__all__ = ["GatedMLP", "MoEMLP", "RopeAttn"]
