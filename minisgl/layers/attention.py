"""Attention layer: fused q/k-norm + RoPE + KV store, then paged attention.

Compared with the reference (python/minisgl/layers/attention.py:47-57), which
launches q-norm, k-norm, RoPE and the KV store separately, one kernel does
all four; the q heads are rewritten in place inside the fused qkv output and
the backend reads them from there (no copy).
"""

from __future__ import annotations

from typing import TYPE_CHECKING, Optional

import torch

from minisgl import ops
from minisgl.core import get_global_ctx
from minisgl.parallel import get_tp_info
from minisgl.utils import div_even

from .base import StateLessOP
from .rotary import get_rope

if TYPE_CHECKING:
    from minisgl.models import RotaryConfig

    from .norm import RMSNorm


class AttentionLayer(StateLessOP):
    def __init__(self, layer_id: int, num_qo_heads: int, num_kv_heads: int, head_dim: int,
                 rotary_config: "RotaryConfig", q_norm: Optional["RMSNorm"] = None,
                 k_norm: Optional["RMSNorm"] = None, eps: float = 1e-6) -> None:
        assert num_qo_heads % num_kv_heads == 0
        tp = get_tp_info().size
        self.layer_id = layer_id
        self.head_dim = head_dim
        self.num_qo_heads = div_even(num_qo_heads, tp)
        self.num_kv_heads = div_even(num_kv_heads, tp, allow_replicate=True)
        self.qo_attn_dim = self.num_qo_heads * head_dim
        self.kv_attn_dim = self.num_kv_heads * head_dim
        scaling = tuple(rotary_config.scaling.items()) if rotary_config.scaling else None
        self.rotary = get_rope(head_dim, rotary_config.rotary_dim, rotary_config.max_position,
                               rotary_config.base, scaling)
        self._q_norm = q_norm
        self._k_norm = k_norm
        self.eps = q_norm.eps if q_norm is not None else eps

    def rope_args(self) -> dict:
        """Arguments of the fused qkv-GEMM epilogue (q/k norm, RoPE, KV store)
        for the current batch."""
        ctx = get_global_ctx()
        batch = ctx.batch
        kv = ctx.kv_cache
        return dict(
            positions=batch.positions, cos_sin=self.rotary.cos_sin_cache, out_loc=batch.out_loc,
            q_norm_w=None if self._q_norm is None else self._q_norm.weight,
            k_norm_w=None if self._k_norm is None else self._k_norm.weight,
            head_eps=self.eps, k_cache=kv.k_cache(self.layer_id), v_cache=kv.v_cache(self.layer_id),
            hq=self.num_qo_heads, hk=self.num_kv_heads, page_size=ctx.page_size,
        )

    def attend(self, qkv: torch.Tensor) -> torch.Tensor:
        """Attention over q heads already rotated in ``qkv`` (KV already stored)."""
        ctx = get_global_ctx()
        return ctx.attn_backend.forward(qkv, self.layer_id, ctx.batch)

    @property
    def fusable(self) -> bool:
        """Whether the fused qkv epilogue can replace ``rope_store``."""
        return self.head_dim == 128

    def forward(self, qkv: torch.Tensor) -> torch.Tensor:
        ctx = get_global_ctx()
        batch = ctx.batch
        kv = ctx.kv_cache
        ops.rope_store(
            qkv, batch.positions, self.rotary.cos_sin_cache,
            None if self._q_norm is None else self._q_norm.weight,
            None if self._k_norm is None else self._k_norm.weight,
            kv.k_cache(self.layer_id), kv.v_cache(self.layer_id), batch.out_loc,
            self.num_qo_heads, self.num_kv_heads, self.head_dim, ctx.page_size, self.eps,
        )
        return ctx.attn_backend.forward(qkv, self.layer_id, batch)
