"""Attention backend for multi-head latent attention (DeepSeek-V3 / Kimi-K2).

The model hands over absorbed queries: q_nope multiplied into the latent
space by W_UK, head-major [heads, T_pad, kv_lora], and the rotated q_pe
[T, heads, rope]. The backend attends over the paged latent cache (every
head reads the same latent rows) and returns the latent output, head-major
[heads, T_pad, kv_lora], which the model maps back to heads with W_UV. Metadata per batch is the GQA backend's:
each request's page-table row, key count and query offset, in one pinned
upload. The reference has no MLA (no DeepSeek-V3 architecture). Under context
parallelism each rank holds the latent rows of the 64-key tiles t with
t % cp == rank and attends over those only; the partial outputs and
log-sum-exps of all ranks are all-gathered and merged (``ops.mla_attention``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Dict, List, Optional

import torch

from minisgl import ops
from minisgl.core import Batch, get_global_ctx
from minisgl.parallel import get_cp_info, get_tp_info
from minisgl.utils import div_even

from .base import BaseAttnBackend, BaseAttnMetadata

if TYPE_CHECKING:
    from minisgl.models import ModelConfig


def mla_softmax_scale(config: "ModelConfig") -> float:
    """1 / sqrt(qk_nope + qk_rope), times mscale^2 of YaRN's mscale_all_dim
    when the checkpoint asks for it (DeepSeek-V3 convention)."""
    from minisgl.layers.rotary import _yarn_mscale

    scale = (config.qk_nope_head_dim + config.qk_rope_head_dim) ** -0.5
    sc = config.rotary_config.scaling or {}
    if sc.get("mscale_all_dim"):
        m = _yarn_mscale(float(sc["factor"]), float(sc["mscale_all_dim"]))
        scale *= m * m
    return scale


@dataclass
class MLAAttnMetadata(BaseAttnMetadata):
    req_rows: torch.Tensor   # int32 [B]
    seq_lens: torch.Tensor   # int32 [B]
    cu_q: torch.Tensor       # int32 [B + 1]
    max_q: int
    last_indices: Optional[torch.Tensor] = None

    def get_last_indices(self, bs: int) -> torch.Tensor:
        if self.last_indices is None:
            return torch.arange(bs, device=self.req_rows.device)
        return self.last_indices[:bs]


class MLAAttnBackend(BaseAttnBackend):
    def __init__(self, config: "ModelConfig", max_batch: int = 256) -> None:
        ctx = get_global_ctx()
        self.heads = div_even(config.num_qo_heads, get_tp_info().size)
        self.kv_lora = config.kv_lora_rank
        self.rope = config.qk_rope_head_dim
        self.scale = mla_softmax_scale(config)
        self.page_size = ctx.page_size
        self.kv = ctx.kv_cache
        self.device = self.kv.device
        self.capture: Optional[Dict[str, torch.Tensor]] = None
        cp = get_cp_info()
        self.cp_size, self.cp_rank = (cp.size, cp.rank) if cp is not None else (1, 0)

    def forward(self, q: torch.Tensor, layer_id: int, batch: Batch) -> torch.Tensor:
        raise TypeError("the MLA backend takes (q_lat, q_pe): call forward_mla")

    def forward_mla(self, q_lat: torch.Tensor, q_pe: torch.Tensor, layer_id: int, batch: Batch) -> torch.Tensor:
        """q_lat [H, T_pad, kv_lora] head-major, q_pe [T, H, rope] ->
        latent output [H, T_pad, kv_lora]."""
        md = batch.attn_metadata
        assert isinstance(md, MLAAttnMetadata)
        group = None
        if self.cp_size > 1:
            import torch.distributed as dist

            group = dist.group.WORLD
        return ops.mla_attention(q_lat, q_pe, self.kv.latent(layer_id), get_global_ctx().page_table, md.req_rows,
                                 md.seq_lens, md.cu_q, self.page_size, self.scale, cp_size=self.cp_size,
                                 cp_rank=self.cp_rank, cp_group=group)

    def prepare_metadata(self, batch: Batch) -> None:
        reqs = batch.padded_reqs
        B = len(reqs)
        rows = [r.table_idx for r in reqs]
        lens = [r.device_len for r in reqs]
        qlens = [1] * B if batch.is_decode else [r.extend_len for r in reqs]
        cu = [0]
        for n in qlens:
            cu.append(cu[-1] + n)
        host = torch.tensor(rows + lens + cu, dtype=torch.int32, pin_memory=self.device.type == "cuda")
        dev = host.to(self.device, non_blocking=True)
        cu_q = dev[2 * B :]
        batch.attn_metadata = MLAAttnMetadata(dev[:B], dev[B : 2 * B], cu_q, max(qlens),
                                              None if batch.is_decode else (cu_q[1:] - 1).long())

    def init_capture_graph(self, max_seq_len: int, bs_list: List[int]) -> None:
        n = max(bs_list)
        self.capture = {
            "req_rows": torch.zeros(n, dtype=torch.int32, device=self.device),
            "seq_lens": torch.ones(n, dtype=torch.int32, device=self.device),
            "cu_q": torch.arange(n + 1, dtype=torch.int32, device=self.device),
        }

    def prepare_for_capture(self, batch: Batch) -> None:
        assert self.capture is not None
        bs = batch.size
        self.capture["req_rows"][:bs].fill_(batch.reqs[0].table_idx)
        self.capture["seq_lens"][:bs].fill_(1)
        batch.attn_metadata = MLAAttnMetadata(self.capture["req_rows"][:bs], self.capture["seq_lens"][:bs],
                                              self.capture["cu_q"][: bs + 1], 1)

    def prepare_for_replay(self, batch: Batch) -> None:
        assert self.capture is not None
        md = batch.attn_metadata
        assert isinstance(md, MLAAttnMetadata)
        bs = batch.padded_size
        self.capture["req_rows"][:bs].copy_(md.req_rows)
        self.capture["seq_lens"][:bs].copy_(md.seq_lens)
