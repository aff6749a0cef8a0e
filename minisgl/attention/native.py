"""The sm_100a paged attention backend (prefill and decode).

Metadata per batch is small: for each request its page-table row, its total
key count and (prefill) its query offset. The kernels read the global page
table directly (token slot of position p = page_table[row, p]), so unlike the
reference backends (python/minisgl/attention/trtllm.py:91-129) no per-batch
block table is gathered. All per-batch integers go to the device in one
pinned host buffer and a single asynchronous copy.

Decode uses split-KV: the number of splits is fixed per batch size so the
grid is identical at capture and replay; each (request, kv head) gets up to
that many CTAs depending on its length.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import TYPE_CHECKING, Dict, List, Optional

import torch

from minisgl import ops
from minisgl.core import Batch, get_global_ctx
from minisgl.parallel import get_tp_info
from minisgl.utils import div_even

from .base import BaseAttnBackend, BaseAttnMetadata

if TYPE_CHECKING:
    from minisgl.models import ModelConfig

NUM_SMS = 148
MAX_SPLITS = 16


def decode_splits(batch_size: int, kv_heads: int) -> int:
    """Splits per (request, kv head) so that about two CTAs run per SM."""
    want = math.ceil(2 * NUM_SMS / max(1, batch_size * kv_heads))
    return max(1, min(MAX_SPLITS, want))


@dataclass
class NativeAttnMetadata(BaseAttnMetadata):
    req_rows: torch.Tensor   # int32 [B]
    seq_lens: torch.Tensor   # int32 [B]
    cu_q: Optional[torch.Tensor]  # int32 [B + 1] (prefill)
    max_q: int
    max_splits: int
    last_indices: Optional[torch.Tensor] = None  # int64 [B] (prefill)

    def get_last_indices(self, bs: int) -> torch.Tensor:
        if self.last_indices is None:  # decode: one token per request
            return torch.arange(bs, device=self.req_rows.device)
        return self.last_indices[:bs]


class NativeAttnBackend(BaseAttnBackend):
    def __init__(self, config: "ModelConfig", max_batch: int = 256) -> None:
        ctx = get_global_ctx()
        tp = get_tp_info().size
        self.hq = div_even(config.num_qo_heads, tp)
        self.hk = div_even(config.num_kv_heads, tp, allow_replicate=True)
        self.d = config.head_dim
        self.scale = config.head_dim ** -0.5
        self.page_size = ctx.page_size
        self.kv = ctx.kv_cache
        self.device = self.kv.device
        self.max_batch = max_batch
        self._scratch_bs = 0
        self.part_o: Optional[torch.Tensor] = None
        self.part_lse: Optional[torch.Tensor] = None
        self._ensure_scratch(max_batch)
        self.capture: Optional[Dict[str, torch.Tensor]] = None
        self.capture_bs: List[int] = []

    # ---------------------------------------------------------------- scratch
    def _ensure_scratch(self, bs: int) -> None:
        if bs <= self._scratch_bs or self.device.type != "cuda":
            return
        self._scratch_bs = bs
        self.part_o = torch.empty(bs * self.hq * MAX_SPLITS * self.d, dtype=torch.float32, device=self.device)
        self.part_lse = torch.empty(bs * self.hq * MAX_SPLITS, dtype=torch.float32, device=self.device)

    # ---------------------------------------------------------------- forward
    def forward(self, qkv: torch.Tensor, layer_id: int, batch: Batch) -> torch.Tensor:
        md = batch.attn_metadata
        assert isinstance(md, NativeAttnMetadata)
        pool = self.kv.pool
        pt = get_global_ctx().page_table
        if batch.is_decode:
            return ops.decode_attention(qkv, pool, layer_id, pt, md.req_rows, md.seq_lens, self.hq, self.hk, self.d,
                                        self.page_size, self.scale, self.part_o, self.part_lse, md.max_splits)
        return ops.prefill_attention(qkv, pool, layer_id, pt, md.req_rows, md.seq_lens, md.cu_q, md.max_q,
                                     self.hq, self.hk, self.d, self.page_size, self.scale)

    # --------------------------------------------------------------- metadata
    def prepare_metadata(self, batch: Batch) -> None:
        reqs = batch.padded_reqs
        B = len(reqs)
        rows = [r.table_idx for r in reqs]
        lens = [r.device_len for r in reqs]
        on_gpu = self.device.type == "cuda"
        if batch.is_decode:
            host = torch.tensor(rows + lens, dtype=torch.int32, pin_memory=on_gpu)
            dev = host.to(self.device, non_blocking=True)
            self._ensure_scratch(B)
            batch.attn_metadata = NativeAttnMetadata(dev[:B], dev[B:], None, 1, decode_splits(B, self.hk))
            return
        qlens = [r.extend_len for r in reqs]
        cu = [0]
        for n in qlens:
            cu.append(cu[-1] + n)
        host = torch.tensor(rows + lens + cu, dtype=torch.int32, pin_memory=on_gpu)
        dev = host.to(self.device, non_blocking=True)
        cu_q = dev[2 * B :]
        batch.attn_metadata = NativeAttnMetadata(
            req_rows=dev[:B], seq_lens=dev[B : 2 * B], cu_q=cu_q, max_q=max(qlens), max_splits=1,
            last_indices=(cu_q[1:] - 1).long(),
        )

    # ------------------------------------------------------------ CUDA graphs
    def init_capture_graph(self, max_seq_len: int, bs_list: List[int]) -> None:
        max_bs = max(bs_list)
        self._ensure_scratch(max_bs)
        self.capture = {
            "req_rows": torch.zeros(max_bs, dtype=torch.int32, device=self.device),
            "seq_lens": torch.ones(max_bs, dtype=torch.int32, device=self.device),
        }
        self.capture_bs = sorted(bs_list)

    def prepare_for_capture(self, batch: Batch) -> None:
        assert self.capture is not None
        bs = batch.size
        dummy_row = batch.reqs[0].table_idx
        self.capture["req_rows"][:bs].fill_(dummy_row)
        self.capture["seq_lens"][:bs].fill_(1)
        batch.attn_metadata = NativeAttnMetadata(self.capture["req_rows"][:bs], self.capture["seq_lens"][:bs], None,
                                                 1, decode_splits(bs, self.hk))

    def prepare_for_replay(self, batch: Batch) -> None:
        assert self.capture is not None
        md = batch.attn_metadata
        assert isinstance(md, NativeAttnMetadata)
        bs = batch.padded_size
        self.capture["req_rows"][:bs].copy_(md.req_rows)
        self.capture["seq_lens"][:bs].copy_(md.seq_lens)
