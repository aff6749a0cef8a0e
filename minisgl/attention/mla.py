"""Attention backend for multi-head latent attention (DeepSeek-V3 / Kimi-K2).

The model hands over absorbed queries: q_nope multiplied into the latent
space by W_UK, head-major [heads, T_pad, kv_lora], and the rotated q_pe
[T, heads, rope]. The backend attends over the paged latent cache (every
head reads the same latent rows) and returns the latent output, head-major
[heads, T_pad, kv_lora], which the model maps back to heads with W_UV. Metadata per batch is the GQA backend's:
each request's page-table row, key count and query offset, in one pinned
upload. The reference has no MLA (no DeepSeek-V3 architecture).

Context parallelism (``--cp N``): rank r holds the latent rows of the
64-key tiles t with t % N == r and attends every query over those only;
``ops.mla_attention_share`` returns the rank's share of the merged output
(only log-sum-exps cross the ranks), and the model reduces the shares after
W_UV. Prefill batches are token-sharded: ``CPShardPlan`` gives each rank
the tokens of its own tiles, so every layer outside attention (projections,
MLP / experts, norms) runs on 1/N of the tokens; decode batches run
replicated and all-reduce the shares.
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


class CPShardPlan:
    """How one prefill batch is split over the context-parallel ranks.

    Token i of the batch (position p) belongs to rank (p // 64) % N, the
    owner of its 64-key tile, so a rank stores the latent rows of exactly
    the tokens it computes. Every rank runs T_max rows (its own tokens,
    then padding rows whose position lies in another rank's tile, so they
    store nothing): the ranks meet at every layer's collectives, so the
    busiest rank sets the pace either way, and equal row counts let the
    collectives run on whole buffers. The rank-major layout [N * T_max]
    (rank k's rows at k * T_max + j) is what all-gathers produce and
    reduce-scatters consume; ``row_map`` maps batch order into it.
    """

    def __init__(self, positions: "np.ndarray", cu: "np.ndarray", cp: int, rank: int, out_loc: torch.Tensor,
                 device: torch.device, group) -> None:
        import numpy as np

        T = len(positions)
        owner = (positions // 64) % cp
        counts = np.bincount(owner, minlength=cp)
        self.cp, self.rank, self.group = cp, rank, group
        self.T, self.T_max = T, int(counts.max())
        self.T_own = int(counts[rank])
        slot = np.empty(T, dtype=np.int64)
        for k in range(cp):
            idx = np.nonzero(owner == k)[0]
            slot[idx] = k * self.T_max + np.arange(len(idx))
        own = np.nonzero(owner == rank)[0]
        pad = self.T_max - len(own)
        local = np.concatenate([own, np.zeros(pad, dtype=np.int64)])
        # padding rows: a position in the next rank's first tile (stored
        # there, never here) and token 0's ids / slot
        pad_pos = 64 * ((rank + 1) % cp)
        local_pos = np.concatenate([positions[own], np.full(pad, pad_pos, dtype=positions.dtype)])
        last = cu[1:] - 1
        mine = owner[last] == rank
        # local row of each last token this rank owns, and its request index
        last_src = slot[last[mine]] - rank * self.T_max
        last_dst = np.nonzero(mine)[0]
        pin = device.type == "cuda"
        host64 = torch.from_numpy(np.concatenate([local, last_src, last_dst]).astype(np.int64))
        host32 = torch.from_numpy(np.concatenate([slot, local_pos]).astype(np.int32))
        if pin:
            host64, host32 = host64.pin_memory(), host32.pin_memory()
        d64 = host64.to(device, non_blocking=True)
        d32 = host32.to(device, non_blocking=True)
        n_last = int(mine.sum())
        self.local = d64[: self.T_max]                          # batch index of each local row
        self.last_src = d64[self.T_max : self.T_max + n_last]   # local rows holding a request's last token
        self.last_dst = d64[self.T_max + n_last :]              # ... and the request index
        self.row_map = d32[:T]                                  # batch token -> rank-major row (int32)
        self.gather_idx = self.row_map.long()
        self.positions = d32[T:]                                # positions of the local rows
        self.out_loc = out_loc.index_select(0, self.local)      # cache slots of the local rows

    # collectives over the context-parallel ranks (NCCL on the GPU, gloo on
    # the CPU, which has no reduce-scatter)
    def gather(self, x: torch.Tensor) -> torch.Tensor:
        """[T_max, C] local rows of every rank -> [T, C] in batch order."""
        import torch.distributed as dist

        if x.is_cuda:
            full = torch.empty(self.cp * self.T_max, *x.shape[1:], dtype=x.dtype, device=x.device)
            dist.all_gather_into_tensor(full, x.contiguous(), group=self.group)
        else:
            parts = [torch.empty_like(x) for _ in range(self.cp)]
            dist.all_gather(parts, x.contiguous(), group=self.group)
            full = torch.cat(parts)
        return full.index_select(0, self.gather_idx)

    def reduce_scatter(self, y: torch.Tensor) -> torch.Tensor:
        """[N * T_max, C] rank-major rows, summed over the ranks -> this
        rank's [T_max, C]."""
        import torch.distributed as dist

        if y.is_cuda:
            out = torch.empty(self.T_max, *y.shape[1:], dtype=y.dtype, device=y.device)
            dist.reduce_scatter_tensor(out, y.contiguous(), group=self.group)
            return out
        dist.all_reduce(y, group=self.group)
        return y[self.rank * self.T_max : (self.rank + 1) * self.T_max]

    def last_rows(self, h: torch.Tensor, B: int) -> torch.Tensor:
        """[T_max, D] local hidden -> [B, D] hidden of each request's last
        token (one owner per row, summed over the ranks)."""
        import torch.distributed as dist

        out = torch.zeros(B, h.shape[1], dtype=h.dtype, device=h.device)
        out.index_copy_(0, self.last_dst, h.index_select(0, self.last_src))
        dist.all_reduce(out, group=self.group)
        return out


@dataclass
class MLAAttnMetadata(BaseAttnMetadata):
    req_rows: torch.Tensor   # int32 [B]
    seq_lens: torch.Tensor   # int32 [B]
    cu_q: torch.Tensor       # int32 [B + 1]
    max_q: int
    last_indices: Optional[torch.Tensor] = None
    cp_plan: Optional[CPShardPlan] = None   # token-sharded prefill under context parallelism
    # non-absorbed prefill (kv_b expansion of every key, then 192 / 128-dim
    # attention) when its FLOPs are below the absorbed form's; the key layout
    # for the GPU kernels (None on the CPU, whose reference needs none)
    expanded: bool = False
    prefill_plan: Optional["ops.MlaPrefillPlan"] = None

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
        self.nope = config.qk_nope_head_dim
        self.v_dim = config.v_head_dim
        self.scale = mla_softmax_scale(config)
        self.page_size = ctx.page_size
        self.kv = ctx.kv_cache
        self.device = self.kv.device
        self.capture: Optional[Dict[str, torch.Tensor]] = None
        cp = get_cp_info()
        self.cp_size, self.cp_rank = (cp.size, cp.rank) if cp is not None else (1, 0)

    def forward(self, q: torch.Tensor, layer_id: int, batch: Batch) -> torch.Tensor:
        raise TypeError("the MLA backend takes (q_lat, q_pe): call forward_mla")

    @property
    def cp_group(self):
        import torch.distributed as dist

        return dist.group.WORLD

    def forward_mla(self, q_lat: torch.Tensor, q_pe: torch.Tensor, layer_id: int, batch: Batch) -> torch.Tensor:
        """q_lat [H, T_pad, kv_lora] head-major, q_pe [T, H, rope] ->
        latent output [H, T_pad, kv_lora]; under context parallelism this
        rank's share of it (the shares of all ranks sum to the output)."""
        md = batch.attn_metadata
        assert isinstance(md, MLAAttnMetadata)
        args = (q_lat, q_pe, self.kv.latent(layer_id), get_global_ctx().page_table, md.req_rows, md.seq_lens,
                md.cu_q, self.page_size, self.scale)
        if self.cp_size > 1:
            return ops.mla_attention_share(*args, self.cp_size, self.cp_rank, self.cp_group)
        return ops.mla_attention(*args)

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
        plan = None
        if self.cp_size > 1 and not batch.is_decode:
            import numpy as np

            starts = np.fromiter((r.cached_len for r in reqs), np.int64, B)
            n = np.asarray(qlens, dtype=np.int64)
            offsets = np.cumsum(n) - n
            positions = np.arange(int(n.sum()), dtype=np.int64) - np.repeat(offsets - starts, n)
            plan = CPShardPlan(positions, np.asarray(cu, dtype=np.int64), self.cp_size, self.cp_rank,
                               batch.out_loc, self.device, self.cp_group)
        # a sharded prefill hands the LM head one row per request already
        last = None if batch.is_decode or plan is not None else (cu_q[1:] - 1).long()
        md = MLAAttnMetadata(dev[:B], dev[B : 2 * B], cu_q, max(qlens), last, plan)
        if not batch.is_decode and self.cp_size <= 1 and self.expanded_prefill(lens, qlens):
            md.expanded = True
            if self.device.type == "cuda":
                md.prefill_plan = ops.MlaPrefillPlan(lens, self.device)
        batch.attn_metadata = md

    def expanded_prefill(self, lens: List[int], qlens: List[int]) -> bool:
        """Whether the non-absorbed form costs fewer FLOPs for this batch: per
        head, expanding every key through kv_b_proj costs 2 * kv_lora *
        (nope + v) FLOPs a key, and each query-key pair 2 * (nope + rope + v)
        instead of 2 * (2 * kv_lora + rope). MINISGL_MLA_PREFILL=absorbed
        or =expanded forces one form."""
        import os

        force = os.environ.get("MINISGL_MLA_PREFILL", "")
        if force in ("absorbed", "expanded"):
            return force == "expanded"
        pairs = sum(n * L for n, L in zip(qlens, lens))
        expand = 2 * self.kv_lora * (self.nope + self.v_dim) * sum(lens)
        return expand + 2 * (self.nope + self.rope + self.v_dim) * pairs < 2 * (2 * self.kv_lora + self.rope) * pairs

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
