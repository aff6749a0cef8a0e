"""Expert parallelism with token dispatch (DP attention).

Under ``--enable-dp-attention`` every rank serves its own requests with a
replicated copy of everything but the routed experts, which are split over
the ranks (rank r holds experts [r E / R, (r + 1) E / R)). Each MoE layer:

1. routes its own tokens over all experts (router kernel);
2. dispatch: sorts the (token, slot) pairs by owning rank and sends each
   pair's hidden row and local expert id to its owner (all-to-all; the
   counts go first so every receiver knows its row count);
3. runs its local experts over the rows it received (the grouped tcgen05
   expert pipeline, bf16 or MXFP4, one slot per row);
4. combine: returns every row to the rank it came from (the reverse
   all-to-all) and sums each token's k rows weighted by the router, in slot
   order (deterministic).

With ``--comm fused`` on GPUs the rows move by peer stores over NVLink from
our own kernels (``minisgl/parallel/ep_comm.py``, ``csrc/ep.cu``: no host
synchronisation); otherwise with ``torch.distributed.all_to_all_single``
(NCCL, or gloo on CPU ranks). The peer-store path launches only kernels
with fixed-capacity buffers, so decode steps run as CUDA graphs even when
the ranks replay graphs of different batch sizes. The reference has neither DP attention nor expert
parallelism (its MoE is the TP-sharded Triton fused_moe kernel:
python/minisgl/moe/fused.py, python/minisgl/kernel/triton/fused_moe.py).
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from minisgl import ops

from .base import BaseMoeBackend
from .fused import FusedMoe


class AllToAllMoe(BaseMoeBackend):
    def __init__(self, ep_size: int, ep_rank: int, group: Optional[dist.ProcessGroup] = None,
                 heap=None) -> None:
        self.ep_size = ep_size
        self.ep_rank = ep_rank
        self.group = group
        self.heap = heap  # EpHeap: the NVLink dispatch (``--comm fused``), else torch.distributed
        self.local = FusedMoe()  # runs this rank's experts on the rows it received
        self._ident: dict = {}

    def _forward_nvlink(self, x, w1, w2, topk_w, topk_ids, e_local, mxfp4):
        """Peer-store dispatch, local experts over the receive buffer, peer-store
        return, weighted combine (no host synchronisation)."""
        heap = self.heap
        T, H = x.shape
        k = topk_ids.shape[1]
        heap.dispatch(x, topk_ids, e_local)
        rows, ids = heap.recv_rows, heap.recv_ids.view(-1, 1)
        ones = torch.ones(rows.shape[0], 1, dtype=torch.float32, device=x.device)
        if mxfp4 is not None:
            ys, pair_pos = ops.moe_experts_rows(rows, ones, ids, mxfp4=mxfp4)
        else:
            ys, pair_pos = ops.moe_experts_rows(rows, ones, ids, w1=w1, w2=w2)
        heap.give_back(ys, pair_pos)
        n = T * k
        ident = self._ident.get(n)
        if ident is None:
            ident = self._ident[n] = torch.arange(n, dtype=torch.int32, device=x.device)
        return ops.moe_combine(heap.back[:n], topk_w, ident, T, k)

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: List[int], in_splits: List[int]) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, gating_output: torch.Tensor,
                topk: int, renormalize: bool, activation: str = "silu", scoring: str = "softmax",
                correction_bias: Optional[torch.Tensor] = None, n_group: int = 1, topk_group: int = 1,
                routed_scale: float = 1.0, interleaved: bool = False, expert_offset: int = 0,
                mxfp4: Optional[tuple] = None) -> torch.Tensor:
        x = hidden_states
        T, H = x.shape
        dev = x.device
        topk_w, topk_ids = ops.moe_route(gating_output, topk, scoring, renormalize, correction_bias, n_group,
                                         topk_group, routed_scale)
        e_local = (mxfp4[0] if mxfp4 is not None else w1).shape[0]
        if self.heap is not None and x.is_cuda:
            return self._forward_nvlink(x, w1, w2, topk_w, topk_ids, e_local, mxfp4)
        ids = topk_ids.reshape(-1).long()
        dest = ids // e_local
        order = torch.argsort(dest, stable=True)  # pairs grouped by owning rank, slot order inside
        send_counts = torch.bincount(dest, minlength=self.ep_size).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, [1] * self.ep_size, [1] * self.ep_size)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        # dispatch: hidden rows and local expert ids to the owners
        send_x = x[order // topk].contiguous()
        send_e = (ids[order] - dest[order] * e_local).to(torch.int32)
        recv_x = x.new_empty(sum(rc), H)
        recv_e = torch.empty(sum(rc), dtype=torch.int32, device=dev)
        self._a2a(recv_x, send_x, rc, sc)
        self._a2a(recv_e, send_e, rc, sc)
        # local experts, one slot per received row (weight 1)
        R = recv_x.shape[0]
        ones = torch.ones(R, 1, dtype=torch.float32, device=dev)
        if R == 0:
            y = recv_x
        elif not x.is_cuda:
            from .fused import moe_reference

            if getattr(mxfp4, "blocked", None) is not None and interleaved:
                from minisgl.quant import moe_experts_mx_reference

                y = moe_experts_mx_reference(recv_x, *mxfp4, ones, recv_e[:, None]).to(recv_x.dtype)
            else:
                lw1, lw2 = self.local._cpu_weights(mxfp4) if mxfp4 is not None else (w1, w2)
                y = moe_reference(recv_x, lw1, lw2, ones, recv_e[:, None], activation, interleaved)
        elif mxfp4 is not None:
            y = ops.moe_experts_quantised(recv_x, mxfp4, ones, recv_e[:, None])
        else:
            y = ops.moe_experts(recv_x, w1, w2, ones, recv_e[:, None])
        # combine: rows back to their source, weighted sum over each token's slots
        back = x.new_empty(send_x.shape[0], H)
        self._a2a(back, y.contiguous(), sc, rc)
        pairs = x.new_empty(T * topk, H)
        pairs[order] = back
        out = (pairs.view(T, topk, H).float() * topk_w.view(T, topk, 1).float()).sum(dim=1)
        return out.to(x.dtype)


class ContextParallelMoe(BaseMoeBackend):
    """Routed experts split over the context-parallel ranks. A token-sharded
    prefill batch holds different tokens on every rank, so its rows go to
    their experts' owners and back (``AllToAllMoe``); a decode batch runs
    replicated, so each rank applies its own experts to every row (the others
    contribute nothing) and one all-reduce over the ranks sums the parts."""

    def __init__(self, ep_size: int, ep_rank: int, group: Optional[dist.ProcessGroup] = None) -> None:
        self.dispatch = AllToAllMoe(ep_size, ep_rank, group)
        self.local = FusedMoe()
        self.group = group

    def forward(self, hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, gating_output: torch.Tensor,
                topk: int, renormalize: bool, activation: str = "silu", scoring: str = "softmax",
                correction_bias: Optional[torch.Tensor] = None, n_group: int = 1, topk_group: int = 1,
                routed_scale: float = 1.0, interleaved: bool = False, expert_offset: int = 0,
                mxfp4: Optional[tuple] = None) -> torch.Tensor:
        from minisgl.core import get_global_ctx

        kw = dict(hidden_states=hidden_states, w1=w1, w2=w2, gating_output=gating_output, topk=topk,
                  renormalize=renormalize, activation=activation, scoring=scoring, correction_bias=correction_bias,
                  n_group=n_group, topk_group=topk_group, routed_scale=routed_scale, interleaved=interleaved,
                  mxfp4=mxfp4)
        md = getattr(get_global_ctx().batch, "attn_metadata", None)
        if getattr(md, "cp_plan", None) is not None:
            return self.dispatch.forward(**kw)
        out = self.local.forward(expert_offset=expert_offset, **kw)
        dist.all_reduce(out, group=self.group)
        return out
