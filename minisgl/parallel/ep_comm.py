"""NVLink token dispatch for expert parallelism (DP attention).

``EpHeap`` allocates one heap per rank (CUDA IPC handles exchanged over a
gloo group, every peer's heap mapped into this process) laid out as
[signals 4 KB][recv ids][recv rows][back rows] (``minisgl/csrc/ep.cu``):

* ``dispatch(x, topk_ids)``: one kernel stores every (token, slot) row into
  its expert owner's recv rows and marks every rank's recv ids, then waits
  (bounded) for all peers; afterwards ``recv_rows`` / ``recv_ids`` of this
  rank hold the rows sent to it ([world * cap] slots, -1 ids unused);
* ``give_back(ys, pair_pos)``: the rows computed here go back to their
  source ranks' back rows, then a second barrier; ``back`` [cap, H] of this
  rank then holds the expert outputs of its own pairs in pair order.

Both kernels are launched on the current stream with no host
synchronisation. A step's pair count must fit the capacity (tokens x k).
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from minisgl import ops

SIGNAL_BYTES = 4096


def _round(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class _DeviceBuffer:
    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class EpHeap:
    def __init__(self, device: torch.device, cap_pairs: int, hidden: int,
                 group: Optional[dist.ProcessGroup] = None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the NVLink dispatch supports up to 8 ranks")
        self.device = device
        self.cap = cap_pairs
        self.H = hidden
        self.ids_off = SIGNAL_BYTES
        self.rows_off = self.ids_off + _round(self.world * cap_pairs * 4)
        self.back_off = self.rows_off + _round(self.world * cap_pairs * hidden * 2)
        total = self.back_off + _round(cap_pairs * hidden * 2)
        native = ops.native()
        ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.world))
        self._cpu_group = dist.new_group(ranks=ranks, backend="gloo")
        with torch.cuda.device(device):
            own, handle = native.symm_create(total)
        handles: List[Optional[bytes]] = [None] * self.world
        dist.all_gather_object(handles, handle, group=self._cpu_group)
        bases: List[int] = []
        self._opened: List[int] = []
        with torch.cuda.device(device):
            for r in range(self.world):
                if r == self.rank:
                    bases.append(own)
                else:
                    p = native.symm_open(handles[r])
                    self._opened.append(p)
                    bases.append(p)
        self._own = own
        self.bases = torch.tensor(bases, dtype=torch.int64, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        mem = torch.as_tensor(_DeviceBuffer(own, total), device=device)
        self.recv_ids = mem[self.ids_off:self.ids_off + self.world * cap_pairs * 4].view(torch.int32)
        self.recv_rows = mem[self.rows_off:self.rows_off + self.world * cap_pairs * hidden * 2].view(
            torch.bfloat16).view(self.world * cap_pairs, hidden)
        self.back = mem[self.back_off:self.back_off + cap_pairs * hidden * 2].view(torch.bfloat16).view(
            cap_pairs, hidden)
        dist.barrier(group=self._cpu_group)  # every heap is mapped before the first dispatch

    def _geometry(self):
        return (self.bases, self.epoch, self.rank, self.world, self.cap, self.ids_off, self.rows_off, self.back_off)

    def dispatch(self, x: torch.Tensor, topk_ids: torch.Tensor, e_local: int) -> None:
        if topk_ids.numel() > self.cap:
            raise RuntimeError(f"EP dispatch: {topk_ids.numel()} pairs exceed the heap capacity {self.cap}")
        ops._count(2)
        ops.native().ep_dispatch(*self._geometry(), x.contiguous(), topk_ids.to(torch.int32).contiguous(), e_local,
                                 ops.error_word(x.device))

    def give_back(self, ys: torch.Tensor, pair_pos: torch.Tensor) -> None:
        ops._count(2)
        ops.native().ep_return(*self._geometry(), ys, pair_pos, ops.error_word(ys.device))

    def shutdown(self) -> None:
        native = ops.native()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self._cpu_group)  # no peer touches this heap any more
        for p in self._opened:
            native.symm_close(p)
        self._opened = []
        if self._own:
            native.symm_free(self._own)
            self._own = 0
