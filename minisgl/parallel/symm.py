"""Tensor-parallel collectives from our own kernels over NVLink peer memory.

``--comm fused`` registers ``SymmMemImpl`` as the communicator plugin. Each
rank allocates a symmetric heap (same size on every rank, CUDA IPC handles
exchanged over a gloo group, every peer's heap mapped into this process) and
the collectives are one kernel each (``minisgl/csrc/symm.cu``): a one-shot
all-reduce that sums every rank's partial over NVLink in rank order, with the
residual add fused, and an all-gather; both synchronise through flags in the
heaps with bounded waits. No NCCL call and no NVLS multicast object is used
on this path.

The row-parallel projections (o_proj, down_proj) go through
``gemm_reduce_into``. For a few rows it is one kernel: every output tile is
computed, written into this rank's heap, exchanged with the same tile of the
other ranks over NVLink and summed with the residual in the GEMM's epilogue,
tile by tile, so the transfer of one tile overlaps the math of the others.
For more rows the tuned plain GEMM writes its partial into the heap and one
NVLink kernel reduces it (faster there: no split-path parking).

The reference's counterpart is the PyNCCL plugin over NCCL symmetric windows
(python/minisgl/kernel/pynccl.py, src/pynccl.cu:72-188).
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from minisgl import ops
from minisgl.utils import fault

from .comm import DistributedImpl, register_plugin

SIGNAL_BYTES = 4096
FLAG_BYTES = 16384  # per-CTA flags of the GEMM with the all-reduce fused
DATA_OFFSET = SIGNAL_BYTES + FLAG_BYTES


class _DeviceBuffer:
    """Exposes a raw device address as a torch tensor (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class SymmMemImpl(DistributedImpl):
    # rows up to which the row-parallel GEMM with the all-reduce in one kernel
    # is used (Qwen3-32B TP2 on B200: 44.0 vs 47.1 us for NCCL at 1 row of
    # down_proj; from 64 rows the GEMM + NVLink-kernel pair is faster)
    ONE_KERNEL_MAX_ROWS = 16

    def __init__(self, device: torch.device, capacity_bytes: int, group: Optional[dist.ProcessGroup] = None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the NVLink collectives support up to 8 ranks")
        self.device = device
        self.capacity = (max(capacity_bytes, 1 << 20) + 255) // 256 * 256
        native = ops.native()
        ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.world))
        self._cpu_group = dist.new_group(ranks=ranks, backend="gloo")
        with torch.cuda.device(device):
            # [signals][GEMM flags][collective data][two GEMM partial halves]
            # [gathered rows of the sequence-parallel collective]
            own, handle = native.symm_create(DATA_OFFSET + 4 * self.capacity)
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
        # call counters: [0] the fused GEMM + all-reduce, [1] the collective kernels
        self.epoch = torch.zeros(2, dtype=torch.int32, device=device)
        self.calls = 0  # collective launches so far (the fault-injection clock)
        self._faults = bool(fault.rules())
        self.data = torch.as_tensor(_DeviceBuffer(own + DATA_OFFSET, self.capacity), device=device)
        self.gather_offset = DATA_OFFSET + 3 * self.capacity
        self.gathered = torch.as_tensor(_DeviceBuffer(own + self.gather_offset, self.capacity), device=device)
        dist.barrier(group=self._cpu_group)  # every heap is mapped before the first collective

    # -------------------------------------------------------------- buffers
    def partial_buffer(self, rows: int, cols: int, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """This rank's heap data region viewed as [rows, cols]: a GEMM writes
        its partial product here and ``reduce_into`` sums the partials."""
        n = rows * cols * torch.finfo(dtype).bits // 8
        if n > self.capacity:
            raise RuntimeError(f"symmetric heap too small: {n} > {self.capacity} bytes")
        return self.data[:n].view(dtype).view(rows, cols)

    def _collective(self, kind: int, out: torch.Tensor, n_elems: int, residual: Optional[torch.Tensor] = None,
                    rows: int = 0, row_elems: int = 0) -> None:
        self.calls += 1
        if self._faults and fault.skip_collective(self.rank, self.calls - 1):
            return  # injected: this rank never arrives, the peers' bounded waits expire
        ops._count(2)
        ops.native().symm_collective(kind, out, residual, self.bases, self.epoch[1:], self.rank, self.world, n_elems,
                                     rows, row_elems, ops.error_word(out.device))

    # ----------------------------------------------- sequence parallelism
    # The decoder keeps the residual stream token-sharded between layers
    # (rank r holds rows [r * T / R, (r + 1) * T / R)); each row-parallel
    # projection writes its partial product into ``sp_partial`` and
    # ``rs_norm_ag`` reduce-scatters it into the residual slice, normalises the
    # new rows and gathers them on every rank for the next column-parallel GEMM.
    sequence_parallel = True

    def sp_partial(self, rows: int, cols: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        """Where a row-parallel GEMM writes its partial product [rows, cols]."""
        return self.partial_buffer(rows, cols, dtype)

    def rs_norm_ag(self, partial: torch.Tensor, resid: torch.Tensor, add_resid: bool,
                   norm_w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
        """Reduce-scatter ``partial`` (an ``sp_partial`` view, [R * rows, H])
        into ``resid`` [rows, H] (added to it when ``add_resid``), RMS-normalise
        the new rows (times ``norm_w`` when given) and return all ranks'
        normalised rows [R * rows, H] (a view of the heap's gather region, valid
        until the next call). One kernel (``minisgl/csrc/symm.cu``)."""
        rows, H = resid.shape
        assert partial.data_ptr() == self.data.data_ptr() and partial.shape == (rows * self.world, H)
        if 2 * rows * self.world * H > self.capacity:
            raise RuntimeError("symmetric heap too small for the sequence-parallel collective")
        self.calls += 1
        if self._faults and fault.skip_collective(self.rank, self.calls - 1):
            return self.gathered[: 2 * rows * self.world * H].view(torch.bfloat16).view(rows * self.world, H)
        ops._count(2)
        ops.native().symm_rsn(resid, add_resid, norm_w, eps, self.bases, self.epoch[1:], self.rank, self.world,
                              DATA_OFFSET, self.gather_offset, ops.error_word(resid.device))
        return self.gathered[: 2 * rows * self.world * H].view(torch.bfloat16).view(rows * self.world, H)

    # ---------------------------------------------------------- collectives
    def gemm_reduce_into(self, x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor],
                         residual: torch.Tensor) -> torch.Tensor:
        """residual += all-reduce over ranks of x @ w^T (+ bias, added by rank
        0): one kernel computes each output tile, exchanges it with the other
        ranks over NVLink and adds the residual, when the whole grid fits on
        the GPU at once; otherwise the GEMM writes into the heap and the
        collective kernel reduces. Plans are the tuned fused-epilogue plans,
        which the engine keeps identical on every rank."""
        M = x.shape[0]
        if M > self.ONE_KERNEL_MAX_ROWS:
            # measured faster beyond a few rows: the tuned plain GEMM (no cluster
            # parking) into the heap, then the NVLink all-reduce kernel
            part = self.partial_buffer(M, w.shape[0])
            ops.gemm(x, w, bias if self.rank == 0 else None, out=part)
            return self.reduce_into(part, residual)
        plan = ops._gemm_fused_plans.get((M, w.shape[0], x.shape[1]), (0, 0, 0))
        ops._count(2)
        ops.native().gemm_allreduce(residual, x, w, bias if self.rank == 0 else None, self.bases, self.epoch,
                                    self._own, self.rank, self.world, self.capacity, plan[0], plan[2], plan[1],
                                    ops.error_word(x.device))
        return residual

    def reduce_into(self, partial: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """residual += sum of every rank's ``partial`` (a ``partial_buffer``),
        in place."""
        self._collective(0, residual, partial.numel(), residual=residual)
        return residual

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != torch.bfloat16 or x.numel() % 8 != 0 or 2 * x.numel() > self.capacity:
            dist.all_reduce(x, group=self.group)  # outside the kernel's domain: library collective
            return x
        buf = self.partial_buffer(x.numel(), 1).view(x.shape)
        buf.copy_(x)
        self._collective(0, x, x.numel())
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """Rows of every rank concatenated; a byte copy, so 16- and 32-bit
        tensors both go through the kernel (as bf16 units)."""
        rows = x.shape[0]
        out = x.new_empty((rows * self.world,) + tuple(x.shape[1:]))
        units = x.contiguous().view(-1).view(torch.bfloat16) if x.element_size() in (2, 4) else None
        row = units.numel() // max(rows, 1) if units is not None else 0
        if units is None or rows == 0 or row % 8 != 0 or 2 * units.numel() > self.capacity:
            dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
            return out
        self.partial_buffer(units.numel(), 1).view(-1).copy_(units)
        self._collective(1, out.view(-1).view(torch.bfloat16), units.numel(), rows=rows, row_elems=row)
        return out

    def shutdown(self) -> None:
        native = ops.native()
        torch.cuda.synchronize(self.device)
        if self._cpu_group is not None:
            dist.barrier(group=self._cpu_group)  # no peer reads this heap any more
        for p in self._opened:
            native.symm_close(p)
        self._opened = []
        if self._own:
            native.symm_free(self._own)
            self._own = 0


def enable_symm_comm(device: torch.device, capacity_bytes: int) -> SymmMemImpl:
    """Register the NVLink collectives as the tensor-parallel communicator."""
    impl = SymmMemImpl(device, capacity_bytes)
    register_plugin(impl)
    return impl
