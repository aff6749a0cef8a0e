"""Tensor-parallel collectives behind a plugin stack.

The layers call ``DistributedCommunicator().all_reduce / all_gather``; the
last registered plugin serves the call (the reference's design,
python/minisgl/distributed/impl.py:63-70). Plugins here:

* ``TorchDistributedImpl``: torch.distributed on the default process group
  (NCCL on GPUs, gloo for CPU ranks). This is the NCCL baseline.
* ``minisgl.parallel.symm.SymmMemImpl`` (registered by the engine when
  ``--comm fused``): one-shot all-reduce / all-gather kernels that read peer
  buffers directly over NVLink from symmetric memory.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import List, Optional

import torch
import torch.distributed as dist


class DistributedImpl(ABC):
    @abstractmethod
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor: ...

    @abstractmethod
    def all_gather(self, x: torch.Tensor) -> torch.Tensor: ...

    def shutdown(self) -> None:
        return None


class TorchDistributedImpl(DistributedImpl):
    """``sequence_parallel``: when set, the decoder keeps a token-sharded
    residual stream and calls ``rs_norm_ag`` (stated with the collectives
    below) instead of all-reducing after every row-parallel projection; it is
    off for this baseline plugin and switched on by tests that compare the two
    forms on CPU ranks."""

    sequence_parallel = False

    def __init__(self, group: Optional[dist.ProcessGroup] = None) -> None:
        self.group = group

    def sp_partial(self, rows: int, cols: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        return torch.empty(rows, cols, dtype=dtype, device=device)

    def rs_norm_ag(self, partial: torch.Tensor, resid: torch.Tensor, add_resid: bool,
                   norm_w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
        return rs_norm_ag_reference(self, partial, resid, add_resid, norm_w, eps)

    def _size(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self._size() > 1:
            dist.all_reduce(x, op=dist.ReduceOp.SUM, group=self.group)
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        n = self._size()
        if n == 1:
            return x
        out = x.new_empty((x.shape[0] * n,) + tuple(x.shape[1:]))
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out


def rs_norm_ag_reference(comm: "DistributedImpl", partial: torch.Tensor, resid: torch.Tensor, add_resid: bool,
                         norm_w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """The sequence-parallel collective stated with library collectives: sum
    the partials of every rank, keep this rank's rows as the new residual
    slice (rounded like a bf16 all-reduce, then the residual added), RMSNorm
    them and gather every rank's normalised rows."""
    from minisgl.ops import reference as ref

    rows = resid.shape[0]
    rank = dist.get_rank(getattr(comm, "group", None)) if dist.is_initialized() else 0
    full = comm.all_reduce(partial)
    mine = full[rank * rows:(rank + 1) * rows]
    new = (mine.float() + resid.float()).to(resid.dtype) if add_resid else mine.to(resid.dtype)
    resid.copy_(new)
    return comm.all_gather(ref.rmsnorm(new, norm_w, eps) if not new.is_cuda else _rmsnorm(new, norm_w, eps))


def _rmsnorm(x: torch.Tensor, w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    from minisgl import ops

    return ops.rmsnorm(x, w, eps)


class DistributedCommunicator:
    plugins: List[DistributedImpl] = [TorchDistributedImpl()]

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return self.plugins[-1].all_reduce(x)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return self.plugins[-1].all_gather(x)


def sequence_parallel_comm() -> Optional[DistributedImpl]:
    """The active plugin when it runs the decoder sequence-parallel (tensor
    parallelism over more than one rank and a plugin with
    ``sequence_parallel`` set), else None."""
    from .info import get_tp_info

    plugin = DistributedCommunicator.plugins[-1]
    if get_tp_info().size > 1 and getattr(plugin, "sequence_parallel", False):
        return plugin
    return None


def register_plugin(impl: DistributedImpl) -> None:
    DistributedCommunicator.plugins.append(impl)


def destroy_distributed() -> None:
    for p in DistributedCommunicator.plugins:
        p.shutdown()
    DistributedCommunicator.plugins = [TorchDistributedImpl()]
