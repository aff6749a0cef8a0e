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
    def __init__(self, group: Optional[dist.ProcessGroup] = None) -> None:
        self.group = group

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


class DistributedCommunicator:
    plugins: List[DistributedImpl] = [TorchDistributedImpl()]

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return self.plugins[-1].all_reduce(x)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return self.plugins[-1].all_gather(x)


def register_plugin(impl: DistributedImpl) -> None:
    DistributedCommunicator.plugins.append(impl)


def destroy_distributed() -> None:
    for p in DistributedCommunicator.plugins:
        p.shutdown()
    DistributedCommunicator.plugins = [TorchDistributedImpl()]
