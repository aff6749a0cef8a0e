"""Tensor-parallel linear layers (Megatron-style sharding).

Column-parallel layers shard output features; row-parallel layers shard
input features and sum partial outputs across ranks. Matmuls run on the
tcgen05 GEMM. Sharding matches the reference (python/minisgl/layers/
linear.py:13-127) so the same checkpoint shards load.
"""

from __future__ import annotations

from typing import List, Optional

import torch

from minisgl import ops
from minisgl.parallel import DistributedCommunicator, get_tp_info
from minisgl.utils import div_even

from .base import BaseOP


class _Linear(BaseOP):
    def __init__(self, full_in: int, full_out: int, local_in: int, local_out: int, has_bias: bool) -> None:
        self.full_input_size = full_in
        self.full_output_size = full_out
        self.local_input_size = local_in
        self.local_output_size = local_out
        self.weight = torch.empty(local_out, local_in)
        self.bias: Optional[torch.Tensor] = torch.empty(local_out) if has_bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.gemm(x, self.weight, self.bias)


class LinearReplicated(_Linear):
    def __init__(self, input_size: int, output_size: int, has_bias: bool) -> None:
        super().__init__(input_size, output_size, input_size, output_size, has_bias)


class LinearColParallelMerged(_Linear):
    """Several column-parallel projections fused along the output (gate|up)."""

    def __init__(self, input_size: int, output_sizes: List[int], has_bias: bool) -> None:
        tp = get_tp_info().size
        local = sum(div_even(s, tp) for s in output_sizes)
        super().__init__(input_size, sum(output_sizes), input_size, local, has_bias)


class LinearQKVMerged(_Linear):
    def __init__(self, hidden_size: int, head_dim: int, num_qo_heads: int, num_kv_heads: int, has_bias: bool) -> None:
        tp = get_tp_info().size
        q = div_even(num_qo_heads, tp)
        kv = div_even(num_kv_heads, tp, allow_replicate=True)
        super().__init__(hidden_size, (num_qo_heads + 2 * num_kv_heads) * head_dim, hidden_size,
                         (q + 2 * kv) * head_dim, has_bias)


class LinearRowParallel(_Linear):
    def __init__(self, input_size: int, output_size: int, has_bias: bool) -> None:
        self._tp = get_tp_info().size
        self._comm = DistributedCommunicator()
        super().__init__(input_size, output_size, div_even(input_size, self._tp), output_size, has_bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = ops.gemm(x, self.weight, self.bias)
        return self._comm.all_reduce(y) if self._tp > 1 else y

    def forward_residual(self, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """residual + x @ w^T with the add fused into the GEMM epilogue. One
        rank: written into ``residual`` in place. Several ranks: rank 0 adds
        the residual to its partial product and the all-reduce sums the
        partials, so every rank gets residual + the full product."""
        if self._tp == 1:
            return ops.gemm_fused(x, self.weight, bias=self.bias, residual=residual, out=residual)
        first = get_tp_info().rank == 0
        plugin = DistributedCommunicator.plugins[-1]
        if hasattr(plugin, "gemm_reduce_into") and x.is_cuda:
            # NVLink collectives: the GEMM exchanges its output tiles with the
            # other ranks and adds the residual in one kernel
            return plugin.gemm_reduce_into(x, self.weight, self.bias, residual)
        y = ops.gemm_fused(x, self.weight, bias=self.bias if first else None, residual=residual if first else None)
        return self._comm.all_reduce(y)


class LinearOProj(LinearRowParallel):
    """The attention output projection (row parallel)."""
