"""RMSNorm layers backed by the native row kernels."""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from minisgl import ops

from .base import BaseOP


class RMSNorm(BaseOP):
    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self.eps)

    def forward_inplace(self, x: torch.Tensor) -> None:
        ops.rmsnorm(x, self.weight, self.eps, out=x)


class RMSNormFused(BaseOP):
    """First call (no residual yet): y = norm(x), residual = x. Later calls:
    residual += x and x = norm(residual), in place."""

    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        if residual is None:
            return ops.rmsnorm(x, self.weight, self.eps), x
        ops.fused_add_rmsnorm(x, residual, self.weight, self.eps)
        return x, residual
