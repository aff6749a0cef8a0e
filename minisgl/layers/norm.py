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
    residual += x and x = norm(residual), in place.

    ``folded`` (set by the owning layer after loading): the weight has been
    multiplied into the columns of the projection that consumes this norm,
    so the norm itself runs without a weight."""

    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size)
        self._folded = False

    def fold(self) -> None:
        self._folded = True

    @property
    def folded(self) -> bool:
        return self._folded

    @property
    def active_weight(self) -> Optional[torch.Tensor]:
        """The weight the norm itself applies (None once folded)."""
        return None if self._folded else self.weight

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        w = None if self._folded else self.weight
        if residual is None:
            return ops.rmsnorm(x, w, self.eps), x
        ops.fused_add_rmsnorm(x, residual, w, self.eps)
        return x, residual
