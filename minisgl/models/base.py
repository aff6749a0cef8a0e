from __future__ import annotations

import torch

from minisgl.layers import BaseOP


class BaseLLMModel(BaseOP):
    """A causal LM: ``forward()`` reads the active batch from the global
    context and returns fp32 logits [batch size, vocab]."""

    def forward(self) -> torch.Tensor:  # pragma: no cover - interface
        raise NotImplementedError
