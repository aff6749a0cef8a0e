from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Optional

import torch


class BaseMoeBackend(ABC):
    @abstractmethod
    def forward(self, hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, gating_output: torch.Tensor,
                topk: int, renormalize: bool, activation: str = "silu", scoring: str = "softmax",
                correction_bias: Optional[torch.Tensor] = None, n_group: int = 1, topk_group: int = 1,
                routed_scale: float = 1.0, interleaved: bool = False, expert_offset: int = 0,
                mxfp4: Optional[tuple] = None) -> torch.Tensor:
        """sum_k w[t, k] * down_e(act(gate_up_e(x_t))) for the k routed experts.
        ``interleaved``: each expert's gate|up rows alternate in 64-row blocks.
        ``expert_offset``: global id of local expert 0 (expert parallelism;
        experts outside the local range contribute nothing here).
        ``mxfp4``: (w1 packed, w1 scales, w2 packed, w2 scales) replacing w1 / w2."""
