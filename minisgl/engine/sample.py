"""Batch sampler: greedy argmax or temperature / top-k / top-p sampling on
the device (sm_100a kernels; see ``minisgl/csrc/sampling.cu``).

Clamping of user parameters follows the reference
(python/minisgl/engine/sample.py:53-68): temperatures and top-p are floored
at 1e-6, top-k < 1 means the whole vocabulary.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Optional

import torch

from minisgl import ops
from minisgl.env import ENV
from minisgl.utils import nvtx_annotate

if TYPE_CHECKING:
    from minisgl.core import Batch


@dataclass
class BatchSamplingArgs:
    temperatures: Optional[torch.Tensor]
    top_k: Optional[torch.Tensor] = None
    top_p: Optional[torch.Tensor] = None


class Sampler:
    def __init__(self, device: torch.device, vocab_size: int, seed: int = 0) -> None:
        self.device = device
        self.vocab_size = vocab_size
        self.seed = seed or ENV.SAMPLING_SEED.value
        # device-resident step counter advanced by the sampling kernel itself
        self.step = torch.zeros((), dtype=torch.int64, device=device)
        self.generator = torch.Generator(device="cpu").manual_seed(self.seed) if device.type == "cpu" else None

    def prepare(self, batch: "Batch") -> BatchSamplingArgs:
        params = [r.sampling_params for r in batch.reqs]
        if all(p.is_greedy for p in params):
            return BatchSamplingArgs(None)
        temps = [max(0.0 if p.is_greedy else p.temperature, 1e-6) for p in params]
        ks = [p.top_k if p.top_k >= 1 else self.vocab_size for p in params]
        ps = [min(max(p.top_p, 1e-6), 1.0) for p in params]
        use_k = any(k != self.vocab_size for k in ks)
        use_p = any(p < 1.0 for p in ps)
        pin = self.device.type == "cuda"
        t = torch.tensor(temps, dtype=torch.float32, pin_memory=pin).to(self.device, non_blocking=True)
        k = torch.tensor(ks, dtype=torch.int32, pin_memory=pin).to(self.device, non_blocking=True) if use_k else None
        p = torch.tensor(ps, dtype=torch.float32, pin_memory=pin).to(self.device, non_blocking=True) if use_p else None
        return BatchSamplingArgs(t, k, p)

    # rows up to which sampling inside the LM-head GEMM is faster than GEMM +
    # sampling kernel on a B200 (Qwen3 vocabulary: 120 vs 140 us at 32 rows;
    # at 256 rows the epilogue's noise work, serial behind each tile's
    # mainloop at one CTA per SM, makes it 2x slower)
    FUSED_MAX_ROWS = 64

    def fusable(self, args: BatchSamplingArgs, rows: int) -> bool:
        """Greedy and temperature-only batches of at most FUSED_MAX_ROWS rows
        are sampled inside the LM-head GEMM (same random stream, same
        tokens); top-k / top-p batches need the logits."""
        return (self.device.type == "cuda" and rows <= self.FUSED_MAX_ROWS and args.top_k is None
                and args.top_p is None and not ENV.NO_FUSED_SAMPLING.value)

    @nvtx_annotate("Sampler")
    def sample(self, logits: torch.Tensor, args: BatchSamplingArgs) -> torch.Tensor:
        if args.temperatures is None:
            return ops.argmax(logits)
        return ops.sample(logits, args.temperatures, args.top_k, args.top_p, self.seed, self.step,
                          generator=self.generator)
