"""Synthetic request pools of the serving benchmarks (standard library
only: ``bench.py`` loads this file by path, also in the reference arm's
process, whose ``minisgl`` package is the reference's).

Shapes:
  qwen3-32b (default)  prompts lognormal (median 1024, in [32, 16384]),
                       outputs lognormal (median 256, in [16, 2048]); 30 %
                       of the prompts start with one of 50 seeded shared
                       prefixes of 512-2048 tokens (the radix cache serves them)
  qwen3-0.6b           prompts and outputs uniform in [100, 1024] (the
                       reference's offline benchmark,
                       benchmark/offline/bench.py:12-30)
  kimi-k2              prompts uniform in [512, 4096], outputs in [128, 1024]

The same (shape, size, seed) gives the same pool on every rank and in both
arms of the benchmark.
"""

from __future__ import annotations

import math
import random
from typing import List, Tuple


def lognormal_len(rng: random.Random, median: float, sigma: float, lo: int, hi: int) -> int:
    return int(min(hi, max(lo, round(median * math.exp(rng.gauss(0.0, sigma))))))


def make_pool(shape: str, num_reqs: int, seed: int, vocab_limit: int = 10000) -> Tuple[List[List[int]], List[int]]:
    """(prompt token ids, output lengths) of ``num_reqs`` requests."""
    rng = random.Random(seed * 1_000_003 + 17)
    prompts: List[List[int]] = []
    outs: List[int] = []
    if shape == "qwen3-0.6b":  # the reference's offline benchmark distributions
        for _ in range(num_reqs):
            prompts.append([rng.randrange(vocab_limit) for _ in range(rng.randint(100, 1024))])
            outs.append(rng.randint(100, 1024))
        return prompts, outs
    if shape == "kimi-k2":  # the expert-parallel serving config
        for _ in range(num_reqs):
            prompts.append([rng.randrange(vocab_limit) for _ in range(rng.randint(512, 4096))])
            outs.append(rng.randint(128, 1024))
        return prompts, outs
    prefixes = [[rng.randrange(vocab_limit) for _ in range(rng.randint(512, 2048))] for _ in range(50)]
    for _ in range(num_reqs):
        n = lognormal_len(rng, 1024, 0.8, 32, 16384)
        if rng.random() < 0.3:
            pre = prefixes[rng.randrange(len(prefixes))]
            tail = max(16, n - len(pre))
            prompts.append(pre + [rng.randrange(vocab_limit) for _ in range(tail)])
        else:
            prompts.append([rng.randrange(vocab_limit) for _ in range(n)])
        outs.append(lognormal_len(rng, 256, 0.8, 16, 2048))
    return prompts, outs
