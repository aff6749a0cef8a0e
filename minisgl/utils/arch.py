"""Device capability probes."""

from __future__ import annotations

import functools
from typing import Optional, Tuple


@functools.lru_cache(maxsize=None)
def device_capability() -> Optional[Tuple[int, int]]:
    import torch

    if not torch.cuda.is_available():
        return None
    return torch.cuda.get_device_capability()


def is_arch_supported(major: int, minor: int = 0) -> bool:
    cap = device_capability()
    return cap is not None and cap >= (major, minor)


def is_sm90_supported() -> bool:
    return is_arch_supported(9, 0)


def is_sm100_supported() -> bool:
    return is_arch_supported(10, 0)
