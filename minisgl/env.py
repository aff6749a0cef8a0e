"""Process-wide settings read from MINISGL_* environment variables.

Same variables and defaults as the reference (python/minisgl/env.py:58-87),
plus the B200-specific switches of this engine.
"""

from __future__ import annotations

import os
from typing import Callable, Generic, Optional, TypeVar

T = TypeVar("T")
PREFIX = "MINISGL_"


def _to_bool(s: str) -> bool:
    return s.strip().lower() in ("1", "true", "yes", "on")


def _to_bytes(s: str) -> int:
    s = s.strip().upper().removesuffix("B")
    units = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    if s and s[-1] in units:
        return int(float(s[:-1]) * units[s[-1]])
    return int(s)


class EnvVar(Generic[T]):
    def __init__(self, default: T, parse: Callable[[str], T]) -> None:
        self.default = default
        self.parse = parse
        self.value: T = default
        self.name = ""

    def load(self, name: str) -> None:
        self.name = name
        raw = os.getenv(name)
        self.value = self.default
        if raw is not None:
            try:
                self.value = self.parse(raw)
            except (ValueError, TypeError):
                pass

    def __bool__(self) -> bool:
        return bool(self.value)

    def __str__(self) -> str:
        return str(self.value)


def _int(d: int) -> EnvVar[int]:
    return EnvVar(d, int)


def _float(d: float) -> EnvVar[float]:
    return EnvVar(d, float)


def _bool(d: bool) -> EnvVar[bool]:
    return EnvVar(d, _to_bool)


def _opt_bool() -> EnvVar[Optional[bool]]:
    return EnvVar(None, _to_bool)


def _mem(d: int) -> EnvVar[int]:
    return EnvVar(d, _to_bytes)


class _Env:
    # interactive shell defaults
    SHELL_MAX_TOKENS = _int(2048)
    SHELL_TOP_K = _int(-1)
    SHELL_TOP_P = _float(1.0)
    SHELL_TEMPERATURE = _float(0.6)
    # runtime
    FLASHINFER_USE_TENSOR_CORES = _opt_bool()  # accepted for compatibility; no effect here
    DISABLE_OVERLAP_SCHEDULING = _bool(False)
    PYNCCL_MAX_BUFFER_SIZE = _mem(1 << 30)
    # B200 engine switches
    DEBUG_CHECK_ERRORS = _bool(False)   # read the kernel error word after every step
    DEBUG_BOUNDS = _bool(False)         # check every KV slot a batch touches against the pool (host, syncs)
    BROADCAST_TIMEOUT_S = _float(60.0)  # a rank's wait for a request message rank 0 counted for it
    STATS_INTERVAL = _int(0)            # log a stats line every N steps (0 = off)
    SAMPLING_SEED = _int(0)
    NO_FUSED_SAMPLING = _bool(False)    # sample from materialised logits even when the LM head could
    CUDA_PROFILER_STEPS = EnvVar("", str)  # "a:b": cudaProfilerStart before step a, Stop before step b

    def __init__(self) -> None:
        self.reload()

    def reload(self) -> None:
        for name in dir(type(self)):
            var = getattr(type(self), name)
            if isinstance(var, EnvVar):
                var.load(PREFIX + name)


ENV = _Env()
