"""Scheduler configuration: the engine's settings plus the prefill budget,
the prefix-cache kind, offline mode and the local IPC endpoints.

The public field names (``max_extend_tokens``, ``cache_type``,
``offline_mode``) and address properties are the ones the launcher, the
server arguments and the offline API use (reference counterpart:
python/minisgl/scheduler/config.py:14-41). Endpoints are named per launch:
``ipc:///tmp/minisgl-<namespace>-<role>``, where the namespace is drawn when
the configuration is created and travels with it to every spawned process,
so two servers on one machine never share a socket.
"""

from __future__ import annotations

import os
import uuid
from dataclasses import dataclass, field

from minisgl.engine import EngineConfig


def _fresh_namespace() -> str:
    return f"{os.getpid()}-{uuid.uuid4().hex[:8]}"


@dataclass(frozen=True)
class SchedulerConfig(EngineConfig):
    max_extend_tokens: int = 8192  # prefill tokens per scheduler step (chunked prefill budget)
    cache_type: str = "radix"      # prefix cache: "radix" or "naive"
    offline_mode: bool = False     # in-process LLM API instead of ZMQ sockets
    ipc_namespace: str = field(default_factory=_fresh_namespace)

    def ipc_endpoint(self, role: str) -> str:
        return f"ipc:///tmp/minisgl-{self.ipc_namespace}-{role}"

    # tokenizer -> scheduler rank 0
    @property
    def zmq_backend_addr(self) -> str:
        return self.ipc_endpoint("backend")

    # scheduler rank 0 -> detokenizer
    @property
    def zmq_detokenizer_addr(self) -> str:
        return self.ipc_endpoint("detokenizer")

    # scheduler rank 0 -> the other ranks (request fan-out)
    @property
    def zmq_scheduler_broadcast_addr(self) -> str:
        return self.ipc_endpoint("rank-fanout")

    @property
    def max_forward_len(self) -> int:
        """Most tokens one forward pass can carry (the prefill budget)."""
        return self.max_extend_tokens

    @property
    def backend_create_detokenizer_link(self) -> bool:
        return True
