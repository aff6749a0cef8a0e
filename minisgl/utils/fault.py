"""Host-side fault injection for failure-detection tests.

``MINISGL_FAULT_INJECT`` holds ``;``-separated rules
``<action>:rank=<r>[:step=<s>][:seconds=<t>]``; a rule fires on rank r (the
tensor-parallel rank) at engine step s (default 0):

* ``raise``  — the engine raises ``InjectedFault`` before the step's forward;
* ``stall``  — the engine sleeps ``seconds`` (default 30) before the forward,
  so its peers' next collective runs into the process-group timeout;
* ``exit``   — the process exits at once with status 17 (a rank that dies);
* ``skip_collective`` — the NVLink collective kernels of that rank are not
  launched from step s on, so the peers' bounded device waits expire and the
  host reports ``CommTimeoutError`` (no kernel faults or hangs: every device
  wait in this code base has a time budget);
* ``drop_broadcast`` — rank 0 of a multi-rank server does not re-publish the
  s-th message (counting from 0) of those it announces in a count broadcast
  (messages taken while idle go out before any count and are never dropped):
  the other ranks' bounded wait for it expires and they raise
  ``MessageLostError`` instead of hanging.

Nothing here touches a GPU: faults are made on the host, as the failure
paths must be exercised without faulting shared devices. The reference has
no fault injection (its failure handling is the gloo / NCCL timeout,
python/minisgl/engine/config.py:27).
"""

from __future__ import annotations

import os
import sys
import time
from dataclasses import dataclass
from typing import List, Optional

ENV = "MINISGL_FAULT_INJECT"


class InjectedFault(RuntimeError):
    """Raised by an injected ``raise`` fault."""


@dataclass(frozen=True)
class FaultRule:
    action: str
    rank: int
    step: int = 0
    seconds: float = 30.0


_ACTIONS = ("raise", "stall", "exit", "skip_collective", "drop_broadcast")


def parse(spec: Optional[str]) -> List[FaultRule]:
    rules: List[FaultRule] = []
    for part in (spec or "").split(";"):
        part = part.strip()
        if not part:
            continue
        fields = part.split(":")
        action = fields[0]
        if action not in _ACTIONS:
            raise ValueError(f"{ENV}: unknown fault {action!r} (have {', '.join(_ACTIONS)})")
        kv = dict(f.split("=", 1) for f in fields[1:])
        if "rank" not in kv:
            raise ValueError(f"{ENV}: rule {part!r} needs rank=<r>")
        rules.append(FaultRule(action, int(kv["rank"]), int(kv.get("step", 0)), float(kv.get("seconds", 30))))
    return rules


def rules() -> List[FaultRule]:
    return parse(os.environ.get(ENV))


def at_step(rank: int, step: int) -> None:
    """Engine hook, called before every forward with this rank's step index."""
    for r in rules():
        if r.rank != rank or r.step != step:
            continue
        if r.action == "raise":
            raise InjectedFault(f"injected fault on rank {rank} at step {step}")
        if r.action == "stall":
            time.sleep(r.seconds)
        elif r.action == "exit":
            sys.stderr.write(f"injected exit on rank {rank} at step {step}\n")
            sys.stderr.flush()
            os._exit(17)


def skip_collective(rank: int, step: int) -> bool:
    """True when this rank's NVLink collective launches are to be skipped."""
    return any(r.action == "skip_collective" and r.rank == rank and step >= r.step for r in rules())


def drops_broadcast(rank: int, index: int) -> bool:
    """Whether rank `rank` must not re-publish its `index`-th message."""
    return any(r.action == "drop_broadcast" and r.rank == rank and r.step == index for r in rules())
