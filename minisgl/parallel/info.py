"""Which tensor-parallel rank this process is (set once per process)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional


@dataclass(frozen=True)
class DistributedInfo:
    rank: int
    size: int

    def __post_init__(self) -> None:
        if not 0 <= self.rank < self.size:
            raise ValueError(f"rank {self.rank} outside world of {self.size}")

    def is_primary(self) -> bool:
        return self.rank == 0


_TP: Optional[DistributedInfo] = None


def set_tp_info(rank: int, size: int) -> None:
    global _TP
    if _TP is not None:
        raise RuntimeError("TP info is already set for this process")
    _TP = DistributedInfo(rank, size)


def get_tp_info() -> DistributedInfo:
    if _TP is None:
        raise RuntimeError("TP info has not been set")
    return _TP


def try_get_tp_info() -> Optional[DistributedInfo]:
    return _TP


def reset_tp_info() -> None:
    """Forget the rank (tests and in-process engine restarts)."""
    global _TP
    _TP = None


# Context parallelism: the ranks of the process group split each sequence's
# KV (attention over the latent cache) while every other layer is replicated;
# layers then see a tensor-parallel size of 1.
_CP: Optional[DistributedInfo] = None


def set_cp_info(rank: int, size: int) -> None:
    global _CP
    _CP = DistributedInfo(rank, size) if size > 1 else None


def get_cp_info() -> Optional[DistributedInfo]:
    return _CP


def reset_cp_info() -> None:
    global _CP
    _CP = None


# DP attention: every rank serves its own requests with a replicated model
# except the routed experts (split over the ranks); layers then see a
# tensor-parallel size of 1 and this records the rank among the replicas.
_DP: Optional[DistributedInfo] = None


def set_dp_info(rank: int, size: int) -> None:
    global _DP
    _DP = DistributedInfo(rank, size) if size > 1 else None


def get_dp_info() -> Optional[DistributedInfo]:
    return _DP


def reset_dp_info() -> None:
    global _DP
    _DP = None
