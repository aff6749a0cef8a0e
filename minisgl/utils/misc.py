"""Small integer helpers and the script-or-test decorator."""

from __future__ import annotations

from typing import Callable


def div_even(a: int, b: int, allow_replicate: bool = False) -> int:
    """a / b for exact divisions. With ``allow_replicate`` a divisor larger
    than ``a`` (e.g. more TP ranks than KV heads) yields 1, provided b is a
    multiple of a, so each head is replicated on b / a ranks."""
    if allow_replicate and b > a:
        if b % a != 0:
            raise ValueError(f"{b} ranks cannot replicate {a} heads evenly")
        return 1
    if a % b != 0:
        raise ValueError(f"{a} is not divisible by {b}")
    return a // b


def div_ceil(a: int, b: int) -> int:
    return -(-a // b)


def align_ceil(a: int, b: int) -> int:
    return div_ceil(a, b) * b


def align_down(a: int, b: int) -> int:
    return a - a % b


def call_if_main(name: str) -> Callable[[Callable], Callable]:
    """Run the decorated function immediately when the defining module is the
    script being executed; otherwise return it unchanged (so pytest collects
    it as a test)."""

    def deco(fn: Callable) -> Callable:
        if name == "__main__":
            fn()
        return fn

    return deco


class Unset:
    """Sentinel type for 'argument not given'."""

    def __repr__(self) -> str:
        return "UNSET"


UNSET = Unset()
