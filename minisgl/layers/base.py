"""Minimal module protocol for inference layers.

Parameters are plain tensor attributes; sub-layers are plain attributes too.
Attributes whose name starts with ``_`` are private (not weights). The
state-dict names this produces (``model.layers.0.self_attn.qkv_proj.weight``)
are what the weight loader emits, mirroring the reference's BaseOP protocol
(python/minisgl/layers/base.py:15-99) so HF checkpoints map the same way.
"""

from __future__ import annotations

from typing import Any, Dict, Generic, Iterator, List, Optional, Tuple, TypeVar

import torch

StateDict = Dict[str, torch.Tensor]


def _join(prefix: str, name: str) -> str:
    return f"{prefix}.{name}" if prefix else name


class BaseOP:
    def forward(self, *args: Any, **kwargs: Any) -> Any:
        raise NotImplementedError

    def named_tensors(self, prefix: str = "") -> Iterator[Tuple[str, "BaseOP", str, torch.Tensor]]:
        """(full name, owner, attribute, tensor) for every public tensor."""
        for name, value in list(vars(self).items()):
            if name.startswith("_"):
                continue
            if isinstance(value, torch.Tensor):
                yield _join(prefix, name), self, name, value
            elif isinstance(value, BaseOP):
                yield from value.named_tensors(_join(prefix, name))

    def state_dict(self, *, prefix: str = "", result: Optional[StateDict] = None) -> StateDict:
        out = {} if result is None else result
        for full, _, _, t in self.named_tensors(prefix):
            out[full] = t
        return out

    def load_state_dict(self, state_dict: StateDict, *, prefix: str = "", _internal: bool = False) -> None:
        for name, value in list(vars(self).items()):
            if name.startswith("_"):
                continue
            key = _join(prefix, name)
            if isinstance(value, torch.Tensor):
                if key not in state_dict:
                    raise KeyError(f"missing weight {key}")
                item = state_dict.pop(key)
                if tuple(item.shape) != tuple(value.shape) or item.dtype != value.dtype:
                    raise ValueError(f"{key}: expected {tuple(value.shape)} {value.dtype}, got "
                                     f"{tuple(item.shape)} {item.dtype}")
                setattr(self, name, item)
            elif isinstance(value, BaseOP):
                value.load_state_dict(state_dict, prefix=key, _internal=True)
        if not _internal and state_dict:
            raise RuntimeError(f"unexpected weights: {sorted(state_dict)[:8]}")
        if not _internal:
            self.post_load()

    def post_load(self) -> None:
        """Hook run once after all weights are in place (recursively)."""
        for name, value in list(vars(self).items()):
            if not name.startswith("_") and isinstance(value, BaseOP):
                value.post_load()


class StateLessOP(BaseOP):
    def state_dict(self, *, prefix: str = "", result: Optional[StateDict] = None) -> StateDict:
        return {} if result is None else result

    def named_tensors(self, prefix: str = ""):
        return iter(())

    def load_state_dict(self, state_dict: StateDict, *, prefix: str = "", _internal: bool = False) -> None:
        if not _internal and state_dict:
            raise RuntimeError(f"unexpected weights: {sorted(state_dict)[:8]}")


T = TypeVar("T", bound=BaseOP)


class OPList(BaseOP, Generic[T]):
    def __init__(self, ops: List[T]) -> None:
        self.op_list = ops

    def named_tensors(self, prefix: str = ""):
        for i, op in enumerate(self.op_list):
            yield from op.named_tensors(_join(prefix, str(i)))

    def load_state_dict(self, state_dict: StateDict, *, prefix: str = "", _internal: bool = False) -> None:
        for i, op in enumerate(self.op_list):
            op.load_state_dict(state_dict, prefix=_join(prefix, str(i)), _internal=True)
        if not _internal and state_dict:
            raise RuntimeError(f"unexpected weights: {sorted(state_dict)[:8]}")

    def post_load(self) -> None:
        for op in self.op_list:
            op.post_load()

    def __iter__(self):
        return iter(self.op_list)

    def __len__(self) -> int:
        return len(self.op_list)

    def __getitem__(self, i: int) -> T:
        return self.op_list[i]
