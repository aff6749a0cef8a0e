"""Dataclass <-> msgpack-ready dict conversion.

A message becomes a dict tagged with ``__type__`` (the class name); nested
dataclasses and lists are converted recursively; 1-D tensors travel as raw
bytes plus a dtype string. The receiver rebuilds objects from a name -> class
map. This wire format mirrors the reference (python/minisgl/message/utils.py)
so frontends and workers of either build speak the same protocol.
"""

from __future__ import annotations

import dataclasses
from typing import Any, Dict, Mapping

import numpy as np
import torch

_TENSOR = "Tensor"


def _encode(v: Any) -> Any:
    if isinstance(v, (int, float, str, bool, bytes)) or v is None:
        return v
    if isinstance(v, dict):
        return {k: _encode(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_encode(x) for x in v]
    return serialize_type(v)


def serialize_type(obj: Any) -> Dict:
    if isinstance(obj, torch.Tensor):
        if obj.dim() != 1:
            raise ValueError("only 1-D tensors can be serialized")
        t = obj.detach().cpu().contiguous()
        return {"__type__": _TENSOR, "buffer": t.numpy().tobytes(), "dtype": str(t.dtype)}
    if dataclasses.is_dataclass(obj):
        out: Dict[str, Any] = {"__type__": type(obj).__name__}
        for f in dataclasses.fields(obj):
            if f.init:
                out[f.name] = _encode(getattr(obj, f.name))
        return out
    out = {"__type__": type(obj).__name__}
    out.update({k: _encode(v) for k, v in vars(obj).items()})
    return out


def _decode(classes: Mapping[str, type], v: Any) -> Any:
    if isinstance(v, dict):
        if "__type__" in v:
            return deserialize_type(classes, v)
        return {k: _decode(classes, x) for k, x in v.items()}
    if isinstance(v, list):
        return [_decode(classes, x) for x in v]
    return v


def deserialize_type(classes: Mapping[str, type], data: Dict) -> Any:
    kind = data["__type__"]
    if kind == _TENSOR:
        np_dtype = getattr(np, data["dtype"].removeprefix("torch."))
        return torch.from_numpy(np.frombuffer(data["buffer"], dtype=np_dtype).copy())
    cls = classes[kind]
    kwargs = {k: _decode(classes, v) for k, v in data.items() if k != "__type__"}
    return cls(**kwargs)
