"""torch helpers: default-dtype scope and NVTX ranges."""

from __future__ import annotations

import functools
from contextlib import contextmanager

import torch


@contextmanager
def torch_dtype(dtype: torch.dtype):
    old = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        yield
    finally:
        torch.set_default_dtype(old)


_NVTX = torch.cuda.is_available()


def nvtx_annotate(name: str, layer_id_field: str | None = None):
    """Wrap a method in an NVTX range; ``{}`` in ``name`` is filled with the
    value of ``layer_id_field`` on the instance (e.g. ``Layer_{}``)."""

    def deco(fn):
        if not _NVTX:
            return fn

        @functools.wraps(fn)
        def wrapper(self, *args, **kwargs):
            label = name.format(getattr(self, layer_id_field)) if layer_id_field else name
            torch.cuda.nvtx.range_push(label)
            try:
                return fn(self, *args, **kwargs)
            finally:
                torch.cuda.nvtx.range_pop()

        return wrapper

    return deco
