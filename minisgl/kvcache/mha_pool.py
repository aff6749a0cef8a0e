"""Paged K/V storage for multi-head (GQA) attention.

One tensor of shape [2, layers, pages, local_kv_heads, page_size, head_dim].
Unlike the reference's token-major NHD pool (python/minisgl/kvcache/
mha_pool.py:25-35), a (page, head) block of page_size x head_dim is
contiguous here, so one TMA box moves a whole block of keys for one head.
The attention kernels address the pool through a single 2-D tensor map.
The pool is zero-initialised so positions past the end of a sequence never
hold non-finite values.
"""

from __future__ import annotations

import torch

from minisgl.parallel import get_tp_info
from minisgl.utils import div_even

from .base import BaseKVCachePool


class MHAKVCache(BaseKVCachePool):
    def __init__(self, num_kv_heads: int, num_layers: int, head_dim: int, num_pages: int, page_size: int,
                 dtype: torch.dtype, device: torch.device) -> None:
        local = div_even(num_kv_heads, get_tp_info().size, allow_replicate=True)
        self.local_kv_heads = local
        self.head_dim = head_dim
        self.page_size = page_size
        self.num_pages = num_pages
        self._num_layers = num_layers
        self._device = torch.device(device)
        self.pool = torch.zeros((2, num_layers, num_pages, local, page_size, head_dim), dtype=dtype, device=device)

    def k_cache(self, layer: int) -> torch.Tensor:
        return self.pool[0, layer]

    def v_cache(self, layer: int) -> torch.Tensor:
        return self.pool[1, layer]

    def store_kv(self, k: torch.Tensor, v: torch.Tensor, out_loc: torch.Tensor, layer: int) -> None:
        loc = out_loc.long()
        page, off = loc // self.page_size, loc % self.page_size
        shape = (-1, self.local_kv_heads, self.head_dim)
        self.pool[0, layer][page, :, off] = k.reshape(shape)
        self.pool[1, layer][page, :, off] = v.reshape(shape)

    @property
    def device(self) -> torch.device:
        return self._device

    @property
    def dtype(self) -> torch.dtype:
        return self.pool.dtype

    @property
    def num_layers(self) -> int:
        return self._num_layers

    @staticmethod
    def bytes_per_page(num_kv_heads: int, num_layers: int, head_dim: int, page_size: int, dtype: torch.dtype) -> int:
        local = div_even(num_kv_heads, get_tp_info().size, allow_replicate=True)
        return 2 * num_layers * local * page_size * head_dim * dtype.itemsize
