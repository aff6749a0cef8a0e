"""Paged latent cache for multi-head latent attention (DeepSeek-V3 / Kimi-K2).

MLA stores one vector per token and layer, shared by every head: the
normalised compressed KV (kv_lora_rank) followed by the rotated positional
key (qk_rope_head_dim), 576 bf16 values for DeepSeek-V3. Layout
[layers, pages, page_size, kv_lora_rank + rope_dim], so a page of one layer
is one contiguous block of page_size x 1152 bytes. The same rows serve as
keys (all 576 values) and values (the first kv_lora_rank), so K and V are the
same tensor. The reference has no MLA (its pools are MHA only,
python/minisgl/kvcache/mha_pool.py); under tensor parallelism every rank
keeps the whole latent (it is not split by heads). Under context
parallelism the pool holds one page in cp: global page g (whose 64 keys
belong to this rank when g % cp == rank, which the page allocator
guarantees) sits at local page g // cp.
"""

from __future__ import annotations

import torch

from .base import BaseKVCachePool


class MLAKVCache(BaseKVCachePool):
    def __init__(self, num_layers: int, kv_lora_rank: int, rope_dim: int, num_pages: int, page_size: int,
                 dtype: torch.dtype, device: torch.device, cp_size: int = 1) -> None:
        self.kv_lora_rank = kv_lora_rank
        self.rope_dim = rope_dim
        self.latent_dim = kv_lora_rank + rope_dim
        self.page_size = page_size
        self.num_pages = num_pages
        self.cp_size = cp_size
        self._num_layers = num_layers
        self._device = torch.device(device)
        # context parallelism: global page g is stored by rank g % cp at local
        # page g // cp (one spare local page for the dummy request's page)
        local = num_pages if cp_size <= 1 else num_pages // cp_size + 2
        self.pool = torch.zeros((num_layers, local, page_size, self.latent_dim), dtype=dtype, device=device)

    def latent(self, layer: int) -> torch.Tensor:
        """[pages, page_size, kv_lora_rank + rope_dim] of one layer."""
        return self.pool[layer]

    def k_cache(self, layer: int) -> torch.Tensor:
        return self.pool[layer]

    def v_cache(self, layer: int) -> torch.Tensor:
        return self.pool[layer][..., : self.kv_lora_rank]

    def store_latent(self, latent: torch.Tensor, out_loc: torch.Tensor, layer: int) -> None:
        loc = out_loc.long()
        self.pool[layer][loc // self.page_size // self.cp_size, loc % self.page_size] = latent.to(self.pool.dtype)

    def store_kv(self, k: torch.Tensor, v: torch.Tensor, out_loc: torch.Tensor, layer: int) -> None:
        """k: the full latent rows (v is the leading part of the same rows)."""
        self.store_latent(k, out_loc, layer)

    @property
    def device(self) -> torch.device:
        return self._device

    @property
    def dtype(self) -> torch.dtype:
        return self.pool.dtype

    @property
    def num_layers(self) -> int:
        return self._num_layers
