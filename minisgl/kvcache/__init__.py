"""KV pools and prefix caches."""

from __future__ import annotations

from typing import TYPE_CHECKING

import torch

from minisgl.utils import Registry

from .base import BaseCacheHandle, BaseKVCachePool, BasePrefixCache, InsertResult, MatchResult, SizeInfo

if TYPE_CHECKING:
    from minisgl.models import ModelConfig

SUPPORTED_CACHE_MANAGER = Registry("Cache Manager")


@SUPPORTED_CACHE_MANAGER.register("naive")
def _naive(device: torch.device, page_size: int = 1) -> BasePrefixCache:
    from .naive_cache import NaivePrefixCache

    return NaivePrefixCache(device, page_size)


@SUPPORTED_CACHE_MANAGER.register("radix")
def _radix(device: torch.device, page_size: int = 1) -> BasePrefixCache:
    from .radix_cache import RadixPrefixCache

    return RadixPrefixCache(device, page_size)


def create_prefix_cache(device: torch.device, type: str, page_size: int = 1) -> BasePrefixCache:
    return SUPPORTED_CACHE_MANAGER[type](device, page_size)


def create_kvcache_pool(model_config: "ModelConfig", num_pages: int, page_size: int, dtype: torch.dtype,
                        device: torch.device, cp_size: int = 1) -> BaseKVCachePool:
    if model_config.is_mla:
        from .mla_pool import MLAKVCache

        return MLAKVCache(model_config.num_layers, model_config.kv_lora_rank, model_config.qk_rope_head_dim,
                          num_pages, page_size, dtype, device, cp_size=cp_size)
    from .mha_pool import MHAKVCache

    return MHAKVCache(model_config.num_kv_heads, model_config.num_layers, model_config.head_dim, num_pages,
                      page_size, dtype, device)


__all__ = [
    "create_kvcache_pool", "create_prefix_cache", "BaseKVCachePool", "BaseCacheHandle", "BasePrefixCache",
    "SizeInfo", "MatchResult", "InsertResult", "SUPPORTED_CACHE_MANAGER",
]
