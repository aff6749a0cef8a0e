from .arch import is_arch_supported, is_sm90_supported, is_sm100_supported
from .hf import cached_load_hf_config, download_hf_weight, load_tokenizer
from .logger import init_logger
from .misc import UNSET, Unset, align_ceil, align_down, call_if_main, div_ceil, div_even
from .mp import (
    ZmqAsyncPullQueue,
    ZmqAsyncPushQueue,
    ZmqPubQueue,
    ZmqPullQueue,
    ZmqPushQueue,
    ZmqSubQueue,
)
from .registry import Registry
from .torch_utils import nvtx_annotate, torch_dtype

__all__ = [
    "cached_load_hf_config", "download_hf_weight", "load_tokenizer", "init_logger",
    "is_arch_supported", "is_sm90_supported", "is_sm100_supported", "call_if_main",
    "div_even", "div_ceil", "align_ceil", "align_down", "UNSET", "Unset", "torch_dtype",
    "nvtx_annotate", "Registry", "ZmqPushQueue", "ZmqPullQueue", "ZmqPubQueue", "ZmqSubQueue",
    "ZmqAsyncPushQueue", "ZmqAsyncPullQueue",
]
