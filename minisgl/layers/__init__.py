from .activation import gelu_and_mul, silu_and_mul
from .attention import AttentionLayer
from .base import BaseOP, OPList, StateLessOP
from .embedding import ParallelLMHead, VocabParallelEmbedding
from .linear import LinearColParallelMerged, LinearOProj, LinearQKVMerged, LinearReplicated, LinearRowParallel
from .moe import MoELayer
from .norm import RMSNorm, RMSNormFused
from .rotary import get_rope, set_rope_device

__all__ = [
    "silu_and_mul", "gelu_and_mul", "AttentionLayer", "BaseOP", "StateLessOP", "OPList",
    "VocabParallelEmbedding", "ParallelLMHead", "LinearColParallelMerged", "LinearRowParallel",
    "LinearOProj", "LinearQKVMerged", "RMSNorm", "RMSNormFused", "get_rope", "set_rope_device",
    "LinearReplicated", "MoELayer",
]
