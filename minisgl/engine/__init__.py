from .config import EngineConfig
from .engine import Engine, ForwardOutput
from .sample import BatchSamplingArgs, Sampler

__all__ = ["Engine", "EngineConfig", "ForwardOutput", "BatchSamplingArgs", "Sampler"]
