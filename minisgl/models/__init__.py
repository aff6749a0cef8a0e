from .base import BaseLLMModel
from .config import ModelConfig, RotaryConfig
from .register import get_model_class, supported_architectures
from .weight import LazyRandomWeights, load_weight, random_weights


def create_model(model_config: ModelConfig) -> BaseLLMModel:
    return get_model_class(model_config.architectures[0], model_config)


__all__ = ["create_model", "load_weight", "random_weights", "LazyRandomWeights", "ModelConfig", "RotaryConfig", "BaseLLMModel",
           "supported_architectures"]
