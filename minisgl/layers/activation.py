"""Gated activations: act(x[:, :d]) * x[:, d:] (sm_100a kernel on CUDA)."""

from minisgl.ops import gelu_and_mul, silu_and_mul

__all__ = ["silu_and_mul", "gelu_and_mul"]
