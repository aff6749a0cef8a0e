"""Weight quantisation formats for the routed experts."""

from .mxfp4 import dequantize_mxfp4, quantize_mxfp4, quantize_mxfp4_reference

__all__ = ["quantize_mxfp4", "quantize_mxfp4_reference", "dequantize_mxfp4"]
