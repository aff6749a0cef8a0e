"""Weight quantisation formats for the routed experts."""

from .mxfp4 import (MxfpExperts, block_scales, dequantize_mx8, dequantize_mxfp4, moe_experts_mx_reference,
                    quantize_mx8_reference, quantize_mxfp4, quantize_mxfp4_reference, scale_block_offsets)

__all__ = ["MxfpExperts", "quantize_mxfp4", "quantize_mxfp4_reference", "dequantize_mxfp4", "block_scales", "scale_block_offsets",
           "quantize_mx8_reference", "dequantize_mx8", "moe_experts_mx_reference"]
