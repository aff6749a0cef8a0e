"""MXFP4 (OCP microscaling v1.0: E2M1 elements, one E8M0 scale per 32).

A weight w [E, N, K] (K a multiple of 64) is stored as

* ``packed`` uint8 [E, N, K / 2]: element 2i in the low nibble of byte i,
  E2M1 codes (sign bit 3, exponent bits 1-2, mantissa bit 0);
* ``scales`` uint8 [E, K / 64, N, 2]: the E8M0 exponent (bias 127) of each
  32-element block, grouped by 64-wide k-block so that the block of 128 rows
  a GEMM tile needs is one contiguous run of 256 bytes.

Per block: e = floor(log2 amax) - 2 (2 is E2M1's largest exponent), scale
byte e + 127, elements x / 2^e rounded to nearest even onto
{0, 0.5, 1, 1.5, 2, 3, 4, 6} with saturation at 6. Blocks whose amax is
below 2^-124 (or zero) get scale byte 0 and zero elements. The reference has
no MXFP4 path (its experts run bf16 through the Triton fused_moe kernel,
python/minisgl/kernel/triton/fused_moe.py); this module and
``csrc/mxfp4.cu`` produce the same bytes.
"""

from __future__ import annotations

from typing import Tuple

import torch

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _codes(a: torch.Tensor) -> torch.Tensor:
    """E2M1 magnitude code of |x| / 2^e (round to nearest even, saturate)."""
    return ((a > 0.25).int() + (a >= 0.75).int() + (a > 1.25).int() + (a >= 1.75).int() + (a > 2.5).int()
            + (a >= 3.5).int() + (a > 5.0).int())


def quantize_mxfp4_reference(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """PyTorch statement of the quantiser (any device, bit-exact with the
    CUDA kernel): w [E, N, K] -> (packed, scales)."""
    E, N, K = w.shape
    if K % 64 != 0:
        raise ValueError("MXFP4 needs K % 64 == 0")
    x = w.float().reshape(E, N, K // 32, 32)
    amax = x.abs().amax(dim=-1)
    ebits = (amax.view(torch.int32) >> 23) & 0xFF
    live = ebits >= 3
    sbyte = torch.where(live, ebits - 2, torch.zeros_like(ebits))
    inv = torch.where(live, ((254 - sbyte) << 23).view(torch.float32), torch.zeros_like(amax))
    y = x * inv[..., None]
    mag = _codes(y.abs())
    code = mag | ((y < 0) & (mag != 0)).int() * 8
    code = code.reshape(E, N, K // 2, 2)
    packed = (code[..., 0] | (code[..., 1] << 4)).to(torch.uint8)
    scales = sbyte.reshape(E, N, K // 64, 2).permute(0, 2, 1, 3).contiguous().to(torch.uint8)
    return packed, scales


def dequantize_mxfp4(packed: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """(packed [E, N, K / 2], scales [E, K / 64, N, 2]) -> w [E, N, K]."""
    E, N, Kh = packed.shape
    K = 2 * Kh
    p = packed.to(torch.int32)
    code = torch.stack([p & 15, p >> 4], dim=-1).reshape(E, N, K)
    lut = _E2M1.to(packed.device)
    mag = lut[(code & 7).long()]
    val = torch.where((code & 8) != 0, -mag, mag)
    sb = scales.to(torch.int32).permute(0, 2, 1, 3).reshape(E, N, K // 32)
    scale = torch.where(sb > 0, (sb << 23).view(torch.float32), torch.zeros_like(sb, dtype=torch.float32))
    return (val.reshape(E, N, K // 32, 32) * scale[..., None]).reshape(E, N, K).to(dtype)


def quantize_mxfp4(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """w [E, N, K] -> (packed, scales); the sm_100a kernel on CUDA tensors."""
    if not w.is_cuda:
        return quantize_mxfp4_reference(w)
    from minisgl import ops

    E, N, K = w.shape
    packed = torch.empty(E, N, K // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(E, K // 64, N, 2, dtype=torch.uint8, device=w.device)
    ops._count()
    ops.native().mxfp4_quantize(packed, scales, w.to(torch.bfloat16).contiguous())
    return packed, scales
