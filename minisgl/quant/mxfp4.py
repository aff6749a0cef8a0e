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

from typing import Optional, Tuple

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


# ----------------------------------------------------------------------------
# Block-scaled tensor-core path: MXFP4 weights x MXFP8 activations
# (csrc/mx_gemm.cu, tcgen05 .kind::mxf8f6f4.block_scale).
#
# Scale block: the E8M0 scales of 128 rows x 128 K elements (4 per row) as
# 512 bytes, byte (r % 32) * 16 + (r / 32) * 4 + j for row r and 32-block j:
# the layout one tcgen05.cp .32x128b.warpx4 moves into TMEM for the MMAs.
# ----------------------------------------------------------------------------


def scale_block_offsets(rows: int = 128) -> torch.Tensor:
    """int64 [rows, 4]: byte of (row r, 32-block j) inside a scale block."""
    r = torch.arange(rows).view(rows, 1)
    j = torch.arange(4).view(1, 4)
    return (r % 32) * 16 + (r // 32) * 4 + j


def block_scales(scales: torch.Tensor) -> torch.Tensor:
    """MXFP4 weight scales [E, K / 64, N, 2] -> scale blocks
    [E, N / 128, K / 128, 512] (N and K multiples of 128)."""
    E, Kb, N, _ = scales.shape
    K = 64 * Kb
    if N % 128 != 0 or K % 128 != 0:
        raise ValueError("the block-scaled MX experts (--moe-quant mxfp4-a8) need hidden and expert "
                         "intermediate sizes that are multiples of 128")
    # [E, N, K / 32] -> [E, N / 128, 128 rows, K / 128, 4]
    per_row = scales.permute(0, 2, 1, 3).reshape(E, N // 128, 128, K // 128, 4)
    out = torch.zeros(E, N // 128, K // 128, 512, dtype=torch.uint8, device=scales.device)
    off = scale_block_offsets().to(scales.device).reshape(-1)  # [128 * 4]
    vals = per_row.permute(0, 1, 3, 2, 4).reshape(E, N // 128, K // 128, 128 * 4)
    out[..., off] = vals
    return out


class MxfpExperts(tuple):
    """MXFP4 routed-expert weights (w1 packed, w1 scales, w2 packed, w2
    scales). ``blocked`` holds (w1, w2) scale blocks when the experts run on
    the block-scaled tensor cores with MXFP8 activations
    (``--moe-quant mxfp4-a8``; every MoE backend routes them through
    ``minisgl.ops.moe_experts_quantised`` / ``moe_experts_rows``)."""

    blocked: Optional[Tuple[torch.Tensor, torch.Tensor]] = None


_E4M3_MAX = 448.0


def quantize_mx8_reference(x: torch.Tensor, tile: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """MXFP8 rows (OCP MX: E4M3 elements, one E8M0 scale per 32) as the CUDA
    quantiser writes them: x [R, K] (R a multiple of `tile`, K of 128) ->
    (q uint8 [R, K] E4M3 bits, sf uint8 [R / tile, K / 128, 512] scale
    blocks; a tile of fewer than 128 rows fills rows 0..tile-1 of its block,
    the rest is zero). Per block: e = ceil(log2(amax / 448)) with amax / 448
    computed in fp32, scale byte e + 127, elements x / 2^e rounded to nearest
    even (within E4M3's +-448 but for the rounding of amax / 448, which a
    clamp absorbs); an all-zero block gets scale byte 0 and zero elements."""
    R, K = x.shape
    if R % tile != 0 or K % 128 != 0 or tile not in (16, 32, 64, 128):
        raise ValueError("MXFP8 rows: R % tile == 0, K % 128 == 0, tile of 16, 32, 64 or 128")
    xb = x.float().reshape(R, K // 32, 32)
    amax = xb.abs().amax(dim=-1)
    sb = (amax * torch.tensor(1.0 / _E4M3_MAX, dtype=torch.float32)).view(torch.int32)
    sbyte = ((sb >> 23) & 0xFF) + ((sb & 0x7FFFFF) != 0).int()
    live = sbyte > 0
    inv = torch.where(live, ((254 - sbyte) << 23).view(torch.float32), torch.zeros_like(amax))
    y = (xb * inv[..., None]).clamp(-_E4M3_MAX, _E4M3_MAX)
    q = y.to(torch.float8_e4m3fn).view(torch.uint8).reshape(R, K)
    sf = torch.zeros(R // tile, K // 128, 512, dtype=torch.uint8, device=x.device)
    off = scale_block_offsets(tile).to(x.device).reshape(-1)  # [tile * 4]
    per = sbyte.to(torch.uint8).reshape(R // tile, tile, K // 128, 4).permute(0, 2, 1, 3)
    sf[..., off] = per.reshape(R // tile, K // 128, tile * 4)
    return q, sf


def dequantize_mx8(q: torch.Tensor, sf: torch.Tensor, tile: int) -> torch.Tensor:
    """(q [R, K] E4M3 bits, sf [R / tile, K / 128, 512]) -> fp32 [R, K]."""
    R, K = q.shape
    off = scale_block_offsets(tile).to(q.device).reshape(-1)
    sb = sf[..., off].reshape(R // tile, K // 128, tile, 4).permute(0, 2, 1, 3).reshape(R, K // 32)
    sb = sb.to(torch.int32)
    scale = torch.where(sb > 0, (sb << 23).view(torch.float32), torch.zeros_like(sb, dtype=torch.float32))
    vals = q.view(torch.float8_e4m3fn).float().reshape(R, K // 32, 32)
    return (vals * scale[..., None]).reshape(R, K)


def moe_experts_mx_reference(x: torch.Tensor, w1q: torch.Tensor, w1s: torch.Tensor, w2q: torch.Tensor,
                             w2s: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
    """PyTorch statement of the block-scaled MX expert path (the GPU oracle):
    token rows and the SiLU x up rows are quantised to MXFP8 as the kernels
    do (per row, so the tile does not matter), weights dequantised from
    MXFP4; the products accumulate in fp32, silu(gate) * up and the expert
    outputs are rounded to bf16 as the kernels store them, and the weighted
    combine sums in fp32. w1 rows are gate|up interleaved in 64-row blocks."""
    from minisgl.ops import reference as ref

    w1 = dequantize_mxfp4(w1q, w1s)
    w2 = dequantize_mxfp4(w2q, w2s)

    def mx8(rows: torch.Tensor) -> torch.Tensor:
        n = rows.shape[0]
        pad = (-n) % 16
        full = torch.cat([rows.float(), rows.new_zeros(pad, rows.shape[1]).float()]) if pad else rows.float()
        q, sf = quantize_mx8_reference(full, 16)
        return dequantize_mx8(q, sf, 16)[:n]

    T, H = x.shape
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    xq = mx8(x.to(torch.bfloat16))
    for e in torch.unique(topk_ids).tolist():
        if e < 0 or e >= w1.shape[0]:
            continue
        tok, slot = (topk_ids == e).nonzero(as_tuple=True)
        h = xq[tok] @ w1[e].t()  # the epilogue applies SiLU x up to the fp32 accumulators
        a = ref.silu_mul_interleaved(h).to(torch.bfloat16)
        y = (mx8(a) @ w2[e].t()).to(torch.bfloat16).float()
        out.index_add_(0, tok, y * topk_w[tok, slot, None].float())
    return out.to(torch.bfloat16)
