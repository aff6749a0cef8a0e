"""Host-side statements of the block-scaled MX expert path (MXFP4 weights x
MXFP8 activations on tcgen05 .kind::mxf8f6f4): the 512-byte scale-block
layout that tcgen05.cp moves into TMEM, the weight-scale re-layout, the
MXFP8 activation quantiser (scale rule, rounding, zero blocks, short tiles)
and the expert-path oracle, checked against plain fp32 PyTorch."""

import pytest
import torch

from minisgl.quant import (block_scales, dequantize_mx8, dequantize_mxfp4, moe_experts_mx_reference,
                           quantize_mx8_reference, quantize_mxfp4_reference, scale_block_offsets)


def test_scale_block_offsets_cover_the_block_once():
    off = scale_block_offsets()
    assert sorted(off.flatten().tolist()) == list(range(512))
    assert ((off[:, 1:] - off[:, :-1]) == 1).all()  # a row's four scales are one 32-bit TMEM word
    # rows r, r + 32, r + 64, r + 96 share the 16 bytes that TMEM lane r % 32 receives
    assert off[5, 0] == 80 and off[37, 0] == 84 and off[101, 3] == 5 * 16 + 3 * 4 + 3


def test_block_scales_place_every_weight_scale():
    g = torch.Generator().manual_seed(1)
    E, N, K = 2, 256, 384
    w = torch.randn(E, N, K, generator=g) * torch.logspace(-3, 3, K // 32).repeat_interleave(32)
    _, scales = quantize_mxfp4_reference(w)
    blk = block_scales(scales)
    assert blk.shape == (E, N // 128, K // 128, 512)
    off = scale_block_offsets()
    per_row = scales.permute(0, 2, 1, 3).reshape(E, N, K // 32)  # scale of (e, n, 32-block)
    for e in range(E):
        for n in (0, 31, 32, 127, 128, 200, 255):
            for j32 in range(K // 32):
                got = blk[e, n // 128, j32 // 4, off[n % 128, j32 % 4]]
                assert got == per_row[e, n, j32]
    with pytest.raises(ValueError):
        block_scales(torch.zeros(1, 1, 64, 2, dtype=torch.uint8))  # K = 64: not a multiple of 128


def _blocks(x):
    return x.float().reshape(x.shape[0], -1, 32)


def test_mx8_quantiser_rule_and_error():
    g = torch.Generator().manual_seed(2)
    R, K = 64, 256
    # magnitudes from 2^-20 to 2^20 per 32-block, one zero block, one exact power of two
    x = torch.randn(R, K, generator=g) * torch.logspace(-6, 6, R * K // 32).reshape(R, K // 32).repeat_interleave(
        32, dim=1)
    x[3, 32:64] = 0.0
    x[5, :32] = 0.0
    x[5, 7] = 448.0 * 4  # amax / 448 exactly 2^2: no rounding up
    q, sf = quantize_mx8_reference(x, 32)
    assert q.dtype == torch.uint8 and q.shape == (R, K) and sf.shape == (R // 32, K // 128, 512)
    deq = dequantize_mx8(q, sf, 32)
    off = scale_block_offsets(32)
    sb = sf[..., off.reshape(-1)].reshape(R // 32, K // 128, 32, 4).permute(0, 2, 1, 3).reshape(R, K // 32)
    amax = _blocks(x).abs().amax(-1)
    live = amax > 0
    scale = torch.pow(2.0, sb.double() - 127)
    # e = ceil(log2(amax / 448)): amax / 2^e in (224, 448]
    ratio = amax.double()[live] / scale[live]
    assert (ratio <= 448).all() and (ratio > 224 * (1 - 1e-6)).all()
    assert sb[5, 0] == 127 + 2
    # zero block: scale byte 0, zero elements
    assert sb[3, 1] == 0 and (deq[3, 32:64] == 0).all()
    # round to nearest E4M3 (3 mantissa bits): half a step of the value, or
    # half the subnormal step 2^-9 of the scale
    err = (deq.double() - x.double()).abs().reshape(R, K // 32, 32)
    bound = x.double().abs().reshape(R, K // 32, 32) * 2.0 ** -4 + scale[..., None] * 2.0 ** -10
    assert (err <= bound * (1 + 1e-9)).all()


def test_mx8_short_tiles_fill_their_block_rows_and_zero_the_rest():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(32, 128, generator=g)
    q16, sf16 = quantize_mx8_reference(x, 16)
    q128, sf128 = quantize_mx8_reference(torch.cat([x, torch.zeros(96, 128)]), 128)
    assert torch.equal(q16, q128[:32])
    off = scale_block_offsets()
    for t in range(2):
        rows = sf16[t, 0, off[:16].reshape(-1)]
        assert torch.equal(rows, sf128[0, 0, off[16 * t:16 * t + 16].reshape(-1)])
        assert (sf16[t, 0, off[16:].reshape(-1)] == 0).all()


def test_mx_expert_oracle_tracks_the_fp32_experts():
    """The MXFP8 rounding of the token and SiLU rows moves the expert output
    by a few per cent of its scale, no more; routing and the gate|up
    interleave are those of the fp32 path."""
    from minisgl.moe.fused import moe_reference

    g = torch.Generator().manual_seed(4)
    T, H, I, E, k = 24, 256, 128, 4, 2
    x = torch.randn(T, H, generator=g)
    w1 = torch.randn(E, 2 * I, H, generator=g) * 0.05
    w2 = torch.randn(E, H, I, generator=g) * 0.05
    w1q, w1s = quantize_mxfp4_reference(w1)
    w2q, w2s = quantize_mxfp4_reference(w2)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int()
    tw = torch.rand(T, k, generator=g)
    got = moe_experts_mx_reference(x, w1q, w1s, w2q, w2s, tw, ids).float()
    want = moe_reference(x, dequantize_mxfp4(w1q, w1s), dequantize_mxfp4(w2q, w2s), tw, ids, "silu",
                         interleaved=True)
    rel = (got - want).norm() / want.norm()
    assert rel < 0.05, rel


def test_mx_experts_engine_on_cpu():
    """--moe-quant mxfp4-a8 through the engine on the CPU (the path's PyTorch
    statement): greedy tokens stay close to those of the bf16-activation
    MXFP4 experts from the same checkpoint."""
    import shutil
    import tempfile

    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_mx_ckpt_")
    shutil.rmtree(folder)
    make_model_dir("tiny-qwen3-moe", folder=folder)
    write_random_checkpoint(folder, seed=5, std=0.05)
    prompts = [[5, 6, 7, 8, 9, 10, 11, 12, 13], [100, 200, 300, 400, 500, 600, 700, 800, 900, 1000, 11, 12]]
    try:
        outs = {}
        for quant in ("mxfp4", "mxfp4-a8"):
            llm = LLM(folder, dtype=torch.float32, device="cpu", page_size=16, num_page_override=64,
                      max_running_req=4, max_seq_len_override=256, max_extend_tokens=64, moe_quant=quant)
            experts = [dl.mlp.experts._mxfp4 for dl in llm.engine.model.model.layers.op_list]
            assert experts and all(w is not None and (w.blocked is not None) == (quant == "mxfp4-a8")
                                   for w in experts)
            res = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
            outs[quant] = [o["token_ids"] for o in res]
            llm.shutdown()
        a, b = outs["mxfp4"], outs["mxfp4-a8"]
        assert all(len(x) == 8 for x in b)
        firsts = sum(x[0] == y[0] for x, y in zip(a, b))
        assert firsts == len(a), (a, b)
    finally:
        shutil.rmtree(folder, ignore_errors=True)


def test_mx8_tiny_blocks_stay_finite():
    """Block maxima down in fp32's subnormal range: amax / 448 has a zero
    exponent field, the scale byte is 1 (2^-126), and the elements stay
    finite and within half an E4M3 step (or half its subnormal step)."""
    x = torch.zeros(16, 128)
    x[0, :32] = torch.linspace(-1e-39, 1e-39, 32)   # subnormal fp32 values
    x[1, 32:64] = 3e-37
    q, sf = quantize_mx8_reference(x, 16)
    deq = dequantize_mx8(q, sf, 16)
    assert torch.isfinite(deq).all()
    off = scale_block_offsets(16)
    assert sf[0, 0, off[0, 0]] == 1 and sf[0, 0, off[1, 1]] >= 1
    scale = 2.0 ** -126
    err = (deq[0, :32].double() - x[0, :32].double()).abs()
    assert (err <= x[0, :32].double().abs() * 2.0 ** -4 + scale * 2.0 ** -10 + 1e-45).all()
    assert deq[1, 32:64].sub(3e-37).abs().max() <= 3e-37 * 2.0 ** -4
