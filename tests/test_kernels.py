"""Numerics of the sm_100a kernels against the fp32 PyTorch reference.

Shape sweeps follow the reference's kernel tests (tests/kernel/test_index.py,
tests/kernel/test_store.py): many batch sizes, exact checks where the op is a
pure copy, tolerance checks where bf16 rounding is involved.
"""

import math

import pytest
import torch

from minisgl import ops
from minisgl.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(out, expect, atol, rtol):
    out, expect = out.float().cpu(), expect.float().cpu()
    err = (out - expect).abs()
    bound = atol + rtol * expect.abs()
    bad = (err > bound).sum().item()
    assert bad == 0, f"{bad} elements out of tolerance; max err {err.max().item():.4g}"


@pytest.mark.parametrize(
    "M,N,K",
    [
        (1, 1024, 1024),
        (7, 4096, 1024),
        (16, 1024, 3072),
        (33, 6144, 1024),
        (64, 1024, 2048),
        (100, 768, 512),
        (128, 2048, 1024),
        (200, 1024, 3072),
        (256, 4096, 1024),
        (1000, 1536, 1024),
        (4096, 4096, 1024),
        (3000, 1024, 72),
        (256, 151936 // 16, 1024),
        (129, 1024, 3072),
        (250, 6144, 1024),
    ],
)
@pytest.mark.parametrize("bias", [False, True])
def test_gemm(M, N, K, bias):
    torch.manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(N, K, device=DEV) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, device=DEV) * 0.1).to(torch.bfloat16) if bias else None
    out = ops.gemm(x, w, b)
    torch.cuda.synchronize()
    expect = ref.gemm(x, w, b, torch.float32)
    _close(out, expect, atol=2e-2 * math.sqrt(K / 1024), rtol=1e-2)


@pytest.mark.parametrize("mode,splits", [(1, 1), (1, 2), (1, 4), (2, 1), (2, 4), (2, 8)])
def test_gemm_forced_paths(mode, splits):
    torch.manual_seed(0)
    M, N, K = 96, 2048, 2048
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(N, K, device=DEV) * 0.05).to(torch.bfloat16)
    out = torch.empty(M, N, device=DEV, dtype=torch.float32)
    ops.native().gemm(out, x, w, None, ops.gemm_workspace(x.device), splits, mode, ops.error_word(x.device))
    torch.cuda.synchronize()
    _close(out, ref.gemm(x, w, None, torch.float32), atol=3e-2, rtol=1e-2)
    ops.check_device_errors(x.device)


@pytest.mark.parametrize("M,N,K", [(1, 1024, 1024), (4, 256, 256), (64, 1024, 2048), (200, 512, 3072)])
def test_gemm_every_plan(M, N, K):
    """Every (tile orientation, N tile, cluster split) plan is numerically right."""
    torch.manual_seed(M + N)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(N, K, device=DEV) * 0.05).to(torch.bfloat16)
    expect = ref.gemm(x, w, None, torch.float32).cpu()
    from minisgl.ops.gemm_tune import candidates, run_plan

    for mode, bn, s in candidates(M, K):
        out = torch.zeros(M, N, device=DEV, dtype=torch.float32)
        run_plan(out, x, w, (mode, bn, s))
        torch.cuda.synchronize()
        err = (out.cpu() - expect).abs().max().item()
        assert err < 3e-2 * (K / 1024) ** 0.5 + 1e-2, (mode, bn, s, err)


@pytest.mark.parametrize("M,N,K", [(1, 1280, 5120), (5, 1000, 1024), (16, 5120, 3200), (33, 640, 64),
                                   (100, 6400, 5120), (256, 5120, 3200), (256, 1536, 25600)])
@pytest.mark.parametrize("R", [1, 2])
def test_gemm_streamk(M, N, K, R):
    """Stream-K weight streaming (plan mode 4): split tiles are summed from
    the per-CTA partials in a fixed order, so two launches give identical
    bits, and the ready flags are reset for the next launch."""
    torch.manual_seed(M * 7 + N + R)
    big = torch.randn(M, K + 64, device=DEV, dtype=torch.bfloat16)
    x = big[:, 64:]  # row stride K + 64
    w = (torch.randn(N, K, device=DEV) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, device=DEV) * 0.1).to(torch.bfloat16)
    ws = ops.streamk_workspace(x.device)
    err = ops.error_word(x.device)
    outs = []
    for f32 in (False, True, True):
        out = torch.full((M, N), float("nan"), device=DEV, dtype=torch.float32 if f32 else torch.bfloat16)
        ops.native().gemm(out, x, w, b, ws, 0, ops.GEMM_STREAMK, err, R, None, 0)
        outs.append(out)
    torch.cuda.synchronize()
    ops.check_device_errors(x.device)
    expect = ref.gemm(x, w, b, torch.float32)
    tol = 2e-2 * math.sqrt(K / 1024) + 1e-2
    _close(outs[0], expect, atol=tol, rtol=1e-2)
    _close(outs[1], expect, atol=tol, rtol=1e-2)
    assert torch.equal(outs[1], outs[2])
    sms = torch.cuda.get_device_properties(x.device).multi_processor_count
    flags = ws[-32 * sms:].view(torch.int32)
    assert int(flags.abs().sum()) == 0


@pytest.mark.parametrize("M,N,K,bn", [(4096, 6144, 1024, 256), (3000, 1000, 576, 256), (129, 4096, 2048, 128),
                                        (1, 512, 64, 256), (8192, 1024, 3072, 128)])
@pytest.mark.parametrize("bias,f32", [(False, False), (True, True)])
def test_gemm_persistent(M, N, K, bn, bias, f32):
    """Persistent tiles (plan mode 3) with ragged edges in M and N."""
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(N, K, device=DEV) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, device=DEV) * 0.1).to(torch.bfloat16) if bias else None
    out = torch.empty(M, N, device=DEV, dtype=torch.float32 if f32 else torch.bfloat16)
    ops.native().gemm(out, x, w, b, None, 1, 3, ops.error_word(x.device), bn)
    torch.cuda.synchronize()
    ops.check_device_errors(x.device)
    _close(out, ref.gemm(x, w, b, torch.float32), atol=2e-2 * math.sqrt(K / 1024) + 1e-2, rtol=1e-2)


@pytest.mark.parametrize("M,N,K", [(4096, 6144, 1024), (3000, 1000, 576), (300, 4096, 2048), (1, 512, 64),
                                   (8192, 1024, 3072)])
@pytest.mark.parametrize("bias,f32", [(False, False), (True, True)])
def test_gemm_cta_pairs(M, N, K, bias, f32):
    """Persistent 256 x 256 tiles on CTA pairs (plan mode 5, cta_group::2
    MMAs) with ragged edges in M and N, including a pair whose odd CTA's rows
    all lie past M."""
    torch.manual_seed(M + N + K + 1)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(N, K, device=DEV) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, device=DEV) * 0.1).to(torch.bfloat16) if bias else None
    out = torch.empty(M, N, device=DEV, dtype=torch.float32 if f32 else torch.bfloat16)
    ops.native().gemm(out, x, w, b, None, 1, ops.GEMM_PAIR, ops.error_word(x.device), 256)
    torch.cuda.synchronize()
    ops.check_device_errors(x.device)
    _close(out, ref.gemm(x, w, b, torch.float32), atol=2e-2 * math.sqrt(K / 1024) + 1e-2, rtol=1e-2)


def test_gemm_strided_input_fp32_out():
    torch.manual_seed(1)
    big = torch.randn(50, 3072, device=DEV, dtype=torch.bfloat16)
    x = big[:, 1024:2048]  # row stride 3072
    w = (torch.randn(512, 1024, device=DEV) * 0.05).to(torch.bfloat16)
    out = ops.gemm(x, w, out_dtype=torch.float32)
    _close(out, ref.gemm(x, w, None, torch.float32), atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("rows,cols", [(1, 1024), (37, 5120), (256, 128), (1000, 2048)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rmsnorm(rows, cols, dtype):
    torch.manual_seed(rows + cols)
    x = torch.randn(rows, cols, device=DEV, dtype=dtype)
    w = torch.rand(cols, device=DEV, dtype=dtype) + 0.5
    _close(ops.rmsnorm(x, w, 1e-6), ref.rmsnorm(x.cpu(), w.cpu(), 1e-6), atol=1e-2, rtol=1e-2)
    r = torch.randn_like(x)
    x2, r2 = x.clone(), r.clone()
    ops.fused_add_rmsnorm(x2, r2, w, 1e-6)
    x3, r3 = x.cpu().clone(), r.cpu().clone()
    ref.fused_add_rmsnorm(x3, r3, w.cpu(), 1e-6)
    assert torch.equal(r2.cpu(), r3)
    _close(x2, x3, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("rows,d", [(1, 3072), (77, 512), (512, 25600 // 8)])
def test_act_and_mul(rows, d):
    x = torch.randn(rows, 2 * d, device=DEV, dtype=torch.bfloat16)
    _close(ops.silu_and_mul(x), ref.act_and_mul(x.cpu(), "silu"), atol=1e-2, rtol=1e-2)
    _close(ops.gelu_and_mul(x), ref.act_and_mul(x.cpu(), "gelu"), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("bs", [1, 7, 512, 4096])
def test_embedding(bs):
    V, H = 1000, 1024
    w = torch.randn(V, H, device=DEV, dtype=torch.bfloat16)
    ids = torch.randint(0, V, (bs,), device=DEV, dtype=torch.int32)
    assert torch.equal(ops.embedding(ids, w), w[ids.long()])
    # vocab-sharded: rows outside [lo, lo + n) are zero
    lo, n = 250, 500
    shard = w[lo : lo + n].contiguous()
    out = ops.embedding(ids, shard, (lo, n))
    assert torch.equal(out.cpu(), ref.embedding(ids.cpu(), shard.cpu(), lo, n))


@pytest.mark.parametrize("hq,hk,d,page", [(16, 8, 128, 16), (8, 1, 128, 64), (4, 2, 64, 32)])
@pytest.mark.parametrize("qk_norm", [True, False])
def test_rope_store(hq, hk, d, page, qk_norm):
    torch.manual_seed(3)
    T, pages = 40, 16
    qkv = torch.randn(T, (hq + 2 * hk) * d, device=DEV, dtype=torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), device=DEV, dtype=torch.int32)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    fr = torch.arange(4096, dtype=torch.float32)[:, None] * inv[None]
    cos_sin = torch.cat([fr.cos(), fr.sin()], -1).to(DEV)
    qn = (torch.rand(d, device=DEV) + 0.5).to(torch.bfloat16) if qk_norm else None
    kn = (torch.rand(d, device=DEV) + 0.5).to(torch.bfloat16) if qk_norm else None
    kc = torch.zeros(pages, hk, page, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    loc = torch.randperm(pages * page, device=DEV)[:T].to(torch.int32)
    a = qkv.clone()
    ops.rope_store(a, pos, cos_sin, qn, kn, kc, vc, loc, hq, hk, d, page, 1e-6)
    b = qkv.cpu().clone()
    kc2, vc2 = torch.zeros_like(kc).cpu(), torch.zeros_like(vc).cpu()
    ref.rope_store(b, pos.cpu(), cos_sin.cpu(), None if qn is None else qn.cpu(), None if kn is None else kn.cpu(),
                   kc2, vc2, loc.cpu(), hq, hk, d, page, 1e-6)
    _close(a[:, : hq * d], b[:, : hq * d], atol=2e-2, rtol=2e-2)
    _close(kc, kc2, atol=2e-2, rtol=2e-2)
    assert torch.equal(vc.cpu(), vc2)
