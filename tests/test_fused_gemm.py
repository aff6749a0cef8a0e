"""Fused-epilogue GEMMs (row RMSNorm, SiLU x up, residual add, q/k-norm +
RoPE + KV store) against the fp32 reference composition."""

import pytest
import torch

from minisgl import ops
from minisgl.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
# (mode, N tile, K splits): weight-major cluster path, token-major cluster
# path, and token-major tiles without split-K (epilogue straight from TMEM)
PLANS = [None, (2, 16, 1), (2, 32, 4), (2, 64, 8), (2, 128, 2), (2, 256, 1), (1, 128, 1), (1, 256, 1),
         (1, 64, 1), (1, 256, 2), (1, 128, 8)]


def _whole_heads(plan):
    return plan is None or plan[0] == 2 or plan[1] % 128 == 0


def _close(out, expect, atol=3e-2, rtol=3e-2):
    out, expect = out.float().cpu(), expect.float().cpu()
    err = (out - expect).abs()
    bad = (err > atol + rtol * expect.abs()).sum().item()
    assert bad == 0, f"{bad} elements out of tolerance; max err {err.max().item():.4g}"


def _inputs(M, N, K, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("M", [1, 5, 32, 77, 256, 300])
@pytest.mark.parametrize("plan", PLANS)
def test_norm_residual(M, plan):
    N, K = 1024, 2048
    x, w = _inputs(M, N, K)
    res = torch.randn(M, N).to(torch.bfloat16)
    bias = (torch.randn(N) * 0.1).to(torch.bfloat16)
    xd, wd, rd = x.to(DEV), w.to(DEV), res.to(DEV)
    out = ops.gemm_fused(xd, wd, norm_eps=1e-6, bias=bias.to(DEV), plan=plan)
    _close(out, ref.gemm_fused(x, w, bias, 1e-6, None, False, None))
    out = ops.gemm_fused(xd, wd, residual=rd, out=rd, plan=plan)  # in place
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device(DEV))
    _close(out, ref.gemm_fused(x, w, None, None, res, False, None))


@pytest.mark.parametrize("M", [1, 16, 33, 128, 256])
@pytest.mark.parametrize("plan", PLANS)
def test_norm_silu(M, plan):
    if not _whole_heads(plan):
        pytest.skip("token-major silu needs N tiles of 128 / 256")
    N, K = 2 * 768, 1024
    x, w = _inputs(M, N, K, seed=1)
    out = ops.gemm_fused(x.to(DEV), w.to(DEV), norm_eps=1e-6, silu=True, plan=plan)
    torch.cuda.synchronize()
    _close(out, ref.gemm_fused(x, w, None, 1e-6, None, True, None))
    # the interleaved activation kernel used by the unfused path agrees
    h = ops.gemm(ops.rmsnorm(x.to(DEV), None, 1e-6), w.to(DEV))
    _close(ops.silu_and_mul(h, interleaved=True), ref.gemm_fused(x, w, None, 1e-6, None, True, None))


@pytest.mark.parametrize("M", [1, 9, 64, 256])
@pytest.mark.parametrize("plan", PLANS)
@pytest.mark.parametrize("qk_norm", [True, False])
def test_norm_rope_store(M, plan, qk_norm):
    if not _whole_heads(plan):
        pytest.skip("token-major rope needs N tiles of 128 / 256")
    hq, hk, K, page = 16, 8, 1024, 16
    N = (hq + 2 * hk) * 128
    x, w = _inputs(M, N, K, seed=2)
    g = torch.Generator().manual_seed(3)
    pages = (M + page - 1) // page + 2
    cos_sin = torch.cat([torch.cos(torch.rand(512, 64, generator=g) * 6),
                         torch.sin(torch.rand(512, 64, generator=g) * 6)], dim=1)
    positions = torch.randint(0, 512, (M,), generator=g, dtype=torch.int32)
    out_loc = torch.randperm(pages * page, generator=g)[:M].to(torch.int32)
    qn = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16) if qk_norm else None
    kc = torch.zeros(pages, hk, page, 128, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)

    def rope(dev, kc_, vc_):
        return dict(positions=positions.to(dev), cos_sin=cos_sin.to(dev), out_loc=out_loc.to(dev),
                    q_norm_w=None if qn is None else qn.to(dev), k_norm_w=None if kn is None else kn.to(dev),
                    head_eps=1e-6, k_cache=kc_, v_cache=vc_, hq=hq, hk=hk, page_size=page)

    kcd, vcd = kc.to(DEV), vc.to(DEV)
    qkv = torch.zeros(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm_fused(x.to(DEV), w.to(DEV), norm_eps=1e-6, rope=rope(DEV, kcd, vcd), out=qkv, plan=plan)
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device(DEV))
    expect = ref.gemm_fused(x, w, None, 1e-6, None, False, rope("cpu", kc, vc))
    _close(qkv[:, : hq * 128], expect[:, : hq * 128])
    _close(kcd, kc)
    _close(vcd, vc)


@pytest.mark.parametrize("M", [1, 7, 64, 256])
@pytest.mark.parametrize("plan", [(16, 1), (32, 2), (64, 1), (256, 1), (32, 8)])
@pytest.mark.parametrize("temps", ["greedy", "mixed"])
def test_lm_head_sample_matches_logit_sampler(M, plan, temps):
    """Sampling inside the LM-head GEMM draws the same tokens as the sampling
    kernel run on the materialised fp32 logits of the same tile plan."""
    N, K = 5000, 1024  # a vocabulary that does not fill its last 128-row tile
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    logits = torch.empty(M, N, device=DEV, dtype=torch.float32)
    ops.native().gemm(logits, x, w, None, None, plan[1], 2, None, plan[0])
    step_a = torch.full((), 5, dtype=torch.int64, device=DEV)
    step_b = step_a.clone()
    if temps == "greedy":
        expect = ops.argmax(logits)
        got = ops.lm_head_sample(x, w, None, None, 123, step_b, plan=plan)
    else:
        t = torch.rand(M, generator=g) * 1.5
        t[::3] = 1e-6  # greedy rows of a mixed batch
        t = t.to(DEV)
        expect = ops.sample(logits, t, None, None, 123, step_a)
        got = ops.lm_head_sample(x, w, None, t, 123, step_b, plan=plan)
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device(DEV))
    assert torch.equal(got.cpu(), expect.cpu())
    assert step_a.item() == step_b.item()  # both paths advance the counter alike
