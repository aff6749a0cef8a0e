"""Device-side index checks: a KV slot outside the cache (rope + KV store,
the qkv GEMM's rope epilogue, the MLA latent store) or a request row outside
the page table (prefill and decode attention) is reported through the error
word (``ops.DeviceIndexError``) and the access is skipped. Every buffer the
kernels get is a view of a larger allocation, so an out-of-range index still
points at memory the test owns, and the test checks that it stays untouched."""

import pytest
import torch

from minisgl import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _expect_index_error():
    torch.cuda.synchronize()
    # the error word is kept per device index: name the current one
    with pytest.raises(ops.DeviceIndexError):
        ops.check_device_errors(torch.device("cuda", torch.cuda.current_device()))


def test_rope_store_reports_slot_outside_cache():
    hq, hk, d, page, pages, T = 8, 2, 128, 16, 4, 6
    qkv = torch.randn(T, (hq + 2 * hk) * d, device=DEV, dtype=torch.bfloat16)
    pos = torch.arange(T, device=DEV, dtype=torch.int32)
    cos_sin = torch.randn(64, d, device=DEV)
    kfull = torch.zeros(pages + 2, hk, page, d, device=DEV, dtype=torch.bfloat16)
    vfull = torch.zeros_like(kfull)
    kc, vc = kfull[:pages], vfull[:pages]
    loc = torch.tensor([0, 1, 2, pages * page + 3, 4, 5], device=DEV, dtype=torch.int32)
    ops.rope_store(qkv, pos, cos_sin, None, None, kc, vc, loc, hq, hk, d, page, 1e-6)
    _expect_index_error()
    assert kfull[pages:].abs().sum().item() == 0 and vfull[pages:].abs().sum().item() == 0
    assert kc.abs().sum().item() > 0  # the valid slots were written


def test_gemm_rope_epilogue_reports_slot_outside_cache():
    hq, hk, page, pages, M, H = 8, 2, 16, 4, 5, 256
    N = (hq + 2 * hk) * 128
    x = torch.randn(M, H, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, H, device=DEV, dtype=torch.bfloat16) * 0.05
    kfull = torch.zeros(pages + 2, hk, page, 128, device=DEV, dtype=torch.bfloat16)
    vfull = torch.zeros_like(kfull)
    pos = torch.arange(M, device=DEV, dtype=torch.int32)
    loc = torch.tensor([0, 1, pages * page + 7, 3, 4], device=DEV, dtype=torch.int32)
    cos_sin = torch.randn(64, 128, device=DEV)
    rope = dict(positions=pos, cos_sin=cos_sin, q_norm_w=None, k_norm_w=None, head_eps=1e-6,
                k_cache=kfull[:pages], v_cache=vfull[:pages], out_loc=loc, hq=hq, hk=hk, page_size=page)
    ops.gemm_fused(x, w, rope=rope, plan=(2, 128, 1))
    _expect_index_error()
    assert kfull[pages:].abs().sum().item() == 0 and vfull[pages:].abs().sum().item() == 0


def test_attention_reports_request_row_outside_page_table():
    hq, hk, d, page, L = 8, 2, 128, 64, 100
    pool = torch.randn(2, 1, 4, hk, page, d, device=DEV, dtype=torch.bfloat16)
    full = torch.zeros(4, 128, device=DEV, dtype=torch.int32)
    full[:, :L] = torch.arange(L, device=DEV, dtype=torch.int32)
    pt = full[:2]  # the kernels see two rows; row 3 is still memory of this test
    rows = torch.tensor([1, 3], device=DEV, dtype=torch.int32)
    seq = torch.tensor([L, L], device=DEV, dtype=torch.int32)
    q = torch.randn(2 * L, hq * d, device=DEV, dtype=torch.bfloat16)
    cu = torch.tensor([0, L, 2 * L], device=DEV, dtype=torch.int32)
    ops.prefill_attention(q, pool, 0, pt, rows, seq, cu, L, hq, hk, d, page, d ** -0.5)
    _expect_index_error()
    qd = torch.randn(2, hq * d, device=DEV, dtype=torch.bfloat16)
    part_o = torch.empty(2 * hq * 4 * d, device=DEV, dtype=torch.float32)
    part_lse = torch.empty(2 * hq * 4, device=DEV, dtype=torch.float32)
    ops.decode_attention(qd, pool, 0, pt, rows, seq, hq, hk, d, page, d ** -0.5, part_o, part_lse, 4)
    _expect_index_error()


def test_mla_latent_store_reports_slot_outside_pool():
    pages, page, T = 3, 64, 4
    full = torch.zeros(pages + 2, page, 576, device=DEV, dtype=torch.bfloat16)
    kv_a = torch.randn(T, 576, device=DEV, dtype=torch.bfloat16)
    norm_w = torch.ones(512, device=DEV, dtype=torch.bfloat16)
    pos = torch.arange(T, device=DEV, dtype=torch.int32)
    cos_sin = torch.randn(64, 64, device=DEV)
    loc = torch.tensor([0, pages * page + 2, 2, 3], device=DEV, dtype=torch.int32)
    ops.mla_store_latent(kv_a, norm_w, 1e-6, pos, cos_sin, full[:pages], loc, page)
    _expect_index_error()
    assert full[pages:].abs().sum().item() == 0
    assert full[0, :4].abs().sum().item() > 0  # the valid rows were stored
