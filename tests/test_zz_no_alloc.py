"""The allocation-free decode attention entry point, called through its
exported C symbol and checked against minisgl.ops.decode_attention and
against the fp32 PyTorch statement of paged attention
(minisgl.ops.reference.attention).

Collected last on purpose: it must also pass after every other GPU test has
run in the same process (with the library's other state already warm).
"""

import ctypes

import pytest
import torch

from minisgl import ops
from minisgl.ops import reference

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCRATCH_BYTES = 8 << 20  # MINISGL_NOALLOC_SCRATCH_BYTES


def _entry():
    lib = ctypes.CDLL(ops.native().__file__)
    fn = lib.minisgl_decode_attention_noalloc
    fn.restype = ctypes.c_int
    i, p = ctypes.c_int, ctypes.c_void_p
    fn.argtypes = [p, p, i, p, i, i, i, p, i, p, p, i, i, i, i, i, ctypes.c_float, i, p, p,
                   ctypes.c_char_p, ctypes.c_size_t]
    return fn


def _make_pool(lens, hk, d, page, layers, seed):
    g = torch.Generator().manual_seed(seed)
    need = [(L + page - 1) // page for L in lens]
    num_pages = sum(need) + 2
    pool = torch.randn(2, layers, num_pages, hk, page, d, generator=g).to(torch.bfloat16)
    width = max(64, (max(lens) + page + 63) // 64 * 64)
    pt = torch.zeros(len(lens) + 1, width, dtype=torch.int32)
    perm = torch.randperm(num_pages, generator=g).tolist()
    rows = []
    for b, L in enumerate(lens):
        row = len(lens) - b
        rows.append(row)
        pages = [perm.pop() for _ in range(need[b])]
        for pos in range(L):
            pt[row, pos] = pages[pos // page] * page + pos % page
    return pool.to(DEV), pt.to(DEV), torch.tensor(rows, dtype=torch.int32, device=DEV)


def _call(fn, out, q, pool, layer, pt, rows, seq, hq, hk, d, page, scale, splits, err):
    msg = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(out.data_ptr(), q.data_ptr(), q.stride(0), pool.data_ptr(), pool.size(1), pool.size(2), layer,
            pt.data_ptr(), pt.stride(0), rows.data_ptr(), seq.data_ptr(), rows.numel(), hq, hk, d, page, scale,
            splits, err.data_ptr() if err is not None else None, stream, msg, len(msg))
    return rc, msg.value.decode()


def _case(lens, hq, hk, page, splits, seed):
    d, layers = 128, 3
    pool, pt, rows = _make_pool(lens, hk, d, page, layers, seed)
    seq = torch.tensor(lens, dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(len(lens), (hq + 2 * hk) * d, device=DEV, dtype=torch.bfloat16, generator=g)
    return dict(q=q, pool=pool, pt=pt, rows=rows, seq=seq, hq=hq, hk=hk, d=d, page=page, splits=splits,
                scale=d ** -0.5, layer=layers - 1)


def _expected(c):
    B = c["rows"].numel()
    part_o = torch.empty(B * c["hq"] * c["splits"] * c["d"], device=DEV, dtype=torch.float32)
    part_lse = torch.empty(B * c["hq"] * c["splits"], device=DEV, dtype=torch.float32)
    return ops.decode_attention(c["q"], c["pool"], c["layer"], c["pt"], c["rows"], c["seq"], c["hq"], c["hk"],
                                c["d"], c["page"], c["scale"], part_o, part_lse, c["splits"])


def _oracle(c):
    """fp32 paged attention over the same pool, page table and queries."""
    B, hq, d = c["rows"].numel(), c["hq"], c["d"]
    q = c["q"][:, : hq * d].float().reshape(B, hq, d)
    cu = torch.arange(B + 1, dtype=torch.int32, device=DEV)
    out = reference.attention(q, c["pool"].float(), c["layer"], c["pt"], c["rows"], c["seq"], cu, hq, c["hk"], d,
                              c["page"], c["scale"])
    return out.reshape(B, hq * d)


def _run(fn, c, err):
    out = torch.empty(c["rows"].numel(), c["hq"] * c["d"], device=DEV, dtype=torch.bfloat16)
    rc, msg = _call(fn, out, c["q"], c["pool"], c["layer"], c["pt"], c["rows"], c["seq"], c["hq"], c["hk"],
                    c["d"], c["page"], c["scale"], c["splits"], err)
    assert rc == 0, msg
    return out


def _close(out, expect, atol=2e-2, rtol=2e-2):
    out, expect = out.float(), expect.float()
    err = (out - expect).abs()
    bad = (err > atol + rtol * expect.abs()).sum().item()
    assert bad == 0, f"{bad} elements out of tolerance; max err {err.max().item():.4g}"


def test_noalloc_matches_regular_entry_twice_in_a_row():
    fn = _entry()
    err = ops.error_word(torch.device(DEV))
    # first call: long sequences, 16 splits, wide GQA group
    a = _case([1, 70, 700, 2000, 333, 64, 129, 1500], hq=16, hk=2, page=64, splits=16, seed=1)
    # second call, right after: a different batch with fewer splits, so the
    # scratch still holds the first call's partials where this one reads none
    b = _case([5, 900, 1200, 17, 4000], hq=8, hk=8, page=16, splits=6, seed=2)
    out_a = _run(fn, a, err)
    out_b = _run(fn, b, err)
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device(DEV))
    _close(out_a, _expected(a))
    _close(out_b, _expected(b))
    _close(out_a, _oracle(a))
    _close(out_b, _oracle(b))
    torch.cuda.synchronize()


def test_noalloc_single_split_and_limits():
    fn = _entry()
    c = _case([3, 300, 77], hq=16, hk=8, page=256, splits=1, seed=3)
    out1 = _run(fn, c, None)
    _close(out1, _expected(c))
    _close(out1, _oracle(c))
    # a request whose scratch would not fit is rejected with a clear error
    B = 64
    big = _case([10] * B, hq=16, hk=8, page=16, splits=16, seed=4)
    assert B * 16 * 16 * 129 * 4 > SCRATCH_BYTES
    out = torch.empty(B, 16 * 128, device=DEV, dtype=torch.bfloat16)
    rc, msg = _call(fn, out, big["q"], big["pool"], big["layer"], big["pt"], big["rows"], big["seq"], 16, 8, 128,
                    16, big["scale"], 16, None)
    assert rc == 2 and "exceeds the fixed" in msg, (rc, msg)
    # unsupported shapes are rejected, not launched
    rc, msg = _call(fn, out, big["q"], big["pool"], big["layer"], big["pt"], big["rows"], big["seq"], 16, 8, 64,
                    16, big["scale"], 1, None)
    assert rc == 1 and "head_dim" in msg, (rc, msg)
    # a page-table row stride below one element (here 0) is rejected before any launch
    pt0 = big["pt"].as_strided(tuple(big["pt"].shape), (0, 1))
    assert pt0.stride(0) == 0
    rc, msg = _call(fn, out, big["q"], big["pool"], big["layer"], pt0, big["rows"], big["seq"], 16, 8, 128, 16,
                    big["scale"], 1, None)
    assert rc == 1 and "ld_pt" in msg, (rc, msg)
    torch.cuda.synchronize()
