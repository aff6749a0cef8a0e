"""Paged attention, sampling and routing kernels against the fp32 reference."""

import pytest
import torch

from minisgl import ops
from minisgl.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(out, expect, atol, rtol):
    out, expect = out.float().cpu(), expect.float().cpu()
    err = (out - expect).abs()
    bad = (err > atol + rtol * expect.abs()).sum().item()
    assert bad == 0, f"{bad} elements out of tolerance; max err {err.max().item():.4g}"


def _make_pool(lens, hk, d, page, layers=2, seed=0):
    """Random KV pool + page table whose rows map positions to token slots."""
    g = torch.Generator().manual_seed(seed)
    need = [(L + page - 1) // page for L in lens]
    num_pages = sum(need) + 3
    pool = torch.randn(2, layers, num_pages, hk, page, d, generator=g).to(torch.bfloat16)
    width = max(64, (max(lens) + page + 63) // 64 * 64)
    pt = torch.zeros(len(lens) + 2, width, dtype=torch.int32)
    perm = torch.randperm(num_pages, generator=g).tolist()
    rows = []
    for b, L in enumerate(lens):
        row = len(lens) + 1 - b  # rows deliberately not equal to b
        rows.append(row)
        pages = [perm.pop() for _ in range(need[b])]
        for p in range(L):
            pt[row, p] = pages[p // page] * page + p % page
    return pool.to(DEV), pt.to(DEV), torch.tensor(rows, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("hq,hk", [(16, 8), (64, 8), (8, 1), (4, 4)])
@pytest.mark.parametrize("page", [16, 64, 256])
@pytest.mark.parametrize("splits", [1, 8])
def test_decode_attention(hq, hk, page, splits):
    d = 128
    lens = [1, 17, 63, 64, 65, 200, 1000, 333]
    B = len(lens)
    pool, pt, rows = _make_pool(lens, hk, d, page)
    seq = torch.tensor(lens, dtype=torch.int32, device=DEV)
    wide = torch.randn(B, (hq + 2 * hk) * d, device=DEV, dtype=torch.bfloat16)  # q inside a qkv row
    scale = d ** -0.5
    part_o = torch.empty(B * hq * splits * d, device=DEV, dtype=torch.float32)
    part_lse = torch.empty(B * hq * splits, device=DEV, dtype=torch.float32)
    out = ops.decode_attention(wide, pool, 1, pt, rows, seq, hq, hk, d, page, scale, part_o, part_lse, splits)
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device(DEV))
    q = wide[:, : hq * d].reshape(B, hq, d).cpu()
    cu = torch.arange(B + 1, dtype=torch.int32)
    expect = ref.attention(q, pool.cpu(), 1, pt.cpu(), rows.cpu(), seq.cpu(), cu, hq, hk, d, page, scale)
    _close(out.view(B, hq, d), expect, atol=2e-2, rtol=2e-2)


def _prefill_case(hq, hk, page, lens, qlens, qmul=1.0, pad=0):
    """Prefill attention against the fp32 reference; `pad` extra columns make
    the q row stride other than a multiple of 8 elements."""
    d = 128
    B = len(lens)
    pool, pt, rows = _make_pool(lens, hk, d, page, seed=1)
    seq = torch.tensor(lens, dtype=torch.int32, device=DEV)
    cu = torch.tensor([0] + torch.tensor(qlens).cumsum(0).tolist(), dtype=torch.int32, device=DEV)
    T = sum(qlens)
    wide = torch.randn(T, (hq + 2 * hk) * d + pad, device=DEV, dtype=torch.bfloat16) * qmul
    scale = d ** -0.5
    out = ops.prefill_attention(wide, pool, 0, pt, rows, seq, cu, max(qlens), hq, hk, d, page, scale)
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device(DEV))
    q = wide[:, : hq * d].reshape(T, hq, d).cpu()
    expect = ref.attention(q, pool.cpu(), 0, pt.cpu(), rows.cpu(), seq.cpu(), cu.cpu(), hq, hk, d, page, scale)
    _close(out.view(T, hq, d), expect, atol=2e-2, rtol=2e-2)


# 128-row query tiles on the tensor cores: partial tiles, cached prefixes,
# several tiles per request, and scores large enough (qmul 6) that running
# maxima grow across tiles and the output rescale runs. Even GQA groups run
# the head-pair kernel, the odd group (12 / 4) the one-head kernel.
@pytest.mark.parametrize("hq,hk", [(16, 8), (8, 1), (12, 4)])
@pytest.mark.parametrize("page", [16, 64, 256])
@pytest.mark.parametrize("qmul", [1.0, 6.0])
def test_prefill_attention(hq, hk, page, qmul):
    _prefill_case(hq, hk, page, [5, 64, 130, 700, 257, 1500], [5, 64, 30, 700, 100, 1300], qmul)


def test_prefill_attention_unaligned_q_stride():
    # a q row stride that TMA cannot take selects the kernel that reads q with plain loads
    _prefill_case(16, 8, 64, [5, 130, 700], [5, 30, 700], pad=2)


@pytest.mark.parametrize("B,V", [(1, 1000), (64, 151936), (3, 32000)])
def test_argmax(B, V):
    x = torch.randn(B, V, device=DEV)
    x[0, V - 1] = 100.0
    assert torch.equal(ops.argmax(x).cpu(), torch.argmax(x, -1).int().cpu())


def test_sample_greedy_limits():
    B, V = 16, 151936
    x = torch.randn(B, V, device=DEV) * 3
    t = torch.full((B,), 1.0, device=DEV)
    k1 = torch.ones(B, dtype=torch.int32, device=DEV)
    # top_k = 1 and a tiny top_p are both greedy
    assert torch.equal(ops.sample(x, t, top_k=k1).cpu(), torch.argmax(x, -1).int().cpu())
    p = torch.full((B,), 1e-6, device=DEV)
    assert torch.equal(ops.sample(x, t, top_p=p).cpu(), torch.argmax(x, -1).int().cpu())
    tiny = torch.full((B,), 1e-5, device=DEV)
    assert torch.equal(ops.sample(x, tiny).cpu(), torch.argmax(x, -1).int().cpu())


@pytest.mark.parametrize("mode", ["plain", "top_k", "top_p", "both"])
def test_sample_distribution(mode):
    """Empirical token frequencies match the filtered softmax."""
    V, draws = 12, 4000
    logits = torch.tensor([[2.0, 1.5, 1.0, 0.5, 0.0, -0.5, -1.0, 0.3, 0.9, 1.2, -2.0, 0.1]])
    x = logits.repeat(draws, 1).to(DEV)
    t = torch.full((draws,), 0.8, device=DEV)
    top_k = torch.full((draws,), 4, dtype=torch.int32, device=DEV) if mode in ("top_k", "both") else None
    top_p = torch.full((draws,), 0.7, device=DEV) if mode in ("top_p", "both") else None
    step = torch.zeros((), dtype=torch.int64, device=DEV)
    counts = torch.zeros(V)
    for _ in range(5):
        ids = ops.sample(x, t, top_k, top_p, seed=1234, step=step).cpu().long()
        counts += torch.bincount(ids, minlength=V).float()
    freq = counts / counts.sum()
    # expected distribution from the reference filter
    lf = logits / 0.8
    keep = torch.ones(V, dtype=torch.bool)
    if top_k is not None:
        keep &= lf[0] >= lf[0].topk(4).values[-1]
    if top_p is not None:
        p = torch.softmax(lf[0].masked_fill(~keep, -1e30), -1)
        sp, idx = p.sort(descending=True)
        drop = (sp.cumsum(0) - sp) >= 0.7
        keep &= ~torch.zeros(V, dtype=torch.bool).scatter(0, idx, drop)
    expect = torch.softmax(lf[0].masked_fill(~keep, -1e30), -1)
    assert (freq[~keep] == 0).all(), "sampled a filtered token"
    assert (freq - expect).abs().max() < 0.02, (freq, expect)
    assert int(step.item()) == 5


@pytest.mark.parametrize("E,k,scoring", [(128, 8, "softmax"), (64, 4, "softmax"), (384, 8, "sigmoid")])
def test_moe_route(E, k, scoring):
    T = 300
    x = torch.randn(T, E, device=DEV)
    bias = torch.randn(E, device=DEV) * 0.1 if scoring == "sigmoid" else None
    w, ids = ops.moe_route(x, k, scoring, True, bias, 1, 1, 2.5 if scoring == "sigmoid" else 1.0)
    w2, ids2 = ref.moe_route(x.cpu(), k, scoring, True, None if bias is None else bias.cpu(), 1, 1,
                             2.5 if scoring == "sigmoid" else 1.0)
    assert torch.equal(ids.cpu().sort(-1).values, ids2.sort(-1).values)
    _close(w.cpu().sort(-1).values, w2.sort(-1).values, atol=1e-5, rtol=1e-4)


def test_moe_route_grouped():
    T, E, k = 64, 256, 8
    x = torch.randn(T, E, device=DEV)
    bias = torch.randn(E, device=DEV) * 0.1
    w, ids = ops.moe_route(x, k, "sigmoid", True, bias, 8, 4, 2.5)
    w2, ids2 = ref.moe_route(x.cpu(), k, "sigmoid", True, bias.cpu(), 8, 4, 2.5)
    assert torch.equal(ids.cpu().sort(-1).values, ids2.sort(-1).values)


class _ConcatGather:
    """Stands in for a tensor-parallel communicator: the 'ranks' are the
    shards of one process, gathered by concatenation in rank order."""

    def __init__(self, parts):
        self.parts = parts

    def all_gather(self, x):
        return torch.cat(self.parts, 0)


@pytest.mark.parametrize("ranks,V", [(2, 151936), (8, 151936), (3, 1000)])
@pytest.mark.parametrize("greedy", [True, False])
def test_sample_sharded_matches_whole_vocabulary(ranks, V, greedy):
    """Sampling from vocabulary shards (tensor parallelism) draws the tokens
    the whole-vocabulary sampler draws for the same seed and step, and
    advances the step counter the same way."""
    B = 37
    x = torch.randn(B, V, device=DEV) * 2
    t = None if greedy else torch.full((B,), 0.7, device=DEV)
    step_full = torch.full((), 5, dtype=torch.int64, device=DEV)
    step_shard = step_full.clone()
    want = ops.argmax(x) if greedy else ops.sample(x, t, seed=99, step=step_full)
    per = -(-V // ranks)
    nat = ops.native()
    chunks = nat.sample_shard_chunks(per)
    ld = (2 * chunks + 3) // 4 * 4
    parts = []
    for r in range(ranks):
        lo, hi = r * per, min(V, (r + 1) * per)
        packed = torch.zeros(B, ld, dtype=torch.int32, device=DEV)
        nat.sample_shard_partials(packed, x[:, lo:hi], t, 99, step_shard, lo)
        parts.append(packed)
    got = torch.empty(B, dtype=torch.int32, device=DEV)
    nat.sample_shard_reduce(got, _ConcatGather(parts).all_gather(None), chunks, ranks, t, step_shard)
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), want.cpu())
    assert int(step_shard) == int(step_full)
