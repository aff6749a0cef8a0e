"""Per-kernel timings at serving shapes, with roofline fractions.

    python -m minisgl.benchmark.kernels [--only <label text>] [--json out.json]
    python -m minisgl.benchmark.kernels --probe M,N,K,mode,bn,splits[,kps] [--trace]

``--probe`` times one forced GEMM tile plan (mode 1 token-major, 2
weight-major, 3 persistent; N tile; split-K factor; k-blocks per stage) over
back-to-back launches cycling 8 weight copies; ``--trace`` adds per-CTA
%globaltimer phase stamps (entry, set-up done, producer past
griddepcontrol.wait, first stage consumed, accumulator ready, exit).

Denominators are the measured B200 peaks in MEASURED_PEAKS.json when present
(STREAM-style copy bandwidth and cuBLAS bf16 GEMM throughput), else the
fallback figures 6650 GB/s and 1590 TFLOP/s. Each line reports the kernel's
time (CUDA events, L2 flushed between calls), its algorithmic bytes / FLOPs
and the achieved fraction of the relevant peak. cuBLAS (torch.matmul) is
timed on the same GEMM shapes as a baseline.
"""

from __future__ import annotations

import argparse
import json
import os
import random
from typing import Dict, List, Optional

import torch

from minisgl import ops

from .perf import SmClockLog, time_graph, time_kernel


def _peaks() -> Dict[str, float]:
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    path = os.path.join(root, "MEASURED_PEAKS.json")
    if os.path.isfile(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "source": "fallback"}


def _pool(lens: List[int], hk: int, d: int, page: int, layers: int = 1):
    pages_per = [(L + page - 1) // page for L in lens]
    num_pages = sum(pages_per) + 1
    pool = torch.randn(2, layers, num_pages, hk, page, d, device="cuda", dtype=torch.bfloat16) * 0.5
    width = (max(lens) + page + 63) // 64 * 64
    pt = torch.zeros(len(lens), width, dtype=torch.int32)
    perm = torch.randperm(num_pages - 1).tolist()
    for b, L in enumerate(lens):
        pages = [perm.pop() for _ in range(pages_per[b])]
        pos = torch.arange(L)
        pt[b, :L] = torch.tensor(pages)[pos // page] * page + pos % page
    return pool, pt.cuda(), torch.arange(len(lens), dtype=torch.int32, device="cuda")


def bench_decode_attention(B: int, L: int, hq: int, hk: int, page: int, peaks) -> Dict:
    d = 128
    lens = [L] * B
    pool, pt, rows = _pool(lens, hk, d, page)
    seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, hq * d, device="cuda", dtype=torch.bfloat16)
    from minisgl.attention.native import MAX_SPLITS, decode_splits

    splits = decode_splits(B, hk)
    part_o = torch.empty(B * hq * MAX_SPLITS * d, device="cuda")
    part_lse = torch.empty(B * hq * MAX_SPLITS, device="cuda")
    ms = time_kernel(lambda: ops.decode_attention(q, pool, 0, pt, rows, seq, hq, hk, d, page, d ** -0.5,
                                                  part_o, part_lse, splits))
    nbytes = 2 * B * L * hk * d * 2
    gbs = nbytes / ms / 1e6
    ms_trt = _trtllm_attention_ms(pool, pt, rows, seq, q, 1, hq, hk, d, page)
    return {"kernel": "decode_attention", "B": B, "L": L, "hq": hq, "hk": hk, "page": page, "splits": splits,
            "ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 3),
            "trtllm_ms": None if ms_trt is None else round(ms_trt, 4),
            "vs_trtllm": None if ms_trt is None else round(ms_trt / ms, 3)}


def bench_decode_attention_varlen(B: int, lo: int, hi: int, hq: int, hk: int, page: int, peaks) -> List[Dict]:
    """Mixed lengths U[lo, hi], the serving mix (bytes: the keys that exist)."""
    d = 128
    g = random.Random(1)
    lens = [g.randint(lo, hi) for _ in range(B)]
    pool, pt, rows = _pool(lens, hk, d, page)
    seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, hq * d, device="cuda", dtype=torch.bfloat16)
    from minisgl.attention.native import MAX_SPLITS, decode_splits

    splits = decode_splits(B, hk)
    part_o = torch.empty(B * hq * MAX_SPLITS * d, device="cuda")
    part_lse = torch.empty(B * hq * MAX_SPLITS, device="cuda")
    nbytes = 2 * sum(lens) * hk * d * 2
    out = []
    ms = time_kernel(lambda: ops.decode_attention(q, pool, 0, pt, rows, seq, hq, hk, d, page, d ** -0.5,
                                                  part_o, part_lse, splits))
    gbs = nbytes / ms / 1e6
    out.append({"kernel": "decode_attention_varlen", "B": B, "L": f"U[{lo},{hi}]", "hq": hq, "hk": hk,
                "page": page, "splits": splits, "ms": round(ms, 4), "GB/s": round(gbs, 1),
                "frac_hbm": round(gbs / peaks["hbm_gbs"], 3)})
    return out


def _trtllm_attention_ms(pool, pt, rows, seq, q, L_q: int, hq: int, hk: int, d: int, page: int) -> Optional[float]:
    """Milliseconds of the TRT-LLM FMHA kernels that flashinfer ships (the
    reference's default attention backend on sm100) on the same paged pool
    (HND pages of this layer) and queries, or None when flashinfer is not
    importable. Prefill when L_q > 1 (every request has L_q new tokens),
    decode otherwise. Timed for comparison only; the engine never calls it."""
    try:
        from flashinfer.decode import trtllm_batch_decode_with_kv_cache
        from flashinfer.prefill import trtllm_batch_context_with_kv_cache
    except Exception:  # noqa: BLE001 - an optional library
        return None
    B = rows.numel()
    kv = (pool[0, 0], pool[1, 0])  # [pages, hk, page, d]
    blocks = (pt[rows.long(), ::page] // page).to(torch.int32).contiguous()
    ws = torch.empty(128 << 20, dtype=torch.uint8, device="cuda")
    qv = q.view(-1, hq, d)
    max_kv = int(seq.max())
    try:
        if L_q > 1:
            cu_q = torch.arange(0, (B + 1) * L_q, L_q, dtype=torch.int32, device="cuda")
            cu_kv = torch.cat([torch.zeros(1, dtype=torch.int32, device="cuda"), seq.cumsum(0).to(torch.int32)])
            fn = lambda: trtllm_batch_context_with_kv_cache(  # noqa: E731
                qv, kv, ws, blocks, seq, L_q, max_kv, d ** -0.5, 1.0, B, cu_q, cu_kv, kv_layout="HND",
                out_dtype=torch.bfloat16)
        else:
            fn = lambda: trtllm_batch_decode_with_kv_cache(  # noqa: E731
                qv, kv, ws, blocks, seq, max_kv, d ** -0.5, 1.0, kv_layout="HND", out_dtype=torch.bfloat16)
        return time_kernel(fn, iters=5)
    except Exception:  # noqa: BLE001 - shapes the library does not take
        return None


def bench_prefill_attention(B: int, L: int, hq: int, hk: int, page: int, peaks) -> Dict:
    """Causal prefill of B requests of L tokens. `ms` is the tcgen05 kernel
    (q read by TMA); `ms_plain_q` the warp-MMA kernel that the launcher takes
    when the q row stride is not a multiple of 8 elements (same inputs, q
    padded by 2 columns)."""
    d = 128
    lens = [L] * B
    pool, pt, rows = _pool(lens, hk, d, page)
    seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
    cu = torch.arange(0, (B + 1) * L, L, dtype=torch.int32, device="cuda")
    qp = torch.randn(B * L, hq * d + 2, device="cuda", dtype=torch.bfloat16)
    q = qp[:, : hq * d].contiguous()
    ms = time_kernel(lambda: ops.prefill_attention(q, pool, 0, pt, rows, seq, cu, L, hq, hk, d, page, d ** -0.5),
                     iters=5)
    ms_old = time_kernel(lambda: ops.prefill_attention(qp, pool, 0, pt, rows, seq, cu, L, hq, hk, d, page,
                                                       d ** -0.5), iters=5)
    flops = 4 * B * hq * d * L * (L + 1) / 2
    tf = flops / ms / 1e9
    ms_trt = _trtllm_attention_ms(pool, pt, rows, seq, q, L, hq, hk, d, page)
    return {"kernel": "prefill_attention", "B": B, "L": L, "hq": hq, "hk": hk, "ms": round(ms, 4),
            "TFLOP/s": round(tf, 1), "frac_tensor": round(tf / peaks["tflops"], 3),
            "ms_plain_q": round(ms_old, 4), "speedup": round(ms_old / ms, 2),
            "trtllm_ms": None if ms_trt is None else round(ms_trt, 4),
            "vs_trtllm": None if ms_trt is None else round(ms_trt / ms, 3)}


def trace_prefill_attention(B: int = 1, L: int = 16384, hq: int = 16, hk: int = 8, page: int = 64) -> Dict:
    """Median per-tile phase times (ns) of one prefill CTA from the kernel's
    %globaltimer trace: the CTA with the longest key range of request 0,
    head 0; tiles 4-59 of its first 64."""
    import statistics

    d = 128
    pool, pt, rows = _pool([L] * B, hk, d, page)
    seq = torch.tensor([L] * B, dtype=torch.int32, device="cuda")
    cu = torch.arange(0, (B + 1) * L, L, dtype=torch.int32, device="cuda")
    q = torch.randn(B * L, hq * d, device="cuda", dtype=torch.bfloat16)
    tr = torch.zeros(512, dtype=torch.int64, device="cuda")
    for _ in range(3):
        ops.prefill_attention(q, pool, 0, pt, rows, seq, cu, L, hq, hk, d, page, d ** -0.5, trace=tr)
    torch.cuda.synchronize()
    t = tr.view(64, 8).cpu().tolist()
    if os.environ.get("MINISGL_PREFILL_PAIR", "1") != "0" and (hq // hk) % 2 == 0:
        # head-pair kernel slots: 0 scores seen (head 0, warp 0), 1-4 P
        # handed over by head 0's warps 0-3, 5 MMA thread saw P, 6 PV issued,
        # 7 next QK issued
        pair = {
            "period": lambda i: t[i][1] - t[i - 1][1],
            "scores_seen_to_p_handed_w0": lambda i: t[i][1] - t[i][0],
            "p_handed_skew_last_minus_first": lambda i: max(t[i][1:5]) - min(t[i][1:5]),
            "last_p_to_mma_sees_p": lambda i: t[i][5] - max(t[i][1:5]),
            "pv_issue": lambda i: t[i][6] - t[i][5],
            "kv_wait_and_qk_issue": lambda i: t[i][7] - t[i][6],
            "qk_issued_to_next_scores": lambda i: t[i + 1][0] - t[i][7],
        }
        out = {"trace": "prefill_attention (head pairs)", "B": B, "L": L, "hq": hq, "hk": hk}
        for k, f in pair.items():
            out[k + "_ns"] = statistics.median(f(i) for i in range(4, 59))
        return out
    # slots: 0 copy issued, 1 QK issued, 2 scores ready, 7 scores loaded, 3 exps done,
    # 4 PV(i - 2) done, 5 P written, 6 PV issued
    phases = {
        "period": lambda i: t[i][5] - t[i - 1][5],
        "copy_to_qk_issue": lambda i: t[i][1] - t[i][0],
        "qk_issue_to_scores": lambda i: t[i][2] - t[i][1],
        "softmax_idle": lambda i: t[i][2] - t[i - 1][5],
        "exps": lambda i: t[i][3] - t[i][7],
        "p_written_to_pv_issue": lambda i: t[i][6] - t[i][5],
        "qk_issue_to_pv_issue": lambda i: t[i][6] - t[i][1],
    }
    out = {"trace": "prefill_attention", "B": B, "L": L, "hq": hq, "hk": hk}
    for k, f in phases.items():
        out[k + "_ns"] = statistics.median(f(i) for i in range(4, 60))
    return out


def bench_mla_decode(B: int, L: int, H: int, page: int, peaks) -> Dict:
    """Absorbed MLA decode over a paged latent cache (576 bf16 per token).
    Bytes: every latent row once (head groups of 64 re-read it from L2);
    FLOPs: 2 * H * L * (576 + 512) per request."""
    lens = [L] * B
    pages_per = (L + page - 1) // page
    num_pages = B * pages_per + 1
    latent = torch.randn(num_pages, page, 576, device="cuda", dtype=torch.bfloat16) * 0.5
    perm = torch.randperm(num_pages - 1)
    pos = torch.arange(pages_per * page)
    pt = (perm[: B * pages_per].view(B, pages_per)[:, pos // page] * page + pos % page).to(torch.int32).cuda()
    rows = torch.arange(B, dtype=torch.int32, device="cuda")
    seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    tile = ops._group_tile(B)
    T_pad = (B + tile - 1) // tile * tile
    q_lat = torch.randn(H, T_pad, 512, device="cuda", dtype=torch.bfloat16) * 0.5
    q_pe = torch.randn(B, H, 64, device="cuda", dtype=torch.bfloat16) * 0.5
    splits = ops.native().mla_num_splits(B, H)
    ms = time_kernel(lambda: ops.mla_attention(q_lat, q_pe, latent, pt, rows, seq, cu, page, 192 ** -0.5))
    nbytes = B * L * 576 * 2
    flops = 2.0 * B * H * L * (576 + 512)
    gbs = nbytes / ms / 1e6
    tf = flops / ms / 1e9
    return {"kernel": "mla_decode", "B": B, "L": L, "heads": H, "page": page, "splits": splits, "ms": round(ms, 4),
            "GB/s": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 3), "TFLOP/s": round(tf, 1),
            "frac_tensor": round(tf / peaks["tflops"], 3)}


def bench_mla_prefill(B: int, L: int, H: int, peaks) -> Dict:
    """Causal MLA prefill of B requests of L new tokens at Kimi-K2 latent
    dims, both forms: absorbed (queries through W_UK, attention over the
    576-dim latent rows, output through W_UV) and non-absorbed (every key
    expanded through kv_b_proj, then 192 / 128-dim attention). FLOPs of the
    non-absorbed form: expansion 2 * 512 * 256 * H per key plus 2 * (192 +
    128) * H per causal query-key pair."""
    page = 64
    lens = [L] * B
    pages_per = (L + page - 1) // page
    num_pages = B * pages_per + 1
    latent = torch.randn(num_pages, page, 576, device="cuda", dtype=torch.bfloat16) * 0.5
    perm = torch.randperm(num_pages - 1)
    pos = torch.arange(pages_per * page)
    pt = (perm[: B * pages_per].view(B, pages_per)[:, pos // page] * page + pos % page).to(torch.int32).cuda()
    rows = torch.arange(B, dtype=torch.int32, device="cuda")
    seq = torch.tensor(lens, dtype=torch.int32, device="cuda")
    cu = torch.arange(0, (B + 1) * L, L, dtype=torch.int32, device="cuda")
    T = B * L
    scale = 192 ** -0.5
    q = torch.randn(T, H, 192, device="cuda", dtype=torch.bfloat16)
    q_rope = torch.randn(T, H, 64, device="cuda", dtype=torch.bfloat16)
    w_kv_b = torch.randn(H * 256, 512, device="cuda", dtype=torch.bfloat16) * 0.05
    w_uk_t = torch.randn(H, 512, 128, device="cuda", dtype=torch.bfloat16) * 0.05
    w_uv = torch.randn(H, 128, 512, device="cuda", dtype=torch.bfloat16) * 0.05
    plan = ops.MlaPrefillPlan(lens, torch.device("cuda"))
    tile = ops._group_tile(T)
    T_pad = (T + tile - 1) // tile * tile

    def absorbed():
        xs = torch.empty(H, T_pad, 128, device="cuda", dtype=torch.bfloat16)
        xs[:, :T] = q[..., :128].transpose(0, 1)
        q_lat = ops.grouped_gemm(xs, w_uk_t, tile)
        o_lat = ops.mla_attention(q_lat, q_rope, latent, pt, rows, seq, cu, page, scale)
        return ops.mla_output(o_lat, w_uv, T)

    def expanded():
        return ops.mla_prefill_attention(q, q_rope, latent, pt, rows, seq, cu, L, w_kv_b, 128, 128, page, scale,
                                         plan)

    ms_abs = time_kernel(absorbed, iters=3)
    ms_exp = time_kernel(expanded, iters=3)
    pairs = B * L * (L + 1) / 2
    flops_exp = 2.0 * 512 * 256 * H * B * L + 2.0 * (192 + 128) * H * pairs
    return {"kernel": "mla_prefill", "B": B, "L": L, "heads": H, "absorbed_ms": round(ms_abs, 3),
            "expanded_ms": round(ms_exp, 3), "speedup": round(ms_abs / ms_exp, 2),
            "expanded_TFLOP/s": round(flops_exp / ms_exp / 1e9, 1),
            "expanded_frac_tensor": round(flops_exp / ms_exp / 1e9 / peaks["tflops"], 3)}


def bench_moe_mxfp4(T: int, E: int, k: int, H: int, I: int, peaks) -> Dict:
    """Routed experts with MXFP4 weights (Kimi-K2 expert dims by default):
    router outputs uniform over E local experts, the full pipeline (align,
    gather, gate_up with SiLU, down, combine) against the same experts in
    bf16. Bytes: the MXFP4 weights of the experts hit (4.25 bits a weight)
    plus activations; the bf16 row reads its bf16 weights."""
    from minisgl.quant import quantize_mxfp4

    g = torch.Generator(device="cuda").manual_seed(0)
    w1 = (torch.randn(E, 2 * I, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    q1, q2 = quantize_mxfp4(w1), quantize_mxfp4(w2)
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, device="cuda", generator=g)[:k] for _ in range(T)]).to(torch.int32)
    tw = torch.full((T, k), 1.0 / k, device="cuda")
    hit = int(torch.unique(ids).numel())
    ms = time_kernel(lambda: ops.moe_experts_mxfp4(x, *q1, *q2, tw, ids))
    tiles = {t: round(time_kernel(lambda t=t: ops.moe_experts_mxfp4(x, *q1, *q2, tw, ids, tile=t)), 4)
             for t in (16, 32, 64, 128) if t <= max(16, 2 * T * k // E)}
    ms_bf16 = time_kernel(lambda: ops.moe_experts(x, w1, w2, tw, ids))
    wbytes = hit * (3 * I * H) * 0.5 * (1 + 1 / 16)  # E2M1 + one E8M0 byte per 32
    nbytes = wbytes + 2 * 2 * T * k * H
    gbs = nbytes / ms / 1e6
    return {"kernel": "moe_experts_mxfp4", "T": T, "E": E, "k": k, "H": H, "I": I, "experts_hit": hit,
            "ms": round(ms, 4), "bf16_ms": round(ms_bf16, 4), "GB/s": round(gbs, 1),
            "frac_hbm": round(gbs / peaks["hbm_gbs"], 3), "ms_by_token_tile": tiles}


def bench_moe_mx(T: int, E: int, k: int, H: int, I: int, peaks) -> Dict:
    """Routed experts on the block-scaled tensor cores (MXFP4 weights x
    MXFP8 activations, ``--moe-quant mxfp4-a8``) at the same shapes as
    bench_moe_mxfp4, with the error against the path's PyTorch statement
    (max |got - want| over max |want|) and the W4A16 time beside it."""
    from minisgl.quant import block_scales, moe_experts_mx_reference, quantize_mxfp4

    g = torch.Generator(device="cuda").manual_seed(0)
    w1 = (torch.randn(E, 2 * I, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    q1, q2 = quantize_mxfp4(w1), quantize_mxfp4(w2)
    b1, b2 = block_scales(q1[1]), block_scales(q2[1])
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, device="cuda", generator=g)[:k] for _ in range(T)]).to(torch.int32)
    tw = torch.full((T, k), 1.0 / k, device="cuda")
    got = ops.moe_experts_mx(x, q1[0], b1, q2[0], b2, tw, ids)
    torch.cuda.synchronize()
    ops.check_device_errors(torch.device("cuda", torch.cuda.current_device()))
    want = moe_experts_mx_reference(x, *q1, *q2, tw, ids).float()  # PyTorch ops, on the GPU
    err = ((got.float() - want).abs().max() / want.abs().max()).item()
    ms = time_kernel(lambda: ops.moe_experts_mx(x, q1[0], b1, q2[0], b2, tw, ids))
    ms_w4a16 = time_kernel(lambda: ops.moe_experts_mxfp4(x, *q1, *q2, tw, ids))
    hit = int(torch.unique(ids).numel())
    wbytes = hit * (3 * I * H) * 0.5 * (1 + 1 / 16)
    nbytes = wbytes + 2 * T * k * H + 2 * T * H  # MXFP4 weights, MXFP8 rows in, bf16 rows out
    gbs = nbytes / ms / 1e6
    return {"kernel": "moe_experts_mx", "T": T, "E": E, "k": k, "H": H, "I": I, "experts_hit": hit,
            "ms": round(ms, 4), "w4a16_ms": round(ms_w4a16, 4), "max_rel_err": round(err, 5),
            "GB/s": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 3)}


def bench_mx8_quantize(P: int, K: int, tile: int, peaks) -> Dict:
    """The MXFP8 row quantiser of the block-scaled expert path alone: bf16
    rows in, E4M3 rows and 512-byte scale blocks out, checked bit for bit
    against its PyTorch statement, timed against the measured HBM copy
    bandwidth."""
    from minisgl.quant import quantize_mx8_reference

    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(P, K, device="cuda", generator=g) * 2).to(torch.bfloat16)
    q, sf = ops.mx8_quantize(x, tile)
    torch.cuda.synchronize()
    wq, wsf = quantize_mx8_reference(x.float(), tile)
    exact = bool(torch.equal(q, wq) and torch.equal(sf, wsf))
    ms = time_kernel(lambda: ops.mx8_quantize(x, tile))
    nbytes = P * K * 2 + P * K + sf.numel()
    gbs = nbytes / ms / 1e6
    return {"kernel": "mx8_quantize", "P": P, "K": K, "tile": tile, "exact": exact, "ms": round(ms, 4),
            "GB/s": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 3)}


def bench_sample(B: int, V: int, peaks) -> List[Dict]:
    """Sampling from fp32 logits [B, V]: argmax (greedy) and Gumbel-max with
    temperature (counter-based noise); bytes = the logits read once."""
    logits = torch.randn(B, V, device="cuda") * 0.7
    temps = torch.full((B,), 0.6, device="cuda")
    out = []
    for name, fn in (("argmax", lambda: ops.argmax(logits)),
                     ("sample_temperature", lambda: ops.sample(logits, temps, None, None, 1234, None))):
        ms = time_kernel(fn)
        gbs = B * V * 4 / ms / 1e6
        out.append({"kernel": name, "B": B, "V": V, "us": round(ms * 1000, 2), "GB/s": round(gbs, 1),
                    "frac_hbm": round(gbs / peaks["hbm_gbs"], 3)})
    return out


def bench_gemm(M: int, N: int, K: int, peaks, label: str) -> Dict:
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ms = time_kernel(lambda: ops.gemm(x, w, out=out))
    ms_cublas = time_kernel(lambda: torch.matmul(x, w.t(), out=out))
    ms_graph = time_graph(lambda: ops.gemm(x, w, out=out), iters=50)
    ms_cublas_graph = time_graph(lambda: torch.matmul(x, w.t(), out=out), iters=50)
    flops = 2 * M * N * K
    nbytes = 2 * (M * K + N * K + M * N)
    tf, gbs = flops / ms / 1e9, nbytes / ms / 1e6
    bound = max(flops / (peaks["tflops"] * 1e9), nbytes / (peaks["hbm_gbs"] * 1e6))  # roofline ms
    row = {"kernel": f"gemm[{label}]", "M": M, "N": N, "K": K, "ms": round(ms, 4), "cublas_ms": round(ms_cublas, 4),
           "graph_ms": round(ms_graph, 4), "cublas_graph_ms": round(ms_cublas_graph, 4),
           "TFLOP/s": round(tf, 1), "GB/s": round(gbs, 1), "frac_roofline": round(bound / ms, 3)}
    if M >= 128 and K % 64 == 0:
        # persistent tiles (plan mode 3), both N tiles
        nat = ops.native()
        for bn in (256, 128):
            t = time_kernel(lambda bn=bn: nat.gemm(out, x, w, None, None, 1, 3, None, bn))
            row[f"persistent{bn}_ms"] = round(t, 4)
            row[f"persistent{bn}_frac_roofline"] = round(bound / t, 3)
    return row


def _cycle_ms(run, ws: List[torch.Tensor], reps: int = 24) -> float:
    """Mean ms of ``run(w)`` over back-to-back launches in a CUDA graph that
    cycles through weight copies larger than L2 in total (weights stream
    from HBM, as in a decode step); best of three replays."""
    run(ws[0])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            run(ws[i % len(ws)])
    best = float("inf")
    for _ in range(3):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e) / reps)
    del g
    return best


def bench_gemm_cold(M: int, N: int, K: int, peaks, label: str) -> Dict:
    """Our GEMM with its autotuned plan vs cuBLAS, weights cold (copies
    cycled beyond L2), back to back in a CUDA graph."""
    from minisgl.ops import gemm_tune

    dev = torch.device("cuda")
    gemm_tune.tune([(N, K)], [M], dev)
    w = torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02
    copies = max(1, min(16, -(-(256 << 20) // w.nbytes)))
    ws = [w] + [w.clone() for _ in range(copies - 1)]
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    ms = _cycle_ms(lambda w_: ops.gemm(x, w_, out=out), ws)
    ms_cublas = _cycle_ms(lambda w_: torch.matmul(x, w_.t(), out=out), ws)
    # the CTA-pair persistent plan, timed on its own for comparison
    ms_pair = None
    if M >= 256 and K % 64 == 0:
        ms_pair = _cycle_ms(lambda w_: gemm_tune.run_plan(out, x, w_, (ops.GEMM_PAIR, 256, 1)), ws)
    flops, nbytes = 2 * M * N * K, 2 * (M * K + N * K + M * N)
    bound = max(flops / (peaks["tflops"] * 1e9), nbytes / (peaks["hbm_gbs"] * 1e6))
    return {"kernel": f"gemm_cold[{label}]", "M": M, "N": N, "K": K, "plan": gemm_tune.lookup(M, N, K),
            "ms": round(ms, 4), "cublas_ms": round(ms_cublas, 4), "vs_cublas": round(ms_cublas / ms, 3),
            "pair_ms": None if ms_pair is None else round(ms_pair, 4),
            "GB/s": round(nbytes / ms / 1e6, 1), "TFLOP/s": round(flops / ms / 1e9, 1),
            "frac_roofline": round(bound / ms, 3), "cublas_frac_roofline": round(bound / ms_cublas, 3)}


def long_gemm_variants(M: int, N: int, K: int) -> Dict:
    """Prefill-sized GEMM: the persistent one-SM plan (3, 256, 1), the
    CTA-pair plan (5, 256, 1) and cuBLAS, each timed back to back in a CUDA
    graph over two weight copies (best of three replays), then each launched
    once inside the NVTX range 'measure'."""
    import os

    from minisgl.ops import gemm_tune

    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(2)]
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    runs = {"persistent": lambda w: gemm_tune.run_plan(out, x, w, (3, 256, 1)),
            "pair": lambda w: gemm_tune.run_plan(out, x, w, (ops.GEMM_PAIR, 256, 1)),
            "cublas": lambda w: torch.matmul(x, w.t(), out=out)}
    res: Dict = {"M": M, "N": N, "K": K, "debug": os.environ.get("MINISGL_GEMM_DEBUG", "0"),
                 "prefetch": os.environ.get("MINISGL_GEMM_PREFETCH", "0")}
    for name, run in runs.items():
        ms = _cycle_ms(run, ws, reps=10)
        res[f"{name}_ms"] = round(ms, 4)
        res[f"{name}_tflops"] = round(2 * M * N * K / ms / 1e9, 1)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("measure")
    for run in runs.values():
        run(ws[0])
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    return res


def bench_layer_chain(M: int, peaks, layers: int = 28) -> List[Dict]:
    """The non-attention kernels of one Qwen3-0.6B decode layer (tp1) at M
    tokens, per layer, over ``layers`` weight copies (~0.9 GB, so weights
    stream from HBM), in a CUDA graph: the fused chain (4 GEMMs with norm /
    RoPE / SiLU / residual epilogues) against the unfused one (norms, RoPE +
    KV store and activation as separate kernels). Attention is left out; a
    fixed tensor stands in for its output."""
    from minisgl.ops import gemm_tune

    H, I, hq, hk, d, page = 1024, 3072, 16, 8, 128, 64
    dev = torch.device("cuda")
    nqkv = (hq + 2 * hk) * d
    gemm_tune.tune([(nqkv, H), (H, hq * d), (2 * I, H), (H, I)], [M], dev, fused={
        (nqkv, H): (ops.EPI_NORM | ops.EPI_ROPE, hq, hk), (H, hq * d): (ops.EPI_RESIDUAL, hq, hk),
        (2 * I, H): (ops.EPI_NORM | ops.EPI_SILU, hq, hk), (H, I): (ops.EPI_RESIDUAL, hq, hk)})
    W = [dict(qkv=torch.randn(nqkv, H, device=dev, dtype=torch.bfloat16) * 0.02,
              o=torch.randn(H, hq * d, device=dev, dtype=torch.bfloat16) * 0.02,
              gu=torch.randn(2 * I, H, device=dev, dtype=torch.bfloat16) * 0.02,
              down=torch.randn(H, I, device=dev, dtype=torch.bfloat16) * 0.02) for _ in range(layers)]
    r = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
    x = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
    attn = torch.randn(M, hq * d, device=dev, dtype=torch.bfloat16)
    pages = (M + page - 1) // page + 1
    kc = torch.zeros(pages, hk, page, d, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    positions = torch.arange(M, device=dev, dtype=torch.int32)
    out_loc = torch.arange(M, device=dev, dtype=torch.int32)
    ang = torch.rand(4096, 64, device=dev) * 6
    cos_sin = torch.cat([ang.cos(), ang.sin()], dim=1).contiguous()
    rope = dict(positions=positions, cos_sin=cos_sin, out_loc=out_loc, q_norm_w=None, k_norm_w=None,
                head_eps=1e-6, k_cache=kc, v_cache=vc, hq=hq, hk=hk, page_size=page)
    q = torch.empty(M, hq * d, device=dev, dtype=torch.bfloat16)
    h = torch.empty(M, I, device=dev, dtype=torch.bfloat16)

    def fused():
        for w in W:
            ops.gemm_fused(r, w["qkv"], norm_eps=1e-6, rope=rope, out=q)
            ops.gemm_fused(attn, w["o"], residual=r, out=r)
            ops.gemm_fused(r, w["gu"], norm_eps=1e-6, silu=True, out=h)
            ops.gemm_fused(h, w["down"], residual=r, out=r)

    def unfused():
        y = x
        for w in W:
            ops.fused_add_rmsnorm(y, r, None, 1e-6)
            qkv = ops.gemm(y, w["qkv"])
            ops.rope_store(qkv, positions, cos_sin, None, None, kc, vc, out_loc, hq, hk, d, page, 1e-6)
            o = ops.gemm(attn, w["o"])
            ops.fused_add_rmsnorm(o, r, None, 1e-6)
            a = ops.silu_and_mul(ops.gemm(o, w["gu"]), interleaved=True)
            y = ops.gemm(a, w["down"])

    out = []
    wbytes = sum(t.numel() * 2 for t in W[0].values())
    for name, fn in (("fused", fused), ("unfused", unfused)):
        ms = time_graph(fn, iters=3) / layers
        out.append({"kernel": f"layer_chain[{name}]", "M": M, "us_per_layer": round(ms * 1000, 2),
                    "weight_GB/s": round(wbytes / ms / 1e6, 1), "frac_hbm": round(wbytes / ms / 1e6 / peaks["hbm_gbs"], 3),
                    "fused_plans": [gemm_tune.FUSED_PLANS.get((M, n, k)) for n, k in
                                    ((nqkv, H), (H, hq * d), (2 * I, H), (H, I))] if name == "fused" else
                    [gemm_tune.PLANS.get((M, n, k)) for n, k in ((nqkv, H), (H, hq * d), (2 * I, H), (H, I))]})
    return out


def bench_row_kernels(M: int, peaks) -> List[Dict]:
    """The decode-sized row kernels (M tokens of Qwen3-0.6B) back to back in a
    CUDA graph: what one launch costs inside a chain."""
    H, I, hq, hk, d, page = 1024, 3072, 16, 8, 128, 64
    dev = torch.device("cuda")
    x = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
    r = torch.randn_like(x)
    gu = torch.randn(M, 2 * I, device=dev, dtype=torch.bfloat16)
    qkv = torch.randn(M, (hq + 2 * hk) * d, device=dev, dtype=torch.bfloat16)
    kc = torch.zeros((M + page - 1) // page + 1, hk, page, d, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    pos = torch.arange(M, device=dev, dtype=torch.int32)
    ang = torch.rand(4096, 64, device=dev) * 6
    cs = torch.cat([ang.cos(), ang.sin()], 1).contiguous()
    out = []
    for name, fn in (("fused_add_rmsnorm", lambda: ops.fused_add_rmsnorm(x, r, None, 1e-6)),
                     ("rmsnorm", lambda: ops.rmsnorm(x, None, 1e-6)),
                     ("silu_and_mul", lambda: ops.silu_and_mul(gu, interleaved=True)),
                     ("rope_store", lambda: ops.rope_store(qkv, pos, cs, None, None, kc, vc, pos, hq, hk, d, page,
                                                           1e-6))):
        ms = time_graph(fn, iters=200)
        out.append({"kernel": f"chain[{name}]", "M": M, "us": round(ms * 1000, 2)})
    return out


def bench_elementwise(peaks) -> List[Dict]:
    out = []
    T, H = 16384, 1024
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
    ms = time_kernel(lambda: ops.fused_add_rmsnorm(x, r, w, 1e-6))
    gbs = 4 * T * H * 2 / ms / 1e6
    out.append({"kernel": "fused_add_rmsnorm", "T": T, "H": H, "ms": round(ms, 4), "GB/s": round(gbs, 1),
                "frac_hbm": round(gbs / peaks["hbm_gbs"], 3)})
    gu = torch.randn(T, 2 * 3072, device="cuda", dtype=torch.bfloat16)
    ms = time_kernel(lambda: ops.silu_and_mul(gu))
    gbs = 3 * T * 3072 * 2 / ms / 1e6
    out.append({"kernel": "silu_and_mul", "T": T, "I": 3072, "ms": round(ms, 4), "GB/s": round(gbs, 1),
                "frac_hbm": round(gbs / peaks["hbm_gbs"], 3)})
    logits = torch.randn(256, 151936, device="cuda")
    t = torch.full((256,), 0.6, device="cuda")
    ms = time_kernel(lambda: ops.sample(logits, t))
    gbs = logits.numel() * 4 / ms / 1e6
    out.append({"kernel": "sample(temperature)", "B": 256, "V": 151936, "ms": round(ms, 4), "GB/s": round(gbs, 1),
                "frac_hbm": round(gbs / peaks["hbm_gbs"], 3)})
    return out


def _quantiles(v: torch.Tensor) -> str:
    v = v.sort().values
    return f"min {v[0]:.2f} med {v[len(v) // 2]:.2f} max {v[-1]:.2f}"


def probe_plan(M: int, N: int, K: int, mode: int, bn: int, splits: int, kps: int = 0, trace: bool = False,
               iters: int = 40) -> Dict:
    """Mean microseconds per launch of one forced tile plan (and, with
    ``trace``, the phase stamps of one more launch, as quantiles over CTAs)."""
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(8)]
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    nat = ops.native()

    scratch = ops.streamk_workspace(x.device) if mode == ops.GEMM_STREAMK else None

    def run(w, tr=None):
        nat.gemm(out, x, w, None, scratch, splits, mode, None, bn, tr, kps)

    for i in range(8):
        run(ws[i % 8])
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        run(ws[i % 8])
    e.record()
    torch.cuda.synchronize()
    row: Dict = {"M": M, "N": N, "K": K, "plan": [mode, bn, splits], "kps": kps,
                 "us_per_launch": round(s.elapsed_time(e) / iters * 1000, 2)}
    if trace:
        # stamps of the last of 16 back-to-back launches (each launch
        # overwrites the buffer), so the overlap with its predecessor shows
        tr = torch.zeros(1 << 16, dtype=torch.int64, device="cuda")
        for i in range(16):
            run(ws[i % 8], tr)
        torch.cuda.synchronize()
        t = tr.view(-1, 8).cpu()
        t = t[t[:, 0] > 0].double()
        rel = (t - t[:, 0].min()) / 1000.0
        if mode == ops.GEMM_STREAMK:
            last = torch.where(t[:, 4] > 0, rel[:, 4], rel[:, 3])
            own = t[:, 5] > 0
            row.update({"ctas": len(t), "entry": _quantiles(rel[:, 0]), "set-up": _quantiles(rel[:, 1] - rel[:, 0]),
                        "producer past wait": _quantiles(rel[:, 2]), "first acc ready": _quantiles(rel[:, 3]),
                        "last acc ready": _quantiles(last),
                        "owner waits": _quantiles(rel[own, 5] - last[own]) if bool(own.any()) else "none",
                        "epilogue after last acc": _quantiles(rel[:, 6] - last), "exit": _quantiles(rel[:, 6])})
            return row
        row.update({"ctas": len(t), "entry": _quantiles(rel[:, 0]), "set-up": _quantiles(rel[:, 1] - rel[:, 0]),
                    "producer past wait": _quantiles(rel[:, 2]),
                    "first stage after wait": _quantiles(rel[:, 3] - rel[:, 2]),
                    "mainloop": _quantiles(rel[:, 4] - rel[:, 3]), "epilogue": _quantiles(rel[:, 5] - rel[:, 4]),
                    "exit": _quantiles(rel[:, 5])})
    return row


def probe_launch_modes(M: int, N: int, K: int, mode: int, bn: int, splits: int, kps: int = 0) -> Dict:
    """Microseconds per launch of one forced plan, launched eagerly and
    from a CUDA graph (one weight, and 8 weight copies cycled beyond L2), and
    the device error word afterwards: separates host launch cost, kernel time
    and inter-launch effects."""
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(8)]
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    nat = ops.native()
    scratch = ops.streamk_workspace(x.device) if mode == ops.GEMM_STREAMK else None
    err = ops.error_word(x.device)

    def run(w):
        nat.gemm(out, x, w, None, scratch, splits, mode, err, bn, None, kps)

    def eager(n=40):
        for i in range(8):
            run(ws[i % 8])
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(n):
            run(ws[i % 8])
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / n * 1000

    def graph(copies, n=40):
        g = torch.cuda.CUDAGraph()
        run(ws[0])
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            for i in range(n):
                run(ws[i % copies])
        g.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        torch.cuda.synchronize()
        del g
        return s.elapsed_time(e) / n * 1000

    row = {"M": M, "N": N, "K": K, "plan": [mode, bn, splits], "eager_us": round(eager(), 2),
           "graph_1copy_us": round(graph(1), 2), "graph_8copies_us": round(graph(8), 2)}
    row["error_word"] = err.tolist()
    return row


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--launch-modes", default="", help="M,N,K,mode,bn,splits[,kps]: eager vs graph launch timing")
    p.add_argument("--probe", default="", help="M,N,K,mode,bn,splits[,kps]: time one forced GEMM tile plan")
    p.add_argument("--trace", action="store_true", help="with --probe: per-CTA phase stamps")
    p.add_argument("--long-gemms", default="", help="M,N,K: the persistent one-SM and CTA-pair plans and cuBLAS, "
                   "timed; each launched once more inside an NVTX range 'measure' (for an ncu --nvtx-include "
                   "capture). MINISGL_GEMM_DEBUG / MINISGL_GEMM_PREFETCH select the kernels' measurement switches")
    p.add_argument("--json", default="")
    p.add_argument("--quick", action="store_true")
    p.add_argument("--only", default="", help="run only cases whose label contains this text")
    p.add_argument("--trace-prefill", action="store_true", help="print the prefill attention phase trace and exit")
    args = p.parse_args()
    if args.launch_modes:
        vals = [int(v) for v in args.launch_modes.split(",")]
        print(json.dumps(probe_launch_modes(*vals[:7])), flush=True)
        return
    if args.long_gemms:
        M, N, K = (int(v) for v in args.long_gemms.split(","))
        print(json.dumps(long_gemm_variants(M, N, K)), flush=True)
        return
    if args.probe:
        vals = [int(v) for v in args.probe.split(",")]
        print(json.dumps(probe_plan(*vals[:7], trace=args.trace)), flush=True)
        return
    if args.trace_prefill:
        print(json.dumps(trace_prefill_attention()), flush=True)
        return
    peaks = _peaks()
    random.seed(0)
    torch.manual_seed(0)
    cases = []
    for B, L in [(256, 800), (128, 800), (32, 2000), (1, 4000)]:
        cases.append((f"decode_attention B={B} L={L}", lambda B=B, L=L: bench_decode_attention(B, L, 16, 8, 64, peaks)))
    for B, lo, hi in [(256, 200, 2000), (64, 200, 2000), (8, 500, 4000), (1, 4000, 4000)]:
        cases.append((f"decode_attention varlen B={B}",
                      lambda B=B, lo=lo, hi=hi: bench_decode_attention_varlen(B, lo, hi, 16, 8, 64, peaks)))
    cases.append(("decode_attention qwen3-32b", lambda: bench_decode_attention(64, 2000, 64, 8, 64, peaks)))
    for B, L in [(8, 2048), (2, 8192), (1, 16384)]:
        cases.append((f"prefill_attention qwen3-32b B={B} L={L}",
                      lambda B=B, L=L: bench_prefill_attention(B, L, 64, 8, 64, peaks)))
    cases.append(("decode_attention qwen3-32b tp8", lambda: bench_decode_attention(64, 2000, 8, 1, 64, peaks)))
    for B, L, hq, hk in [(16, 1024, 16, 8), (4, 4096, 16, 8), (1, 16384, 16, 8), (2, 4096, 64, 8)]:
        cases.append((f"prefill_attention B={B} L={L} hq={hq}",
                      lambda B=B, L=L, hq=hq, hk=hk: bench_prefill_attention(B, L, hq, hk, 64, peaks)))
    for B, L, Hh in [(256, 1024, 64), (128, 2048, 64), (64, 4096, 64), (8, 4096, 64), (1, 8192, 64), (32, 4096, 16),
                     (64, 2048, 128)]:
        cases.append((f"mla_decode B={B} L={L} H={Hh}",
                      lambda B=B, L=L, Hh=Hh: bench_mla_decode(B, L, Hh, 64, peaks)))
    for B, L in ((1, 4096), (1, 16384), (4, 2048)):
        cases.append((f"mla_prefill B={B} L={L}", lambda B=B, L=L: bench_mla_prefill(B, L, 64, peaks)))
    H, I, V = 1024, 3072, 151936
    for M in (1, 64, 256):
        for lab, N, K in (("qkv", 4096, H), ("o", H, 2048), ("gate_up", 2 * I, H), ("down", H, I)):
            name = f"{lab} M={M}"
            cases.append((f"gemm[{name}]", lambda M=M, N=N, K=K, name=name: bench_gemm(M, N, K, peaks, name)))
    cases.append(("gemm[lm_head M=256]", lambda: bench_gemm(256, V, H, peaks, "lm_head M=256")))
    cases.append(("gemm[gate_up prefill]", lambda: bench_gemm(16384, 2 * I, H, peaks, "gate_up prefill")))
    cases.append(("gemm[square 8192]", lambda: bench_gemm(8192, 8192, 8192, peaks, "square 8192")))
    for lab, N, K in (("qkv", 4096, H), ("o", H, 2048), ("down", H, I)):
        cases.append((f"gemm[{lab} prefill]", lambda N=N, K=K, lab=lab: bench_gemm(16384, N, K, peaks,
                                                                                 f"{lab} prefill")))
    cases.append(("elementwise", lambda: bench_elementwise(peaks)))
    # Qwen3-32B projections at TP1 / 2 / 4 / 8, decode batch sizes and a prefill chunk
    H32, I32, d = 5120, 25600, 128
    for tp in (1, 2, 4, 8):
        for lab, N, K in (("qkv", (64 + 16) * d // tp, H32), ("o", H32, 64 * d // tp),
                          ("gate_up", 2 * I32 // tp, H32), ("down", H32, I32 // tp)):
            for M in (1, 32, 128, 256, 8192):
                name = f"32b tp{tp} {lab} M={M}"
                cases.append((f"gemm32b[{name}]", lambda M=M, N=N, K=K, name=name: bench_gemm_cold(M, N, K, peaks,
                                                                                                  name)))
    for T in (16, 256):
        cases.append((f"moe_mxfp4 T={T}", lambda T=T: bench_moe_mxfp4(T, 16, 8, 7168, 2048, peaks)))
    for M in (1, 8, 32, 64, 128, 192, 256):
        cases.append((f"layer_chain M={M};", lambda M=M: bench_layer_chain(M, peaks)))
    cases.append(("rowkernels M=256", lambda: bench_row_kernels(256, peaks)))
    for B in (64, 256):
        cases.append((f"sample B={B}", lambda B=B: bench_sample(B, 151936, peaks)))
    # the block-scaled MX expert path last (the newest kernels), its quantiser first
    for P, tile in ((2048, 16), (16384, 128)):
        cases.append((f"mx8_quantize P={P}", lambda P=P, tile=tile: bench_mx8_quantize(P, 7168, tile, peaks)))
    for T in (16, 256):
        cases.append((f"moe_mx T={T}", lambda T=T: bench_moe_mx(T, 16, 8, 7168, 2048, peaks)))
    rows: List[Dict] = []
    clocks = SmClockLog(torch.cuda.current_device()).start()
    for label, fn in cases:
        if args.only and args.only not in label:
            continue
        r = fn()
        rows.extend(r if isinstance(r, list) else [r])
    clock_summary = clocks.stop()
    for r in rows:
        r["peaks"] = peaks["source"]
        print(json.dumps(r), flush=True)
    # SM clocks over the whole run, to read the timings above against
    print(json.dumps(clock_summary), flush=True)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
