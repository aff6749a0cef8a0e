"""Plain-PyTorch restatement of every native op (fp32 math).

This is the CPU oracle: the CPU engine path runs on it, and the GPU kernel
tests compare the sm_100a kernels against it. Semantics (layouts, rounding
points, masking) match the CUDA kernels in ``minisgl/csrc``.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch


def gemm(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], out_dtype: torch.dtype) -> torch.Tensor:
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(out_dtype)


def rmsnorm(x: torch.Tensor, w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = xf * inv if w is None else xf * inv * w.float()
    return y.to(x.dtype)


def silu_mul_interleaved(h: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up for gate|up rows interleaved in blocks of 64 columns."""
    M, N = h.shape
    hv = h.float().view(M, N // 128, 2, 64)
    g, u = hv[:, :, 0], hv[:, :, 1]
    return (torch.nn.functional.silu(g) * u).reshape(M, N // 2).to(h.dtype)


def gemm_fused(
    x: torch.Tensor,
    w: torch.Tensor,
    bias: Optional[torch.Tensor],
    norm_eps: Optional[float],
    residual: Optional[torch.Tensor],
    silu: bool,
    rope: Optional[dict],
) -> torch.Tensor:
    """The fused decode GEMM: optional row RMSNorm of x (weight folded into
    w), bias, then one of silu(gate) * up (interleaved rows), residual add,
    or q/k-norm + RoPE + KV store (returns the qkv rows, q heads rotated)."""
    y = x.float() @ w.float().t()
    if norm_eps is not None:
        xf = x.float()
        y = y * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + norm_eps)
    if bias is not None:
        y = y + bias.float()
    y = y.to(x.dtype)
    if silu:
        return silu_mul_interleaved(y)
    if residual is not None:
        return (y.float() + residual.float()).to(x.dtype)
    if rope is not None:
        rope_store(y, rope["positions"], rope["cos_sin"], rope.get("q_norm_w"), rope.get("k_norm_w"),
                   rope["k_cache"], rope["v_cache"], rope["out_loc"], rope["hq"], rope["hk"], 128,
                   rope["page_size"], rope["head_eps"])
    return y


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: Optional[torch.Tensor], eps: float) -> None:
    s = (x.float() + residual.float()).to(x.dtype)
    residual.copy_(s)
    x.copy_(rmsnorm(s, w, eps))


def act_and_mul(x: torch.Tensor, act: str) -> torch.Tensor:
    d = x.shape[-1] // 2
    g, u = x[..., :d].float(), x[..., d:].float()
    if act == "silu":
        a = g / (1.0 + torch.exp(-g))
    elif act == "gelu":
        a = 0.5 * g * (1.0 + torch.erf(g / math.sqrt(2.0)))
    else:
        raise ValueError(f"unsupported activation {act}")
    return (a * u).to(x.dtype)


def embedding(ids: torch.Tensor, weight: torch.Tensor, lo: int, n: int) -> torch.Tensor:
    local = ids.long() - lo
    inside = (local >= 0) & (local < n)
    out = weight[local.clamp(0, max(n - 1, 0))]
    return torch.where(inside.unsqueeze(-1), out, torch.zeros_like(out))


def rope_store(
    qkv: torch.Tensor,
    positions: torch.Tensor,
    cos_sin: torch.Tensor,
    q_norm_w: Optional[torch.Tensor],
    k_norm_w: Optional[torch.Tensor],
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    out_loc: torch.Tensor,
    hq: int,
    hk: int,
    d: int,
    page_size: int,
    eps: float,
) -> None:
    """q/k per-head RMSNorm + NeoX RoPE in place in ``qkv``; k/v stored to the
    paged cache (per-layer layout [pages, hk, page_size, d])."""
    T = qkv.shape[0]
    dt = qkv.dtype
    q = qkv[:, : hq * d].view(T, hq, d)
    k = qkv[:, hq * d : (hq + hk) * d].view(T, hk, d)
    v = qkv[:, (hq + hk) * d : (hq + 2 * hk) * d].view(T, hk, d)

    def norm_rope(x: torch.Tensor, w: Optional[torch.Tensor]) -> torch.Tensor:
        xf = x.float()
        if w is not None:
            xf = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(dt).float()
        cs = cos_sin[positions.long()]  # [T, d]
        h = d // 2
        cos, sin = cs[:, None, :h], cs[:, None, h:]
        x1, x2 = xf[..., :h], xf[..., h:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(dt)

    q.copy_(norm_rope(q, q_norm_w))
    k.copy_(norm_rope(k, k_norm_w))
    loc = out_loc.long()
    page, off = loc // page_size, loc % page_size
    k_cache[page, :, off] = k
    v_cache[page, :, off] = v


def gather_kv(
    kv_pool: torch.Tensor, layer: int, page_table: torch.Tensor, row: int, length: int, page_size: int
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Keys/values [length, hk, d] of one request from the paged pool."""
    slots = page_table[row, :length].long()
    page, off = slots // page_size, slots % page_size
    k = kv_pool[0, layer][page, :, off]
    v = kv_pool[1, layer][page, :, off]
    return k, v


def attention(
    q: torch.Tensor,  # [T, hq, d]
    kv_pool: torch.Tensor,
    layer: int,
    page_table: torch.Tensor,
    req_rows: torch.Tensor,
    seq_lens: torch.Tensor,
    cu_q: torch.Tensor,
    hq: int,
    hk: int,
    d: int,
    page_size: int,
    scale: float,
) -> torch.Tensor:
    """Causal paged attention: query i of request b sits at position
    seq_len_b - q_len_b + i and sees keys [0, position]."""
    out = torch.zeros(q.shape[0], hq, d, dtype=q.dtype, device=q.device)
    G = hq // hk
    rows = req_rows.tolist()
    lens = seq_lens.tolist()
    cu = cu_q.tolist()
    for b, (row, L) in enumerate(zip(rows, lens)):
        s, e = cu[b], cu[b + 1]
        n = e - s
        if n == 0 or L <= 0:
            continue
        k, v = gather_kv(kv_pool, layer, page_table, row, L, page_size)
        qb = q[s:e].float()  # [n, hq, d]
        kf = k.float().repeat_interleave(G, dim=1)  # [L, hq, d]
        vf = v.float().repeat_interleave(G, dim=1)
        scores = torch.einsum("nhd,lhd->hnl", qb, kf) * scale
        qpos = torch.arange(L - n, L, device=q.device)
        kpos = torch.arange(L, device=q.device)
        mask = kpos[None, :] > qpos[:, None]
        scores = scores.masked_fill(mask[None], float("-inf"))
        p = torch.softmax(scores, dim=-1)
        out[s:e] = torch.einsum("hnl,lhd->nhd", p, vf).to(q.dtype)
    return out


def rope_interleaved(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """DeepSeek (GPT-J) rotary embedding: pairs (2i, 2i + 1) rotate by
    frequency i. x [T, ..., d]; cos_sin [max_pos, d] = d/2 cos then d/2 sin."""
    d = x.shape[-1]
    cs = cos_sin[positions.long()].float()
    shape = (x.shape[0],) + (1,) * (x.dim() - 2) + (d // 2,)
    c, s = cs[:, : d // 2].reshape(shape), cs[:, d // 2 :].reshape(shape)
    xf = x.float()
    even, odd = xf[..., 0::2], xf[..., 1::2]
    out = torch.empty_like(xf)
    out[..., 0::2] = even * c - odd * s
    out[..., 1::2] = odd * c + even * s
    return out.to(x.dtype)


CP_TILE = 64  # keys per context-parallel ownership unit: tile t belongs to rank t % cp


def cp_owned(positions: torch.Tensor, cp_size: int, cp_rank: int) -> torch.Tensor:
    """Which key positions this context-parallel rank holds."""
    return (positions.long() // CP_TILE) % cp_size == cp_rank


def mla_store_latent(kv_a: torch.Tensor, norm_w: torch.Tensor, eps: float, positions: torch.Tensor,
                     cos_sin: torch.Tensor, latent: torch.Tensor, out_loc: torch.Tensor, page_size: int,
                     cp_size: int = 1, cp_rank: int = 0) -> None:
    """Latent row [rmsnorm(c_kv) | rope(k_pe)] of every token into the paged
    cache; under context parallelism only the rows of this rank's 64-key
    tiles, at local page (global page) // cp."""
    kv_lora = norm_w.shape[0]
    c = rmsnorm(kv_a[:, :kv_lora], norm_w, eps)
    k_pe = rope_interleaved(kv_a[:, kv_lora:], positions, cos_sin)
    loc = out_loc.long()
    rows = torch.cat([c, k_pe], dim=-1).to(latent.dtype)
    page = loc // page_size
    if cp_size > 1:
        keep = cp_owned(positions, cp_size, cp_rank)
        loc, rows, page = loc[keep], rows[keep], page[keep] // cp_size
    latent[page, loc % page_size] = rows


def mla_prepare_q(q: torch.Tensor, w_uk_t: torch.Tensor, positions: torch.Tensor,
                  cos_sin: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Absorbed queries (q_lat [H, T, kv_lora] = q_nope W_UK per head,
    head-major; q_pe [T, H, rope] rotated). w_uk_t is [H, kv_lora, nope]
    (W_UK of each head, transposed)."""
    nope = w_uk_t.shape[2]
    q_pe = rope_interleaved(q[..., nope:], positions, cos_sin).contiguous()
    q_lat = torch.einsum("thn,hcn->htc", q[..., :nope].float(), w_uk_t.float()).to(q.dtype)
    return q_lat, q_pe


def mla_prepare(q: torch.Tensor, kv_a: torch.Tensor, w_uk_t: torch.Tensor, norm_w: torch.Tensor, eps: float,
                positions: torch.Tensor, cos_sin: torch.Tensor, latent: torch.Tensor, out_loc: torch.Tensor,
                page_size: int, cp_size: int = 1, cp_rank: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Both halves for one token set: the cache rows, then the queries."""
    mla_store_latent(kv_a, norm_w, eps, positions, cos_sin, latent, out_loc, page_size, cp_size, cp_rank)
    return mla_prepare_q(q, w_uk_t, positions, cos_sin)


def mla_rope_q(q: torch.Tensor, rope: int, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """The rotated rope part [T, H, rope] of q [T, H, nope + rope]."""
    return rope_interleaved(q[..., q.shape[-1] - rope:], positions, cos_sin).contiguous()


def mla_prefill_attention(q: torch.Tensor, q_rope: torch.Tensor, latent: torch.Tensor, page_table: torch.Tensor,
                          req_rows: torch.Tensor, seq_lens: torch.Tensor, cu_q: torch.Tensor, w_kv_b: torch.Tensor,
                          kv_lora: int, nope: int, v_dim: int, page_size: int, scale: float) -> torch.Tensor:
    """Non-absorbed causal MLA for prefill: every key's c_kv goes through
    kv_b_proj (w_kv_b [H * (nope + v), kv_lora], per head nope rows then v
    rows) into per-head k_nope / v; scores are q_nope . k_nope + q_rope .
    k_rope (the key's cached, rotated rope part, shared by the heads);
    returns [T, H * v] in q's dtype (fp32 math)."""
    T, H, qk = q.shape
    rope = qk - nope
    out = torch.zeros(T, H, v_dim, dtype=torch.float32, device=q.device)
    w = w_kv_b.float().view(H, nope + v_dim, kv_lora)
    flat = latent.reshape(-1, latent.shape[-1])
    rows, lens, cu = req_rows.tolist(), seq_lens.tolist(), cu_q.tolist()
    for b, (row, L) in enumerate(zip(rows, lens)):
        s, e = cu[b], cu[b + 1]
        n = e - s
        if n == 0 or L <= 0:
            continue
        kv = flat[page_table[row, :L].long()].float()               # [L, kv_lora + rope]
        k_nope = torch.einsum("lc,hnc->lhn", kv[:, :kv_lora], w[:, :nope])
        v = torch.einsum("lc,hvc->lhv", kv[:, :kv_lora], w[:, nope:])
        k_rope = kv[:, kv_lora:kv_lora + rope]
        qb = q[s:e].float()
        scores = (torch.einsum("nhd,lhd->hnl", qb[..., :nope], k_nope)
                  + torch.einsum("nhd,ld->hnl", q_rope[s:e].float(), k_rope)) * scale
        qpos = torch.arange(L - n, L, device=q.device)
        mask = torch.arange(L, device=q.device)[None, :] > qpos[:, None]
        p = torch.softmax(scores.masked_fill(mask[None], float("-inf")), dim=-1)
        out[s:e] = torch.einsum("hnl,lhv->nhv", p, v)
    return out.reshape(T, H * v_dim).to(q.dtype)


def mla_output(o_lat: torch.Tensor, w_uv: torch.Tensor, T: int, row_map: Optional[torch.Tensor] = None,
               out_rows: Optional[int] = None) -> torch.Tensor:
    """Latent attention output back to heads: o_lat [H, >= T, kv_lora] x
    W_UV [H, v, kv_lora] -> [T, H * v]; with a row map, token t goes to row
    row_map[t] of [out_rows, H * v] (other rows zero)."""
    o = torch.einsum("htc,hvc->thv", o_lat[:, :T].float(), w_uv.float())
    o = o.reshape(T, -1).to(o_lat.dtype)
    if row_map is None:
        return o
    out = torch.zeros(out_rows, o.shape[1], dtype=o.dtype, device=o.device)
    out[row_map.long()] = o
    return out


def mla_share(o_own: torch.Tensor, lse_all: torch.Tensor, rank: int) -> torch.Tensor:
    """This context-parallel rank's share of the merged attention output:
    its own partial o_own [T, H, C] weighted by exp(lse_rank - lse_total),
    where lse_all [R, T, H] holds every rank's log-sum-exp. The shares of
    all ranks sum to the merged output."""
    m = lse_all.amax(dim=0)
    fin = torch.isfinite(m)
    m0 = torch.where(fin, m, torch.zeros_like(m))
    w = torch.where(torch.isfinite(lse_all), torch.exp(lse_all - m0), torch.zeros_like(lse_all))
    share = o_own * (w[rank] / w.sum(0).clamp_min(1e-30))[..., None]
    return share.transpose(0, 1)


def mla_attention_partial(q_lat: torch.Tensor, q_pe: torch.Tensor, latent: torch.Tensor, page_table: torch.Tensor,
                          req_rows: torch.Tensor, seq_lens: torch.Tensor, cu_q: torch.Tensor, page_size: int,
                          scale: float, cp_size: int, cp_rank: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Causal absorbed MLA over the keys this context-parallel rank holds:
    (o [T, H, kv_lora] normalised over those keys, lse [T, H] natural log;
    -inf and zeros where the rank holds none of a token's keys)."""
    T, H, _ = q_pe.shape
    kv_lora = q_lat.shape[2]
    q = torch.cat([q_lat[:, :T].transpose(0, 1), q_pe], dim=-1).float()
    D = q.shape[-1]
    o = torch.zeros(T, H, kv_lora, dtype=torch.float32, device=q.device)
    lse = torch.full((T, H), float("-inf"), dtype=torch.float32, device=q.device)
    rows, lens, cu = req_rows.tolist(), seq_lens.tolist(), cu_q.tolist()
    for b, (row, L) in enumerate(zip(rows, lens)):
        s, e = cu[b], cu[b + 1]
        n = e - s
        if n == 0 or L <= 0:
            continue
        pos = torch.arange(L, device=q.device)
        mine = cp_owned(pos, cp_size, cp_rank)
        if not bool(mine.any()):
            continue
        slots = page_table[row, :L].long()
        local = (slots // page_size // cp_size) * page_size + slots % page_size  # this rank's local page
        kv = latent.reshape(-1, D)[torch.where(mine, local, torch.zeros_like(local))].float()
        scores = torch.einsum("nhd,ld->nhl", q[s:e], kv) * scale
        qpos = torch.arange(L - n, L, device=q.device)
        mask = (pos[None, :] > qpos[:, None]) | ~mine[None, :]
        scores = scores.masked_fill(mask[:, None, :], float("-inf"))
        m = scores.amax(dim=-1, keepdim=True)
        has = torch.isfinite(m)
        p = torch.where(has, torch.exp(scores - torch.where(has, m, torch.zeros_like(m))), torch.zeros_like(scores))
        l = p.sum(-1, keepdim=True)
        o[s:e] = torch.where(has, torch.einsum("nhl,lc->nhc", p, kv[:, :kv_lora]) / l.clamp_min(1e-30), 0.0)
        lse[s:e] = torch.where(has, m + torch.log(l.clamp_min(1e-30)), torch.full_like(m, float("-inf")))[..., 0]
    return o, lse


def merge_partials(o: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
    """o [R, T, H, C], lse [R, T, H] (natural log) -> the softmax-weighted
    merge [T, H, C] over the R parts."""
    m = lse.amax(dim=0, keepdim=True)
    w = torch.where(torch.isfinite(lse), torch.exp(lse - torch.where(torch.isfinite(m), m, torch.zeros_like(m))),
                    torch.zeros_like(lse))
    return (o * w[..., None]).sum(0) / w.sum(0)[..., None].clamp_min(1e-30)


def mla_attention(
    q_lat: torch.Tensor,  # [H, >= T, kv_lora]: absorbed queries, head-major
    q_pe: torch.Tensor,  # [T, H, rope]
    latent: torch.Tensor,  # [pages, page_size, kv_lora + rope] of one layer
    page_table: torch.Tensor,
    req_rows: torch.Tensor,
    seq_lens: torch.Tensor,
    cu_q: torch.Tensor,
    page_size: int,
    scale: float,
) -> torch.Tensor:
    """Causal absorbed multi-head latent attention over the paged latent
    cache: scores = [q_lat | q_pe] . [c_kv | k_pe], output = softmax(scores)
    @ c_kv, returned head-major like q_lat ([H, T, kv_lora], fp32 math)."""
    T, H, _ = q_pe.shape
    kv_lora = q_lat.shape[2]
    q = torch.cat([q_lat[:, :T].transpose(0, 1), q_pe], dim=-1)
    D = q.shape[-1]
    out = torch.zeros(T, H, kv_lora, dtype=q.dtype, device=q.device)
    rows, lens, cu = req_rows.tolist(), seq_lens.tolist(), cu_q.tolist()
    for b, (row, L) in enumerate(zip(rows, lens)):
        s, e = cu[b], cu[b + 1]
        n = e - s
        if n == 0 or L <= 0:
            continue
        slots = page_table[row, :L].long()
        kv = latent.reshape(-1, D)[slots].float()  # [L, D]
        qb = q[s:e].float()  # [n, H, D]
        scores = torch.einsum("nhd,ld->hnl", qb, kv) * scale
        qpos = torch.arange(L - n, L, device=q.device)
        mask = torch.arange(L, device=q.device)[None, :] > qpos[:, None]
        scores = scores.masked_fill(mask[None], float("-inf"))
        p = torch.softmax(scores, dim=-1)
        out[s:e] = torch.einsum("hnl,lc->nhc", p, kv[:, :kv_lora]).to(q.dtype)
    return out.transpose(0, 1).contiguous()


def argmax(logits: torch.Tensor) -> torch.Tensor:
    return torch.argmax(logits.float(), dim=-1).to(torch.int32)


def sample(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: Optional[torch.Tensor],
    top_p: Optional[torch.Tensor],
    generator: Optional[torch.Generator] = None,
) -> torch.Tensor:
    """Multinomial draw from softmax(logits / T) restricted to top-k / top-p."""
    lf = logits.float() / temperature.float().clamp_min(1e-6)[:, None]
    B, V = lf.shape
    keep = torch.ones_like(lf, dtype=torch.bool)
    if top_k is not None:
        k = top_k.long().clamp(1, V)
        kth = torch.sort(lf, dim=-1, descending=True).values.gather(1, (k - 1)[:, None])
        use = (top_k > 0) & (top_k < V)
        keep &= ~use[:, None] | (lf >= kth)
    if top_p is not None:
        masked = lf.masked_fill(~keep, float("-inf"))
        probs = torch.softmax(masked, dim=-1)
        sp, idx = torch.sort(probs, dim=-1, descending=True)
        cum = sp.cumsum(-1)
        # keep the smallest prefix whose mass reaches p
        drop_sorted = (cum - sp) >= top_p.float()[:, None]
        drop = torch.zeros_like(drop_sorted).scatter(1, idx, drop_sorted)
        keep &= ~drop
    probs = torch.softmax(lf.masked_fill(~keep, float("-inf")), dim=-1)
    return torch.multinomial(probs, 1, generator=generator).view(-1).to(torch.int32)


def moe_route(
    logits: torch.Tensor,
    k: int,
    scoring: str,
    renormalize: bool,
    bias: Optional[torch.Tensor] = None,
    n_group: int = 1,
    topk_group: int = 1,
    routed_scale: float = 1.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    lf = logits.float()
    if scoring == "softmax":
        scores = torch.softmax(lf, dim=-1)
        choice = scores
    else:
        scores = torch.sigmoid(lf)
        choice = scores + (bias.float() if bias is not None else 0.0)
        if n_group > 1 and topk_group < n_group:
            T, E = choice.shape
            g = choice.view(T, n_group, E // n_group)
            gs = g.topk(2, dim=-1).values.sum(-1)
            keep = torch.zeros_like(gs, dtype=torch.bool).scatter(1, gs.topk(topk_group, dim=-1).indices, True)
            choice = g.masked_fill(~keep[..., None], float("-inf")).view(T, E)
    ids = choice.topk(k, dim=-1).indices
    w = scores.gather(1, ids)
    if renormalize:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return (w * routed_scale).float(), ids.to(torch.int32)


def fast_compare_key(a: torch.Tensor, b: torch.Tensor) -> int:
    n = min(len(a), len(b))
    if n == 0:
        return 0
    diff = (a[:n].long() != b[:n].long()).nonzero()
    return int(diff[0, 0]) if len(diff) > 0 else n
