"""Dense, cache-free fp32 restatement of the decoder math (the oracle).

``dense_logits(state, cfg, tokens)`` runs one full causal forward over a
token sequence straight from the weight dictionary: no paging, no chunking,
no KV cache, no fused kernels. Engine tests compare the paged / chunked /
graph-captured engine against it.
"""

from __future__ import annotations

from typing import Dict, List

import torch

from .config import ModelConfig


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _ones_if(flag: bool, w: torch.Tensor) -> torch.Tensor:
    return torch.ones_like(w) if flag else w


def _rope_tables(cfg: ModelConfig, n: int):
    from minisgl.layers.rotary import RotaryEmbedding

    rc = cfg.rotary_config
    with torch.device("cpu"):
        emb = RotaryEmbedding(rc.head_dim, rc.rotary_dim, max(n, 1), rc.base, rc.scaling)
    cs = emb.cos_sin_cache[:n]
    h = rc.rotary_dim // 2
    return cs[:, :h], cs[:, h:]


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


@torch.no_grad()
def dense_logits(state: Dict[str, torch.Tensor], cfg: ModelConfig, tokens: List[int],
                 qk_norm: bool = True, fused_layout: bool = False) -> torch.Tensor:
    """fp32 logits [len(tokens), vocab] for a dense (non-MoE, non-MLA) decoder.

    ``fused_layout``: the state comes from a model whose input / post-
    attention norm weights are folded into qkv / gate_up and whose gate|up
    rows alternate in 64-row blocks; the oracle then skips those norm weights
    and reads gate and up from the interleaved rows."""
    W = {k: v.detach().float().cpu() for k, v in state.items()}
    n = len(tokens)
    ids = torch.tensor(tokens, dtype=torch.long)
    x = W["model.embed_tokens.weight"][ids]
    hq, hk, d = cfg.num_qo_heads, cfg.num_kv_heads, cfg.head_dim
    cos, sin = _rope_tables(cfg, n)
    causal = torch.ones(n, n, dtype=torch.bool).tril()
    eps = cfg.rms_norm_eps
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        h = _rms(x, _ones_if(fused_layout, W[p + "input_layernorm.weight"]), eps)
        qkv = h @ W[p + "self_attn.qkv_proj.weight"].t()
        if (p + "self_attn.qkv_proj.bias") in W:
            qkv = qkv + W[p + "self_attn.qkv_proj.bias"]
        q = qkv[:, : hq * d].view(n, hq, d)
        k = qkv[:, hq * d : (hq + hk) * d].view(n, hk, d)
        v = qkv[:, (hq + hk) * d :].view(n, hk, d)
        if qk_norm and (p + "self_attn.q_norm.weight") in W:
            q = _rms(q, W[p + "self_attn.q_norm.weight"], eps)
            k = _rms(k, W[p + "self_attn.k_norm.weight"], eps)
        q, k = _rotate(q, cos, sin), _rotate(k, cos, sin)
        g = hq // hk
        k, v = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) * d ** -0.5
        s = s.masked_fill(~causal[None], float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(n, hq * d)
        x = x + o @ W[p + "self_attn.o_proj.weight"].t()
        h = _rms(x, _ones_if(fused_layout, W[p + "post_attention_layernorm.weight"]), eps)
        gu = h @ W[p + "mlp.gate_up_proj.weight"].t()
        inter = gu.shape[-1] // 2
        if fused_layout:
            blocks = gu.view(n, inter // 64, 2, 64)
            a = (torch.nn.functional.silu(blocks[:, :, 0]) * blocks[:, :, 1]).reshape(n, inter)
        else:
            a = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
        x = x + a @ W[p + "mlp.down_proj.weight"].t()
    x = _rms(x, W["model.norm.weight"], eps)
    head = W.get("lm_head.weight", W["model.embed_tokens.weight"])
    return x @ head.t()


def greedy_generate(state: Dict[str, torch.Tensor], cfg: ModelConfig, prompt: List[int], steps: int,
                    qk_norm: bool = True, fused_layout: bool = False) -> List[int]:
    seq = list(prompt)
    out = []
    for _ in range(steps):
        logits = (dense_logits_mla(state, cfg, seq) if cfg.kv_lora_rank > 0
                  else dense_logits(state, cfg, seq, qk_norm, fused_layout))
        nxt = int(logits[-1].argmax())
        out.append(nxt)
        seq.append(nxt)
    return out


def _rope_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """pairs (2i, 2i + 1) rotate by frequency i; cos / sin [n, d / 2]"""
    shape = (x.shape[0],) + (1,) * (x.dim() - 2) + (cos.shape[-1],)
    c, s = cos.reshape(shape), sin.reshape(shape)
    even, odd = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = even * c - odd * s
    out[..., 1::2] = odd * c + even * s
    return out


@torch.no_grad()
def dense_logits_mla(state: Dict[str, torch.Tensor], cfg: ModelConfig, tokens: List[int]) -> torch.Tensor:
    """fp32 logits of a DeepSeek-V3-style decoder, computed the direct way:
    keys and values decompressed from the latent through kv_b_proj for every
    head (no absorption, no paging), dense SwiGLU or routed + shared experts."""
    from minisgl.attention.mla import mla_softmax_scale
    from minisgl.moe.fused import moe_reference
    from minisgl.ops import reference as ref

    W = {k: v.detach().float().cpu() for k, v in state.items()}
    n = len(tokens)
    x = W["model.embed_tokens.weight"][torch.tensor(tokens, dtype=torch.long)]
    H = cfg.num_qo_heads
    nope, rope, vd, lora = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
    cos, sin = _rope_tables(cfg, n)
    causal = torch.ones(n, n, dtype=torch.bool).tril()
    eps = cfg.rms_norm_eps
    scale = mla_softmax_scale(cfg)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        h = _rms(x, W[p + "input_layernorm.weight"], eps)
        if cfg.q_lora_rank > 0:
            q = _rms(h @ W[a + "q_a_proj.weight"].t(), W[a + "q_a_layernorm.weight"], eps) @ W[a + "q_b_proj.weight"].t()
        else:
            q = h @ W[a + "q_proj.weight"].t()
        q = q.view(n, H, nope + rope)
        kv_a = h @ W[a + "kv_a_proj_with_mqa.weight"].t()
        c = _rms(kv_a[:, :lora], W[a + "kv_a_layernorm.weight"], eps)
        k_pe = _rope_interleaved(kv_a[:, lora:], cos, sin)  # [n, rope], shared by all heads
        kv = (c @ W[a + "kv_b_proj.weight"].t()).view(n, H, nope + vd)
        k = torch.cat([kv[..., :nope], k_pe[:, None, :].expand(n, H, rope)], dim=-1)
        qf = torch.cat([q[..., :nope], _rope_interleaved(q[..., nope:], cos, sin)], dim=-1)
        s = torch.einsum("qhd,khd->hqk", qf, k) * scale
        s = s.masked_fill(~causal[None], float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), kv[..., nope:]).reshape(n, H * vd)
        x = x + o @ W[a + "o_proj.weight"].t()
        h = _rms(x, W[p + "post_attention_layernorm.weight"], eps)
        m = p + "mlp."
        if (m + "gate.weight") in W:
            logits = h @ W[m + "gate.weight"].t()
            topk_w, topk_ids = ref.moe_route(logits, cfg.num_experts_per_tok, cfg.scoring_func, cfg.norm_topk_prob,
                                             W.get(m + "gate.e_score_correction_bias"), cfg.n_group, cfg.topk_group,
                                             cfg.routed_scaling_factor)
            out = moe_reference(h, W[m + "experts.gate_up_proj"], W[m + "experts.down_proj"], topk_w, topk_ids,
                                "silu", interleaved=True).float()
            if (m + "shared_experts.gate_up_proj.weight") in W:
                gu = h @ W[m + "shared_experts.gate_up_proj.weight"].t()
                half = gu.shape[-1] // 2
                out = out + (torch.nn.functional.silu(gu[:, :half]) * gu[:, half:]) @ \
                    W[m + "shared_experts.down_proj.weight"].t()
        else:
            gu = h @ W[m + "gate_up_proj.weight"].t()
            half = gu.shape[-1] // 2
            out = (torch.nn.functional.silu(gu[:, :half]) * gu[:, half:]) @ W[m + "down_proj.weight"].t()
        x = x + out
    x = _rms(x, W["model.norm.weight"], eps)
    head = W.get("lm_head.weight", W["model.embed_tokens.weight"])
    return x @ head.t()
