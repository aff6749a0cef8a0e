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
        nxt = int(dense_logits(state, cfg, seq, qk_norm, fused_layout)[-1].argmax())
        out.append(nxt)
        seq.append(nxt)
    return out
