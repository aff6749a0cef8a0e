"""Rotary position embedding tables.

Builds the fp32 [max_position, rotary_dim] table (cos of the rotary_dim/2
frequencies followed by their sin) that the fused norm + RoPE + KV-store
kernel reads. Frequency schedules:

* default: inv_freq_i = base^(-2i / d) (Su et al., RoFormer, 2021);
* llama3: the piecewise low/high-frequency rescaling published with
  Llama 3.1 (wavelengths above original_max / low_freq_factor are divided
  by ``factor``, below original_max / high_freq_factor are kept, a linear
  blend in between);
* yarn: YaRN (Peng et al., 2023) "NTK-by-parts" interpolation with a linear
  ramp between the beta_fast / beta_slow correction dimensions, plus the
  attention temperature factor 0.1 ln(s) + 1 folded into cos/sin when the
  config asks for it (DeepSeek-V3 style ``mscale`` / ``mscale_all_dim``).

Tables are cached per configuration and device.
"""

from __future__ import annotations

import functools
import math
from typing import Any, Dict, Optional, Tuple

import torch

from .base import StateLessOP


def _inv_freq(dim: int, base: float) -> torch.Tensor:
    return 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))


def _llama3(inv: torch.Tensor, s: Dict[str, Any]) -> torch.Tensor:
    factor = float(s["factor"])
    lo, hi = float(s.get("low_freq_factor", 1.0)), float(s.get("high_freq_factor", 4.0))
    orig = float(s["original_max_position_embeddings"])
    wavelen = 2 * math.pi / inv
    if lo == hi:
        return torch.where(wavelen < orig / hi, inv, inv / factor)
    smooth = ((orig / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
    return inv * ((1 - smooth) / factor + smooth)


def _yarn_mscale(scale: float, m: float) -> float:
    return 1.0 if scale <= 1.0 else 0.1 * m * math.log(scale) + 1.0


def _yarn(inv: torch.Tensor, dim: int, base: float, s: Dict[str, Any]) -> Tuple[torch.Tensor, float]:
    factor = float(s["factor"])
    beta_fast = float(s.get("beta_fast", 32.0))
    beta_slow = float(s.get("beta_slow", 1.0))
    orig = float(s["original_max_position_embeddings"])

    def corr_dim(rot: float) -> float:
        return dim * math.log(orig / (rot * 2 * math.pi)) / (2 * math.log(base))

    lo = max(math.floor(corr_dim(beta_fast)), 0)
    hi = min(math.ceil(corr_dim(beta_slow)), dim // 2 - 1)
    ramp = ((torch.arange(dim // 2, dtype=torch.float64) - lo) / max(hi - lo, 1)).clamp(0, 1)
    blended = inv / factor * ramp + inv * (1 - ramp)
    if s.get("mscale_all_dim"):
        mscale = _yarn_mscale(factor, float(s.get("mscale", 1.0))) / _yarn_mscale(factor, float(s["mscale_all_dim"]))
    elif "mscale" in s:
        mscale = _yarn_mscale(factor, float(s["mscale"]))
    else:
        mscale = float(s.get("attention_factor") or _yarn_mscale(factor, 1.0))
    return blended, mscale


class RotaryEmbedding(StateLessOP):
    def __init__(self, head_size: int, rotary_dim: int, max_position: int, base: float,
                 scaling: Optional[Dict[str, Any]] = None) -> None:
        if rotary_dim != head_size:
            raise ValueError("partial rotary embeddings are not supported")
        self.head_size = head_size
        inv = _inv_freq(rotary_dim, base)
        mscale = 1.0
        kind = (scaling or {}).get("rope_type", (scaling or {}).get("type", "default"))
        if kind in (None, "default"):
            pass
        elif kind == "llama3":
            inv = _llama3(inv, scaling)
        elif kind in ("yarn", "deepseek_yarn"):
            inv, mscale = _yarn(inv, rotary_dim, base, scaling)
        elif kind == "linear":
            inv = inv / float(scaling["factor"])
        else:
            raise ValueError(f"unsupported rope scaling {scaling}")
        t = torch.arange(max_position, dtype=torch.float64)
        freqs = torch.outer(t, inv)
        self._cos_sin_cache = (torch.cat([freqs.cos(), freqs.sin()], dim=-1) * mscale).float()

    @property
    def cos_sin_cache(self) -> torch.Tensor:
        return self._cos_sin_cache

    def forward(self, positions: torch.Tensor, q: torch.Tensor, k: torch.Tensor):
        """Rotate q [T, hq, d] and k [T, hk, d] (NeoX layout); used by paths
        that do not go through the fused store kernel (MLA rope part)."""
        cs = self._cos_sin_cache[positions.long()]
        h = self.head_size // 2
        cos, sin = cs[:, None, :h], cs[:, None, h:]

        def rot(x: torch.Tensor) -> torch.Tensor:
            xf = x.float()
            x1, x2 = xf[..., :h], xf[..., h:]
            return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).to(x.dtype)

        return rot(q), rot(k)


_ROPE_DEVICE: Optional[torch.device] = None


def set_rope_device(device: torch.device) -> None:
    global _ROPE_DEVICE
    _ROPE_DEVICE = torch.device(device)


@functools.lru_cache(maxsize=None)
def _cached(head_dim: int, rotary_dim: int, max_position: int, base: float, scaling_items, device) -> RotaryEmbedding:
    with torch.device("cpu"):  # models are built under a meta-device scope
        emb = RotaryEmbedding(head_dim, rotary_dim, max_position, base, dict(scaling_items) if scaling_items else None)
    emb._cos_sin_cache = emb._cos_sin_cache.to(device)
    return emb


def get_rope(head_dim: int, rotary_dim: int, max_position: int, base: float,
             rope_scaling: Optional[Tuple[Tuple[str, Any], ...]] = None) -> RotaryEmbedding:
    """Shared table for a configuration. Models are built on the meta device,
    so the table goes to the device registered with ``set_rope_device``."""
    device = _ROPE_DEVICE or torch.device("cpu")
    items = tuple(sorted((k, _freeze(v)) for k, v in dict(rope_scaling).items())) if rope_scaling else None
    return _cached(head_dim, rotary_dim, max_position, float(base), items, device)


def _freeze(v: Any) -> Any:
    if isinstance(v, list):
        return tuple(v)
    if isinstance(v, dict):
        return tuple(sorted(v.items()))
    return v


def reset_rope_cache() -> None:
    _cached.cache_clear()
