"""Weights: streaming HF safetensors loader and seeded random initialisation.

Loader rules (same checkpoint layout as the reference,
python/minisgl/models/weight.py:13-124):

* tensor parallel shards: q/k/v/gate/up split on dim 0; o/down on dim 1;
  embed/lm_head split by vocabulary rows (ceil(V / tp) per rank). When there
  are fewer KV heads than ranks, rank r keeps head r * kv / tp.
* merges: q, k, v -> qkv_proj; gate, up -> gate_up_proj.
* experts ``...experts.{i}.{name}`` are stacked into ``...experts.{name}``
  of shape [E, ...]; under expert parallelism each rank keeps its own block
  of experts and the intermediate dimension is not split.
* multimodal wrappers: ``language_model.`` is stripped, vision tower and
  projector weights are skipped.

Random init draws every weight matrix from N(0, 0.02) and sets norm
weights to one, deterministically from a seed (synthetic benchmarks have no
checkpoint).
"""

from __future__ import annotations

import glob
import os
import re
from typing import Dict, Iterator, Optional, Tuple

import torch

from minisgl.parallel import get_tp_info
from minisgl.utils import cached_load_hf_config, div_ceil, download_hf_weight

_SPLIT_ROWS = (".q_proj", ".k_proj", ".v_proj", ".gate_proj", ".up_proj", ".q_b_proj", ".kv_b_proj")
_SPLIT_COLS = (".o_proj", ".down_proj")
_MERGE = {
    ".q_proj": (".qkv_proj", "q", ("q", "k", "v")),
    ".k_proj": (".qkv_proj", "k", ("q", "k", "v")),
    ".v_proj": (".qkv_proj", "v", ("q", "k", "v")),
    ".gate_proj": (".gate_up_proj", "gate", ("gate", "up")),
    ".up_proj": (".gate_up_proj", "up", ("gate", "up")),
}
_EXPERT = re.compile(r"^(?P<prefix>.+\.experts)\.(?P<idx>\d+)\.(?P<name>.+?)(?:\.weight)?$")
# MLA projections that are not tensor-parallel sharded in this engine
_REPLICATED_HINTS = ("kv_a_proj_with_mqa", "q_a_proj", "kv_a_layernorm", "q_a_layernorm")


def _has(name: str, parts) -> bool:
    return any(p in name for p in parts)


def shard_tensor(name: str, t: torch.Tensor, rank: int, size: int, num_kv_heads: Optional[int],
                 expert_parallel: bool = False) -> torch.Tensor:
    if size == 1 or _has(name, _REPLICATED_HINTS):
        return t
    if expert_parallel and ".experts." in name and "shared_experts" not in name:
        return t  # whole experts per rank: no intra-expert split
    if _has(name, _SPLIT_ROWS):
        if _has(name, (".k_proj", ".v_proj")) and num_kv_heads is not None and num_kv_heads < size:
            hd = t.shape[0] // num_kv_heads
            h = rank * num_kv_heads // size
            return t[h * hd : (h + 1) * hd].clone()
        return t.chunk(size, dim=0)[rank].clone()
    if _has(name, _SPLIT_COLS):
        return t.chunk(size, dim=1)[rank].clone()
    if "lm_head" in name or "embed_tokens" in name:
        per = div_ceil(t.shape[0], size)
        return t[rank * per : min((rank + 1) * per, t.shape[0])].clone()
    return t


def _merge_info(name: str):
    for suffix, (fused, slot, slots) in _MERGE.items():
        if suffix in name:
            return name.replace(suffix, fused), slot, slots
    return None


def load_weight(model_path: str, device: torch.device, *, ep_size: int = 1,
                ep_rank: int = 0) -> Iterator[Tuple[str, torch.Tensor]]:
    """Yield (runtime name, tensor on ``device``), sharded and merged.

    Peak host memory is one checkpoint tensor plus pending merge parts."""
    import safetensors

    from .config import ModelConfig

    folder = download_hf_weight(model_path)
    config = ModelConfig.from_hf(cached_load_hf_config(model_path))
    files = sorted(glob.glob(os.path.join(folder, "*.safetensors")))
    files = [f for f in files if not f.endswith("consolidated.safetensors")] or files
    info = get_tp_info()
    ep = ep_size > 1
    per_rank_experts = config.num_experts // ep_size if ep else config.num_experts
    first_expert = ep_rank * per_rank_experts if ep else 0
    merges: Dict[str, Dict[str, torch.Tensor]] = {}
    experts: Dict[str, Dict[int, torch.Tensor]] = {}
    for file in files:
        with safetensors.safe_open(file, framework="pt", device=str(device)) as f:
            for raw_name in f.keys():
                if raw_name.startswith(("vision_tower.", "multi_modal_projector.", "model.vision")):
                    continue
                name = raw_name.removeprefix("language_model.")
                m = _EXPERT.match(name)
                if ep and m is not None and not (first_expert <= int(m.group("idx")) < first_expert + per_rank_experts):
                    continue
                t = shard_tensor(name, f.get_tensor(raw_name), info.rank, info.size, config.num_kv_heads, ep)
                mi = _merge_info(name)
                if mi is not None:
                    key, slot, slots = mi
                    parts = merges.setdefault(key, {})
                    parts[slot] = t
                    if len(parts) < len(slots):
                        continue
                    name, t = key, torch.cat([parts[s] for s in slots], dim=0)
                    del merges[key]
                m = _EXPERT.match(name)
                if config.is_moe and m is not None and "shared_experts" not in name:
                    packed = f"{m.group('prefix')}.{m.group('name')}"
                    slots_e = experts.setdefault(packed, {})
                    slots_e[int(m.group("idx")) - first_expert] = t
                    if len(slots_e) < per_rank_experts:
                        continue
                    yield packed, torch.stack([slots_e[i] for i in range(per_rank_experts)])
                    del experts[packed]
                    continue
                yield name, t
    if merges or experts:
        raise RuntimeError(f"checkpoint is incomplete: {sorted(merges)[:4]} {sorted(experts)[:4]}")


def _random_tensor(name: str, ref: torch.Tensor, device: torch.device, gen: torch.Generator,
                   gen_dev: torch.device, seed: int, std: float, first_expert: int) -> torch.Tensor:
    """The random-init value of one named weight (its seed depends only on
    the name, so the order in which weights are drawn does not matter)."""
    import zlib

    dt = ref.dtype  # the model was built with the right dtype per tensor
    if name.endswith("norm.weight") or "layernorm" in name or name.endswith("_norm.weight"):
        return torch.ones(ref.shape, dtype=dt, device=device)
    if "bias" in name:
        return torch.zeros(ref.shape, dtype=dt, device=device)
    if name.endswith(("experts.gate_up_proj", "experts.down_proj")) and ref.dim() == 3:
        # stacked routed experts: one seed per global expert, so under
        # expert parallelism every rank holds its own experts' values
        t = torch.empty(ref.shape, dtype=dt, device=device)
        for e in range(ref.shape[0]):
            gen.manual_seed(seed * 1000003 + zlib.crc32(f"{name}.{first_expert + e}".encode()))
            part = torch.empty(ref.shape[1:], dtype=torch.float32 if gen_dev.type == "cpu" else dt, device=gen_dev)
            part.normal_(0.0, std, generator=gen)
            t[e].copy_(part)
        return t
    # per-name seed: identical on every rank, so replicated weights agree
    gen.manual_seed(seed * 1000003 + zlib.crc32(name.encode()))
    t = torch.empty(ref.shape, dtype=torch.float32 if gen_dev.type == "cpu" else dt, device=gen_dev)
    t.normal_(0.0, std, generator=gen)
    return t.to(device=device, dtype=dt)


def random_weights(shapes: Dict[str, torch.Tensor], device: torch.device, seed: int = 0,
                   std: float = 0.02, gen_device: Optional[torch.device] = None,
                   first_expert: int = 0) -> Dict[str, torch.Tensor]:
    """N(0, std) for matrices, ones for norm weights, zeros for biases.
    ``shapes`` maps names to (meta) tensors giving shape and dtype. With
    ``gen_device`` the numbers are drawn there (e.g. on the CPU, so a GPU
    engine and the CPU oracle get identical weights) and then moved."""
    lazy = LazyRandomWeights(shapes, device, seed, std, gen_device, first_expert)
    return {name: lazy[name] for name in sorted(shapes)}


class LazyRandomWeights:
    """``random_weights`` drawn one tensor at a time, when the model's
    ``load_state_dict`` takes it (``pop``): the same values, but the peak
    memory of loading is the model plus one tensor instead of two copies of
    the model. With quantised experts, whose layer quantises them as soon as
    they are loaded, only one layer's bf16 experts exist at any time (a
    Kimi-K2-shape model holds 254 GB of bf16 experts per rank at EP8, 67 GB
    once quantised to MXFP4). Supports what ``load_state_dict`` uses: ``in``,
    ``pop``, ``len`` and iteration over the names not yet taken."""

    def __init__(self, shapes: Dict[str, torch.Tensor], device: torch.device, seed: int = 0, std: float = 0.02,
                 gen_device: Optional[torch.device] = None, first_expert: int = 0) -> None:
        self._shapes = dict(shapes)
        self._device = torch.device(device)
        self._gen_dev = torch.device(gen_device) if gen_device is not None else self._device
        self._gen = torch.Generator(device=self._gen_dev)
        self._seed, self._std, self._first = seed, std, first_expert

    def __contains__(self, name: object) -> bool:
        return name in self._shapes

    def __len__(self) -> int:
        return len(self._shapes)

    def __iter__(self):
        return iter(list(self._shapes))

    def keys(self):
        return list(self._shapes)

    def __getitem__(self, name: str) -> torch.Tensor:
        return _random_tensor(name, self._shapes[name], self._device, self._gen, self._gen_dev, self._seed,
                              self._std, self._first)

    def pop(self, name: str, *default):
        if name not in self._shapes:
            if default:
                return default[0]
            raise KeyError(name)
        t = self[name]
        del self._shapes[name]
        return t
