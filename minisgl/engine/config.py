"""Engine configuration (a frozen dataclass the scheduler and server extend).

Field names and defaults of the reference's EngineConfig
(python/minisgl/engine/config.py:15-55) are kept; the additions select the
device, expert / context parallelism and the collective implementation.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from functools import cached_property
from typing import TYPE_CHECKING, Any, Dict, List, Optional

import torch

from minisgl.parallel import DistributedInfo

if TYPE_CHECKING:
    from minisgl.models import ModelConfig


@dataclass(frozen=True)
class EngineConfig:
    model_path: str
    tp_info: DistributedInfo
    dtype: torch.dtype
    max_running_req: int = 256
    attention_backend: str = "auto"
    moe_backend: str = "auto"
    cuda_graph_bs: Optional[List[int]] = None
    cuda_graph_max_bs: Optional[int] = None
    page_size: int = 1
    memory_ratio: float = 0.9
    distributed_timeout: float = 60.0
    use_dummy_weight: bool = False
    use_pynccl: bool = True
    max_seq_len_override: Optional[int] = None
    num_page_override: Optional[int] = None
    # --- additions of this engine
    device: str = "cuda"              # "cpu" runs the fp32 reference path (tests, tiny models)
    ep_size: int = 1                  # expert parallelism (routed experts split across ranks)
    cp_size: int = 1                  # context parallelism (sequence split across ranks)
    enable_dp_attention: bool = False
    moe_quant: str = "none"           # "none" | "mxfp4" | "mxfp4-a8"
    comm: str = "fused"               # "fused" (in-kernel NVLink collectives) | "nccl" (baseline)
    weight_seed: int = 0
    dummy_weight_device: Optional[str] = None  # draw random weights here ("cpu" for bit-identical tests)
    hf_config_override: Optional[Dict[str, Any]] = field(default=None, hash=False, compare=False)
    distributed_port: Optional[int] = None
    gemm_autotune: bool = True        # time GEMM tile plans for the decode batch sizes at start-up

    @cached_property
    def hf_config(self):
        from minisgl.utils import cached_load_hf_config

        cfg = cached_load_hf_config(self.model_path)
        for k, v in (self.hf_config_override or {}).items():
            setattr(cfg, k, v)
        return cfg

    @cached_property
    def model_config(self) -> "ModelConfig":
        import dataclasses

        from minisgl.models import ModelConfig

        cfg = ModelConfig.from_hf(self.hf_config)
        # DP attention splits the routed experts over every rank
        ep = self.tp_info.size if self.enable_dp_attention else (self.ep_size if self.ep_size > 1 else 1)
        return dataclasses.replace(cfg, moe_quant=self.moe_quant, ep_size=ep,
                                   ep_rank=self.tp_info.rank % ep if ep > 1 else 0)

    @property
    def max_seq_len(self) -> int:
        if self.max_seq_len_override is not None:
            return self.max_seq_len_override
        return self.model_config.rotary_config.max_position

    @property
    def max_forward_len(self) -> int:
        return self.max_seq_len

    @property
    def distributed_addr(self) -> str:
        return f"tcp://127.0.0.1:{self.distributed_port or 2333}"
