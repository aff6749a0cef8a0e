"""Model hyper-parameters read from a Hugging Face config.

Handles the wrappers and renames seen across model families: a
``text_config`` sub-config (Mistral-3 style multimodal checkpoints),
``num_local_experts`` vs ``num_experts``, rope settings stored either as
``rope_theta`` / ``rope_scaling`` (transformers 4) or ``rope_parameters``
(transformers 5), and the MLA / routed-expert fields of DeepSeek-V3-style
models (Kimi-K2).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional


@dataclass(frozen=True)
class RotaryConfig:
    head_dim: int
    rotary_dim: int
    max_position: int
    base: float
    scaling: Optional[Dict[str, Any]]


@dataclass(frozen=True)
class ModelConfig:
    num_layers: int
    num_qo_heads: int
    num_kv_heads: int
    head_dim: int
    hidden_size: int
    vocab_size: int
    intermediate_size: int
    rms_norm_eps: float
    rotary_config: RotaryConfig
    hidden_act: str
    tie_word_embeddings: bool
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    norm_topk_prob: bool
    model_type: str
    architectures: List[str]
    # DeepSeek-V3 / Kimi-K2 (MLA + routed experts with a shared expert)
    q_lora_rank: int = 0
    kv_lora_rank: int = 0
    qk_nope_head_dim: int = 0
    qk_rope_head_dim: int = 0
    v_head_dim: int = 0
    n_shared_experts: int = 0
    first_k_dense_replace: int = 0
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0
    scoring_func: str = "softmax"
    attention_bias: bool = False
    # runtime choices that shape the layers (not part of the HF config)
    moe_quant: str = "none"      # "none" | "mxfp4" | "mxfp4-a8": routed expert weights in MXFP4 (a8: MXFP8 activations)
    ep_size: int = 1             # routed experts split over this many ranks
    ep_rank: int = 0
    extra: Dict[str, Any] = field(default_factory=dict)

    @property
    def is_moe(self) -> bool:
        return "moe" in self.model_type or self.num_experts > 0

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    @classmethod
    def from_hf(cls, config: Any) -> "ModelConfig":
        text = getattr(config, "text_config", None)
        if text is not None:
            for attr in ("architectures", "rope_theta", "rope_scaling", "rope_parameters"):
                if not getattr(text, attr, None) and getattr(config, attr, None):
                    setattr(text, attr, getattr(config, attr))
            config = text

        def get(name: str, default: Any = None) -> Any:
            v = getattr(config, name, default)
            return default if v is None else v

        heads = config.num_attention_heads
        head_dim = get("head_dim") or config.hidden_size // heads
        rope_params = get("rope_parameters") or {}
        scaling = get("rope_scaling") or None
        if scaling is None and rope_params and rope_params.get("rope_type", "default") != "default":
            scaling = dict(rope_params)
        theta = get("rope_theta") or rope_params.get("rope_theta") or (scaling or {}).get("rope_theta") or 10000.0
        num_experts = get("num_local_experts", 0) or get("num_experts", 0) or get("n_routed_experts", 0)
        kv_lora = get("kv_lora_rank", 0)
        rope_dim = get("qk_rope_head_dim", 0) if kv_lora else head_dim
        return cls(
            num_layers=config.num_hidden_layers,
            num_qo_heads=heads,
            num_kv_heads=get("num_key_value_heads", heads),
            head_dim=head_dim,
            hidden_size=config.hidden_size,
            vocab_size=config.vocab_size,
            intermediate_size=get("intermediate_size", 0),
            rms_norm_eps=get("rms_norm_eps", 1e-6),
            rotary_config=RotaryConfig(
                head_dim=rope_dim,
                rotary_dim=rope_dim,
                max_position=get("max_position_embeddings", 4096),
                base=float(theta),
                scaling=scaling,
            ),
            hidden_act=get("hidden_act", "silu"),
            tie_word_embeddings=bool(get("tie_word_embeddings", False)),
            num_experts=num_experts,
            num_experts_per_tok=get("num_experts_per_tok", 0),
            moe_intermediate_size=get("moe_intermediate_size", 0),
            norm_topk_prob=bool(get("norm_topk_prob", False)),
            model_type=get("model_type", "llama"),
            architectures=list(get("architectures", ["LlamaForCausalLM"])),
            q_lora_rank=get("q_lora_rank", 0) or 0,
            kv_lora_rank=kv_lora or 0,
            qk_nope_head_dim=get("qk_nope_head_dim", 0),
            qk_rope_head_dim=get("qk_rope_head_dim", 0),
            v_head_dim=get("v_head_dim", 0),
            n_shared_experts=get("n_shared_experts", 0) or 0,
            first_k_dense_replace=get("first_k_dense_replace", 0),
            n_group=get("n_group", 1) or 1,
            topk_group=get("topk_group", 1) or 1,
            routed_scaling_factor=float(get("routed_scaling_factor", 1.0)),
            scoring_func=get("scoring_func", "softmax"),
            attention_bias=bool(get("attention_bias", False)),
        )
