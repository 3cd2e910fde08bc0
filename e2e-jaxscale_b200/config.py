"""Model configuration (configs/model_config.py:11-98): same field names and
GLM-4-9B defaults; from_pretrained reads a HF config.json directory."""

from __future__ import annotations

import json
import os
from dataclasses import dataclass


@dataclass
class ModelConfig:
    hidden_size: int = 4096
    num_hidden_layers: int = 40
    num_attention_heads: int = 32
    num_key_value_heads: int = 2
    head_dim: int | None = None
    intermediate_size: int = 13696
    vocab_size: int = 151552
    max_position_embeddings: int = 131072
    rms_norm_eps: float = 1.5625e-07
    hidden_act: str = "silu"
    attention_bias: bool = True
    rope_theta: float = 10000.0
    partial_rotary_factor: float = 0.5
    tie_word_embeddings: bool = False
    n_routed_experts: int | None = None
    n_shared_experts: int | None = None
    num_experts_per_tok: int | None = None
    moe_intermediate_size: int | None = None
    routed_scaling_factor: float = 1.0
    topk_method: str = "greedy"
    norm_topk_prob: bool = True
    first_k_dense_replace: int = 0
    # width of the MoE layers' shared expert; None: moe_intermediate_size x n_shared_experts (the
    # GLM-4.7-Flash checkpoint's shape, which replaces the reference's intermediate_size placeholder
    # at load time, layers/linear.py:45-49)
    shared_expert_intermediate_size: int | None = None
    q_lora_rank: int | None = None
    kv_lora_rank: int | None = None
    qk_nope_head_dim: int | None = None
    qk_rope_head_dim: int | None = None
    v_head_dim: int | None = None
    model_path: str = ""
    model_type: str = "glm"
    eos_token_id: int | list[int] | None = None

    def __post_init__(self):
        if self.head_dim is None:
            if self.is_mla:
                self.head_dim = self.qk_nope_head_dim + self.qk_rope_head_dim
            else:
                self.head_dim = self.hidden_size // self.num_attention_heads

    @property
    def shared_intermediate_size(self) -> int:
        if self.shared_expert_intermediate_size is not None:
            return self.shared_expert_intermediate_size
        return self.moe_intermediate_size * (self.n_shared_experts or 1)

    @property
    def is_moe(self) -> bool:
        return self.n_routed_experts is not None

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank is not None

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @classmethod
    def from_pretrained(cls, model_path: str) -> "ModelConfig":
        with open(os.path.join(model_path, "config.json")) as f:
            raw = json.load(f)
        known = set(cls.__dataclass_fields__)
        kwargs = {k: v for k, v in raw.items() if k in known}
        gen = os.path.join(model_path, "generation_config.json")
        if os.path.exists(gen):
            with open(gen) as f:
                g = json.load(f)
            if "eos_token_id" in g:
                kwargs["eos_token_id"] = g["eos_token_id"]
        kwargs["model_path"] = model_path
        return cls(**kwargs)
