"""GLM-4.7-Flash (models/glm4_flash.py:26-205) on the library's layers:

    Embed -> N x [RMSNorm -> MLAAttention -> + residual -> RMSNorm ->
                  DenseMLP (layer < first_k_dense_replace) or MoELayer -> + residual]
          -> RMSNorm -> ParallelLMHead

MLAAttention (layers/mla_attention.py), MoELayer / DenseMLP (layers/moe.py) carry
the kernels: low-rank projections with fused latent RMSNorms, the MLA RoPE +
cache-write kernel and the decode attention kernel, the router, the grouped
expert GEMVs and the single exchange that sums the routed and shared-expert
partials over the expert x tensor ranks.  Residual adds are bf16 like the
reference's.  __call__ keeps the reference signature and runs prompt positions
one at a time (MLAAttention is a decode-path layer).
"""

from __future__ import annotations

import numpy as np
import torch

from . import kernels as K
from .config import ModelConfig
from .layers.embedding import Embed, ParallelLMHead
from .layers.kv_cache import KVCache
from .layers.mla_attention import MLAAttention
from .layers.moe import DenseMLP, MoELayer
from .layers.normalization import RMSNorm


class GLM4FlashDecoderLayer:
    """models/glm4_flash.py:26-110."""

    def __init__(self, config: ModelConfig, mesh, layer_id: int = 0, dtype=torch.bfloat16,
                 absorbed_mla: bool = False):
        c = config
        self.layer_id = layer_id
        self.self_attn = MLAAttention(c.hidden_size, c.num_attention_heads, c.q_lora_rank, c.kv_lora_rank,
                                      c.qk_nope_head_dim, c.qk_rope_head_dim, c.v_head_dim,
                                      c.max_position_embeddings, c.rope_theta, c.rms_norm_eps, mesh, dtype,
                                      absorbed=absorbed_mla)
        if layer_id < c.first_k_dense_replace:
            self.mlp = DenseMLP(c.hidden_size, c.intermediate_size, mesh, dtype)
        else:
            self.mlp = MoELayer(c.hidden_size, c.moe_intermediate_size, c.shared_intermediate_size,
                                c.n_routed_experts, c.num_experts_per_tok, c.routed_scaling_factor,
                                c.norm_topk_prob, mesh, dtype)
        self.input_layernorm = RMSNorm(c.hidden_size, epsilon=c.rms_norm_eps, param_dtype=dtype)
        self.post_attention_layernorm = RMSNorm(c.hidden_size, epsilon=c.rms_norm_eps, param_dtype=dtype)

    def __call__(self, hidden_states, positions, attention_mask=None, kv_cache=None, cache_position=None):
        residual = hidden_states
        x = self.input_layernorm(hidden_states)
        a, kv_cache = self.self_attn(x, positions, attention_mask, kv_cache=kv_cache,
                                     cache_position=cache_position)
        h = residual + a
        residual = h
        y = self.mlp(self.post_attention_layernorm(h))
        return residual + y, kv_cache


class GLM4FlashForCausalLM:
    """models/glm4_flash.py:113-205: __call__(input_ids, positions, attention_mask,
    kv_caches, cache_position) -> (logits [B, S, V], caches).  absorbed_mla: the
    attention runs in the latent-cache form (MLAAttention(absorbed=True)) and
    init_kv_caches returns latent caches."""

    def __init__(self, config: ModelConfig, mesh, dtype=torch.bfloat16, absorbed_mla: bool = False):
        self.config, self.mesh, self.dtype = config, mesh, dtype
        self.absorbed_mla = absorbed_mla
        self.device = mesh.device if mesh is not None and mesh.device is not None else torch.device("cuda")
        c = config
        self.embed_tokens = Embed(c.vocab_size, c.hidden_size, dtype, mesh)
        self.layers = [GLM4FlashDecoderLayer(c, mesh, i, dtype, absorbed_mla) for i in range(c.num_hidden_layers)]
        self.norm = RMSNorm(c.hidden_size, epsilon=c.rms_norm_eps, param_dtype=dtype)
        self.lm_head = ParallelLMHead(c.vocab_size, c.hidden_size, dtype, mesh)

    def init_random(self, seed: int = 0, std: float = 0.02) -> None:
        """Synthetic N(0, std) bf16 weights drawn on the device (gains 1, router
        correction bias 0), in the attribute order of models/glm4_flash.py."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        dev, c = self.device, self.config

        def normal(*shape):
            return (torch.randn(*shape, generator=g, device=dev) * std).to(torch.bfloat16)

        self.embed_tokens.embedding.value = normal(c.vocab_size, c.hidden_size)
        H, nh = c.hidden_size, c.num_attention_heads
        qd = c.qk_nope_head_dim + c.qk_rope_head_dim
        for lyr in self.layers:
            at = lyr.self_attn
            at.q_a_proj.weight.value = normal(H, c.q_lora_rank)
            at.q_b_proj.weight.value = normal(c.q_lora_rank, nh * qd)
            at.kv_a_proj_with_mqa.weight.value = normal(H, c.kv_lora_rank + c.qk_rope_head_dim)
            at.kv_b_proj.weight.value = normal(c.kv_lora_rank, nh * (c.qk_nope_head_dim + c.v_head_dim))
            at.o_proj.weight.value = normal(nh * c.v_head_dim, H)
            m = lyr.mlp
            if isinstance(m, DenseMLP):
                m.gate_proj.weight.value = normal(H, c.intermediate_size)
                m.up_proj.weight.value = normal(H, c.intermediate_size)
                m.down_proj.weight.value = normal(c.intermediate_size, H)
            else:
                E, I, Is = c.n_routed_experts, c.moe_intermediate_size, c.shared_intermediate_size
                m.gate.weight.weight.value = normal(H, E)
                m.expert_gate_weight.value = normal(E, H, I)
                m.expert_up_weight.value = normal(E, H, I)
                m.expert_down_weight.value = normal(E, I, H)
                m.shared_experts.gate_proj.weight.value = normal(H, Is)
                m.shared_experts.up_proj.weight.value = normal(H, Is)
                m.shared_experts.down_proj.weight.value = normal(Is, H)
        self.lm_head.embedding.value = normal(c.vocab_size, H)

    def init_kv_caches(self, batch_size: int, max_seq_len: int) -> list[KVCache]:
        """Expanded per-head caches (layers/mla_attention.py:125-139): k [B, L, nh_l, nope + rope],
        v [B, L, nh_l, v_head_dim] per layer, zero-initialised; with absorbed_mla the latent
        caches k [B, L, kv_lora + rope] (v empty)."""
        if self.absorbed_mla:
            return [lyr.self_attn.init_latent_cache(batch_size, max_seq_len, self.device) for lyr in self.layers]
        c = self.config
        tp = 1 if self.mesh is None else self.mesh.shape.get("tensor", 1)
        nh = c.num_attention_heads // tp
        qd = c.qk_nope_head_dim + c.qk_rope_head_dim
        mk = (lambda d: torch.zeros(batch_size, max_seq_len, nh, d, dtype=torch.bfloat16, device=self.device))
        return [KVCache(mk(qd), mk(c.v_head_dim)) for _ in self.layers]

    def __call__(self, input_ids, positions, attention_mask=None, kv_caches=None, cache_position=None):
        """input_ids / positions: host arrays, or device tensors (then the call issues no
        host<->device copy and can be captured in a CUDA graph; pass cache_position=None)."""
        ids = input_ids if torch.is_tensor(input_ids) else torch.as_tensor(np.asarray(input_ids), dtype=torch.int32)
        h = self.embed_tokens(ids)
        new = []
        for i, lyr in enumerate(self.layers):
            cache = kv_caches[i] if kv_caches is not None else None
            h, cache = lyr(h, positions, attention_mask, kv_cache=cache, cache_position=cache_position)
            new.append(cache)
        logits = self.lm_head(self.norm(h))
        return logits, (new if kv_caches is not None else None)
