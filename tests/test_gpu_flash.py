"""GLM-4.7-Flash model (e2e-jaxscale_b200/flash.py: MLA attention, a dense MLP in
layer 0, MoE layers after) against the oracle's composition of the pinned MLA and
MoE restatements (oracle/glm4_ref.py flash_forward, models/glm4_flash.py:93-205),
on seeded random weights: a 4-token prompt and one decode step.  Bar: the
model-level tolerance on logits (max relative error 2e-2, cosine 0.999)."""

import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _np(t):
    return t.float().cpu().numpy()


def small_flash_config(jsx, layers=3):
    return jsx.ModelConfig(hidden_size=256, num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=4,
                           intermediate_size=192, vocab_size=1000, rms_norm_eps=1e-5, rope_theta=1000000.0,
                           n_routed_experts=8, n_shared_experts=1, num_experts_per_tok=4, moe_intermediate_size=64,
                           routed_scaling_factor=1.8, norm_topk_prob=True, first_k_dense_replace=1,
                           q_lora_rank=96, kv_lora_rank=64, qk_nope_head_dim=48, qk_rope_head_dim=16,
                           v_head_dim=64, attention_bias=False, partial_rotary_factor=1.0)


def oracle_params(ref, model, c):
    layers = []
    for lyr in model.layers:
        at = lyr.self_attn
        mla = ref.MLAParams(q_a=_np(at.q_a_proj.weight.value), q_a_ln=np.ones(c.q_lora_rank, np.float32),
                            q_b=_np(at.q_b_proj.weight.value), kv_a=_np(at.kv_a_proj_with_mqa.weight.value),
                            kv_a_ln=np.ones(c.kv_lora_rank, np.float32), kv_b=_np(at.kv_b_proj.weight.value),
                            o=_np(at.o_proj.weight.value))
        m = lyr.mlp
        if hasattr(m, "gate_proj"):
            fl = ref.FlashLayerParams(ln1=np.ones(c.hidden_size, np.float32), mla=mla,
                                      ln2=np.ones(c.hidden_size, np.float32),
                                      dense=(_np(m.gate_proj.weight.value), _np(m.up_proj.weight.value),
                                             _np(m.down_proj.weight.value)))
        else:
            fl = ref.FlashLayerParams(ln1=np.ones(c.hidden_size, np.float32), mla=mla,
                                      ln2=np.ones(c.hidden_size, np.float32),
                                      moe=dict(router=_np(m.gate.weight.weight.value), bias=None,
                                               eg=_np(m.expert_gate_weight.value), eu=_np(m.expert_up_weight.value),
                                               ed=_np(m.expert_down_weight.value),
                                               sg=_np(m.shared_experts.gate_proj.weight.value),
                                               su=_np(m.shared_experts.up_proj.weight.value),
                                               sd=_np(m.shared_experts.down_proj.weight.value)))
        layers.append(fl)
    return ref.FlashParams(embed=_np(model.embed_tokens.embedding.value), layers=layers,
                           norm=np.ones(c.hidden_size, np.float32), lm_head=_np(model.lm_head.embedding.value),
                           nh=c.num_attention_heads, nope=c.qk_nope_head_dim, rope_d=c.qk_rope_head_dim,
                           vdim=c.v_head_dim, eps=c.rms_norm_eps, rope_theta=c.rope_theta,
                           top_k=c.num_experts_per_tok, scale=c.routed_scaling_factor)


def test_flash_model_matches_oracle(jsx, ref, cuda):
    c = small_flash_config(jsx)
    model = jsx.GLM4FlashForCausalLM(c, jsx.create_mesh(1))
    model.init_random(seed=5, std=0.05)
    p = oracle_params(ref, model, c)
    B, S, L = 2, 4, 8
    ids = np.random.default_rng(6).integers(0, c.vocab_size, (B, S))
    pos = np.broadcast_to(np.arange(S), (B, S))
    caches = model.init_kv_caches(B, L)
    logits, caches = model(ids, pos, None, kv_caches=caches, cache_position=np.arange(S))
    qd = c.qk_nope_head_dim + c.qk_rope_head_dim
    kv = [(np.zeros((B, L, c.num_attention_heads, qd), np.float32),
           np.zeros((B, L, c.num_attention_heads, c.v_head_dim), np.float32)) for _ in range(c.num_hidden_layers)]
    want = ref.flash_forward(p, ids, pos, ref.make_prefill_mask(S, L), kv, np.arange(S))
    for got, exp in ((_np(logits), want),):
        err = np.max(np.abs(got - exp)) / np.max(np.abs(exp))
        cos = float(np.sum(got * exp) / (np.linalg.norm(got) * np.linalg.norm(exp)))
        assert err <= 2e-2 and cos >= 0.999, (err, cos)
    nxt = ref.argmax_first(want[:, -1])
    logits2, _ = model(nxt[:, None], np.full((B, 1), S), None, kv_caches=caches, cache_position=[S])
    want2 = ref.flash_forward(p, nxt[:, None], np.full((B, 1), S), ref.make_decode_mask(S, L), kv, [S])
    got2 = _np(logits2)
    err2 = np.max(np.abs(got2 - want2)) / np.max(np.abs(want2))
    cos2 = float(np.sum(got2 * want2) / (np.linalg.norm(got2) * np.linalg.norm(want2)))
    assert err2 <= 2e-2 and cos2 >= 0.999, (err2, cos2)
