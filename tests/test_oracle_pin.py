"""Pins the CPU oracle to the reference's own code: tests/golden/reference_golden.npz
was produced by running the reference's layers/, models/glm4.py, models/glm4_flash.py
and runner.py (greedy loop and sampling step)
(through the numpy stand-in for jax/flax, tests/golden/make_golden.py).  The
oracle must reproduce every recorded output bit for bit on the same inputs."""

import hashlib
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_golden.npz")


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def same(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert np.array_equal(a, b), f"max diff {np.max(np.abs(a - b))}"


def test_rmsnorm(ref, g):
    same(ref.rmsnorm(g["rms_x"], g["rms_scale"], 1.5625e-07), g["rms_y"])


def test_linear_bias_after_round(ref, g):
    same(ref.linear(g["lin_x"], g["lin_w"], g["lin_b"]), g["lin_y"])


def test_rope_half_split(ref, g):
    inv = ref.rope_inv_freq(128)
    qo, ko = ref.rope(g["rope_pos"], g["rope_q"], g["rope_k"], inv)
    same(qo, g["rope_qo"])
    same(ko, g["rope_ko"])


def test_gqa_attention_prefill_then_decode(ref, g):
    cfg = ref.GLMConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=128)
    lp = ref.LayerParams(ln1=None, wq=g["att_q_proj_w"], bq=g["att_q_proj_b"], wk=g["att_k_proj_w"],
                         bk=g["att_k_proj_b"], wv=g["att_v_proj_w"], bv=g["att_v_proj_b"],
                         wo=g["att_o_proj_w"], ln2=None, wg=None, wu=None, wd=None)
    B, S, L = 2, 5, 12
    inv = ref.rope_inv_freq(128)
    kc = np.zeros((B, L, 2, 128), np.float32)
    vc = np.zeros_like(kc)
    pos = np.broadcast_to(np.arange(S), (B, S))
    y = ref.attention(lp, cfg, g["att_h"], pos, ref.make_prefill_mask(S, L), (kc, vc), np.arange(S), inv)
    same(y, g["att_y"])
    y2 = ref.attention(lp, cfg, g["att_h2"], np.full((B, 1), S), ref.make_decode_mask(S, L), (kc, vc),
                       np.array([S]), inv)
    same(y2, g["att_y2"])
    same(kc, g["att_k"])
    same(vc, g["att_v"])


def test_moe_gate(ref, g):
    w0, i0 = ref.moe_gate(g["moe_x"], g["moe_w"], 4, 1.8, True)
    same(w0, g["moe_w0"])
    assert np.array_equal(i0, g["moe_i0"])
    w1, i1 = ref.moe_gate(g["moe_x"], g["moe_w"], 4, 1.8, True, g["moe_bias"])
    same(w1, g["moe_w1"])
    assert np.array_equal(i1, g["moe_i1"])


def test_greedy_generation_and_logits(ref, g):
    rc = ref.GLMConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=128, intermediate_size=384, vocab_size=1000)
    p = ref.init_params(rc, seed=0)
    h = hashlib.sha256()
    for a in [p.embed] + [getattr(lp, n) for lp in p.layers for n in
                          ("ln1", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "ln2", "wg", "wu", "wd")] + \
            [p.norm, p.lm_head]:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    assert h.hexdigest() == str(g["model_params_sha256"]), "numpy generator stream changed"
    prompt = g["model_prompt"]
    record = []
    gen = ref.greedy_generate(p, prompt, 6, max_cache_len=16, record=record)
    assert np.array_equal(gen, g["model_gen"])
    same(record[0][0], g["model_prefill_logits"])
    same(record[1][0], g["model_decode_logits"])


def test_moe_layer(ref, g):
    """MoELayer without expert parallelism: router, top-4 experts accumulated in k
    order in bf16 (_topk_local_forward), shared SwiGLU expert, bf16 sum."""
    y = ref.moe_layer(g["moel_x"], g["moel_router"], g["moel_bias"], 4, 1.8, True, g["moel_eg"], g["moel_eu"],
                      g["moel_ed"], g["moel_sg"], g["moel_su"], g["moel_sd"])
    same(y, g["moel_y"])


def test_mla_attention_prefill_then_decode(ref, g):
    """MLAAttention: low-rank q/kv with latent RMSNorms, RoPE on the rope slice and the
    shared key, expanded per-head cache, bf16 scores, fp32 softmax."""
    p = ref.MLAParams(q_a=g["mla_q_a_proj"], q_a_ln=g["mla_q_a_ln"], q_b=g["mla_q_b_proj"],
                      kv_a=g["mla_kv_a_proj_with_mqa"], kv_a_ln=g["mla_kv_a_ln"], kv_b=g["mla_kv_b_proj"],
                      o=g["mla_o_proj"])
    B, S, L = 2, 5, 12
    kc = np.zeros((B, L, 4, 64), np.float32)
    vc = np.zeros((B, L, 4, 64), np.float32)
    inv = ref.rope_inv_freq(16, theta=1000000.0, partial=1.0)
    pos = np.broadcast_to(np.arange(S), (B, S))
    y = ref.mla_attention(p, g["mla_h"], pos, ref.make_prefill_mask(S, L), (kc, vc), np.arange(S), 4, 48, 16, 64,
                          1.5625e-07, inv)
    same(y, g["mla_y"])
    y2 = ref.mla_attention(p, g["mla_h2"], np.full((B, 1), S), ref.make_decode_mask(S, L), (kc, vc), [S], 4, 48,
                           16, 64, 1.5625e-07, inv)
    same(y2, g["mla_y2"])
    same(kc, g["mla_k"])
    same(vc, g["mla_v"])


def flash_params_from_golden(ref, g, layers=3, hidden=256):
    """The reference GLM4FlashForCausalLM's weights as recorded by make_golden.py."""
    out = []
    for i in range(layers):
        mla = ref.MLAParams(q_a=g[f"flash_{i}_q_a_proj"], q_a_ln=np.ones(96, np.float32), q_b=g[f"flash_{i}_q_b_proj"],
                            kv_a=g[f"flash_{i}_kv_a_proj_with_mqa"], kv_a_ln=np.ones(64, np.float32),
                            kv_b=g[f"flash_{i}_kv_b_proj"], o=g[f"flash_{i}_o_proj"])
        ones = np.ones(hidden, np.float32)
        if i == 0:
            out.append(ref.FlashLayerParams(ln1=ones, mla=mla, ln2=ones,
                                            dense=(g["flash_0_gate_proj"], g["flash_0_up_proj"],
                                                   g["flash_0_down_proj"])))
        else:
            out.append(ref.FlashLayerParams(ln1=ones, mla=mla, ln2=ones, moe=dict(
                router=g[f"flash_{i}_router"], bias=None, eg=g[f"flash_{i}_eg"], eu=g[f"flash_{i}_eu"],
                ed=g[f"flash_{i}_ed"], sg=g[f"flash_{i}_sg"], su=g[f"flash_{i}_su"], sd=g[f"flash_{i}_sd"])))
    return ref.FlashParams(embed=g["flash_embed"], layers=out, norm=np.ones(hidden, np.float32),
                           lm_head=g["flash_lm_head"], nh=4, nope=48, rope_d=16, vdim=64, eps=1e-5,
                           rope_theta=1000000.0, top_k=4, scale=1.8)


def test_flash_model_prefill_then_decode(ref, g):
    """models/glm4_flash.py (GLM4FlashForCausalLM: MLA, dense MLP in layer 0, MoE after)."""
    p = flash_params_from_golden(ref, g)
    B, S, L = 2, 4, 8
    kv = [(np.zeros((B, L, 4, 64), np.float32), np.zeros((B, L, 4, 64), np.float32)) for _ in range(3)]
    lg = ref.flash_forward(p, g["flash_prompt"], np.broadcast_to(np.arange(S), (B, S)), ref.make_prefill_mask(S, L),
                           kv, np.arange(S))
    same(lg, g["flash_logits"])
    lg2 = ref.flash_forward(p, g["flash_next"], np.full((B, 1), S), ref.make_decode_mask(S, L), kv, [S])
    same(lg2, g["flash_logits2"])


def test_sampling_step(ref, g):
    """runner.py:315-359 (_jit_sample): penalty, temperature, top-k, top-p and the
    categorical draw with the recorded Gumbel noise, three parameter sets."""
    for j in range(3):
        rp, temp, tk, tp = g[f"samp{j}_params"]
        tok, _ = ref.sample_tokens(g["samp_logits"], g["samp_presence"] > 0, g[f"samp{j}_noise"], float(rp),
                                   float(temp), int(tk), float(tp))
        assert np.array_equal(tok, g[f"samp{j}_tokens"]), j
