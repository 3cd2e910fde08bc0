"""Generates tests/golden/reference_golden.npz by executing the REFERENCE's own
source files (layers/*.py incl. the MoE and MLA layers, models/glm4.py,
models/glm4_flash.py, runner.py incl. its sampling step, of sdh1014/e2e-JaxScale)
on the CPU through the numpy stand-in under tests/golden/jaxshim/ (JAX and Flax
are not installable here).  The fixture pins the oracle (oracle/glm4_ref.py)
to the reference's composition of operations: where it rounds to bf16, adds
biases and residuals, splits RoPE halves, builds masks and loops greedily.

    python tests/golden/make_golden.py --reference PATH
    (or with JSX_REFERENCE_DIR=PATH in the environment)

Inputs are seeded; model weights come from oracle.glm4_ref.init_params (a
checksum of them is stored so a drift of the numpy generator is detected).
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def params_checksum(p) -> str:
    h = hashlib.sha256()
    arrs = [p.embed] + [getattr(lp, n) for lp in p.layers for n in
                        ("ln1", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "ln2", "wg", "wu", "wd")]
    arrs += [p.norm, p.lm_head]
    for a in arrs:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("JSX_REFERENCE_DIR"),
                    help="checkout of the reference (default: $JSX_REFERENCE_DIR)")
    ap.add_argument("--out", default=os.path.join(HERE, "reference_golden.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference PATH (or JSX_REFERENCE_DIR) is required")

    sys.path.insert(0, os.path.join(HERE, "jaxshim"))
    sys.path.insert(1, args.reference)
    sys.path.insert(2, ROOT)
    import ml_dtypes

    from configs.model_config import ModelConfig  # reference
    from layers.attention import GQAAttention  # reference
    from layers.kv_cache import init_kv_caches  # reference
    from layers.linear import LinearBase  # reference
    from layers.moe import MoEGate  # reference
    from layers.normalization import RMSNorm  # reference
    from layers.rotary import RotaryEmbedding  # reference
    from models.glm4 import GLM4ForCausalLM  # reference
    import runner  # reference

    from oracle import glm4_ref as ref

    BF = ml_dtypes.bfloat16
    rng = np.random.default_rng(2024)

    def rnd(shape, std=1.0):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(BF)

    out = {}
    eps = 1.5625e-07

    # RMSNorm (layers/normalization.py)
    x = rnd((3, 5, 256), 2.0)
    norm = RMSNorm(256, epsilon=eps, param_dtype=BF)
    norm.scale.value = rnd((256,), 1.0)
    out.update(rms_x=x, rms_scale=norm.scale.value, rms_y=norm(x))

    # LinearBase with bias (layers/linear.py), no mesh
    lin = LinearBase(256, 96, None, use_bias=True, params_dtype=BF)
    lin.weight.value = rnd((256, 96), 0.05)
    lin.bias.value = rnd((96,), 0.05)
    xl = rnd((2, 3, 256))
    out.update(lin_x=xl, lin_w=lin.weight.value, lin_b=lin.bias.value, lin_y=lin(xl))

    # RotaryEmbedding (layers/rotary.py)
    rope = RotaryEmbedding(head_dim=128, rope_theta=10000.0, dtype=BF)
    pos = np.array([0, 1, 7, 300, 1023, 4095], np.int32)
    q = rnd((6, 4, 128))
    k = rnd((6, 2, 128))
    qo, ko = rope(pos, q, k)
    out.update(rope_pos=pos, rope_q=q, rope_k=k, rope_qo=qo, rope_ko=ko)

    # GQAAttention prefill into a static cache, then one decode step (layers/attention.py)
    att = GQAAttention(256, 4, 2, 128, 4096, 10000.0, None, attention_bias=True, dtype=BF)
    for name, (i, o) in {"q_proj": (256, 512), "k_proj": (256, 256), "v_proj": (256, 256),
                         "o_proj": (512, 256)}.items():
        lay = getattr(att, name)
        lay.weight.value = rnd((i, o), 0.05)
        if lay.bias is not None:
            lay.bias.value = rnd((o,), 0.05)
        out[f"att_{name}_w"] = lay.weight.value
        if lay.bias is not None:
            out[f"att_{name}_b"] = lay.bias.value
    B, S, L = 2, 5, 12
    hs = rnd((B, S, 256))
    caches = init_kv_caches(B, L, 1, 2, 128, dtype=BF, mesh=None)
    mask = runner.make_prefill_mask(S, L, dtype=BF)
    y, c1 = att(hs, runner.make_positions(S, B), mask, kv_cache=caches[0],
                cache_position=np.arange(S, dtype=np.int32))
    hd1 = rnd((B, 1, 256))
    y2, c2 = att(hd1, np.full((B, 1), S, np.int32), runner.make_decode_mask(S, L, dtype=BF),
                 kv_cache=c1, cache_position=np.array([S], np.int32))
    out.update(att_h=hs, att_y=y, att_h2=hd1, att_y2=y2, att_k=c2.k, att_v=c2.v)

    # MoEGate (layers/moe.py), with and without a correction bias
    gate = MoEGate(256, 64, 4, 1.8, True, None, dtype=BF)
    gate.weight.weight.value = rnd((256, 64), 0.05)
    xg = rnd((2, 7, 256))
    gate.e_score_correction_bias.value = np.zeros(64, np.float32)
    w0, i0 = gate(xg)
    gate.e_score_correction_bias.value = (rng.standard_normal(64).astype(np.float32) * np.float32(1e-3))
    w1, i1 = gate(xg)
    out.update(moe_x=xg, moe_w=gate.weight.weight.value, moe_bias=gate.e_score_correction_bias.value,
               moe_w0=w0, moe_i0=i0, moe_w1=w1, moe_i1=i1)

    # Full model + greedy generation (models/glm4.py, runner.py)
    rc = ref.GLMConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=128, intermediate_size=384, vocab_size=1000)
    p = ref.init_params(rc, seed=0)
    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=128, intermediate_size=384, vocab_size=1000)
    model = GLM4ForCausalLM(cfg, None, dtype=BF)
    m = model.model
    m.embed_tokens.embedding.value = p.embed.astype(BF)
    for lay, lp in zip(m.layers, p.layers):
        a = lay.self_attn
        a.q_proj.weight.value, a.q_proj.bias.value = lp.wq.astype(BF), lp.bq.astype(BF)
        a.k_proj.weight.value, a.k_proj.bias.value = lp.wk.astype(BF), lp.bk.astype(BF)
        a.v_proj.weight.value, a.v_proj.bias.value = lp.wv.astype(BF), lp.bv.astype(BF)
        a.o_proj.weight.value = lp.wo.astype(BF)
        lay.mlp.gate_proj.weight.value = lp.wg.astype(BF)
        lay.mlp.up_proj.weight.value = lp.wu.astype(BF)
        lay.mlp.down_proj.weight.value = lp.wd.astype(BF)
        lay.input_layernorm.scale.value = lp.ln1.astype(BF)
        lay.post_attention_layernorm.scale.value = lp.ln2.astype(BF)
    m.norm.scale.value = p.norm.astype(BF)
    model.lm_head.embedding.value = p.lm_head.astype(BF)
    prompt = np.random.default_rng(1).integers(0, 1000, (2, 7)).astype(np.int32)
    gen = runner.greedy_generate(model, prompt, max_new_tokens=6, max_cache_len=16)
    # logits of the prefill's last position and of the first decode step
    kv = init_kv_caches(2, 16, 2, 2, 128, dtype=BF, mesh=None)
    lg, kv = model(prompt, runner.make_positions(7, 2), runner.make_prefill_mask(7, 16, dtype=BF),
                   kv_caches=kv, cache_position=np.arange(7, dtype=np.int32))
    nxt = np.asarray(gen[:, 7:8], np.int32)
    lg2, kv = model(nxt, np.full((2, 1), 7, np.int32), runner.make_decode_mask(7, 16, dtype=BF),
                    kv_caches=kv, cache_position=np.array([7], np.int32))
    out.update(model_prompt=prompt, model_gen=np.asarray(gen), model_prefill_logits=lg[:, -1],
               model_decode_logits=lg2[:, -1], model_params_sha256=np.array(params_checksum(p)))

    # MoELayer without expert parallelism (layers/moe.py:156-192, _topk_local_forward
    # :247-267, SharedExpertMLP :110-113), 8 experts, top-4.  A mesh object whose
    # "expert" axis has size 1 selects the local path.
    from jax.sharding import Mesh
    from layers.moe import MoELayer  # reference
    mesh1 = Mesh()
    mesh1.shape = {"expert": 1}
    E, Hm, Im, Is = 8, 128, 64, 64
    moe = MoELayer(Hm, Im, Is, E, 4, 1.8, True, mesh1, dtype=BF)
    moe.gate.weight.weight.value = rnd((Hm, E), 0.05)
    moe.gate.e_score_correction_bias.value = (rng.standard_normal(E).astype(np.float32) * np.float32(1e-3))
    moe.expert_gate_weight.value = rnd((E, Hm, Im), 0.05)
    moe.expert_up_weight.value = rnd((E, Hm, Im), 0.05)
    moe.expert_down_weight.value = rnd((E, Im, Hm), 0.05)
    moe.shared_experts.gate_proj.weight.value = rnd((Hm, Is), 0.05)
    moe.shared_experts.up_proj.weight.value = rnd((Hm, Is), 0.05)
    moe.shared_experts.down_proj.weight.value = rnd((Is, Hm), 0.05)
    xm = rnd((2, 5, Hm))
    out.update(moel_x=xm, moel_router=moe.gate.weight.weight.value,
               moel_bias=moe.gate.e_score_correction_bias.value,
               moel_eg=moe.expert_gate_weight.value, moel_eu=moe.expert_up_weight.value,
               moel_ed=moe.expert_down_weight.value, moel_sg=moe.shared_experts.gate_proj.weight.value,
               moel_su=moe.shared_experts.up_proj.weight.value, moel_sd=moe.shared_experts.down_proj.weight.value,
               moel_y=moe(xm))

    # MLAAttention (layers/mla_attention.py): prefill into an expanded per-head cache,
    # then one decode step; 4 heads, q_lora 96, kv_lora 64, nope 48 + rope 16, v 64.
    from layers.mla_attention import MLAAttention  # reference
    mla = MLAAttention(256, 4, 96, 64, 48, 16, 64, 4096, 1000000.0, eps, None, dtype=BF)
    for name, shp in {"q_a_proj": (256, 96), "q_b_proj": (96, 4 * 64), "kv_a_proj_with_mqa": (256, 64 + 16),
                      "kv_b_proj": (64, 4 * (48 + 64)), "o_proj": (4 * 64, 256)}.items():
        getattr(mla, name).weight.value = rnd(shp, 0.05)
        out[f"mla_{name}"] = getattr(mla, name).weight.value
    mla.q_a_layernorm.scale.value = rnd((96,), 1.0)
    mla.kv_a_layernorm.scale.value = rnd((64,), 1.0)
    out.update(mla_q_a_ln=mla.q_a_layernorm.scale.value, mla_kv_a_ln=mla.kv_a_layernorm.scale.value)
    B, S, L = 2, 5, 12
    hm = rnd((B, S, 256))
    from layers.kv_cache import KVCache  # reference
    cache = KVCache(k=np.zeros((B, L, 4, 64), BF), v=np.zeros((B, L, 4, 64), BF))
    ym, cm = mla(hm, runner.make_positions(S, B), runner.make_prefill_mask(S, L, dtype=BF), kv_cache=cache,
                 cache_position=np.arange(S, dtype=np.int32))
    hm2 = rnd((B, 1, 256))
    ym2, cm2 = mla(hm2, np.full((B, 1), S, np.int32), runner.make_decode_mask(S, L, dtype=BF), kv_cache=cm,
                   cache_position=np.array([S], np.int32))
    out.update(mla_h=hm, mla_y=ym, mla_h2=hm2, mla_y2=ym2, mla_k=cm2.k, mla_v=cm2.v)

    # GLM-4.7-Flash model (models/glm4_flash.py): MLA in every layer, a dense MLP in layer 0,
    # MoE (8 experts, top-4, shared expert of 64) in layers 1-2; a 4-token prefill and one
    # decode step through the reference's own model class
    from models.glm4_flash import GLM4FlashForCausalLM  # reference
    fcfg = ModelConfig(hidden_size=256, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=4,
                       intermediate_size=192, vocab_size=1000, rms_norm_eps=1e-5, rope_theta=1000000.0,
                       n_routed_experts=8, n_shared_experts=1, num_experts_per_tok=4, moe_intermediate_size=64,
                       routed_scaling_factor=1.8, norm_topk_prob=True, first_k_dense_replace=1, q_lora_rank=96,
                       kv_lora_rank=64, qk_nope_head_dim=48, qk_rope_head_dim=16, v_head_dim=64,
                       attention_bias=False)
    fm = GLM4FlashForCausalLM(fcfg, mesh1, dtype=BF)
    fm.model.embed_tokens.embedding.value = rnd((1000, 256), 0.05)
    out["flash_embed"] = fm.model.embed_tokens.embedding.value
    for i, lay in enumerate(fm.model.layers):
        at = lay.self_attn
        for name, shp in {"q_a_proj": (256, 96), "q_b_proj": (96, 4 * 64), "kv_a_proj_with_mqa": (256, 64 + 16),
                          "kv_b_proj": (64, 4 * (48 + 64)), "o_proj": (4 * 64, 256)}.items():
            getattr(at, name).weight.value = rnd(shp, 0.05)
            out[f"flash_{i}_{name}"] = getattr(at, name).weight.value
        if i == 0:
            for name, shp in {"gate_proj": (256, 192), "up_proj": (256, 192), "down_proj": (192, 256)}.items():
                getattr(lay.mlp, name).weight.value = rnd(shp, 0.05)
                out[f"flash_{i}_{name}"] = getattr(lay.mlp, name).weight.value
        else:
            mo = lay.mlp
            mo.gate.weight.weight.value = rnd((256, 8), 0.05)
            mo.expert_gate_weight.value = rnd((8, 256, 64), 0.05)
            mo.expert_up_weight.value = rnd((8, 256, 64), 0.05)
            mo.expert_down_weight.value = rnd((8, 64, 256), 0.05)
            mo.shared_experts.gate_proj.weight.value = rnd((256, 64), 0.05)
            mo.shared_experts.up_proj.weight.value = rnd((256, 64), 0.05)
            mo.shared_experts.down_proj.weight.value = rnd((64, 256), 0.05)
            out.update({f"flash_{i}_router": mo.gate.weight.weight.value, f"flash_{i}_eg": mo.expert_gate_weight.value,
                        f"flash_{i}_eu": mo.expert_up_weight.value, f"flash_{i}_ed": mo.expert_down_weight.value,
                        f"flash_{i}_sg": mo.shared_experts.gate_proj.weight.value,
                        f"flash_{i}_su": mo.shared_experts.up_proj.weight.value,
                        f"flash_{i}_sd": mo.shared_experts.down_proj.weight.value})
    fm.lm_head.embedding.value = rnd((1000, 256), 0.05)
    out["flash_lm_head"] = fm.lm_head.embedding.value
    Bf, Sf, Lf = 2, 4, 8
    fprompt = np.random.default_rng(3).integers(0, 1000, (Bf, Sf)).astype(np.int32)
    fkv = [KVCache(k=np.zeros((Bf, Lf, 4, 64), BF), v=np.zeros((Bf, Lf, 4, 64), BF)) for _ in range(3)]
    flg, fkv = fm(fprompt, runner.make_positions(Sf, Bf), runner.make_prefill_mask(Sf, Lf, dtype=BF),
                  kv_caches=fkv, cache_position=np.arange(Sf, dtype=np.int32))
    fnext = np.argmax(np.asarray(flg[:, -1], np.float32), axis=-1).astype(np.int32)[:, None]
    flg2, fkv = fm(fnext, np.full((Bf, 1), Sf, np.int32), runner.make_decode_mask(Sf, Lf, dtype=BF),
                   kv_caches=fkv, cache_position=np.array([Sf], np.int32))
    out.update(flash_prompt=fprompt, flash_logits=flg, flash_next=fnext, flash_logits2=flg2)

    # Sampling step (runner.py:315-359, _jit_sample): penalty, temperature, top-k, top-p and the
    # categorical draw, the draw's Gumbel noise carried by the key (jaxshim NoiseKey)
    from jax import random as jrandom
    Bs, Vs = 4, 3000
    s_logits = rnd((Bs, Vs), 2.0)
    s_pres = (rng.random((Bs, Vs)) < 0.05).astype(np.float32)
    out.update(samp_logits=s_logits, samp_presence=s_pres)
    for j, (rp, temp, tk, tp) in enumerate(((1.1, 0.8, 0, 0.8), (1.3, 1.0, 50, 1.0), (1.0, 1.5, 10, 0.5))):
        kk = tk if tk > 0 else 200
        noise = (-np.log(-np.log(rng.random((Bs, kk))))).astype(np.float32).astype(BF)
        # a Python float meeting a bf16 array stays bf16 in JAX (weak typing): the scalars
        # are given as bf16 values so that numpy keeps the reference's arithmetic in bf16
        tok, _ = runner._jit_sample(s_logits, s_pres, jrandom.NoiseKey(noise), BF(rp), BF(temp), tk, tp)
        out[f"samp{j}_noise"] = noise
        out[f"samp{j}_tokens"] = np.asarray(tok).reshape(-1)
        out[f"samp{j}_params"] = np.array([rp, temp, tk, tp], np.float64)

    ser = {}
    for k_, v in out.items():
        v = np.asarray(v)
        ser[k_] = v.astype(np.float32) if v.dtype == BF else v
    np.savez_compressed(args.out, **ser)
    print(f"wrote {args.out}: {len(ser)} arrays, {os.path.getsize(args.out)} bytes")


if __name__ == "__main__":
    main()
