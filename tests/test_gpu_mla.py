"""MLA attention (GLM-4.7-Flash, layers/mla_attention.py) on the library's kernels
against the reference's own outputs (tests/golden, recorded from MLAAttention) and
against the oracle (oracle/glm4_ref.py mla_attention, pinned to those outputs) at
the GLM-4.7-Flash widths.  Bar: max relative error <= 2e-2 and cosine >= 0.999
(the reference rounds q.k to bf16 before the softmax; the kernel keeps fp32)."""

import importlib
import os

import numpy as np
import pytest
import torch

from test_gpu_ops import bf, close, npf, rand_bf16

pytestmark = pytest.mark.gpu


def within(got, want, tol=2e-2, cos_min=0.999):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.max(np.abs(got - want)) / np.max(np.abs(want))
    cos = float(np.sum(got * want) / (np.linalg.norm(got) * np.linalg.norm(want)))
    assert err <= tol and cos >= cos_min, (err, cos)


def make_layer(jsx, H, nh, ql, kl, nope, rope, vd, theta, eps, p, dev):
    mod = importlib.import_module("e2e-jaxscale_b200.layers.mla_attention")
    m = mod.MLAAttention(H, nh, ql, kl, nope, rope, vd, 4096, theta, eps, None)
    m.q_a_proj.weight.value = p.q_a
    m.q_a_layernorm.scale.value = p.q_a_ln
    m.q_b_proj.weight.value = p.q_b
    m.kv_a_proj_with_mqa.weight.value = p.kv_a
    m.kv_a_layernorm.scale.value = p.kv_a_ln
    m.kv_b_proj.weight.value = p.kv_b
    m.o_proj.weight.value = p.o
    return m


def test_mla_matches_reference_golden(jsx, ref, cuda):
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_golden.npz"))
    p = ref.MLAParams(q_a=g["mla_q_a_proj"], q_a_ln=g["mla_q_a_ln"], q_b=g["mla_q_b_proj"],
                      kv_a=g["mla_kv_a_proj_with_mqa"], kv_a_ln=g["mla_kv_a_ln"], kv_b=g["mla_kv_b_proj"],
                      o=g["mla_o_proj"])
    layer = make_layer(jsx, 256, 4, 96, 64, 48, 16, 64, 1000000.0, 1.5625e-07, p, cuda)
    KV = importlib.import_module("e2e-jaxscale_b200.layers.kv_cache").KVCache
    B, S, L = 2, 5, 12
    cache = KV(torch.zeros(B, L, 4, 64, dtype=torch.bfloat16, device=cuda),
               torch.zeros(B, L, 4, 64, dtype=torch.bfloat16, device=cuda))
    pos = np.broadcast_to(np.arange(S), (B, S))
    y, cache = layer(bf(g["mla_h"], cuda), pos, None, kv_cache=cache, cache_position=np.arange(S))
    within(npf(y), g["mla_y"])
    y2, cache = layer(bf(g["mla_h2"], cuda), np.full((B, 1), S), None, kv_cache=cache, cache_position=[S])
    within(npf(y2), g["mla_y2"])
    within(npf(cache.k), g["mla_k"])
    within(npf(cache.v), g["mla_v"])


def test_mla_flash_shapes(jsx, ref, cuda):
    """GLM-4.7-Flash: hidden 2048, 20 heads, q_lora 768, kv_lora 512, nope 192 + rope 64, v 256,
    theta 1e6; batch 2, a 4-token prefill and one decode step."""
    rng = np.random.default_rng(31)
    H, nh, ql, kl, nope, rope, vd = 2048, 20, 768, 512, 192, 64, 256
    p = ref.MLAParams(q_a=rand_bf16(ref, rng, (H, ql), 0.02), q_a_ln=rand_bf16(ref, rng, (ql,), 1.0),
                      q_b=rand_bf16(ref, rng, (ql, nh * (nope + rope)), 0.02), kv_a=rand_bf16(ref, rng, (H, kl + rope), 0.02),
                      kv_a_ln=rand_bf16(ref, rng, (kl,), 1.0), kv_b=rand_bf16(ref, rng, (kl, nh * (nope + vd)), 0.02),
                      o=rand_bf16(ref, rng, (nh * vd, H), 0.02))
    eps = 1e-5
    layer = make_layer(jsx, H, nh, ql, kl, nope, rope, vd, 1000000.0, eps, p, cuda)
    KV = importlib.import_module("e2e-jaxscale_b200.layers.kv_cache").KVCache
    B, S, L = 2, 4, 16
    kc = np.zeros((B, L, nh, nope + rope), np.float32)
    vc = np.zeros((B, L, nh, vd), np.float32)
    cache = KV(torch.zeros(B, L, nh, nope + rope, dtype=torch.bfloat16, device=cuda),
               torch.zeros(B, L, nh, vd, dtype=torch.bfloat16, device=cuda))
    inv = ref.rope_inv_freq(rope, theta=1000000.0, partial=1.0)
    x = rand_bf16(ref, rng, (B, S, H), 1.0)
    pos = np.broadcast_to(np.arange(S), (B, S))
    want = ref.mla_attention(p, x, pos, ref.make_prefill_mask(S, L), (kc, vc), np.arange(S), nh, nope, rope, vd,
                             eps, inv)
    y, cache = layer(bf(x, cuda), pos, None, kv_cache=cache, cache_position=np.arange(S))
    within(npf(y), want)
    x2 = rand_bf16(ref, rng, (B, 1, H), 1.0)
    want2 = ref.mla_attention(p, x2, np.full((B, 1), S), ref.make_decode_mask(S, L), (kc, vc), [S], nh, nope, rope,
                              vd, eps, inv)
    y2, cache = layer(bf(x2, cuda), np.full((B, 1), S), None, kv_cache=cache, cache_position=[S])
    within(npf(y2), want2)
    within(npf(cache.k), kc)
    within(npf(cache.v), vc)


def test_mla_rope_cache_kernel(jsx, ref, cuda):
    """The RoPE + concatenation + cache write step alone, against the oracle's rope()."""
    rng = np.random.default_rng(3)
    M, nh, nope, rope, vd, L = 3, 4, 48, 16, 64, 20
    q_in = rand_bf16(ref, rng, (M, nh, nope + rope))
    kv_in = rand_bf16(ref, rng, (M, nh, nope + vd))
    k_rope = rand_bf16(ref, rng, (M, rope))
    pos = np.array([0, 7, 19], np.int32)
    inv = ref.rope_inv_freq(rope, theta=1000000.0, partial=1.0)
    K = jsx.kernels
    q_out = torch.empty(M, nh, nope + rope, dtype=torch.bfloat16, device=cuda)
    kc = torch.zeros(M, L, nh, nope + rope, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros(M, L, nh, vd, dtype=torch.bfloat16, device=cuda)
    K.mla_rope_cache(bf(q_in, cuda), bf(kv_in, cuda), bf(k_rope, cuda), torch.from_numpy(inv).to(cuda),
                     torch.from_numpy(pos).to(cuda), q_out, kc, vc, nh, nope, rope, vd)
    qr, kr = ref.rope(pos, q_in[..., nope:], np.broadcast_to(k_rope[:, None, :], (M, nh, rope)), inv)
    close(npf(q_out)[..., nope:], qr, exact_min=0.98)
    assert np.array_equal(npf(q_out)[..., :nope], q_in[..., :nope])
    kcn, vcn = npf(kc), npf(vc)
    for m, p_ in enumerate(pos):
        assert np.array_equal(kcn[m, p_, :, :nope], kv_in[m, :, :nope])
        close(kcn[m, p_, :, nope:], kr[m], exact_min=0.98)
        assert np.array_equal(vcn[m, p_], kv_in[m, :, nope:])


# ---------------------------------------------------------------------------
# absorbed-weight (latent-cache) decode form
# ---------------------------------------------------------------------------

def _mla_flash_params(ref, rng, H=2048, nh=20, ql=768, kl=512, nope=192, rope=64, vd=256):
    return ref.MLAParams(q_a=rand_bf16(ref, rng, (H, ql), 0.02), q_a_ln=rand_bf16(ref, rng, (ql,), 1.0),
                         q_b=rand_bf16(ref, rng, (ql, nh * (nope + rope)), 0.02),
                         kv_a=rand_bf16(ref, rng, (H, kl + rope), 0.02), kv_a_ln=rand_bf16(ref, rng, (kl,), 1.0),
                         kv_b=rand_bf16(ref, rng, (kl, nh * (nope + vd)), 0.02),
                         o=rand_bf16(ref, rng, (nh * vd, H), 0.02))


@pytest.mark.parametrize("nh", [20, 10])
def test_mla_absorbed_flash_shapes(jsx, ref, cuda, nh):
    """MLAAttention(absorbed=True) at the GLM-4.7-Flash widths (20 heads: TP=1, two
    16-row head tiles; 10 heads: the TP=2 shard, one tile): a 4-token prefill and a
    decode step against the oracle's latent form (mla_attention_absorbed) and the
    reference's expanded form (mla_attention); the latent cache rows against the
    oracle's."""
    rng = np.random.default_rng(41 + nh)
    H, ql, kl, nope, rope, vd = 2048, 768, 512, 192, 64, 256
    p = _mla_flash_params(ref, rng, H, nh, ql, kl, nope, rope, vd)
    eps = 1e-5
    mod = importlib.import_module("e2e-jaxscale_b200.layers.mla_attention")
    layer = mod.MLAAttention(H, nh, ql, kl, nope, rope, vd, 4096, 1000000.0, eps, None, absorbed=True)
    for name, val in (("q_a_proj", p.q_a), ("q_b_proj", p.q_b), ("kv_a_proj_with_mqa", p.kv_a),
                      ("kv_b_proj", p.kv_b), ("o_proj", p.o)):
        getattr(layer, name).weight.value = val
    layer.q_a_layernorm.scale.value = p.q_a_ln
    layer.kv_a_layernorm.scale.value = p.kv_a_ln
    B, S, L = 2, 4, 16
    cache = layer.init_latent_cache(B, L, cuda)
    lat = np.zeros((B, L, kl + rope), np.float32)
    kc = np.zeros((B, L, nh, nope + rope), np.float32)
    vc = np.zeros((B, L, nh, vd), np.float32)
    inv = ref.rope_inv_freq(rope, theta=1000000.0, partial=1.0)
    x = rand_bf16(ref, rng, (B, S, H), 1.0)
    x2 = rand_bf16(ref, rng, (B, 1, H), 1.0)
    pos = np.broadcast_to(np.arange(S), (B, S))
    for xi, pi, mask, cp in ((x, pos, ref.make_prefill_mask(S, L), np.arange(S)),
                             (x2, np.full((B, 1), S), ref.make_decode_mask(S, L), [S])):
        want_lat = ref.mla_attention_absorbed(p, xi, pi, mask, lat, cp, nh, nope, rope, vd, eps, inv)
        want_exp = ref.mla_attention(p, xi, pi, mask, (kc, vc), cp, nh, nope, rope, vd, eps, inv)
        y, cache = layer(bf(xi, cuda), pi, None, kv_cache=cache, cache_position=cp)
        within(npf(y), want_lat)
        within(npf(y), want_exp)
    within(npf(cache.k), lat)


@pytest.mark.parametrize("nh,B,L,pos", [
    (20, 3, 1100, [1024, 37, 1099]),   # 18 splits, two head tiles
    (10, 2, 200, [0, 130]),            # the first row alone; 3 splits
    (16, 1, 64, [63]),                 # one full split
])
def test_mla_decode_kernel(jsx, ref, cuda, nh, B, L, pos):
    """jsx_mla_decode alone (split context + merge) against the oracle's latent
    attention step on random latent rows, at long context."""
    rng = np.random.default_rng(7)
    kl, rope = 512, 64
    K = jsx.kernels
    q_abs = rand_bf16(ref, rng, (B, nh, kl), 0.2)
    q_rope = rand_bf16(ref, rng, (B, nh, rope), 1.0)
    lat = rand_bf16(ref, rng, (B, L, kl + rope), 1.0)
    scale = (192 + 64) ** -0.5
    ctx = torch.full((B, nh, kl), float("nan"), dtype=torch.bfloat16, device=cuda)
    ws = K.mla_decode_workspace(B, nh, kl, L, cuda)
    K.mla_decode(bf(q_abs, cuda), bf(q_rope, cuda), bf(lat, cuda), ctx,
                 torch.tensor(pos, dtype=torch.int32, device=cuda), scale, ws)
    got = npf(ctx)
    for b, cur in enumerate(pos):
        mask = ref.make_decode_mask(cur, L)
        want = ref.mla_latent_attention(q_abs[b:b + 1, None], q_rope[b:b + 1, None], lat[b:b + 1], mask, scale)
        within(got[b], want[0, 0])


@pytest.mark.parametrize("M,nh,R,K", [(1, 20, 512, 192), (5, 10, 256, 512), (32, 20, 512, 192), (9, 3, 70, 40)])
def test_mla_absorb_kernel(jsx, ref, cuda, M, nh, R, K):
    """jsx_mla_absorb (per-head GEMV) against fp32 numpy, with a strided x (q_nope
    inside the q rows of width nope + rope)."""
    rng = np.random.default_rng(M * 100 + nh)
    width = K + 64
    x = rand_bf16(ref, rng, (M, nh, width), 1.0)
    w = rand_bf16(ref, rng, (nh, R, K), 0.05)
    out = torch.empty(M, nh, R, dtype=torch.bfloat16, device=cuda)
    jsx.kernels.mla_absorb(bf(x, cuda), nh * width, width, bf(w, cuda), out, M, nh, R, K)
    want = ref.bf16(np.einsum("mhk,hrk->mhr", x[..., :K], w, dtype=np.float32))
    close(npf(out), want, exact_min=0.95)


def test_flash_model_absorbed_matches_expanded_oracle(jsx, ref, cuda):
    """GLM4FlashForCausalLM(absorbed_mla=True) at reduced width (kv_lora 256) against the
    oracle's flash_forward, which composes the reference's expanded MLA: a 4-token prompt
    and one decode step, model-level tolerance on the logits."""
    from test_gpu_flash import oracle_params, small_flash_config
    c = small_flash_config(jsx)
    c.kv_lora_rank = 256
    model = jsx.GLM4FlashForCausalLM(c, jsx.create_mesh(1), absorbed_mla=True)
    model.init_random(seed=5, std=0.05)
    p = oracle_params(ref, model, c)
    B, S, L = 2, 4, 8
    ids = np.random.default_rng(6).integers(0, c.vocab_size, (B, S))
    pos = np.broadcast_to(np.arange(S), (B, S))
    caches = model.init_kv_caches(B, L)
    assert caches[0].k.shape == (B, L, 256 + 16)
    logits, caches = model(ids, pos, None, kv_caches=caches, cache_position=np.arange(S))
    qd = c.qk_nope_head_dim + c.qk_rope_head_dim
    kv = [(np.zeros((B, L, c.num_attention_heads, qd), np.float32),
           np.zeros((B, L, c.num_attention_heads, c.v_head_dim), np.float32)) for _ in range(c.num_hidden_layers)]
    want = ref.flash_forward(p, ids, pos, ref.make_prefill_mask(S, L), kv, np.arange(S))
    within(npf(logits), want)
    nxt = ref.argmax_first(want[:, -1])
    logits2, _ = model(nxt[:, None], np.full((B, 1), S), None, kv_caches=caches, cache_position=[S])
    want2 = ref.flash_forward(p, nxt[:, None], np.full((B, 1), S), ref.make_decode_mask(S, L), kv, [S])
    within(npf(logits2), want2)
