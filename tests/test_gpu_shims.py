"""The reference-API layers (the drop-in boundary) driven directly: GQAAttention
(layers/attention.py) against the reference's own recorded outputs
(tests/golden/reference_golden.npz, GQAAttention prefill + decode into a static
cache) and, for the one-pass prompt path, against the oracle's attention (pinned
to the same recording); LinearBase with a bias against the recorded
LinearBase output.  Row-parallel LinearBase with a bias runs across ranks in
tests/test_gpu_tp.py.  Bar: max relative error 2e-2, cosine 0.999."""

import importlib
import os

import numpy as np
import pytest
import torch

from test_gpu_ops import bf, npf

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_golden.npz")


def within(got, want, tol=2e-2, cos_min=0.999):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.max(np.abs(got - want)) / np.max(np.abs(want))
    cos = float(np.sum(got * want) / (np.linalg.norm(got) * np.linalg.norm(want)))
    assert err <= tol and cos >= cos_min, (err, cos)


def make_gqa(g):
    mod = importlib.import_module("e2e-jaxscale_b200.layers.attention")
    att = mod.GQAAttention(256, 4, 2, 128, 4096, 10000.0, None, attention_bias=True)
    for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
        lay = getattr(att, name)
        lay.weight.value = g[f"att_{name}_w"]
        if lay.bias is not None:
            lay.bias.value = g[f"att_{name}_b"]
    return att


def test_gqa_attention_matches_reference_recording(jsx, cuda):
    g = np.load(GOLDEN)
    att = make_gqa(g)
    KV = importlib.import_module("e2e-jaxscale_b200.layers.kv_cache")
    B, S, L = 2, 5, 12
    cache = KV.init_kv_caches(B, L, 1, 2, 128, device=cuda)[0]
    pos = torch.arange(S, dtype=torch.int32).expand(B, S)
    y, cache = att(bf(g["att_h"], cuda), pos, None, kv_cache=cache, cache_position=torch.arange(S))
    within(npf(y), g["att_y"])
    y2, cache = att(bf(g["att_h2"], cuda), torch.full((B, 1), S, dtype=torch.int32), None, kv_cache=cache,
                    cache_position=torch.tensor([S]))
    within(npf(y2), g["att_y2"])
    within(npf(cache.k), g["att_k"])
    within(npf(cache.v), g["att_v"])
    # the same call again reuses the layer's workspace and scratch buffers
    n = len(att._bufs)
    att(bf(g["att_h2"], cuda), torch.full((B, 1), S, dtype=torch.int32), None, kv_cache=cache,
        cache_position=torch.tensor([S]))
    assert len(att._bufs) == n


def test_gqa_attention_one_pass_prompt(jsx, ref, cuda):
    """A 2 x 40-token prompt (80 tokens: the one-pass tensor-core path) then a decode
    step, against the oracle's GQAAttention restatement with the recorded weights."""
    g = np.load(GOLDEN)
    att = make_gqa(g)
    cfg = ref.GLMConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=128)
    lp = ref.LayerParams(ln1=None, wq=g["att_q_proj_w"], bq=g["att_q_proj_b"], wk=g["att_k_proj_w"],
                         bk=g["att_k_proj_b"], wv=g["att_v_proj_w"], bv=g["att_v_proj_b"],
                         wo=g["att_o_proj_w"], ln2=None, wg=None, wu=None, wd=None)
    rng = np.random.default_rng(17)
    B, S, L = 2, 40, 48
    x = ref.bf16(rng.standard_normal((B, S, 256), dtype=np.float32))
    x2 = ref.bf16(rng.standard_normal((B, 1, 256), dtype=np.float32))
    inv = ref.rope_inv_freq(128)
    kc = np.zeros((B, L, 2, 128), np.float32)
    vc = np.zeros_like(kc)
    pos = np.broadcast_to(np.arange(S), (B, S))
    want = ref.attention(lp, cfg, x, pos, ref.make_prefill_mask(S, L), (kc, vc), np.arange(S), inv)
    want2 = ref.attention(lp, cfg, x2, np.full((B, 1), S), ref.make_decode_mask(S, L), (kc, vc), np.array([S]), inv)
    KV = importlib.import_module("e2e-jaxscale_b200.layers.kv_cache")
    cache = KV.init_kv_caches(B, L, 1, 2, 128, device=cuda)[0]
    y, cache = att(bf(x, cuda), torch.from_numpy(np.ascontiguousarray(pos, np.int32)), None, kv_cache=cache,
                   cache_position=torch.arange(S))
    assert any(k[0] == "wide" for k in att._bufs)
    within(npf(y), want)
    y2, cache = att(bf(x2, cuda), torch.full((B, 1), S, dtype=torch.int32), None, kv_cache=cache,
                    cache_position=torch.tensor([S]))
    within(npf(y2), want2)
    within(npf(cache.k), kc)
    within(npf(cache.v), vc)


def test_linear_with_bias_matches_reference_recording(jsx, cuda):
    g = np.load(GOLDEN)
    mod = importlib.import_module("e2e-jaxscale_b200.layers.linear")
    lin = mod.LinearBase(256, 96, None, use_bias=True, kernel_axes=(None, "tensor"))
    lin.weight.value = g["lin_w"]
    lin.bias.value = g["lin_b"]
    y = lin(bf(g["lin_x"], cuda))
    within(npf(y), g["lin_y"])
