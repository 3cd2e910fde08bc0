"""Self-consistency of the CPU oracle, mirroring the reference's own checks
(benchmarks/verify_kvcache.py) and the algebra the kernels rely on."""

import numpy as np
import pytest


def small(ref, layers=2):
    return ref.GLMConfig(hidden_size=128, num_hidden_layers=layers, num_attention_heads=4,
                         num_key_value_heads=2, head_dim=64, intermediate_size=192, vocab_size=300)


def test_cache_vs_no_cache_prefill(ref):
    """verify_kvcache.py:36-78: cached and uncached prefill agree (< 1e-3)."""
    rc = small(ref)
    p = ref.init_params(rc, seed=1)
    ids = np.random.default_rng(0).integers(0, rc.vocab_size, (2, 9))
    pos = np.broadcast_to(np.arange(9), (2, 9))
    kv = ref.init_kv_caches(rc, 2, 16)
    a = ref.forward(p, ids, pos, ref.make_prefill_mask(9, 16), kv, np.arange(9))
    causal = np.triu(np.full((9, 9), ref.NEG, np.float32), k=1)[None, None]
    b = ref.forward(p, ids, pos, causal, None, None)
    assert np.max(np.abs(a - b)) < 1e-3


def test_teacher_forced_decode_matches_recompute(ref):
    """verify_kvcache.py:81-183: decode with the cache vs full recompute (< 2.0, same tokens)."""
    rc = small(ref)
    p = ref.init_params(rc, seed=2)
    ids = np.random.default_rng(1).integers(0, rc.vocab_size, (1, 6))
    rec = []
    out = ref.greedy_generate(p, ids, 5, max_cache_len=16, record=rec)
    for t in range(1, 5):
        seq = out[:, :6 + t]
        S = seq.shape[1]
        causal = np.triu(np.full((S, S), ref.NEG, np.float32), k=1)[None, None]
        full = ref.forward(p, seq, np.broadcast_to(np.arange(S), (1, S)), causal, None, None)[:, -1]
        assert np.max(np.abs(full - rec[t][0])) < 2.0
        assert ref.argmax_first(full)[0] == out[0, 6 + t]


def test_masked_rows_contribute_nothing(ref):
    """The decode mask's -1e9 rows give exactly zero weight, so attending to rows
    [0, cur] only (what the kernel does) is the same function."""
    rng = np.random.default_rng(3)
    q = ref.bf16(rng.standard_normal((1, 1, 8, 64)))
    k = ref.bf16(rng.standard_normal((1, 40, 2, 64)))
    v = ref.bf16(rng.standard_normal((1, 40, 2, 64)))
    cur = 17
    full = ref.sdpa(q, k, v, ref.make_decode_mask(cur, 40), 64 ** -0.5)
    trunc = ref.sdpa(q, k[:, :cur + 1], v[:, :cur + 1], None, 64 ** -0.5)
    assert np.array_equal(full, trunc)


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_row_parallel_shards_sum_to_the_full_product(ref, tp):
    rng = np.random.default_rng(tp)
    x = ref.bf16(rng.standard_normal((3, 512)))
    w = ref.bf16(rng.standard_normal((512, 64)) * 0.02)
    xs = [ref.shard_columns(x, tp, r) for r in range(tp)]
    ws = [ref.shard_rows(w, tp, r) for r in range(tp)]
    y = ref.row_parallel_reference(xs, ws)
    full = ref.linear(x, w)
    assert np.max(np.abs(y - full)) <= 2 ** -7 * np.max(np.abs(full))


def test_rope_is_identity_at_position_zero(ref):
    rng = np.random.default_rng(4)
    q = ref.bf16(rng.standard_normal((1, 2, 128)))
    k = ref.bf16(rng.standard_normal((1, 1, 128)))
    qo, ko = ref.rope(np.array([0]), q, k, ref.rope_inv_freq(128))
    assert np.array_equal(qo, q) and np.array_equal(ko, k)


def test_moe_gate_weights(ref):
    rng = np.random.default_rng(5)
    x = ref.bf16(rng.standard_normal((10, 64)))
    w = ref.bf16(rng.standard_normal((64, 16)) * 0.1)
    wts, idx = ref.moe_gate(x, w, 4, 1.8, True)
    assert idx.shape == (10, 4) and len(set(idx[0])) == 4
    assert np.allclose(wts.sum(-1), 1.8, atol=0.03)
    logits = ref.linear(x, w)
    assert np.array_equal(idx[:, 0], np.argmax(logits, -1))


def test_argmax_ties_pick_first(ref):
    assert ref.argmax_first(np.array([[1.0, 3.0, 3.0, 2.0]]))[0] == 1


def test_sample_tokens_limits(ref):
    """The sampling restatement: zero noise and no filtering is the first argmax; a
    top-p that keeps only the leading candidate returns it whatever the noise."""
    rng = np.random.default_rng(0)
    lg = ref.bf16(rng.standard_normal((3, 500), dtype=np.float32))
    tok, _ = ref.sample_tokens(lg, None, np.zeros((3, 200), np.float32), 1.0, 1.0, 0, 1.0)
    assert np.array_equal(tok, ref.argmax_first(lg))
    noise = ref.bf16(rng.standard_normal((3, 10), dtype=np.float32) * np.float32(5.0))
    tok, _ = ref.sample_tokens(lg, None, noise, 1.0, 1.0, 10, 1e-6)
    assert np.array_equal(tok, ref.argmax_first(lg))


def test_mla_absorbed_matches_expanded(ref):
    """The latent-cache (absorbed) MLA form against the reference's expanded form
    (pinned by test_oracle_pin), GLM-4.7-Flash head shapes at reduced width: a
    5-token prefill then a decode step; the latent cache holds 64 + 16 values per
    token instead of 4 x (64 + 64)."""
    rng = np.random.default_rng(21)
    H, nh, ql, kl, nope, rd, vd = 256, 4, 96, 64, 48, 16, 64
    r = lambda *s_: ref.bf16(rng.standard_normal(s_, dtype=np.float32) * np.float32(0.05))
    p = ref.MLAParams(q_a=r(H, ql), q_a_ln=ref.bf16(1 + 0.1 * rng.standard_normal(ql).astype(np.float32)),
                      q_b=r(ql, nh * (nope + rd)), kv_a=r(H, kl + rd),
                      kv_a_ln=ref.bf16(1 + 0.1 * rng.standard_normal(kl).astype(np.float32)),
                      kv_b=r(kl, nh * (nope + vd)), o=r(nh * vd, H))
    inv = ref.rope_inv_freq(rd, theta=1000000.0, partial=1.0)
    B, S, L = 2, 5, 12
    x = ref.bf16(rng.standard_normal((B, S, H), dtype=np.float32))
    x2 = ref.bf16(rng.standard_normal((B, 1, H), dtype=np.float32))
    kv = (np.zeros((B, L, nh, nope + rd), np.float32), np.zeros((B, L, nh, vd), np.float32))
    lat = np.zeros((B, L, kl + rd), np.float32)
    pos = np.broadcast_to(np.arange(S), (B, S))
    for xi, pi, mask, cp in ((x, pos, ref.make_prefill_mask(S, L), np.arange(S)),
                             (x2, np.full((B, 1), S), ref.make_decode_mask(S, L), [S])):
        want = ref.mla_attention(p, xi, pi, mask, kv, cp, nh, nope, rd, vd, 1e-5, inv)
        got = ref.mla_attention_absorbed(p, xi, pi, mask, lat, cp, nh, nope, rd, vd, 1e-5, inv)
        err = np.max(np.abs(got - want)) / np.max(np.abs(want))
        cos = float(np.sum(got * want) / (np.linalg.norm(got) * np.linalg.norm(want)))
        assert err <= 2e-2 and cos >= 0.999, (err, cos)
