"""CPU oracle: a numpy + ml_dtypes restatement of JaxScale's GLM-4 decoder step.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline legs import this module, and only to check results or as the timed
CPU baseline.  The product path (the e2e-jaxscale_b200 package) never imports it.

Parity status: PINNED ONLY AGAINST THE REFERENCE'S OWN CODE THROUGH A STAND-IN.
The reference is pure JAX/Flax and neither is installed here (no wheel, no
network), so it cannot be run.  tests/golden/make_golden.py executes the
reference's own layer/model source files against a small numpy-backed stand-in
for the jax/flax names they use, and this restatement is checked against that
run (tests/test_oracle_pin.py).  The stand-in restates the third-party
primitives (lax.dot_general, jax.nn.dot_product_attention, softmax, top_k) from
their published semantics, so those primitives themselves stay unpinned.

Every array that the reference materialises in bf16 is rounded here with
round-to-nearest-even (ml_dtypes) and carried as float32 holding a bf16 value.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import ml_dtypes
import numpy as np

BF16 = ml_dtypes.bfloat16


def bf16(x) -> np.ndarray:
    """Round to bfloat16 (RNE) and return float32 holding the bf16 value."""
    return np.asarray(x, dtype=np.float32).astype(BF16).astype(np.float32)


# ---------------------------------------------------------------------------
# config (configs/model_config.py:11-72)
# ---------------------------------------------------------------------------

@dataclass
class GLMConfig:
    hidden_size: int = 4096
    num_hidden_layers: int = 40
    num_attention_heads: int = 32
    num_key_value_heads: int = 2
    head_dim: int = 128
    intermediate_size: int = 13696
    vocab_size: int = 151552
    rms_norm_eps: float = 1.5625e-07
    rope_theta: float = 10000.0
    partial_rotary_factor: float = 0.5
    attention_bias: bool = True


# ---------------------------------------------------------------------------
# layers
# ---------------------------------------------------------------------------

def rmsnorm(x, scale, eps):
    """layers/normalization.py:31-37: fp32 x*rsqrt(mean(x^2)+eps)*scale -> input dtype (bf16)."""
    x32 = np.asarray(x, np.float32)
    var = np.mean(np.square(x32), axis=-1, keepdims=True, dtype=np.float32)
    normed = x32 * (np.float32(1.0) / np.sqrt(var + np.float32(eps), dtype=np.float32))
    return bf16(normed * np.asarray(scale, np.float32))


def linear(x, w, b=None):
    """layers/linear.py:57-82: bf16(dot(x, W) with fp32 accumulation); then bias in bf16.

    W is [in, out] (layers/linear.py:16).  The bias is added after the sharding
    constraint, on the rounded bf16 product (layers/linear.py:80-81)."""
    y = bf16(np.matmul(np.asarray(x, np.float32), np.asarray(w, np.float32)))
    if b is not None:
        y = bf16(y + np.asarray(b, np.float32))
    return y


def rope_inv_freq(head_dim, theta=10000.0, partial=0.5):
    """layers/rotary.py:29-34 (numpy float32, computed once)."""
    rot = int(head_dim * partial)
    return (1.0 / (theta ** (np.arange(0, rot, 2, dtype=np.float32) / rot))).astype(np.float32)


def rope(positions, q, k, inv_freq):
    """layers/rotary.py:36-93: fp32 angle, cos/sin rounded to bf16, neox half split
    of the first rotary_dim dims, each product and sum rounded to bf16.

    q: [T, nq, hd], k: [T, nkv, hd], positions: [T]."""
    rot = 2 * inv_freq.shape[0]
    freqs = positions.astype(np.float32)[:, None] * inv_freq[None, :]
    cos = bf16(np.cos(freqs))[:, None, :]
    sin = bf16(np.sin(freqs))[:, None, :]

    def apply(x):
        x = np.asarray(x, np.float32)
        x1, x2 = x[..., : rot // 2], x[..., rot // 2 : rot]
        o1 = bf16(bf16(x1 * cos) - bf16(x2 * sin))
        o2 = bf16(bf16(x2 * cos) + bf16(x1 * sin))
        return np.concatenate([o1, o2, x[..., rot:]], axis=-1)

    return apply(q), apply(k)


def sdpa(q, k, v, bias, scale):
    """jax.nn.dot_product_attention(implementation="xla") as called at
    layers/attention.py:148-153: fp32 logits of bf16 q.k, times scale, plus the
    additive mask, fp32 softmax, probabilities cast to bf16, P.V with fp32
    accumulation, bf16 output.  GQA: query head h uses kv head h // (nq/nkv).

    q: [B,S,nq,hd], k/v: [B,L,nkv,hd], bias: broadcastable to [B,nq,S,L]."""
    B, S, nq, hd = q.shape
    nkv = k.shape[2]
    g = nq // nkv
    kk = np.repeat(np.asarray(k, np.float32), g, axis=2)
    vv = np.repeat(np.asarray(v, np.float32), g, axis=2)
    logits = np.einsum("bsnh,blnh->bnsl", np.asarray(q, np.float32), kk, dtype=np.float32)
    logits = logits * np.float32(scale)
    if bias is not None:
        logits = logits + np.asarray(bias, np.float32)
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - m)
    probs = bf16(e / e.sum(axis=-1, keepdims=True, dtype=np.float32))
    out = np.einsum("bnsl,blnh->bsnh", probs, vv, dtype=np.float32)
    return bf16(out)


def silu(x):
    """jax.nn.silu on bf16: x * bf16(sigmoid(x)), rounded to bf16."""
    x = np.asarray(x, np.float32)
    s = bf16(np.float32(1.0) / (np.float32(1.0) + np.exp(-x)))
    return bf16(x * s)


def argmax_first(logits):
    """jnp.argmax along the last axis (runner.py:281, :297): first index of the max."""
    return np.argmax(np.asarray(logits, np.float32), axis=-1).astype(np.int32)


# ---------------------------------------------------------------------------
# masks and positions (runner.py:23-73)
# ---------------------------------------------------------------------------

NEG = float(bf16(np.float32(-1e9)))


def make_prefill_mask(S, L):
    m = np.full((S, L), NEG, np.float32)
    m[:, :S] = np.triu(np.full((S, S), NEG, np.float32), k=1)
    return m[None, None]


def make_decode_mask(cur, L):
    m = np.where(np.arange(L) <= cur, 0.0, NEG).astype(np.float32)
    return m[None, None, None, :]


# ---------------------------------------------------------------------------
# parameters (random init, deterministic order)
# ---------------------------------------------------------------------------

@dataclass
class LayerParams:
    ln1: np.ndarray
    wq: np.ndarray
    bq: np.ndarray
    wk: np.ndarray
    bk: np.ndarray
    wv: np.ndarray
    bv: np.ndarray
    wo: np.ndarray
    ln2: np.ndarray
    wg: np.ndarray
    wu: np.ndarray
    wd: np.ndarray


@dataclass
class ModelParams:
    cfg: GLMConfig
    embed: np.ndarray
    layers: list = field(default_factory=list)
    norm: np.ndarray = None
    lm_head: np.ndarray = None  # [V, H] (layers/embedding.py:74-77)


def _normal_bf16(rng, shape, std=0.02):
    return bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def init_params(cfg: GLMConfig, seed: int = 0) -> ModelParams:
    """N(0, 0.02) drawn in float32 from default_rng(seed), rounded to bf16, in the
    attribute order of models/glm4.py (embed, per layer q/k/v/o with biases,
    gate/up/down, final norm, lm_head); RMSNorm gains are 1."""
    rng = np.random.default_rng(seed)
    H, hd, nq, nkv, I = (cfg.hidden_size, cfg.head_dim, cfg.num_attention_heads,
                         cfg.num_key_value_heads, cfg.intermediate_size)
    p = ModelParams(cfg=cfg, embed=_normal_bf16(rng, (cfg.vocab_size, H)))
    for _ in range(cfg.num_hidden_layers):
        p.layers.append(LayerParams(
            ln1=np.ones(H, np.float32),
            wq=_normal_bf16(rng, (H, nq * hd)), bq=_normal_bf16(rng, (nq * hd,)),
            wk=_normal_bf16(rng, (H, nkv * hd)), bk=_normal_bf16(rng, (nkv * hd,)),
            wv=_normal_bf16(rng, (H, nkv * hd)), bv=_normal_bf16(rng, (nkv * hd,)),
            wo=_normal_bf16(rng, (nq * hd, H)),
            ln2=np.ones(H, np.float32),
            wg=_normal_bf16(rng, (H, I)), wu=_normal_bf16(rng, (H, I)),
            wd=_normal_bf16(rng, (I, H)),
        ))
    p.norm = np.ones(H, np.float32)
    p.lm_head = _normal_bf16(rng, (cfg.vocab_size, H))
    return p


# ---------------------------------------------------------------------------
# model (models/glm4.py:20-260)
# ---------------------------------------------------------------------------

def attention(lp: LayerParams, cfg: GLMConfig, x, positions, mask, kv, cache_position, inv_freq):
    """layers/attention.py:101-160.  kv = (k_cache, v_cache) [B, L, nkv, hd] updated in place."""
    B, S, _ = x.shape
    nq, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    q = linear(x, lp.wq, lp.bq).reshape(B, S, nq, hd)
    k = linear(x, lp.wk, lp.bk).reshape(B, S, nkv, hd)
    v = linear(x, lp.wv, lp.bv).reshape(B, S, nkv, hd)
    qf, kf = rope(positions.reshape(-1), q.reshape(-1, nq, hd), k.reshape(-1, nkv, hd), inv_freq)
    q = qf.reshape(B, S, nq, hd)
    k = kf.reshape(B, S, nkv, hd)
    if kv is not None:
        kc, vc = kv
        c0 = int(cache_position[0])
        kc[:, c0:c0 + S] = k
        vc[:, c0:c0 + S] = v
        kfull, vfull = kc, vc
    else:
        kfull, vfull = k, v
    o = sdpa(q, kfull, vfull, mask, hd ** -0.5).reshape(B, S, nq * hd)
    return linear(o, lp.wo)


def mlp(lp: LayerParams, x):
    """models/glm4.py:46-49."""
    return linear(bf16(silu(linear(x, lp.wg)) * linear(x, lp.wu)), lp.wd)


def decoder_layer(lp, cfg, h, positions, mask, kv, cache_position, inv_freq):
    """models/glm4.py:97-132 (pre-norm, bf16 residual adds)."""
    r = h
    x = rmsnorm(h, lp.ln1, cfg.rms_norm_eps)
    h = bf16(r + attention(lp, cfg, x, positions, mask, kv, cache_position, inv_freq))
    r = h
    x = rmsnorm(h, lp.ln2, cfg.rms_norm_eps)
    return bf16(r + mlp(lp, x))


def init_kv_caches(cfg: GLMConfig, B: int, L: int):
    """layers/kv_cache.py:36-61 (zero-init, [B, L, nkv, hd] per layer)."""
    shp = (B, L, cfg.num_key_value_heads, cfg.head_dim)
    return [(np.zeros(shp, np.float32), np.zeros(shp, np.float32)) for _ in range(cfg.num_hidden_layers)]


def forward(p: ModelParams, input_ids, positions, mask, kv_caches, cache_position,
            return_hidden=False):
    """models/glm4.py:162-195 and :226-260: logits [B, S, V] (bf16 values)."""
    cfg = p.cfg
    inv = rope_inv_freq(cfg.head_dim, cfg.rope_theta, cfg.partial_rotary_factor)
    h = p.embed[np.asarray(input_ids)]
    for i, lp in enumerate(p.layers):
        kv = kv_caches[i] if kv_caches is not None else None
        h = decoder_layer(lp, cfg, h, np.asarray(positions), mask, kv, cache_position, inv)
    hn = rmsnorm(h, p.norm, cfg.rms_norm_eps)
    # layers/embedding.py:88-92: einsum('...h,vh->...v') with fp32 accumulation, bf16 result
    logits = bf16(np.einsum("bsh,vh->bsv", hn, p.lm_head, dtype=np.float32))
    if return_hidden:
        return logits, h
    return logits


def greedy_generate(p: ModelParams, input_ids, max_new_tokens, max_cache_len=None,
                    teacher_tokens=None, record=None):
    """runner.py:240-308 (no EOS).  With teacher_tokens [B, T] the fed token at
    decode step s is teacher_tokens[:, s] instead of the model's own argmax
    (teacher forcing, benchmarks/verify_kvcache.py:111-166).  `record`, when a
    list, receives (logits_last[B,V], h_last[B,H]) per produced token."""
    input_ids = np.asarray(input_ids)
    B, S = input_ids.shape
    L = max_cache_len or (S + max_new_tokens)
    cfg = p.cfg
    kv = init_kv_caches(cfg, B, L)
    pos = np.broadcast_to(np.arange(S, dtype=np.int32)[None], (B, S))
    logits, h = forward(p, input_ids, pos, make_prefill_mask(S, L), kv, np.arange(S),
                        return_hidden=True)
    nxt = argmax_first(logits[:, -1])
    out = [nxt]
    if record is not None:
        record.append((logits[:, -1].copy(), h[:, -1].copy()))
    for step in range(max_new_tokens - 1):
        cur = S + step
        fed = nxt if teacher_tokens is None else np.asarray(teacher_tokens)[:, step]
        pos = np.full((B, 1), cur, np.int32)
        logits, h = forward(p, fed[:, None], pos, make_decode_mask(cur, L), kv,
                            np.array([cur]), return_hidden=True)
        nxt = argmax_first(logits[:, -1])
        out.append(nxt)
        if record is not None:
            record.append((logits[:, -1].copy(), h[:, -1].copy()))
    return np.concatenate([input_ids] + [t[:, None] for t in out], axis=1)


# ---------------------------------------------------------------------------
# tensor parallelism (utils/weight_utils.py:248-265, layers/linear.py:72-78)
# ---------------------------------------------------------------------------

def shard_columns(w, tp, rank):
    """Column-parallel split of W[in, out] on the output dim."""
    n = w.shape[-1] // tp
    return w[..., rank * n:(rank + 1) * n]


def shard_rows(w, tp, rank):
    """Row-parallel split of W[in, out] on the input dim."""
    k = w.shape[0] // tp
    return w[rank * k:(rank + 1) * k]


def row_parallel_reference(x_shards, w_shards):
    """What the reference's XLA all-reduce computes for a row-parallel LinearBase:
    bf16 per-rank partials summed (as fp32 here) and rounded once."""
    acc = np.zeros((x_shards[0].shape[0], w_shards[0].shape[1]), np.float32)
    for xr, wr in zip(x_shards, w_shards):
        acc += bf16(np.matmul(np.asarray(xr, np.float32), np.asarray(wr, np.float32)))
    return bf16(acc)


# ---------------------------------------------------------------------------
# MoE router (layers/moe.py:54-79)
# ---------------------------------------------------------------------------

def moe_gate(x, w, k, scale, norm=True, correction_bias=None):
    """logits = bf16(x @ W) -> f32 softmax -> + correction bias -> top_k (ties: lower
    index first, like lax.top_k) -> gather uncorrected probs -> renormalise
    (+1e-20) -> * scale -> bf16."""
    logits = linear(x, w).astype(np.float32)
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - m)
    scores = e / e.sum(axis=-1, keepdims=True, dtype=np.float32)
    corrected = scores + (np.float32(0) if correction_bias is None
                          else np.asarray(correction_bias, np.float32))
    # stable sort on -value keeps the lower index first among equal values
    idx = np.argsort(-corrected, axis=-1, kind="stable")[..., :k].astype(np.int32)
    wts = np.take_along_axis(scores, idx, axis=-1)
    if norm:
        wts = wts / (wts.sum(axis=-1, keepdims=True, dtype=np.float32) + np.float32(1e-20))
    wts = wts * np.float32(scale)
    return bf16(wts), idx


# ---------------------------------------------------------------------------
# MoE experts (layers/moe.py:247-267) and the MoE layer (layers/moe.py:156-192)
# ---------------------------------------------------------------------------

def moe_experts(x, tk_w, tk_i, gate_w, up_w, down_w):
    """_topk_local_forward (layers/moe.py:247-267): for k = 0..K-1 in order, each
    token's k-th expert SwiGLU with bf16 einsums (fp32 accumulate), then
    output = bf16(output + bf16(expert_out * w_k)).  x [N, H], tk_w [N, K] bf16,
    tk_i [N, K], gate_w/up_w [E, H, I], down_w [E, I, H]."""
    x = bf16(x)
    N, H = x.shape
    out = np.zeros((N, H), np.float32)
    for k in range(tk_i.shape[1]):
        ids = np.asarray(tk_i[:, k])
        g = bf16(np.einsum("nh,nhi->ni", x, np.asarray(gate_w, np.float32)[ids], dtype=np.float32))
        u = bf16(np.einsum("nh,nhi->ni", x, np.asarray(up_w, np.float32)[ids], dtype=np.float32))
        act = bf16(silu(g) * u)
        eo = bf16(np.einsum("ni,nih->nh", act, np.asarray(down_w, np.float32)[ids], dtype=np.float32))
        out = bf16(out + bf16(eo * np.asarray(tk_w[:, k:k + 1], np.float32)))
    return out


def moe_layer(x, router_w, correction_bias, k, scale, norm, gate_w, up_w, down_w, sh_g, sh_u, sh_d):
    """MoELayer.__call__ without expert parallelism (layers/moe.py:156-192): router,
    routed experts, shared SwiGLU expert (layers/moe.py:110-113), bf16 sum."""
    lead = x.shape[:-1]
    xf = bf16(x).reshape(-1, x.shape[-1])
    w, i = moe_gate(xf, router_w, k, scale, norm, correction_bias)
    routed = moe_experts(xf, w, i, gate_w, up_w, down_w)
    shared = linear(bf16(silu(linear(xf, sh_g)) * linear(xf, sh_u)), sh_d)
    return bf16(routed + shared).reshape(*lead, -1)


# ---------------------------------------------------------------------------
# MLA attention (layers/mla_attention.py:101-193), expanded per-head cache
# ---------------------------------------------------------------------------

@dataclass
class MLAParams:
    q_a: np.ndarray        # [H, q_lora]
    q_a_ln: np.ndarray     # [q_lora]
    q_b: np.ndarray        # [q_lora, nh * (nope + rope)]
    kv_a: np.ndarray       # [H, kv_lora + rope]
    kv_a_ln: np.ndarray    # [kv_lora]
    kv_b: np.ndarray       # [kv_lora, nh * (nope + v)]
    o: np.ndarray          # [nh * v, H]


def mla_attention(p: MLAParams, x, positions, mask, kv, cache_position, nh, nope, rope_d, vdim, eps,
                  inv_freq):
    """MLAAttention.__call__: low-rank q (q_a -> RMSNorm -> q_b) and kv (kv_a -> split
    latent | shared rope key -> RMSNorm on the latent -> kv_b), neox RoPE on the rope
    slice of q and on the shared key (broadcast to every head), concatenation, cache
    write, scores = bf16(bf16(q k^T) * scale) + mask, fp32 softmax, bf16
    probabilities, bf16(P v), o_proj.  x [B, S, H]; kv = (k [B, L, nh, nope+rope],
    v [B, L, nh, vdim]) updated in place; returns the output [B, S, H]."""
    B, S, _ = x.shape
    kv_lora = p.kv_a_ln.shape[0]
    qc = rmsnorm(linear(x, p.q_a), p.q_a_ln, eps)
    q = linear(qc, p.q_b).reshape(B, S, nh, nope + rope_d)
    kvc = linear(x, p.kv_a)
    kv_lat, k_rope_sh = kvc[..., :kv_lora], kvc[..., kv_lora:]
    kvb = linear(rmsnorm(kv_lat, p.kv_a_ln, eps), p.kv_b).reshape(B, S, nh, nope + vdim)
    k_nope, v = kvb[..., :nope], kvb[..., nope:]
    k_rope = np.broadcast_to(k_rope_sh[:, :, None, :], (B, S, nh, rope_d))
    qr, kr = rope(np.asarray(positions).reshape(-1), q[..., nope:].reshape(-1, nh, rope_d),
                  k_rope.reshape(-1, nh, rope_d), inv_freq)
    q = np.concatenate([q[..., :nope], qr.reshape(B, S, nh, rope_d)], axis=-1)
    k = np.concatenate([k_nope, kr.reshape(B, S, nh, rope_d)], axis=-1)
    kc, vc = kv
    start = min(max(int(np.asarray(cache_position)[0]), 0), kc.shape[1] - S)
    kc[:, start:start + S] = k
    vc[:, start:start + S] = v
    scale = np.float32((nope + rope_d) ** -0.5)
    scores = bf16(np.einsum("bshd,blhd->bhsl", q, kc, dtype=np.float32))
    scores = bf16(scores * scale)
    if mask is not None:
        scores = bf16(scores + np.asarray(mask, np.float32))
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - m)
    probs = bf16(e / e.sum(axis=-1, keepdims=True, dtype=np.float32))
    out = bf16(np.einsum("bhsl,blhd->bshd", probs, vc, dtype=np.float32)).reshape(B, S, nh * vdim)
    return linear(out, p.o)


# ---------------------------------------------------------------------------
# GLM-4.7-Flash decoder (models/glm4_flash.py:26-205): MLA attention in every
# layer, a dense SwiGLU MLP in the first first_k_dense_replace layers
# (layers/moe.py:270-300), the MoE layer after; pre-norm with bf16 residual adds
# ---------------------------------------------------------------------------

@dataclass
class FlashLayerParams:
    ln1: np.ndarray
    mla: MLAParams
    ln2: np.ndarray
    dense: tuple | None = None   # (wg, wu, wd) [in, out]
    moe: dict | None = None      # router, bias, eg, eu, ed, sg, su, sd


@dataclass
class FlashParams:
    embed: np.ndarray
    layers: list
    norm: np.ndarray
    lm_head: np.ndarray          # [V, H]
    nh: int
    nope: int
    rope_d: int
    vdim: int
    eps: float
    rope_theta: float
    top_k: int
    scale: float
    norm_topk: bool = True


def flash_forward(p: FlashParams, input_ids, positions, mask, kv_caches, cache_position):
    """GLM4FlashForCausalLM.__call__ (models/glm4_flash.py:93-110, :140-205): logits
    [B, S, V] (bf16 values); kv_caches [(k, v)] per layer updated in place."""
    inv = rope_inv_freq(p.rope_d, theta=p.rope_theta, partial=1.0)
    h = p.embed[np.asarray(input_ids)]
    for lp, kv in zip(p.layers, kv_caches):
        r = h
        x = rmsnorm(h, lp.ln1, p.eps)
        a = mla_attention(lp.mla, x, positions, mask, kv, cache_position, p.nh, p.nope, p.rope_d, p.vdim,
                          p.eps, inv)
        h = bf16(r + a)
        r = h
        x = rmsnorm(h, lp.ln2, p.eps)
        if lp.dense is not None:
            wg, wu, wd = lp.dense
            y = linear(bf16(silu(linear(x, wg)) * linear(x, wu)), wd)
        else:
            m = lp.moe
            y = moe_layer(x, m["router"], m["bias"], p.top_k, p.scale, p.norm_topk, m["eg"], m["eu"], m["ed"],
                          m["sg"], m["su"], m["sd"])
        h = bf16(r + y)
    hn = rmsnorm(h, p.norm, p.eps)
    return bf16(np.einsum("bsh,vh->bsv", hn, p.lm_head, dtype=np.float32))


# ---------------------------------------------------------------------------
# sampling (runner.py:315-359, _jit_sample) with the categorical draw's Gumbel
# noise given (jax.random.categorical = argmax(logits + gumbel noise))
# ---------------------------------------------------------------------------

def sample_tokens(logits, presence, gumbel, repetition_penalty, temperature, top_k, top_p):
    """logits [B, V] (bf16 values), presence [B, V] bool or None, gumbel [B, k] (bf16
    values, one per top-k candidate in lax.top_k order).  bf16 arithmetic with the
    Python scalars rounded to bf16 (weak typing).  Returns (tokens [B] int32, the
    smallest |preceding mass - top_p| over the candidates of each row, for
    near-tie reporting)."""
    x = bf16(logits)
    rp = np.float32(bf16(np.float32(repetition_penalty)))
    pen = bf16(np.where(x > 0, x / rp, x * rp))
    if presence is not None:
        x = np.where(np.asarray(presence, bool), pen, x)
    if temperature != 1.0:
        x = bf16(x / np.float32(bf16(np.float32(temperature))))
    k = top_k if top_k > 0 else 200
    B = x.shape[0]
    tokens = np.zeros(B, np.int32)
    margins = np.full(B, np.inf, np.float32)
    for b in range(B):
        order = np.argsort(-x[b], kind="stable")[:k]   # lax.top_k: descending, lower index first on ties
        vals = x[b, order].astype(np.float32)
        if top_p < 1.0:
            e = np.exp(vals - vals.max(), dtype=np.float32)
            probs = (e / e.sum(dtype=np.float32)).astype(np.float32)
            cum = np.cumsum(probs, dtype=np.float32)
            before = cum - probs
            margins[b] = np.min(np.abs(before - np.float32(top_p)))
            vals = np.where(before >= np.float32(top_p), np.float32(bf16(np.float32(-1e9))), vals)
        z = bf16(vals + np.asarray(gumbel[b], np.float32))
        tokens[b] = order[int(np.argmax(z))]
    return tokens, margins


def mla_attention_absorbed(p: MLAParams, x, positions, mask, latent, cache_position, nh, nope, rope_d, vdim, eps,
                           inv_freq):
    """MLA with the kv_b projection absorbed into the query and the output (the
    latent-cache decode form; the reference computes the expanded form,
    layers/mla_attention.py:101-193).  The cache holds per token the normalised
    latent c (kv_lora values) and the rotated shared rope key (rope_d values):
    latent [B, L, kv_lora + rope_d], updated in place.  With W_k[h] and W_v[h]
    the key and value columns of kv_b for head h:
        q.k = (W_k[h] q_nope) . c + q_rope . k_rope,     out_h = (sum_l p_l c_l) W_v[h]
    equal to the expanded form up to where it rounds to bf16 (k_nope and v are
    never materialised here), so it agrees with mla_attention to the bf16
    tolerance, not bit for bit.  Returns the output [B, S, H]."""
    B, S, _ = x.shape
    kv_lora = p.kv_a_ln.shape[0]
    qc = rmsnorm(linear(x, p.q_a), p.q_a_ln, eps)
    q = linear(qc, p.q_b).reshape(B, S, nh, nope + rope_d)
    kvc = linear(x, p.kv_a)
    c = rmsnorm(kvc[..., :kv_lora], p.kv_a_ln, eps)                        # [B, S, kv_lora]
    k_rope = kvc[..., kv_lora:]                                             # [B, S, rope_d]
    qr, kr = rope(np.asarray(positions).reshape(-1), q[..., nope:].reshape(-1, nh, rope_d),
                  k_rope.reshape(-1, 1, rope_d), inv_freq)
    q_rope = qr.reshape(B, S, nh, rope_d)
    start = min(max(int(np.asarray(cache_position)[0]), 0), latent.shape[1] - S)
    latent[:, start:start + S, :kv_lora] = c
    latent[:, start:start + S, kv_lora:] = kr.reshape(B, S, rope_d)
    wkv = np.asarray(p.kv_b, np.float32).reshape(kv_lora, nh, nope + vdim)
    w_k, w_v = wkv[..., :nope], wkv[..., nope:]                             # [kv_lora, nh, nope|vdim]
    q_abs = bf16(np.einsum("bshn,lhn->bshl", q[..., :nope], w_k, dtype=np.float32))   # [B, S, nh, kv_lora]
    scale = np.float32((nope + rope_d) ** -0.5)
    ctx = mla_latent_attention(q_abs, q_rope, latent, mask, scale)         # [B, S, nh, kv_lora]
    out = bf16(np.einsum("bshl,lhv->bshv", ctx, w_v, dtype=np.float32)).reshape(B, S, nh * vdim)
    return linear(out, p.o)


def mla_latent_attention(q_abs, q_rope, latent, mask, scale):
    """The attention step of mla_attention_absorbed: every head of q_abs [B, S, nh, kv_lora]
    / q_rope [B, S, nh, rope] against the latent cache [B, L, kv_lora + rope] (key = the
    whole row, value = its first kv_lora columns), scores rounded like the expanded form
    (bf16(q.k), then bf16(* scale), layers/mla_attention.py:176-184), + mask [.., S, L],
    fp32 softmax, bf16 probabilities; returns ctx = bf16(P . c) [B, S, nh, kv_lora]."""
    kv_lora = q_abs.shape[-1]
    lat = np.asarray(latent, np.float32)
    scores = (np.einsum("bshl,btl->bhst", q_abs, lat[..., :kv_lora], dtype=np.float32) +
              np.einsum("bshr,btr->bhst", q_rope, lat[..., kv_lora:], dtype=np.float32))
    scores = bf16(bf16(scores) * np.float32(scale))
    if mask is not None:
        scores = bf16(scores + np.asarray(mask, np.float32))
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - m)
    probs = bf16(e / e.sum(axis=-1, keepdims=True, dtype=np.float32))
    return bf16(np.einsum("bhst,btl->bshl", probs, lat[..., :kv_lora], dtype=np.float32))
