"""torch-tensor front end of the C ABI (include/jsx.h).

Each function checks devices/dtypes/contiguity, then calls one jsx_* entry
point on torch's current CUDA stream.  Tensors are plain device memory here:
torch is the allocator and stream provider, the arithmetic is in libjsx.so.
"""

from __future__ import annotations

import ctypes

import torch

from ._lib import JSX_LAUNCH_PDL, call, lib  # noqa: F401  (re-exported)

BF16 = torch.bfloat16
MAX_DECODE_TOKENS = 8  # rows per GEMV call (include/jsx.h: 1 <= M <= 8)
TC_MAX_TOKENS = 32     # rows per tensor-core call (jsx_tc_*: 1 <= M <= 32)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t, name, dtype=BF16):
    if t is None:
        raise ValueError(f"{name} is required")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device})")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype} (got {t.dtype})")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def _opt(t, name, dtype=BF16):
    return None if t is None else _need(t, name, dtype)


def set_pdl(enabled: bool) -> None:
    call("jsx_set_launch_flags", JSX_LAUNCH_PDL if enabled else 0)


def pdl_enabled() -> bool:
    return bool(lib.jsx_get_launch_flags() & JSX_LAUNCH_PDL)


def device_error() -> int:
    """jsx_device_error: JSX_ETIMEDOUT (3) when a bounded wait of the whole-step kernel,
    the streaming GEMV or the tensor-core projections gave up since the last call,
    else 0 (reads and clears the error words; synchronous)."""
    out = ctypes.c_int(0)
    call("jsx_device_error", ctypes.byref(out))
    return out.value


def sm_count() -> int:
    out = ctypes.c_int(0)
    call("jsx_device_sm_count", ctypes.byref(out))
    return out.value


# ---- packing ------------------------------------------------------------------
def pack_transpose(w_kn: torch.Tensor) -> torch.Tensor:
    _need(w_kn, "w")
    K, N = w_kn.shape
    out = torch.empty((N, K), dtype=BF16, device=w_kn.device)
    call("jsx_pack_transpose", _p(w_kn), _p(out), K, N, _stream())
    return out


def pack_qkv(wq, wk, wv, nq, nkv, head_dim, rotary_dim) -> torch.Tensor:
    for t, n in ((wq, "wq"), (wk, "wk"), (wv, "wv")):
        _need(t, n)
    K = wq.shape[0]
    out = torch.empty(((nq + 2 * nkv) * head_dim, K), dtype=BF16, device=wq.device)
    call("jsx_pack_qkv", _p(wq), _p(wk), _p(wv), _p(out), K, nq, nkv, head_dim, rotary_dim, _stream())
    return out


def pack_gate_up(wg, wu) -> torch.Tensor:
    _need(wg, "w_gate")
    _need(wu, "w_up")
    K, I = wg.shape
    out = torch.empty((2 * I, K), dtype=BF16, device=wg.device)
    call("jsx_pack_gate_up", _p(wg), _p(wu), _p(out), K, I, _stream())
    return out


# ---- ops --------------------------------------------------------------------------
def rmsnorm(x, gamma, eps, out=None):
    _need(x, "x")
    _need(gamma, "gamma")
    hidden = x.shape[-1]
    rows = x.numel() // hidden
    out = torch.empty_like(x) if out is None else _need(out, "out")
    call("jsx_rmsnorm", _p(x), _p(gamma), _p(out), rows, hidden, ctypes.c_float(eps), _stream())
    return out


def embed(ids, table, out=None):
    _need(ids, "ids", torch.int32)
    _need(table, "table")
    V, H = table.shape
    M = ids.numel()
    out = torch.empty((M, H), dtype=BF16, device=table.device) if out is None else _need(out, "out")
    call("jsx_embed", _p(ids), _p(table), _p(out), M, H, V, _stream())
    return out


def linear(x, w_nk, bias=None, gamma=None, eps=0.0, out=None):
    """y = bf16(x @ W) (+ bias in bf16); RMSNorm prologue when gamma is given."""
    _need(x, "x")
    _need(w_nk, "w_nk")
    _opt(bias, "bias")
    _opt(gamma, "gamma")
    N, K = w_nk.shape
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=BF16, device=x.device) if out is None else _need(out, "out")
    for m0 in range(0, M, MAX_DECODE_TOKENS):
        m = min(MAX_DECODE_TOKENS, M - m0)
        call("jsx_linear", _p(x2[m0:m0 + m]), _p(gamma), ctypes.c_float(eps), _p(w_nk), _p(bias),
             _p(out[m0:m0 + m]), m, K, N, _stream())
    return out.reshape(*x.shape[:-1], N)


def qkv_rope_cache(h, ln_gamma, eps, w_qkv, b_qkv, inv_freq, positions, q_out, k_cache, v_cache,
                   nq, nkv, head_dim, rotary_dim, tokens_per_seq=1):
    _need(h, "h")
    _opt(ln_gamma, "ln_gamma")
    _need(w_qkv, "w_qkv")
    _opt(b_qkv, "b_qkv")
    _need(inv_freq, "inv_freq", torch.float32)
    _need(positions, "positions", torch.int32)
    _need(q_out, "q_out")
    _need(k_cache, "k_cache")
    _need(v_cache, "v_cache")
    M, K = h.shape
    max_seq = k_cache.shape[1]
    call("jsx_qkv_rope_cache", _p(h), _p(ln_gamma), ctypes.c_float(eps), _p(w_qkv), _p(b_qkv),
         _p(inv_freq), _p(positions), _p(q_out), _p(k_cache), _p(v_cache), M, tokens_per_seq, K,
         nq, nkv, head_dim, rotary_dim, max_seq, _stream())


def gate_up_swiglu(h, ln_gamma, eps, w_gu, act):
    _need(h, "h")
    _opt(ln_gamma, "ln_gamma")
    _need(w_gu, "w_gu")
    _need(act, "act")
    M, K = h.shape
    I = w_gu.shape[0] // 2
    call("jsx_gate_up_swiglu", _p(h), _p(ln_gamma), ctypes.c_float(eps), _p(w_gu), _p(act), M, K, I,
         _stream())


def attn_workspace(B, nq, nkv, head_dim, max_seq, device) -> torch.Tensor:
    n = ctypes.c_size_t(0)
    call("jsx_attn_decode_workspace_size", B, nq, nkv, head_dim, max_seq, ctypes.byref(n))
    return torch.zeros(n.value, dtype=torch.uint8, device=device)


def attn_decode(q, k_cache, v_cache, out, positions, scale, workspace):
    _need(q, "q")
    _need(k_cache, "k_cache")
    _need(v_cache, "v_cache")
    _need(out, "out")
    _need(positions, "positions", torch.int32)
    _need(workspace, "workspace", torch.uint8)
    B, max_seq, nkv, hd = k_cache.shape
    nq = q.numel() // (B * hd)
    call("jsx_attn_decode", _p(q), _p(k_cache), _p(v_cache), _p(out), _p(positions), B, nq, nkv, hd,
         max_seq, ctypes.c_float(scale), _p(workspace), workspace.numel(), _stream())


def row_linear_allreduce(comm, x, w_nk, h):
    """h = bf16(h + bf16(sum over ranks of x_r @ W_r)); comm None for one rank."""
    _need(x, "x")
    _need(w_nk, "w_nk")
    _need(h, "h")
    N, K = w_nk.shape
    M = x.numel() // K
    handle = None if comm is None else comm.handle
    call("jsx_row_linear_allreduce", handle, _p(x), _p(w_nk), _p(h), M, K, N, _stream())


def lmhead_workspace(M, device) -> torch.Tensor:
    n = ctypes.c_size_t(0)
    call("jsx_lmhead_workspace_size", M, ctypes.byref(n))
    return torch.zeros(n.value, dtype=torch.uint8, device=device)


def lmhead_argmax(comm, h, norm_gamma, eps, w_vocab, vocab_offset, ids_out, workspace,
                  logits_out=None):
    _need(h, "h")
    _opt(norm_gamma, "norm_gamma")
    _need(w_vocab, "w_vocab")
    _need(ids_out, "ids_out", torch.int32)
    _need(workspace, "workspace", torch.uint8)
    _opt(logits_out, "logits_out")
    M, H = h.shape
    Vl = w_vocab.shape[0]
    handle = None if comm is None else comm.handle
    call("jsx_lmhead_argmax", handle, _p(h), _p(norm_gamma), ctypes.c_float(eps), _p(w_vocab), Vl,
         vocab_offset, M, H, _p(logits_out), _p(ids_out), _p(workspace), workspace.numel(), _stream())


# ---- tensor-core projections (jsx_tc_*), 9..32 tokens per call ----
def tc_workspace(M, shapes, device) -> torch.Tensor:
    """Zeroed workspace large enough for every (K, N) in shapes at M tokens."""
    best = 0
    for K_, N_ in shapes:
        n = ctypes.c_size_t(0)
        call("jsx_tc_workspace_size", M, K_, N_, ctypes.byref(n))
        best = max(best, n.value)
    return torch.zeros(best, dtype=torch.uint8, device=device)


def tc_linear(x, w_nk, workspace, bias=None, gamma=None, eps=0.0, out=None):
    _need(x, "x")
    _need(w_nk, "w_nk")
    _opt(bias, "bias")
    _opt(gamma, "gamma")
    _need(workspace, "workspace", torch.uint8)
    N, K_ = w_nk.shape
    x2 = x.reshape(-1, K_)
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=BF16, device=x.device) if out is None else _need(out, "out")
    call("jsx_tc_linear", _p(x2), _p(gamma), ctypes.c_float(eps), _p(w_nk), _p(bias), _p(out), M, K_, N,
         _p(workspace), workspace.numel(), _stream())
    return out.reshape(*x.shape[:-1], N)


def tc_qkv_rope_cache(h, ln_gamma, eps, w_qkv, b_qkv, inv_freq, positions, q_out, k_cache, v_cache,
                      nq, nkv, head_dim, rotary_dim, workspace, tokens_per_seq=1):
    for t, n in ((h, "h"), (w_qkv, "w_qkv"), (q_out, "q_out"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(t, n)
    _opt(ln_gamma, "ln_gamma")
    _opt(b_qkv, "b_qkv")
    _need(inv_freq, "inv_freq", torch.float32)
    _need(positions, "positions", torch.int32)
    _need(workspace, "workspace", torch.uint8)
    M, K_ = h.shape
    max_seq = k_cache.shape[1]
    call("jsx_tc_qkv_rope_cache", _p(h), _p(ln_gamma), ctypes.c_float(eps), _p(w_qkv), _p(b_qkv),
         _p(inv_freq), _p(positions), _p(q_out), _p(k_cache), _p(v_cache), M, tokens_per_seq, K_,
         nq, nkv, head_dim, rotary_dim, max_seq, _p(workspace), workspace.numel(), _stream())


def tc_gate_up_swiglu(h, ln_gamma, eps, w_gu, act, workspace):
    _need(h, "h")
    _opt(ln_gamma, "ln_gamma")
    _need(w_gu, "w_gu")
    _need(act, "act")
    _need(workspace, "workspace", torch.uint8)
    M, K_ = h.shape
    I = w_gu.shape[0] // 2
    call("jsx_tc_gate_up_swiglu", _p(h), _p(ln_gamma), ctypes.c_float(eps), _p(w_gu), _p(act), M, K_, I,
         _p(workspace), workspace.numel(), _stream())


def tc_row_linear_allreduce(comm, x, w_nk, h, workspace):
    _need(x, "x")
    _need(w_nk, "w_nk")
    _need(h, "h")
    _need(workspace, "workspace", torch.uint8)
    N, K_ = w_nk.shape
    M = x.numel() // K_
    handle = None if comm is None else comm.handle
    call("jsx_tc_row_linear_allreduce", handle, _p(x), _p(w_nk), _p(h), M, K_, N, _p(workspace),
         workspace.numel(), _stream())


def attn_prefill(q, k_cache, v_cache, nq, nkv, head_dim, S, start_pos=0, scale=None, out=None):
    """Causal prefill attention: q [B*S, nq*hd] -> out [B*S, nq*hd] over cache rows [0, start_pos + i]."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(t, n)
    B, L = k_cache.shape[0], k_cache.shape[1]
    scale = head_dim ** -0.5 if scale is None else scale
    out = torch.empty((B * S, nq * head_dim), dtype=BF16, device=q.device) if out is None else _need(out, "out")
    call("jsx_attn_prefill", _p(q), _p(k_cache), _p(v_cache), _p(out), B, S, start_pos, nq, nkv, head_dim, L,
         ctypes.c_float(scale), _stream())
    return out


def sample(logits, gumbel, presence=None, repetition_penalty=1.0, temperature=1.0, top_k=0, top_p=1.0,
           out=None):
    """runner.py:315-359: next tokens [B] int32 from logits [B, V] bf16; gumbel [B, k] bf16 is the
    categorical draw's noise for the k = (top_k or 200) candidates; presence [B, V] bool/uint8."""
    _need(logits, "logits")
    _need(gumbel, "gumbel")
    B, V = logits.shape
    pres = None
    if presence is not None:
        pres = presence.to(torch.uint8).contiguous()
        if pres.shape != logits.shape or pres.device != logits.device:
            raise ValueError("presence must be [B, V] on the logits' device")
    out = torch.empty(B, dtype=torch.int32, device=logits.device) if out is None else _need(out, "out", torch.int32)
    call("jsx_sample", _p(logits), None if pres is None else ctypes.c_void_p(pres.data_ptr()), _p(gumbel),
         _p(out), B, V, ctypes.c_float(repetition_penalty), ctypes.c_float(temperature), top_k,
         ctypes.c_float(top_p), _stream())
    return out


# ---- wide tensor-core projections (prefill / many tokens) ----------------------------
def wide_workspace(M, shapes, device, norm=True) -> torch.Tensor:
    """Workspace for every (K, N) in shapes at M tokens (with room for the
    normalised activations when norm)."""
    best = 0
    for K_, N_ in shapes:
        n = ctypes.c_size_t(0)
        call("jsx_wide_workspace_size", M, K_, N_, int(norm), ctypes.byref(n))
        best = max(best, n.value)
    return torch.empty(best, dtype=torch.uint8, device=device)


def wide_linear(x, w_nk, workspace, bias=None, gamma=None, eps=0.0, out=None):
    _need(x, "x")
    _need(w_nk, "w_nk")
    _opt(bias, "bias")
    _opt(gamma, "gamma")
    _need(workspace, "workspace", torch.uint8)
    N, K_ = w_nk.shape
    x2 = x.reshape(-1, K_)
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=BF16, device=x.device) if out is None else _need(out, "out")
    call("jsx_wide_linear", _p(x2), _p(gamma), ctypes.c_float(eps), _p(w_nk), _p(bias), _p(out), M, K_, N,
         _p(workspace), workspace.numel(), _stream())
    return out.reshape(*x.shape[:-1], N)


def wide_qkv_rope_cache(h, ln_gamma, eps, w_qkv, b_qkv, inv_freq, positions, q_out, k_cache, v_cache,
                        nq, nkv, head_dim, rotary_dim, workspace, tokens_per_seq=1):
    for t, n in ((h, "h"), (w_qkv, "w_qkv"), (q_out, "q_out"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(t, n)
    _opt(ln_gamma, "ln_gamma")
    _opt(b_qkv, "b_qkv")
    _need(inv_freq, "inv_freq", torch.float32)
    _need(positions, "positions", torch.int32)
    _need(workspace, "workspace", torch.uint8)
    M, K_ = h.shape
    max_seq = k_cache.shape[1]
    call("jsx_wide_qkv_rope_cache", _p(h), _p(ln_gamma), ctypes.c_float(eps), _p(w_qkv), _p(b_qkv),
         _p(inv_freq), _p(positions), _p(q_out), _p(k_cache), _p(v_cache), M, tokens_per_seq, K_,
         nq, nkv, head_dim, rotary_dim, max_seq, _p(workspace), workspace.numel(), _stream())


def wide_gate_up_swiglu(h, ln_gamma, eps, w_gu, act, workspace):
    _need(h, "h")
    _opt(ln_gamma, "ln_gamma")
    _need(w_gu, "w_gu")
    _need(act, "act")
    _need(workspace, "workspace", torch.uint8)
    M, K_ = h.shape
    I = w_gu.shape[0] // 2
    call("jsx_wide_gate_up_swiglu", _p(h), _p(ln_gamma), ctypes.c_float(eps), _p(w_gu), _p(act), M, K_, I,
         _p(workspace), workspace.numel(), _stream())


def wide_row_linear_allreduce(comm, x, w_nk, h, workspace):
    """h += all-reduce over the comm's ranks of x @ w_nk^T (comm None: one rank);
    comm: a tile-exchange Comm (mesh.Comm(..., tiles=True))."""
    _need(x, "x")
    _need(w_nk, "w_nk")
    _need(h, "h")
    _need(workspace, "workspace", torch.uint8)
    N, K_ = w_nk.shape
    M = x.numel() // K_
    handle = None if comm is None else comm.handle
    call("jsx_wide_row_linear_allreduce", handle, _p(x), _p(w_nk), _p(h), M, K_, N, _p(workspace),
         workspace.numel(), _stream())


def tc_lmhead_argmax(comm, h, norm_gamma, eps, w_vocab, vocab_offset, ids_out, workspace, logits_out=None):
    _need(h, "h")
    _opt(norm_gamma, "norm_gamma")
    _need(w_vocab, "w_vocab")
    _need(ids_out, "ids_out", torch.int32)
    _need(workspace, "workspace", torch.uint8)
    _opt(logits_out, "logits_out")
    M, H = h.shape
    Vl = w_vocab.shape[0]
    handle = None if comm is None else comm.handle
    call("jsx_tc_lmhead_argmax", handle, _p(h), _p(norm_gamma), ctypes.c_float(eps), _p(w_vocab), Vl,
         vocab_offset, M, H, _p(logits_out), _p(ids_out), _p(workspace), workspace.numel(), _stream())


def row_linear_allreduce_add(comm, x, w_nk, addend, h):
    """h = bf16(h + bf16(sum over ranks of (x_r @ W_r + addend_r))); addend may be None."""
    _need(x, "x")
    _need(w_nk, "w_nk")
    _opt(addend, "addend")
    _need(h, "h")
    N, K_ = w_nk.shape
    M = x.numel() // K_
    handle = None if comm is None else comm.handle
    call("jsx_row_linear_allreduce_add", handle, _p(x), _p(w_nk), _p(addend), _p(h), M, K_, N, _stream())


def moe_workspace(N, K_, E, H, I, device) -> torch.Tensor:
    n = ctypes.c_size_t(0)
    call("jsx_moe_experts_workspace_size", N, K_, E, H, I, ctypes.byref(n))
    return torch.zeros(n.value, dtype=torch.uint8, device=device)


def moe_experts(x, topk_w, topk_idx, w_gu, w_d, out, workspace, owner=None, rank=0):
    """Routed partial of this rank's experts (include/jsx.h jsx_moe_experts).
    w_gu [E, 2I, H] (packed per expert), w_d [E, H, I]; owner: int32 [E] device tensor or None."""
    _need(x, "x")
    _need(topk_w, "topk_w")
    _need(topk_idx, "topk_idx", torch.int32)
    _need(w_gu, "w_gu")
    _need(w_d, "w_d")
    _need(out, "out")
    _need(workspace, "workspace", torch.uint8)
    _opt(owner, "owner", torch.int32)
    N, H = x.shape
    E, I2, _ = w_gu.shape
    call("jsx_moe_experts", _p(x), _p(topk_w), _p(topk_idx), _p(owner), rank, N, topk_idx.shape[1], E, H,
         I2 // 2, _p(w_gu), _p(w_d), _p(out), _p(workspace), workspace.numel(), _stream())


def mla_rope_cache(q_in, kv_in, k_rope, inv_freq, positions, q_out, k_cache, v_cache, nh, nope, rope, vdim,
                   tokens_per_seq=1):
    for t, n in ((q_in, "q_in"), (kv_in, "kv_in"), (k_rope, "k_rope"), (q_out, "q_out"), (k_cache, "k_cache"),
                 (v_cache, "v_cache")):
        _need(t, n)
    _need(inv_freq, "inv_freq", torch.float32)
    _need(positions, "positions", torch.int32)
    M = positions.numel()
    call("jsx_mla_rope_cache", _p(q_in), _p(kv_in), _p(k_rope), _p(inv_freq), _p(positions), _p(q_out),
         _p(k_cache), _p(v_cache), M, tokens_per_seq, nh, nope, rope, vdim, k_cache.shape[1], _stream())


def mla_latent_cache(q_in, c, k_rope, inv_freq, positions, q_rope, latent_cache, nh, nope, rope,
                     tokens_per_seq=1):
    """Absorbed-weight MLA: RoPE of the query's rope slice -> q_rope [M, nh, rope], and the
    latent cache row [c | rope(k_rope)] of every token at its position
    (latent_cache [B, L, kv_lora + rope])."""
    for t, n in ((q_in, "q_in"), (c, "c"), (k_rope, "k_rope"), (q_rope, "q_rope"),
                 (latent_cache, "latent_cache")):
        _need(t, n)
    _need(inv_freq, "inv_freq", torch.float32)
    _need(positions, "positions", torch.int32)
    M = positions.numel()
    kv_lora = c.shape[-1]
    call("jsx_mla_latent_cache", _p(q_in), _p(c), _p(k_rope), _p(inv_freq), _p(positions), _p(q_rope),
         _p(latent_cache), M, tokens_per_seq, nh, nope, rope, kv_lora, latent_cache.shape[1], _stream())


def mla_absorb(x, token_stride, head_stride, w, out, M, nh, R, K):
    """out[m, h, r] = bf16(sum_k w[h, r, k] x[m, h, k]); x of token m, head h starts at
    element m * token_stride + h * head_stride; w [nh, R, K]; out [M, nh, R]."""
    _need(x, "x")
    _need(w, "w")
    _need(out, "out")
    call("jsx_mla_absorb", _p(x), token_stride, head_stride, _p(w), _p(out), M, nh, R, K, _stream())


def mla_decode_workspace(B, nh, kv_lora, max_seq, device) -> torch.Tensor:
    n = ctypes.c_size_t(0)
    call("jsx_mla_decode_workspace_size", B, nh, kv_lora, max_seq, ctypes.byref(n))
    return torch.empty(n.value, dtype=torch.uint8, device=device)


def mla_decode(q_abs, q_rope, latent_cache, ctx, positions, scale, workspace):
    """Multi-query attention of every head over the latent cache rows [0, position]:
    ctx [B, nh, kv_lora] = bf16(softmax(bf16(bf16(q_abs.c + q_rope.kr) * scale)) . c)."""
    for t, n in ((q_abs, "q_abs"), (q_rope, "q_rope"), (latent_cache, "latent_cache"), (ctx, "ctx")):
        _need(t, n)
    _need(positions, "positions", torch.int32)
    _need(workspace, "workspace", torch.uint8)
    B, L, D = latent_cache.shape
    nh, kv_lora = ctx.shape[-2], ctx.shape[-1]
    call("jsx_mla_decode", _p(q_abs), _p(q_rope), _p(latent_cache), _p(ctx), _p(positions), B, nh, kv_lora,
         D - kv_lora, L, ctypes.c_float(scale), _p(workspace), workspace.numel(), _stream())


def moe_gate(x, w_nk, k, scale, norm=True, correction_bias=None, logits_given=False):
    """Router of layers/moe.py:54-79.  With logits_given, x holds bf16 logits [N, E]."""
    _need(x, "x")
    _opt(correction_bias, "correction_bias", torch.float32)
    if logits_given:
        N, E = x.shape
        H = 0
        w = None
    else:
        _need(w_nk, "w_nk")
        E, H = w_nk.shape
        N = x.numel() // H
        w = w_nk
    topk_w = torch.empty((N, k), dtype=BF16, device=x.device)
    topk_i = torch.empty((N, k), dtype=torch.int32, device=x.device)
    call("jsx_moe_gate", _p(x), _p(w), _p(correction_bias), _p(topk_w), _p(topk_i), N, H, E, k,
         ctypes.c_float(scale), int(bool(norm)), _stream())
    return topk_w, topk_i


# ---- whole decode step (jsx_decode_step) --------------------------------------
class LayerWeights(ctypes.Structure):
    """jsx_layer_weights (include/jsx.h)."""
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("ln1", "w_qkv", "b_qkv", "w_o", "ln2", "w_gu", "w_d", "k_cache", "v_cache")]


class StepArgs(ctypes.Structure):
    """jsx_decode_step_args (include/jsx.h)."""
    _fields_ = ([(n, ctypes.c_int) for n in ("batch", "hidden", "n_heads", "n_kv_heads", "head_dim",
                                            "rotary_dim", "inter", "vocab", "vocab_local", "vocab_offset",
                                            "max_seq", "n_layers")]
                + [("eps", ctypes.c_float), ("scale", ctypes.c_float)]
                + [(n, ctypes.c_void_p) for n in ("layers", "embed", "final_norm", "lm_head", "inv_freq",
                                                  "ids", "positions")]
                + [("advance", ctypes.c_int), ("head", ctypes.c_int)]
                + [(n, ctypes.c_void_p) for n in ("h", "q", "attn", "act", "logits", "workspace")]
                + [("workspace_bytes", ctypes.c_size_t), ("trace", ctypes.c_void_p),
                   ("trace_ar", ctypes.c_void_p), ("l2_next_bytes", ctypes.c_uint32),
                   ("l2_attn_bytes", ctypes.c_uint32), ("trace_phase", ctypes.c_void_p)])


def layer_table(layers, caches, device) -> torch.Tensor:
    """Device array of jsx_layer_weights for the whole-step kernel."""
    arr = (LayerWeights * len(layers))()
    for e, lp, c in zip(arr, layers, caches):
        e.ln1, e.w_qkv = lp.ln1.data_ptr(), lp.w_qkv.data_ptr()
        e.b_qkv = None if lp.b_qkv is None else lp.b_qkv.data_ptr()
        e.w_o, e.ln2, e.w_gu, e.w_d = lp.w_o.data_ptr(), lp.ln2.data_ptr(), lp.w_gu.data_ptr(), lp.w_d.data_ptr()
        e.k_cache, e.v_cache = c.k.data_ptr(), c.v.data_ptr()
    raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
    return raw.to(device)


def step_workspace(args: StepArgs, device) -> torch.Tensor:
    n = ctypes.c_size_t(0)
    call("jsx_decode_step_workspace_size", ctypes.byref(args), ctypes.byref(n))
    return torch.zeros(n.value, dtype=torch.uint8, device=device)


def decode_step(comm, args: StepArgs) -> None:
    handle = None if comm is None else comm.handle
    call("jsx_decode_step", handle, ctypes.byref(args), _stream())
