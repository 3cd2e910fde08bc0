"""GQAAttention (layers/attention.py:20-160): q/k/v projections (column-
parallel, bias), partial neox RoPE, static-cache write, SDPA over the cache,
o_proj (row-parallel, all-reduced over the tensor axis).

Kernels, decode (one new position per sequence, or short prompts):
jsx_qkv_rope_cache (projections + bias + RoPE + cache write in one weight
stream), jsx_attn_decode (GQA over cache rows [0, position]),
jsx_row_linear_allreduce (o_proj + all-reduce), one position at a time.
Prompt blocks of 64 tokens or more whose positions run start .. start + S - 1
for every sequence go through in one pass: jsx_wide_qkv_rope_cache (tcgen05
projections + bias + RoPE + cache write), jsx_attn_prefill (causal, rows
[0, start + i]), jsx_wide_row_linear_allreduce (o_proj + the tile-exchange
all-reduce) — the reference's prefill with the mask of runner.py:33-46.
Workspaces and scratch buffers are allocated once per shape and reused.

Masks: the attention_mask argument is accepted for signature compatibility and
not read; attention always covers cache rows [0, position], which is exactly
what the runner's prefill and decode masks select.  positions must equal
cache_position (true for every call the runner makes).
"""

from __future__ import annotations

import numpy as np
import torch

from .. import kernels as K
from ._param import to_device
from .kv_cache import KVCache, local_kv_heads
from .linear import LinearBase
from .rotary import RotaryEmbedding


class GQAAttention:
    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 max_position_embeddings: int, rope_theta: float, mesh, attention_bias: bool = True,
                 dtype=torch.bfloat16, partial_rotary_factor: float = 0.5):
        assert num_heads % num_kv_heads == 0
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.num_kv_groups = num_heads // num_kv_heads
        self.scaling = head_dim ** -0.5
        self.mesh = mesh
        self.q_proj = LinearBase(hidden_size, num_heads * head_dim, mesh, use_bias=attention_bias,
                                 params_dtype=dtype, kernel_axes=(None, "tensor"))
        self.k_proj = LinearBase(hidden_size, num_kv_heads * head_dim, mesh, use_bias=attention_bias,
                                 params_dtype=dtype, kernel_axes=(None, "tensor"))
        self.v_proj = LinearBase(hidden_size, num_kv_heads * head_dim, mesh, use_bias=attention_bias,
                                 params_dtype=dtype, kernel_axes=(None, "tensor"))
        self.o_proj = LinearBase(num_heads * head_dim, hidden_size, mesh, use_bias=False,
                                 params_dtype=dtype, kernel_axes=("tensor", None))
        self.rotary_emb = RotaryEmbedding(head_dim, max_position_embeddings, rope_theta, dtype,
                                          partial_rotary_factor)
        self._packed = None
        self._key = None
        self._bufs = {}

    # --- per-rank shapes ---
    @property
    def tp(self) -> int:
        return 1 if self.mesh is None else self.mesh.shape.get("tensor", 1)

    @property
    def local_heads(self) -> int:
        return self.num_heads // self.tp

    def kv_range(self) -> tuple[int, int]:
        if self.tp == 1:
            return 0, self.num_kv_heads
        return local_kv_heads(self.num_heads, self.num_kv_heads, self.tp, self.mesh.tp_rank)

    def packed(self, device):
        """(w_qkv packed, b_qkv, w_o [H, nq_l*hd]) of this rank."""
        key = tuple(id(p.value) for p in (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight,
                                           self.o_proj.weight)) + (str(device),)
        if self._key == key:
            return self._packed
        hd, tp = self.head_dim, self.tp
        r = 0 if tp == 1 else self.mesh.tp_rank
        nq_l = self.local_heads
        kv0, nkv_l = self.kv_range()
        wq = to_device(self.q_proj.weight.value, device)[:, r * nq_l * hd:(r + 1) * nq_l * hd].contiguous()
        wk = to_device(self.k_proj.weight.value, device)[:, kv0 * hd:(kv0 + nkv_l) * hd].contiguous()
        wv = to_device(self.v_proj.weight.value, device)[:, kv0 * hd:(kv0 + nkv_l) * hd].contiguous()
        w_qkv = K.pack_qkv(wq, wk, wv, nq_l, nkv_l, hd, self.rotary_emb.rotary_dim)
        b_qkv = None
        if self.q_proj.bias is not None:
            bq = to_device(self.q_proj.bias.value, device)[r * nq_l * hd:(r + 1) * nq_l * hd]
            bk = to_device(self.k_proj.bias.value, device)[kv0 * hd:(kv0 + nkv_l) * hd]
            bv = to_device(self.v_proj.bias.value, device)[kv0 * hd:(kv0 + nkv_l) * hd]
            b_qkv = torch.cat([bq, bk, bv]).contiguous()
        w_o = K.pack_transpose(self.o_proj.local_weight(device))
        self._packed = (w_qkv, b_qkv, w_o)
        self._key = key
        return self._packed

    def __call__(self, hidden_states: torch.Tensor, positions: torch.Tensor, attention_mask=None,
                 kv_cache: KVCache | None = None, cache_position: torch.Tensor | None = None,
                 ln_gamma: torch.Tensor | None = None, eps: float = 0.0):
        """hidden_states [B, S, H] -> (out [B, S, H], kv_cache).  ln_gamma (optional)
        fuses the decoder layer's input_layernorm into the projection prologue."""
        dev = hidden_states.device
        B, S, H = hidden_states.shape
        hd = self.head_dim
        nq_l = self.local_heads
        _, nkv_l = self.kv_range()
        w_qkv, b_qkv, w_o = self.packed(dev)
        pos = torch.as_tensor(np.asarray(positions) if not torch.is_tensor(positions) else positions)
        pos = pos.to(device=dev, dtype=torch.int32).reshape(B, S)
        if cache_position is not None:
            cp = torch.as_tensor(np.asarray(cache_position) if not torch.is_tensor(cache_position)
                                 else cache_position)
            cp = cp.to(device=dev, dtype=torch.int32).reshape(1, S)
            if not torch.equal(pos, cp.expand(B, S)):
                raise ValueError("positions must equal cache_position for every sequence")
        if kv_cache is None:
            kc = torch.zeros((B, int(pos.max()) + 1, nkv_l, hd), dtype=torch.bfloat16, device=dev)
            cache = KVCache(kc, torch.zeros_like(kc))
        else:
            cache = kv_cache
        L = cache.k.shape[1]
        inv = self.rotary_emb.inv_freq(dev)
        x = hidden_states.contiguous()
        rot = self.rotary_emb.rotary_dim
        start = int(pos[0, 0])
        if S > 1 and B * S >= 64 and torch.equal(
                pos, (torch.arange(S, dtype=torch.int32, device=dev) + start).expand(B, S)):
            # the whole block in one pass
            M = B * S
            key = ("wide", M, str(dev))
            if key not in self._bufs:
                self._bufs[key] = (
                    K.wide_workspace(M, [(H, w_qkv.shape[0]), (nq_l * hd, H)], dev),
                    torch.empty((M, nq_l * hd), dtype=torch.bfloat16, device=dev),
                    torch.empty((M, nq_l * hd), dtype=torch.bfloat16, device=dev))
            ws, q, o = self._bufs[key]
            K.wide_qkv_rope_cache(x.reshape(M, H), ln_gamma, eps, w_qkv, b_qkv, inv, pos.reshape(-1), q,
                                  cache.k, cache.v, nq_l, nkv_l, hd, rot, ws, tokens_per_seq=S)
            K.attn_prefill(q, cache.k, cache.v, nq_l, nkv_l, hd, S, start_pos=start, scale=self.scaling, out=o)
            y = torch.zeros((M, H), dtype=torch.bfloat16, device=dev)
            K.wide_row_linear_allreduce(self.mesh.comm_tiles(M, H) if self.tp > 1 else None, o, w_o, y, ws)
            return y.reshape(B, S, H), (cache if kv_cache is not None else None)
        key = ("decode", B, L, str(dev))
        if key not in self._bufs:
            self._bufs[key] = (K.attn_workspace(B, nq_l, nkv_l, hd, L, dev),
                               torch.empty((B, nq_l * hd), dtype=torch.bfloat16, device=dev),
                               torch.empty((B, nq_l * hd), dtype=torch.bfloat16, device=dev))
        ws, q, o = self._bufs[key]
        comm = self.mesh.comm(K.MAX_DECODE_TOKENS, H) if self.tp > 1 else None
        out = torch.zeros((B, S, H), dtype=torch.bfloat16, device=dev)
        step = K.MAX_DECODE_TOKENS
        for s in range(S):
            xs = x[:, s].contiguous()
            ps = pos[:, s].contiguous()
            for b0 in range(0, B, step):
                b1 = min(B, b0 + step)
                K.qkv_rope_cache(xs[b0:b1], ln_gamma, eps, w_qkv, b_qkv, inv, ps[b0:b1], q[b0:b1],
                                 cache.k[b0:b1], cache.v[b0:b1], nq_l, nkv_l, hd, rot)
            K.attn_decode(q, cache.k, cache.v, o, ps, self.scaling, ws)
            ys = out[:, s]
            for b0 in range(0, B, step):
                b1 = min(B, b0 + step)
                yb = torch.zeros((b1 - b0, H), dtype=torch.bfloat16, device=dev)
                K.row_linear_allreduce(comm, o[b0:b1], w_o, yb)
                ys[b0:b1] = yb
        return out, (cache if kv_cache is not None else None)
