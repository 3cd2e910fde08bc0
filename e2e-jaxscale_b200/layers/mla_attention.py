"""MLAAttention (layers/mla_attention.py:34-193): GLM-4.7-Flash multi-head latent
attention with the reference's expanded per-head cache.

Per query position: q_a (replicated) -> q_b with the q_a RMSNorm fused as its
prologue (column-parallel over heads); kv_a_proj_with_mqa split into its latent
columns and its shared rope-key columns (replicated) -> kv_b with the kv_a
RMSNorm as prologue (column-parallel); jsx_mla_rope_cache (RoPE on the rope
slice of q and on the shared key, [nope | rope] concatenation, cache write);
jsx_attn_decode with one query head per kv head (MHA) over cache rows
[0, position]; o_proj row-parallel with the fused all-reduce.

The reference rounds the scores q.k to bf16 before scaling (jnp.matmul on bf16
operands); the attention kernel keeps them in fp32 (within the tolerance).  The
attention_mask argument is accepted and not read: rows [0, position] are what the
runner's prefill/decode masks select.  positions must equal cache_position.

absorbed=True: the latent-cache decode form (the reference's own named fix for
MLA's share of layer time, README.md:67).  The cache is KVCache(k=latent
[B, L, kv_lora + rope], v=empty): per token the normalised kv latent and the
rotated shared rope key, 576 values for GLM-4.7-Flash instead of the expanded
nh * 512.  Per position: q_a -> q_b (fused RMSNorm), kv_a -> RMSNorm -> c;
jsx_mla_latent_cache (RoPE of q's rope slice, cache row [c | RoPE(k_rope)]);
q_abs = the key columns of kv_b applied to q_nope per head (jsx_mla_absorb);
jsx_mla_decode (one multi-query attention of all local heads over the latent
rows [0, position]); the value columns of kv_b applied to the latent context
(jsx_mla_absorb); o_proj with the fused all-reduce.  It agrees with the
expanded form to bf16 rounding (k_nope and v are never materialised).
"""

from __future__ import annotations

import numpy as np
import torch

from .. import kernels as K
from ._param import to_device
from .kv_cache import KVCache
from .linear import LinearBase
from .normalization import RMSNorm
from .rotary import RotaryEmbedding


class MLAAttention:
    def __init__(self, hidden_size: int, num_heads: int, q_lora_rank: int, kv_lora_rank: int,
                 qk_nope_head_dim: int, qk_rope_head_dim: int, v_head_dim: int, max_position_embeddings: int,
                 rope_theta: float, rms_norm_eps: float, mesh, dtype=torch.bfloat16, absorbed: bool = False):
        self.absorbed = absorbed
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.qk_nope_head_dim = qk_nope_head_dim
        self.qk_rope_head_dim = qk_rope_head_dim
        self.v_head_dim = v_head_dim
        self.qk_head_dim = qk_nope_head_dim + qk_rope_head_dim
        self.scaling = self.qk_head_dim ** -0.5
        self.kv_lora_rank = kv_lora_rank
        self.mesh = mesh
        self.q_a_proj = LinearBase(hidden_size, q_lora_rank, mesh, params_dtype=dtype, kernel_axes=(None, None))
        self.q_a_layernorm = RMSNorm(q_lora_rank, epsilon=rms_norm_eps, param_dtype=dtype)
        self.q_b_proj = LinearBase(q_lora_rank, num_heads * self.qk_head_dim, mesh, params_dtype=dtype,
                                   kernel_axes=(None, "tensor"))
        self.kv_a_proj_with_mqa = LinearBase(hidden_size, kv_lora_rank + qk_rope_head_dim, mesh,
                                             params_dtype=dtype, kernel_axes=(None, None))
        self.kv_a_layernorm = RMSNorm(kv_lora_rank, epsilon=rms_norm_eps, param_dtype=dtype)
        self.kv_b_proj = LinearBase(kv_lora_rank, num_heads * (qk_nope_head_dim + v_head_dim), mesh,
                                    params_dtype=dtype, kernel_axes=(None, "tensor"))
        self.o_proj = LinearBase(num_heads * v_head_dim, hidden_size, mesh, params_dtype=dtype,
                                 kernel_axes=("tensor", None))
        self.rotary_emb = RotaryEmbedding(qk_rope_head_dim, max_position_embeddings, rope_theta, dtype,
                                          partial_rotary_factor=1.0)
        self._key = None

    @property
    def tp(self) -> int:
        return 1 if self.mesh is None else self.mesh.shape.get("tensor", 1)

    @property
    def local_heads(self) -> int:
        return self.num_heads // self.tp

    def _pack(self, device):
        key = tuple(id(l.weight.value) for l in (self.q_a_proj, self.q_b_proj, self.kv_a_proj_with_mqa,
                                                  self.kv_b_proj, self.o_proj)) + (str(device),)
        if self._key == key:
            return
        kvl = self.kv_lora_rank
        kva = to_device(self.kv_a_proj_with_mqa.weight.value, device)
        self.w_qa = K.pack_transpose(to_device(self.q_a_proj.weight.value, device))
        self.w_qb = K.pack_transpose(self.q_b_proj.local_weight(device))
        self.w_kva_lat = K.pack_transpose(kva[:, :kvl].contiguous())
        self.w_kva_rope = K.pack_transpose(kva[:, kvl:].contiguous())
        self.w_kvb = K.pack_transpose(self.kv_b_proj.local_weight(device))
        self.w_o = K.pack_transpose(self.o_proj.local_weight(device))
        self.g_qa = self.q_a_layernorm.gain(device)
        self.g_kva = self.kv_a_layernorm.gain(device)
        if self.absorbed:
            # kv_b [kv_lora, nh_l (nope + v)] -> per head the key columns transposed
            # [nh_l, kv_lora, nope] and the value columns transposed [nh_l, v, kv_lora]
            nh, nope, vd = self.local_heads, self.qk_nope_head_dim, self.v_head_dim
            wkv = to_device(self.kv_b_proj.local_weight(device), device).reshape(kvl, nh, nope + vd)
            self.w_k_abs = wkv[..., :nope].permute(1, 0, 2).contiguous()
            self.w_v_abs = wkv[..., nope:].permute(1, 2, 0).contiguous()
            del wkv
        self._key = key

    def __call__(self, hidden_states: torch.Tensor, positions: torch.Tensor, attention_mask=None,
                 kv_cache: KVCache | None = None, cache_position: torch.Tensor | None = None):
        """hidden_states [B, S, H] -> (out [B, S, H], kv_cache with k [B, L, nh_l, nope+rope],
        v [B, L, nh_l, v])."""
        dev = hidden_states.device
        self._pack(dev)
        B, S, H = hidden_states.shape
        nh, nope, rope, vd = self.local_heads, self.qk_nope_head_dim, self.qk_rope_head_dim, self.v_head_dim
        qd = nope + rope
        if torch.is_tensor(positions):  # device positions: no host round trip (graph capture)
            pos = positions.to(device=dev, dtype=torch.int32).reshape(B, S)
        else:
            pos = torch.as_tensor(np.array(positions)).to(device=dev, dtype=torch.int32).reshape(B, S)
        if cache_position is not None:
            cp = torch.as_tensor(np.array(cache_position)).to(device=dev, dtype=torch.int32).reshape(1, S)
            if not torch.equal(pos, cp.expand(B, S)):
                raise ValueError("positions must equal cache_position for every sequence")
        if self.absorbed:
            return self._call_absorbed(hidden_states, pos, kv_cache)
        if kv_cache is None:
            L = int(pos.max()) + 1
            cache = KVCache(torch.zeros((B, L, nh, qd), dtype=torch.bfloat16, device=dev),
                            torch.zeros((B, L, nh, vd), dtype=torch.bfloat16, device=dev))
        else:
            cache = kv_cache
        if qd != vd:
            raise NotImplementedError("the decode attention kernel takes one head_dim for K and V")
        L = cache.k.shape[1]
        inv = self.rotary_emb.inv_freq(dev)
        ws = K.attn_workspace(B, nh, nh, qd, L, dev)
        comm = self.mesh.comm(K.MAX_DECODE_TOKENS, H) if self.tp > 1 else None
        eps_q, eps_kv = self.q_a_layernorm.epsilon, self.kv_a_layernorm.epsilon
        x = hidden_states.contiguous()
        out = torch.zeros((B, S, H), dtype=torch.bfloat16, device=dev)
        step = K.MAX_DECODE_TOKENS
        qc = torch.empty((B, self.w_qa.shape[0]), dtype=torch.bfloat16, device=dev)
        q = torch.empty((B, nh * qd), dtype=torch.bfloat16, device=dev)
        kvl = torch.empty((B, self.kv_lora_rank), dtype=torch.bfloat16, device=dev)
        kr = torch.empty((B, rope), dtype=torch.bfloat16, device=dev)
        kv = torch.empty((B, nh * (nope + vd)), dtype=torch.bfloat16, device=dev)
        qr = torch.empty((B, nh * qd), dtype=torch.bfloat16, device=dev)
        o = torch.empty((B, nh * vd), dtype=torch.bfloat16, device=dev)
        for s in range(S):
            xs = x[:, s].contiguous()
            ps = pos[:, s].contiguous()
            for b0 in range(0, B, step):
                b1 = min(B, b0 + step)
                K.linear(xs[b0:b1], self.w_qa, out=qc[b0:b1])
                K.linear(qc[b0:b1], self.w_qb, gamma=self.g_qa, eps=eps_q, out=q[b0:b1])
                K.linear(xs[b0:b1], self.w_kva_lat, out=kvl[b0:b1])
                K.linear(xs[b0:b1], self.w_kva_rope, out=kr[b0:b1])
                K.linear(kvl[b0:b1], self.w_kvb, gamma=self.g_kva, eps=eps_kv, out=kv[b0:b1])
            K.mla_rope_cache(q, kv, kr, inv, ps, qr, cache.k, cache.v, nh, nope, rope, vd)
            K.attn_decode(qr, cache.k, cache.v, o, ps, self.scaling, ws)
            ys = torch.zeros((B, H), dtype=torch.bfloat16, device=dev)
            for b0 in range(0, B, step):
                b1 = min(B, b0 + step)
                K.row_linear_allreduce(comm, o[b0:b1], self.w_o, ys[b0:b1])
            out[:, s] = ys
        return out, (cache if kv_cache is not None else None)

    def init_latent_cache(self, batch_size: int, max_seq_len: int, device) -> KVCache:
        """Zero latent cache of the absorbed form: k [B, L, kv_lora + rope], v empty."""
        return KVCache(torch.zeros((batch_size, max_seq_len, self.kv_lora_rank + self.qk_rope_head_dim),
                                   dtype=torch.bfloat16, device=device),
                       torch.empty(0, dtype=torch.bfloat16, device=device))

    def _call_absorbed(self, hidden_states, pos, kv_cache):
        dev = hidden_states.device
        B, S, H = hidden_states.shape
        nh, nope, rope, vd = self.local_heads, self.qk_nope_head_dim, self.qk_rope_head_dim, self.v_head_dim
        kvl = self.kv_lora_rank
        qd = nope + rope
        cache = kv_cache if kv_cache is not None else self.init_latent_cache(B, int(pos.max()) + 1, dev)
        if cache.k.dim() != 3 or cache.k.shape[-1] != kvl + rope or cache.k.shape[0] != B:
            raise ValueError(f"absorbed MLA needs a latent cache [B, L, {kvl + rope}], got {tuple(cache.k.shape)}")
        L = cache.k.shape[1]
        inv = self.rotary_emb.inv_freq(dev)
        ws = K.mla_decode_workspace(B, nh, kvl, L, dev)
        comm = self.mesh.comm(K.MAX_DECODE_TOKENS, H) if self.tp > 1 else None
        eps_q, eps_kv = self.q_a_layernorm.epsilon, self.kv_a_layernorm.epsilon
        x = hidden_states.contiguous()
        out = torch.zeros((B, S, H), dtype=torch.bfloat16, device=dev)
        step = K.MAX_DECODE_TOKENS
        qc = torch.empty((B, self.w_qa.shape[0]), dtype=torch.bfloat16, device=dev)
        q = torch.empty((B, nh * qd), dtype=torch.bfloat16, device=dev)
        lat = torch.empty((B, kvl), dtype=torch.bfloat16, device=dev)
        c = torch.empty((B, kvl), dtype=torch.bfloat16, device=dev)
        kr = torch.empty((B, rope), dtype=torch.bfloat16, device=dev)
        q_rope = torch.empty((B, nh, rope), dtype=torch.bfloat16, device=dev)
        q_abs = torch.empty((B, nh, kvl), dtype=torch.bfloat16, device=dev)
        ctx = torch.empty((B, nh, kvl), dtype=torch.bfloat16, device=dev)
        o = torch.empty((B, nh * vd), dtype=torch.bfloat16, device=dev)
        for s in range(S):
            xs = x[:, s].contiguous()
            ps = pos[:, s].contiguous()
            for b0 in range(0, B, step):
                b1 = min(B, b0 + step)
                K.linear(xs[b0:b1], self.w_qa, out=qc[b0:b1])
                K.linear(qc[b0:b1], self.w_qb, gamma=self.g_qa, eps=eps_q, out=q[b0:b1])
                K.linear(xs[b0:b1], self.w_kva_lat, out=lat[b0:b1])
                K.linear(xs[b0:b1], self.w_kva_rope, out=kr[b0:b1])
            K.rmsnorm(lat, self.g_kva, eps_kv, out=c)
            K.mla_latent_cache(q, c, kr, inv, ps, q_rope, cache.k, nh, nope, rope)
            for b0 in range(0, B, 32):
                b1 = min(B, b0 + 32)
                K.mla_absorb(q[b0:b1], nh * qd, qd, self.w_k_abs, q_abs[b0:b1], b1 - b0, nh, kvl, nope)
            K.mla_decode(q_abs, q_rope, cache.k, ctx, ps, self.scaling, ws)
            for b0 in range(0, B, 32):
                b1 = min(B, b0 + 32)
                K.mla_absorb(ctx[b0:b1], nh * kvl, kvl, self.w_v_abs, o[b0:b1], b1 - b0, nh, vd, kvl)
            ys = torch.zeros((B, H), dtype=torch.bfloat16, device=dev)
            for b0 in range(0, B, step):
                b1 = min(B, b0 + step)
                K.row_linear_allreduce(comm, o[b0:b1], self.w_o, ys[b0:b1])
            out[:, s] = ys
        return out, (cache if kv_cache is not None else None)
