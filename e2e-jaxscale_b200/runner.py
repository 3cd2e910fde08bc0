"""Generation runner (runner.py:1-460): masks, positions, greedy and sampling generation.

The reference jit-compiles one XLA program per shape and syncs with the host
after every decode step (the EOS check, runner.py:300-306).  Here each step is
a CUDA-graph replay of the per-rank kernel sequence (glm4.DecodeGraph); the
greedy token stays on the device and feeds the next step, and the host reads
it back every step (the same sync the reference performs) only to collect the
output and test for EOS.
"""

from __future__ import annotations

import torch

from . import kernels as K
from .glm4 import WIDE_MIN_TOKENS, DecodeGraph, DecodeState, GLM4ForCausalLM, PrefillState

NEG = -1e9


def make_causal_mask(seq_len: int, dtype=torch.bfloat16) -> torch.Tensor:
    """runner.py:23-30."""
    m = torch.triu(torch.full((seq_len, seq_len), NEG, dtype=dtype), diagonal=1)
    return m[None, None]


def make_prefill_mask(seq_len: int, max_cache_len: int, dtype=torch.bfloat16) -> torch.Tensor:
    """runner.py:33-46."""
    causal = torch.triu(torch.full((seq_len, seq_len), NEG, dtype=dtype), diagonal=1)
    pad = torch.full((seq_len, max_cache_len - seq_len), NEG, dtype=dtype)
    return torch.cat([causal, pad], dim=1)[None, None]


def make_decode_mask(cache_position: int, max_cache_len: int, dtype=torch.bfloat16) -> torch.Tensor:
    """runner.py:49-63."""
    m = torch.where(torch.arange(max_cache_len) <= cache_position,
                    torch.zeros(max_cache_len, dtype=dtype), torch.full((max_cache_len,), NEG, dtype=dtype))
    return m[None, None, None]


def make_positions(seq_len: int, batch_size: int = 1) -> torch.Tensor:
    """runner.py:70-73."""
    return torch.arange(seq_len, dtype=torch.int32)[None].expand(batch_size, seq_len)


class JittedModel:
    """runner.py:113-233 counterpart: same call signature; warmup() builds the
    decode/prefill CUDA graphs for one batch size and cache length."""

    def __init__(self, model: GLM4ForCausalLM):
        self.model = model
        self.config = model.config
        self.dtype = model.dtype
        self.mesh = model.mesh
        self._graphs = {}

    def __call__(self, input_ids, positions, attention_mask, kv_caches=None, cache_position=None):
        return self.model(input_ids, positions, attention_mask, kv_caches=kv_caches,
                          cache_position=cache_position)

    def graph(self, batch_size: int, max_cache_len: int) -> DecodeGraph:
        key = (batch_size, max_cache_len)
        if key not in self._graphs:
            st = DecodeState(self.model, batch_size, max_cache_len)
            self._graphs[key] = DecodeGraph(self.model, st)
        return self._graphs[key]

    def warmup(self, batch_size: int = 1, prompt_len: int = 128, max_cache_len: int = 256):
        self.graph(batch_size, max_cache_len)


def _eos_hit(tok: torch.Tensor, eos) -> bool:
    if eos is None:
        return False
    eos = [eos] if isinstance(eos, int) else list(eos)
    return bool(torch.isin(tok, torch.tensor(eos, dtype=tok.dtype)).all())


def greedy_generate(model, input_ids, max_new_tokens: int = 128, max_cache_len: int | None = None,
                    eos_token_id=None, graph: DecodeGraph | None = None) -> torch.Tensor:
    """runner.py:240-308: prefill the prompt, then greedy decode with the static
    KV cache; stops early when every sequence produced an EOS id.  Returns
    [B, prompt_len + generated] int32 on the host."""
    jm = model if isinstance(model, JittedModel) else JittedModel(model)
    ids = torch.as_tensor(input_ids, dtype=torch.int32)
    B, S = ids.shape
    L = max_cache_len or (S + max_new_tokens)
    g = graph if graph is not None else jm.graph(B, L)
    st = g.st
    dev = jm.model.device
    for cache in st.caches:  # fresh cache (layers/kv_cache.py zero-init)
        cache.k.zero_()
        cache.v.zero_()
    st.pos.zero_()
    host_ids = ids.pin_memory() if torch.cuda.is_available() else ids
    if S > 1 and B * S >= WIDE_MIN_TOKENS:
        # the whole prompt in one pass (wide tensor-core projections + prefill attention)
        ps = PrefillState(jm.model, B, S, L, caches=st.caches)
        st.ids.copy_(jm.model.prefill(ps, host_ids.to(dev, non_blocking=True)))
        st.pos.fill_(S)
    else:
        for s in range(S):
            st.ids.copy_(host_ids[:, s].to(dev, non_blocking=True))
            if s < S - 1:
                g.prefill()
            else:
                g.decode()
    out = [st.ids.to("cpu")]
    for _ in range(max_new_tokens - 1):
        g.decode()
        out.append(st.ids.to("cpu"))
        if _eos_hit(out[-1], eos_token_id):
            break
    return torch.cat([ids] + [t[:, None] for t in out], dim=1)


def _full_logits(model: GLM4ForCausalLM, local: torch.Tensor) -> torch.Tensor:
    """[B, V/tp] vocab shard -> [B, V] (all-gather over the tensor axis)."""
    if model.tp == 1:
        return local
    import torch.distributed as dist
    parts = [torch.empty_like(local) for _ in range(model.tp)]
    dist.all_gather(parts, local.contiguous(), group=model.mesh.group("tensor"))
    return torch.cat(parts, dim=-1).contiguous()


def sample_generate(model: GLM4ForCausalLM, input_ids, max_new_tokens: int = 128, max_cache_len: int | None = None,
                    temperature: float = 0.8, top_k: int = 0, top_p: float = 0.8, repetition_penalty: float = 1.1,
                    eos_token_id=None, seed: int = 42) -> torch.Tensor:
    """runner.py:366-460: prefill, then decode with the sampling of runner.py:315-359
    (jsx_sample) on the full-vocabulary logits of every step.  The presence mask of the
    repetition penalty marks the prompt tokens and every sampled token.  The categorical
    draw's Gumbel noise comes from a torch generator seeded with `seed` (the reference
    draws the same distribution from jax.random with its own key, so the sampled ids
    are not the reference's).  Returns [B, prompt_len + generated] int32 on the host."""
    m = model
    dev, V = m.device, m.config.vocab_size
    ids = torch.as_tensor(input_ids, dtype=torch.int32)
    B, S = ids.shape
    L = max_cache_len or (S + max_new_tokens)
    k = top_k if top_k > 0 else 200
    gen = torch.Generator(device=dev).manual_seed(seed)
    ids_dev = ids.to(dev)
    presence = torch.zeros(B, V, dtype=torch.uint8, device=dev)
    presence.scatter_(1, ids_dev.long(), 1)
    st = DecodeState(m, B, L, want_logits=True)

    def draw(local_logits):
        u = torch.rand(B, k, generator=gen, device=dev).clamp_(1e-20, 1.0)
        g = (-torch.log(-torch.log(u))).to(torch.bfloat16)
        tok = K.sample(_full_logits(m, local_logits), g, presence=presence, repetition_penalty=repetition_penalty,
                       temperature=temperature, top_k=top_k, top_p=top_p)
        presence.scatter_(1, tok.long()[:, None], 1)
        return tok

    if S > 1 and B * S >= WIDE_MIN_TOKENS:
        ps = PrefillState(m, B, S, L, caches=st.caches, want_logits=True)
        m.prefill(ps, ids_dev)
        st.ids.copy_(draw(ps.logits))
    else:
        for s in range(S):
            st.ids.copy_(ids_dev[:, s])
            m.step(st, head=(s == S - 1))
        st.pos.fill_(S)
        st.ids.copy_(draw(st.logits))
    st.pos.fill_(S)
    out = [st.ids.to("cpu")]
    for _ in range(max_new_tokens - 1):
        m.step(st, head=True)  # logits of the fed token's next position
        st.ids.copy_(draw(st.logits))
        out.append(st.ids.to("cpu"))
        if _eos_hit(out[-1], eos_token_id):
            break
    return torch.cat([ids] + [t[:, None] for t in out], dim=1)
