"""GLM-4-9B dense decoder (models/glm4.py:20-260) on libjsx kernels.

One decode step per rank is 5 kernels per layer plus 2:

    jsx_embed                                  Embed (layers/embedding.py:35-51)
    per layer:
      jsx_qkv_rope_cache   input_layernorm + q/k/v + bias + RoPE + KV write (models/glm4.py:118-120)
      jsx_attn_decode      SDPA over cache rows [0, pos] (layers/attention.py:148-153)
      jsx_row_linear_allreduce  o_proj + TP all-reduce + residual (layers/attention.py:159, models/glm4.py:124)
      jsx_gate_up_swiglu   post_attention_layernorm + gate/up + SwiGLU (models/glm4.py:128, :46-48)
      jsx_row_linear_allreduce  down_proj + TP all-reduce + residual (models/glm4.py:49, :130)
    jsx_lmhead_argmax                          final norm + LM head + argmax (models/glm4.py:193, :251; runner.py:297)

The greedy token is written back into the step's input-id buffer, so
consecutive steps chain on the device and a whole step can be captured in a
CUDA graph (DecodeGraph).
"""

from __future__ import annotations

import math
import os

import torch
import torch.distributed as dist

from . import kernels as K
from .config import ModelConfig
from .layers._param import to_device
from .layers.kv_cache import KVCache, init_kv_caches, local_kv_heads
from .layers.rotary import RotaryEmbedding
from .weights import PackedLayer, RandomLayerSource, pack_layer

CHUNK = K.MAX_DECODE_TOKENS
TC_CHUNK = K.TC_MAX_TOKENS
# smallest batch whose projections run on the tensor cores (jsx_tc_*); smaller
# batches stream the weights through the CUDA-core GEMV / whole-step kernel
TC_MIN_BATCH = int(os.environ.get("JSX_TC_MIN_BATCH", "3"))
# smallest prompt block (batch x prompt tokens) prefilled in one pass on the wide
# tensor-core GEMM and the prefill attention; smaller prompts run token by token
WIDE_MIN_TOKENS = int(os.environ.get("JSX_WIDE_MIN_TOKENS", "64"))
# whole-step kernel: per warp, bytes of the next projection's rows requested into
# L2 once the warp has read its rows of the current one, and bytes of the
# gate/up rows requested while the attention runs (multiples of 16; 0 = none).
# Off by default: at TP=1, batch 1 and 2, every setting measured slower (the
# prefetches compete with the current phase's last reads and the attention's).
L2_NEXT_BYTES = int(os.environ.get("JSX_L2_NEXT_BYTES", "0")) & ~15
L2_ATTN_BYTES = int(os.environ.get("JSX_L2_ATTN_BYTES", "0")) & ~15


class DecodeState:
    """Device buffers of one batch: token ids, positions, activations, caches, workspaces."""

    def __init__(self, model: "GLM4ForCausalLM", batch: int, max_seq: int, caches=None,
                 want_logits: bool = False):
        dev, c = model.device, model.config
        self.batch, self.max_seq = batch, max_seq
        self.ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.h = torch.zeros(batch, c.hidden_size, dtype=torch.bfloat16, device=dev)
        self.q = torch.zeros(batch, model.nq_l * c.head_dim, dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros_like(self.q)
        self.act = torch.zeros(batch, model.I_l, dtype=torch.bfloat16, device=dev)
        self.caches = caches if caches is not None else init_kv_caches(
            batch, max_seq, c.num_hidden_layers, c.num_key_value_heads, c.head_dim, mesh=model.mesh,
            num_heads=c.num_attention_heads, device=dev)
        self.attn_ws = K.attn_workspace(batch, model.nq_l, model.nkv_l, c.head_dim, max_seq, dev)
        self.lm_ws = K.lmhead_workspace(CHUNK, dev)
        self.logits = (torch.zeros(batch, model.V_l, dtype=torch.bfloat16, device=dev)
                       if want_logits else None)
        # batches from TC_MIN_BATCH run the projections on the tensor cores
        self.tc = batch >= TC_MIN_BATCH or batch > CHUNK
        self.step_args = None
        if not self.tc and model.layers:
            self._build_step_args(model)
        self.tc_ws = None
        if self.tc and model.layers:
            lp, H = model.layers[0], c.hidden_size
            shapes = [tuple(reversed(lp.w_qkv.shape)), tuple(reversed(lp.w_o.shape)),
                      tuple(reversed(lp.w_gu.shape)), tuple(reversed(lp.w_d.shape)), (H, model.V_l)]
            self.tc_ws = K.tc_workspace(min(batch, TC_CHUNK), shapes, dev)

    def _build_step_args(self, model: "GLM4ForCausalLM") -> None:
        """Arguments of the whole-step kernel (jsx_decode_step) over these buffers."""
        c, dev = model.config, model.device
        a = K.StepArgs()
        a.batch, a.hidden, a.n_heads, a.n_kv_heads = self.batch, c.hidden_size, model.nq_l, model.nkv_l
        a.head_dim, a.rotary_dim, a.inter = c.head_dim, model.rotary.rotary_dim, model.I_l
        a.vocab, a.vocab_local, a.vocab_offset = c.vocab_size, model.V_l, model.vocab_offset
        a.max_seq, a.n_layers = self.max_seq, len(model.layers)
        a.eps, a.scale = c.rms_norm_eps, model.scale
        self.layer_table = K.layer_table(model.layers, self.caches, dev)
        a.layers = self.layer_table.data_ptr()
        a.embed, a.final_norm, a.lm_head = model.embed.data_ptr(), model.norm.data_ptr(), model.lm_head.data_ptr()
        a.inv_freq = model.inv_freq.data_ptr()
        a.ids, a.positions = self.ids.data_ptr(), self.pos.data_ptr()
        a.advance, a.head = 1, 1
        a.h, a.q, a.attn, a.act = self.h.data_ptr(), self.q.data_ptr(), self.attn.data_ptr(), self.act.data_ptr()
        a.logits = None if self.logits is None else self.logits.data_ptr()
        a.l2_next_bytes, a.l2_attn_bytes = L2_NEXT_BYTES, L2_ATTN_BYTES
        self.step_ws = K.step_workspace(a, dev)
        a.workspace, a.workspace_bytes = self.step_ws.data_ptr(), self.step_ws.numel()
        self.step_args = a


class PrefillState:
    """Device buffers of one prefill block: B sequences x S prompt tokens at
    positions start .. start + S - 1, all processed in one pass (the reference's
    prefill forward, models/glm4.py:162-195 with S > 1)."""

    def __init__(self, model: "GLM4ForCausalLM", batch: int, seq: int, max_seq: int, caches=None,
                 want_logits: bool = False):
        dev, c = model.device, model.config
        M = batch * seq
        self.batch, self.seq, self.max_seq = batch, seq, max_seq
        self.ids = torch.zeros(M, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(M, dtype=torch.int32, device=dev)
        self.h = torch.zeros(M, c.hidden_size, dtype=torch.bfloat16, device=dev)
        self.q = torch.zeros(M, model.nq_l * c.head_dim, dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros_like(self.q)
        self.act = torch.zeros(M, model.I_l, dtype=torch.bfloat16, device=dev)
        self.caches = caches if caches is not None else init_kv_caches(
            batch, max_seq, c.num_hidden_layers, c.num_key_value_heads, c.head_dim, mesh=model.mesh,
            num_heads=c.num_attention_heads, device=dev)
        H = c.hidden_size
        lp = model.layers[0]
        shapes = [tuple(reversed(lp.w_qkv.shape)), tuple(reversed(lp.w_o.shape)),
                  tuple(reversed(lp.w_gu.shape)), tuple(reversed(lp.w_d.shape))]
        self.ws = K.wide_workspace(M, shapes + [(H, model.V_l)], dev)
        # the head: last prompt position of every sequence
        self.last_h = torch.zeros(batch, H, dtype=torch.bfloat16, device=dev)
        self.next_ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.logits = (torch.zeros(batch, model.V_l, dtype=torch.bfloat16, device=dev)
                       if want_logits else None)
        self.tc_ws = K.tc_workspace(min(batch, TC_CHUNK), [(H, model.V_l)], dev)
        self.comm = model.mesh.comm_tiles(M, H) if model.tp > 1 else None


class GLM4ForCausalLM:
    """models/glm4.py:198-260.  __call__ keeps the reference signature; the
    decode fast path is step()/DecodeGraph, the prompt fast path prefill()."""

    def __init__(self, config: ModelConfig, mesh, dtype=torch.bfloat16):
        c = config
        self.config, self.mesh, self.dtype = c, mesh, dtype
        self.device = mesh.device if mesh.device is not None else torch.device("cuda")
        self.tp = mesh.shape.get("tensor", 1)
        self.rank = mesh.tp_rank
        t = self.tp
        if c.num_attention_heads % t or c.intermediate_size % t or c.vocab_size % t:
            raise ValueError(f"tp={t} must divide heads, intermediate_size and vocab_size")
        self.nq_l = c.num_attention_heads // t
        self.kv0, self.nkv_l = ((0, c.num_key_value_heads) if t == 1 else
                                local_kv_heads(c.num_attention_heads, c.num_key_value_heads, t, self.rank))
        self.I_l = c.intermediate_size // t
        self.V_l = c.vocab_size // t
        self.vocab_offset = self.rank * self.V_l
        self.rotary = RotaryEmbedding(c.head_dim, c.max_position_embeddings, c.rope_theta, dtype,
                                      c.partial_rotary_factor)
        self.inv_freq = self.rotary.inv_freq(self.device)
        self.scale = c.head_dim ** -0.5
        self.layers: list[PackedLayer] = []
        self.embed = None     # [V, H] replicated
        self.norm = None      # [H]
        self.lm_head = None   # [V_l, H]
        self.comm = mesh.comm(TC_CHUNK, c.hidden_size) if t > 1 else None
        self.fused_step = os.environ.get("JSX_FUSED_STEP", "1") != "0"

    # ---- weights ----
    def load_state(self, params) -> None:
        """params: reference-layout parameters (attributes or keys embed, layers[i].{ln1, wq, bq,
        wk, bk, wv, bv, wo, ln2, wg, wu, wd}, norm, lm_head [V, H])."""
        g = (lambda o, n: o[n] if isinstance(o, dict) else getattr(o, n))
        dev, c = self.device, self.config
        self.layers = [pack_layer(lp, c, self.tp, self.rank, dev) for lp in g(params, "layers")]
        self.embed = to_device(g(params, "embed"), dev)
        self.norm = to_device(g(params, "norm"), dev)
        lm = to_device(g(params, "lm_head"), dev)
        self.lm_head = lm[self.vocab_offset:self.vocab_offset + self.V_l].contiguous()
        del lm
        torch.cuda.synchronize(dev)

    def load_weights(self, model_config: ModelConfig | None = None) -> None:
        """models/glm4.py:262-274: this rank's shards of the HF safetensors checkpoint in
        (model_config or self.config).model_path (checkpoint.py holds the name mapping)."""
        from .checkpoint import load_glm4
        load_glm4(self, (model_config or self.config).model_path)

    def init_random(self, seed: int = 0) -> None:
        """Synthetic N(0, 0.02) bf16 weights generated on the device, gains = 1."""
        dev, c = self.device, self.config
        src = RandomLayerSource(c, dev, seed)
        self.embed = src.normal(c.vocab_size, c.hidden_size)
        self.layers = []
        for _ in range(c.num_hidden_layers):
            lp = src.layer()
            self.layers.append(pack_layer(lp, c, self.tp, self.rank, dev))
            del lp
        self.norm = torch.ones(c.hidden_size, dtype=torch.bfloat16, device=dev)
        lm = src.normal(c.vocab_size, c.hidden_size)
        self.lm_head = lm[self.vocab_offset:self.vocab_offset + self.V_l].contiguous()
        del lm
        torch.cuda.synchronize(dev)

    def weight_bytes(self) -> int:
        """Bytes of weights this rank streams per decode step (layers + LM-head shard + norm)."""
        n = sum(lp.nbytes() for lp in self.layers)
        return n + self.lm_head.numel() * 2 + self.norm.numel() * 2

    # ---- the decode step ----
    def run_body(self, st: DecodeState) -> None:
        """Embedding + all decoder layers for one token per sequence at st.pos."""
        c = self.config
        B, eps, hd, rot = st.batch, c.rms_norm_eps, c.head_dim, self.rotary.rotary_dim
        K.embed(st.ids, self.embed, out=st.h)
        if st.tc:
            self._run_body_tc(st)
            return
        for lp, cache in zip(self.layers, st.caches):
            for b0 in range(0, B, CHUNK):
                b1 = min(B, b0 + CHUNK)
                K.qkv_rope_cache(st.h[b0:b1], lp.ln1, eps, lp.w_qkv, lp.b_qkv, self.inv_freq,
                                 st.pos[b0:b1], st.q[b0:b1], cache.k[b0:b1], cache.v[b0:b1],
                                 self.nq_l, self.nkv_l, hd, rot)
            K.attn_decode(st.q, cache.k, cache.v, st.attn, st.pos, self.scale, st.attn_ws)
            for b0 in range(0, B, CHUNK):
                b1 = min(B, b0 + CHUNK)
                K.row_linear_allreduce(self.comm, st.attn[b0:b1], lp.w_o, st.h[b0:b1])
            for b0 in range(0, B, CHUNK):
                b1 = min(B, b0 + CHUNK)
                K.gate_up_swiglu(st.h[b0:b1], lp.ln2, eps, lp.w_gu, st.act[b0:b1])
            for b0 in range(0, B, CHUNK):
                b1 = min(B, b0 + CHUNK)
                K.row_linear_allreduce(self.comm, st.act[b0:b1], lp.w_d, st.h[b0:b1])

    def _run_body_tc(self, st: DecodeState) -> None:
        """Decoder layers with the projections on the tensor cores (jsx_tc_*), up to 32 tokens a call."""
        c = self.config
        B, eps, hd, rot, ws = st.batch, c.rms_norm_eps, c.head_dim, self.rotary.rotary_dim, st.tc_ws
        spans = [(b0, min(B, b0 + TC_CHUNK)) for b0 in range(0, B, TC_CHUNK)]
        for lp, cache in zip(self.layers, st.caches):
            for b0, b1 in spans:
                K.tc_qkv_rope_cache(st.h[b0:b1], lp.ln1, eps, lp.w_qkv, lp.b_qkv, self.inv_freq,
                                    st.pos[b0:b1], st.q[b0:b1], cache.k[b0:b1], cache.v[b0:b1],
                                    self.nq_l, self.nkv_l, hd, rot, ws)
            K.attn_decode(st.q, cache.k, cache.v, st.attn, st.pos, self.scale, st.attn_ws)
            for b0, b1 in spans:
                K.tc_row_linear_allreduce(self.comm, st.attn[b0:b1], lp.w_o, st.h[b0:b1], ws)
            for b0, b1 in spans:
                K.tc_gate_up_swiglu(st.h[b0:b1], lp.ln2, eps, lp.w_gu, st.act[b0:b1], ws)
            for b0, b1 in spans:
                K.tc_row_linear_allreduce(self.comm, st.act[b0:b1], lp.w_d, st.h[b0:b1], ws)

    def run_head(self, st: DecodeState) -> None:
        """Final norm + LM head + greedy argmax; the token ids overwrite st.ids."""
        if st.tc:
            for b0 in range(0, st.batch, TC_CHUNK):
                b1 = min(st.batch, b0 + TC_CHUNK)
                K.tc_lmhead_argmax(self.comm, st.h[b0:b1], self.norm, self.config.rms_norm_eps, self.lm_head,
                                   self.vocab_offset, st.ids[b0:b1], st.tc_ws,
                                   None if st.logits is None else st.logits[b0:b1])
            return
        for b0 in range(0, st.batch, CHUNK):
            b1 = min(st.batch, b0 + CHUNK)
            K.lmhead_argmax(self.comm, st.h[b0:b1], self.norm, self.config.rms_norm_eps, self.lm_head,
                            self.vocab_offset, st.ids[b0:b1], st.lm_ws,
                            None if st.logits is None else st.logits[b0:b1])

    def step(self, st: DecodeState, head: bool = True) -> None:
        """One token per sequence at st.pos; st.ids <- greedy tokens (head), st.pos += 1.
        Small batches run the whole step as one kernel (jsx_decode_step) unless
        self.fused_step is False; batches from TC_MIN_BATCH chain the tensor-core
        projections and the attention kernel."""
        if self.fused_step and st.step_args is not None:
            st.step_args.head = 1 if head else 0
            K.decode_step(self.comm, st.step_args)
            return
        self.run_body(st)
        if head:
            self.run_head(st)
        st.pos.add_(1)

    # ---- prefill: the whole prompt block in one pass ----
    def prefill_body(self, ps: PrefillState, input_ids, start: int = 0) -> None:
        """Embedding + all decoder layers over B x S prompt tokens at positions
        start .. start + S - 1 (models/glm4.py:162-195 at prefill; the caches
        receive rows [start, start + S)).  input_ids: [B, S] on the device."""
        c = self.config
        B, S = ps.batch, ps.seq
        eps, hd, rot, ws = c.rms_norm_eps, c.head_dim, self.rotary.rotary_dim, ps.ws
        ps.ids.copy_(input_ids.reshape(-1))
        ps.pos.copy_((torch.arange(S, dtype=torch.int32, device=self.device) + start).repeat(B))
        K.embed(ps.ids, self.embed, out=ps.h)
        for lp, cache in zip(self.layers, ps.caches):
            K.wide_qkv_rope_cache(ps.h, lp.ln1, eps, lp.w_qkv, lp.b_qkv, self.inv_freq, ps.pos, ps.q,
                                  cache.k, cache.v, self.nq_l, self.nkv_l, hd, rot, ws, tokens_per_seq=S)
            K.attn_prefill(ps.q, cache.k, cache.v, self.nq_l, self.nkv_l, hd, S, start_pos=start,
                           scale=self.scale, out=ps.attn)
            K.wide_row_linear_allreduce(ps.comm, ps.attn, lp.w_o, ps.h, ws)
            K.wide_gate_up_swiglu(ps.h, lp.ln2, eps, lp.w_gu, ps.act, ws)
            K.wide_row_linear_allreduce(ps.comm, ps.act, lp.w_d, ps.h, ws)

    def prefill(self, ps: PrefillState, input_ids, start: int = 0) -> torch.Tensor:
        """prefill_body, then the final norm + LM head + greedy argmax at the last
        prompt position of every sequence (runner.py:281); returns ps.next_ids."""
        self.prefill_body(ps, input_ids, start)
        ps.last_h.copy_(ps.h.view(ps.batch, ps.seq, -1)[:, -1])
        for b0 in range(0, ps.batch, TC_CHUNK):
            b1 = min(ps.batch, b0 + TC_CHUNK)
            K.tc_lmhead_argmax(self.comm, ps.last_h[b0:b1], self.norm, self.config.rms_norm_eps, self.lm_head,
                               self.vocab_offset, ps.next_ids[b0:b1], ps.tc_ws,
                               None if ps.logits is None else ps.logits[b0:b1])
        return ps.next_ids

    def kernels_per_step(self, batch: int, head: bool = True) -> int:
        tc = batch >= TC_MIN_BATCH or batch > CHUNK
        if self.fused_step and not tc:
            return 1
        if tc:
            # per layer and 32-token chunk: RMSNorm + GEMM (qkv, gate_up), GEMM (o, down; plus the
            # NVLink all-reduce kernel when tp > 1); attention once per layer; LM head RMSNorm + GEMM
            ch = math.ceil(batch / TC_CHUNK)
            per = 6 + (2 if self.tp > 1 else 0)
            n = 1 + self.config.num_hidden_layers * (1 + per * ch)
            return n + (2 * ch if head else 0)
        ch = math.ceil(batch / CHUNK)
        n = 1 + self.config.num_hidden_layers * (1 + 4 * ch)
        return n + (ch if head else 0)

    # ---- reference-signature forward (models/glm4.py:226-260) ----
    def __call__(self, input_ids, positions, attention_mask=None, kv_caches=None, cache_position=None):
        """logits [B, S, V] (bf16, gathered over TP ranks) and the updated caches.
        Tokens are run one position at a time (causal, exactly the reference's
        prefill/decode masks); positions must equal cache_position."""
        dev = self.device
        ids = torch.as_tensor(input_ids).to(device=dev, dtype=torch.int32)
        B, S = ids.shape
        pos = torch.as_tensor(positions).to(device=dev, dtype=torch.int32).reshape(B, S)
        if cache_position is not None:
            cp = torch.as_tensor(cache_position).to(device=dev, dtype=torch.int32).reshape(1, S)
            if not torch.equal(pos, cp.expand(B, S)):
                raise ValueError("positions must equal cache_position for every sequence")
        L = kv_caches[0].k.shape[1] if kv_caches is not None else int(pos.max()) + 1
        start = int(pos[0, 0])
        if S > 1 and B * S >= WIDE_MIN_TOKENS and torch.equal(
                pos, (torch.arange(S, dtype=torch.int32, device=dev) + start).expand(B, S)):
            # one pass over the whole block; logits of every position (layers/embedding.py:88-92)
            ps = PrefillState(self, B, S, L, caches=kv_caches)
            self.prefill_body(ps, ids, start)
            local = K.wide_linear(ps.h, self.lm_head, ps.ws, gamma=self.norm, eps=self.config.rms_norm_eps)
            if self.tp > 1:
                parts = [torch.empty_like(local) for _ in range(self.tp)]
                dist.all_gather(parts, local, group=self.mesh.group("tensor"))
                local = torch.cat(parts, dim=-1)
            return local.reshape(B, S, -1), (ps.caches if kv_caches is not None else None)
        st = DecodeState(self, B, L, caches=kv_caches, want_logits=True)
        logits = torch.empty(B, S, self.config.vocab_size, dtype=torch.bfloat16, device=dev)
        for s in range(S):
            st.ids.copy_(ids[:, s])
            st.pos.copy_(pos[:, s])
            self.run_body(st)
            self.run_head(st)
            if self.tp > 1:
                parts = [torch.empty_like(st.logits) for _ in range(self.tp)]
                dist.all_gather(parts, st.logits, group=self.mesh.group("tensor"))
                logits[:, s] = torch.cat(parts, dim=-1)
            else:
                logits[:, s] = st.logits
        return logits, (st.caches if kv_caches is not None else None)

    def init_kv_caches(self, batch_size: int, max_seq_len: int) -> list[KVCache]:
        c = self.config
        return init_kv_caches(batch_size, max_seq_len, c.num_hidden_layers, c.num_key_value_heads,
                              c.head_dim, mesh=self.mesh, num_heads=c.num_attention_heads,
                              device=self.device)


class DecodeGraph:
    """CUDA graphs of one decode step (body + head + pos advance) and of one
    prefill step (body + pos advance) over a DecodeState."""

    def __init__(self, model: GLM4ForCausalLM, st: DecodeState, warmup: bool = True):
        self.model, self.st = model, st
        if warmup:
            # one eager pass per graph so every lazily-initialised resource exists
            # before capture; restore the state afterwards
            ids, pos = st.ids.clone(), st.pos.clone()
            model.step(st, head=True)
            st.ids.copy_(ids)
            st.pos.copy_(pos)
            torch.cuda.synchronize(model.device)
        self.pool = torch.cuda.graph_pool_handle()
        self.g_decode = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g_decode, pool=self.pool):
            model.step(st, head=True)
        self.g_prefill = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g_prefill, pool=self.pool):
            model.step(st, head=False)

    def decode(self) -> None:
        self.g_decode.replay()

    def prefill(self) -> None:
        self.g_prefill.replay()

    def release(self) -> None:
        self.g_decode = None
        self.g_prefill = None
