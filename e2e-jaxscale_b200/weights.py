"""Per-rank weight placement and packing (utils/weight_utils.py:164-265), and
the synthetic random-init used when no checkpoint is available.

Input: reference-layout parameters of one decoder layer — W[in, out] matrices
(layers/linear.py:16), biases, RMSNorm gains — as numpy arrays or torch
tensors, under the names ln1, wq, bq, wk, bk, wv, bv, wo, ln2, wg, wu, wd
(attributes or dict keys).  Output: this rank's packed device tensors.

Sharding follows the reference's kernel_axes: q/k/v/gate/up split on the
output dim, o/down on the input dim, column biases split with their columns.
KV heads: split when tp <= num_kv_heads, else each rank keeps the one head its
query heads read (the reference's P(None, None, "tensor", None) cache sharding
only divides at tp <= 2).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import kernels as K
from .layers._param import to_device
from .layers.kv_cache import local_kv_heads


def _get(obj, name):
    return obj[name] if isinstance(obj, dict) else getattr(obj, name)


@dataclass
class PackedLayer:
    ln1: torch.Tensor    # [H] bf16
    w_qkv: torch.Tensor  # [(nq_l + 2 nkv_l) hd, H] packed (jsx_pack_qkv)
    b_qkv: torch.Tensor  # [(nq_l + 2 nkv_l) hd] (q | k | v) or None
    w_o: torch.Tensor    # [H, nq_l hd]
    ln2: torch.Tensor
    w_gu: torch.Tensor   # [2 I_l, H] packed (jsx_pack_gate_up)
    w_d: torch.Tensor    # [H, I_l]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.ln1, self.w_qkv, self.b_qkv, self.w_o, self.ln2, self.w_gu, self.w_d)
                   if t is not None)


def pack_layer(lp, cfg, tp: int, rank: int, device) -> PackedLayer:
    hd, nq, nkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    H, I = cfg.hidden_size, cfg.intermediate_size
    nq_l, I_l = nq // tp, I // tp
    kv0, nkv_l = (0, nkv) if tp == 1 else local_kv_heads(nq, nkv, tp, rank)
    qc = slice(rank * nq_l * hd, (rank + 1) * nq_l * hd)
    kvc = slice(kv0 * hd, (kv0 + nkv_l) * hd)
    ic = slice(rank * I_l, (rank + 1) * I_l)

    def dev(name):
        return to_device(_get(lp, name), device)

    wq = dev("wq")[:, qc].contiguous()
    wk = dev("wk")[:, kvc].contiguous()
    wv = dev("wv")[:, kvc].contiguous()
    w_qkv = K.pack_qkv(wq, wk, wv, nq_l, nkv_l, hd, cfg.rotary_dim)
    del wq, wk, wv
    b_qkv = None
    if cfg.attention_bias:
        b_qkv = torch.cat([dev("bq")[qc], dev("bk")[kvc], dev("bv")[kvc]]).contiguous()
    w_o = K.pack_transpose(dev("wo")[qc].contiguous())
    wg = dev("wg")[:, ic].contiguous()
    wu = dev("wu")[:, ic].contiguous()
    w_gu = K.pack_gate_up(wg, wu)
    del wg, wu
    w_d = K.pack_transpose(dev("wd")[ic].contiguous())
    return PackedLayer(ln1=dev("ln1"), w_qkv=w_qkv, b_qkv=b_qkv, w_o=w_o, ln2=dev("ln2"), w_gu=w_gu,
                       w_d=w_d)


class RandomLayerSource:
    """Seeded on-device N(0, std) weights in reference layout, one layer at a
    time (fp32 draws from a CUDA torch.Generator, rounded to bf16).  Every rank
    draws the same global tensors and slices its shard, so TP = 1 and TP = N
    hold the same model."""

    def __init__(self, cfg, device, seed: int = 0, std: float = 0.02):
        self.cfg, self.device, self.std = cfg, device, std
        self.gen = torch.Generator(device=device)
        self.gen.manual_seed(seed)

    def normal(self, *shape) -> torch.Tensor:
        t = torch.randn(*shape, generator=self.gen, device=self.device, dtype=torch.float32)
        return (t * self.std).to(torch.bfloat16)

    def layer(self) -> dict:
        c = self.cfg
        H, hd, nq, nkv, I = c.hidden_size, c.head_dim, c.num_attention_heads, c.num_key_value_heads, \
            c.intermediate_size
        d = {"ln1": torch.ones(H, dtype=torch.bfloat16, device=self.device)}
        d["wq"] = self.normal(H, nq * hd)
        d["bq"] = self.normal(nq * hd)
        d["wk"] = self.normal(H, nkv * hd)
        d["bk"] = self.normal(nkv * hd)
        d["wv"] = self.normal(H, nkv * hd)
        d["bv"] = self.normal(nkv * hd)
        d["wo"] = self.normal(nq * hd, H)
        d["ln2"] = torch.ones(H, dtype=torch.bfloat16, device=self.device)
        d["wg"] = self.normal(H, I)
        d["wu"] = self.normal(H, I)
        d["wd"] = self.normal(I, H)
        return d


def random_reference_params(cfg, seed: int = 0, std: float = 0.02) -> dict:
    """A whole model's reference-layout parameters drawn on the host: N(0, std)
    bf16 from torch's CPU generator seeded `seed` (the same values on every
    host with the same torch build), in the draw order of
    GLM4ForCausalLM.init_random (embedding, each layer's q/k/v/o with biases and
    gate/up/down, LM head); RMSNorm gains are 1.  For load_state on any number
    of ranks, and for checking a run against stored outputs of the same model."""
    src = RandomLayerSource(cfg, torch.device("cpu"), seed, std)
    H = cfg.hidden_size
    params = {"embed": src.normal(cfg.vocab_size, H)}
    params["layers"] = [src.layer() for _ in range(cfg.num_hidden_layers)]
    params["norm"] = torch.ones(H, dtype=torch.bfloat16)
    params["lm_head"] = src.normal(cfg.vocab_size, H)
    return params
