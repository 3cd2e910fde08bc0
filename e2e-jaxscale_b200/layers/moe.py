"""MoEGate (layers/moe.py:27-79): the GLM-4.7-Flash router.

logits = bf16(x @ W_g) -> f32 softmax -> + e_score_correction_bias -> top-k
(lower index first on ties, like lax.top_k) -> uncorrected probabilities of the
chosen experts -> renormalised (+1e-20) when norm_topk_prob -> * routed_scaling_factor
-> bf16.  One kernel (jsx_moe_gate).
"""

from __future__ import annotations

import torch

from .. import kernels as K
from ._param import Param, to_device
from .linear import LinearBase


class MoEGate:
    def __init__(self, hidden_size: int, num_experts: int, num_experts_per_tok: int,
                 routed_scaling_factor: float, norm_topk_prob: bool, mesh, dtype=torch.bfloat16):
        self.num_experts = num_experts
        self.num_experts_per_tok = num_experts_per_tok
        self.routed_scaling_factor = routed_scaling_factor
        self.norm_topk_prob = norm_topk_prob
        self.weight = LinearBase(hidden_size, num_experts, mesh, use_bias=False, params_dtype=dtype,
                                 kernel_axes=(None, None))
        self.e_score_correction_bias = Param(None)

    def __call__(self, hidden_states: torch.Tensor):
        dev = hidden_states.device
        w_nk, _ = self.weight._ensure_packed(dev)
        bias = self.e_score_correction_bias.value
        bias = None if bias is None else to_device(bias, dev, torch.float32)
        lead = hidden_states.shape[:-1]
        w, i = K.moe_gate(hidden_states.contiguous(), w_nk, self.num_experts_per_tok,
                          self.routed_scaling_factor, self.norm_topk_prob, bias)
        k = self.num_experts_per_tok
        return w.reshape(*lead, k), i.reshape(*lead, k)
