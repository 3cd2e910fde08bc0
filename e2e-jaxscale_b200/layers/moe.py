"""GLM-4.7-Flash MoE (layers/moe.py): MoEGate (:27-79, the router), SharedExpertMLP
(:80-113) and MoELayer (:116-244, routed experts + shared expert + expert-parallel sum).

MoEGate:
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


def _owner_table(E: int, ep: int, tp: int) -> list[int]:
    """Rank (expert-major, tensor-minor) that computes each expert: experts are split
    over the expert axis like the reference (layers/moe.py:210-214); inside an expert
    group the tensor ranks take every tp-th expert instead of repeating the group's work."""
    per = E // ep
    return [(e // per) * tp + (e % per) % tp for e in range(E)]


class SharedExpertMLP:
    """layers/moe.py:80-113: down(silu(gate(x)) * up(x)), the gate/up/down LinearBase
    parameters in the reference's [in, out] layout.  Under MoELayer its intermediate
    dimension is split over every expert x tensor rank (one all-reduce for the layer)."""

    def __init__(self, hidden_size: int, intermediate_size: int, mesh, dtype=torch.bfloat16):
        self.gate_proj = LinearBase(hidden_size, intermediate_size, mesh, params_dtype=dtype,
                                    kernel_axes=(None, "tensor"))
        self.up_proj = LinearBase(hidden_size, intermediate_size, mesh, params_dtype=dtype,
                                  kernel_axes=(None, "tensor"))
        self.down_proj = LinearBase(intermediate_size, hidden_size, mesh, params_dtype=dtype,
                                    kernel_axes=("tensor", None))


class MoELayer:
    """layers/moe.py:116-244.  Router (jsx_moe_gate), this rank's routed experts
    (jsx_moe_experts), the shared expert's slice (jsx_gate_up_swiglu), and one
    all-reduce that sums every rank's shared-expert and routed partials into the
    output (jsx_row_linear_allreduce_add): the reference's psum("expert") and the
    shared expert's tensor all-reduce in one exchange."""

    def __init__(self, hidden_size: int, moe_intermediate_size: int, shared_intermediate_size: int,
                 num_experts: int, num_experts_per_tok: int, routed_scaling_factor: float,
                 norm_topk_prob: bool, mesh, dtype=torch.bfloat16):
        self.hidden_size = hidden_size
        self.moe_intermediate_size = moe_intermediate_size
        self.num_experts = num_experts
        self.num_experts_per_tok = num_experts_per_tok
        self.mesh = mesh
        self.gate = MoEGate(hidden_size, num_experts, num_experts_per_tok, routed_scaling_factor,
                            norm_topk_prob, mesh, dtype)
        # stacked expert weights [E, H, I], [E, H, I], [E, I, H] (load_and_stack_experts)
        self.expert_gate_weight = Param(None)
        self.expert_up_weight = Param(None)
        self.expert_down_weight = Param(None)
        self.shared_experts = SharedExpertMLP(hidden_size, shared_intermediate_size, mesh, dtype)
        self._dev = None

    # --- placement of this rank's weights ---
    def _rank_world(self):
        m = self.mesh
        if m is None or not hasattr(m, "moe_rank"):
            return 0, 1
        return m.moe_rank, m.moe_world

    def _prepare(self, device):
        key = (str(device), id(self.expert_gate_weight.value), id(self.shared_experts.down_proj.weight.value))
        if self._dev == key:
            return
        E = self.num_experts
        rank, world = self._rank_world()
        ep = 1 if self.mesh is None else self.mesh.shape.get("expert", 1)
        tp = world // ep
        owner = _owner_table(E, ep, tp)
        eg = to_device(self.expert_gate_weight.value, device)
        eu = to_device(self.expert_up_weight.value, device)
        ed = to_device(self.expert_down_weight.value, device)
        I = eg.shape[2]
        H = self.hidden_size
        self.w_gu = torch.zeros(E, 2 * I, H, dtype=torch.bfloat16, device=device)
        self.w_d = torch.zeros(E, H, I, dtype=torch.bfloat16, device=device)
        for e in range(E):
            if owner[e] == rank:  # other ranks' experts are never read here
                self.w_gu[e] = K.pack_gate_up(eg[e].contiguous(), eu[e].contiguous())
                self.w_d[e] = K.pack_transpose(ed[e].contiguous())
        del eg, eu, ed
        self.owner = torch.tensor(owner, dtype=torch.int32, device=device) if world > 1 else None
        se = self.shared_experts
        sg = to_device(se.gate_proj.weight.value, device)
        su = to_device(se.up_proj.weight.value, device)
        sd = to_device(se.down_proj.weight.value, device)
        Is = sg.shape[1]
        if Is % world:
            raise ValueError(f"shared intermediate {Is} not divisible by {world} ranks")
        n = Is // world
        sl = slice(rank * n, (rank + 1) * n)
        self.s_gu = K.pack_gate_up(sg[:, sl].contiguous(), su[:, sl].contiguous())
        self.s_d = K.pack_transpose(sd[sl].contiguous())
        self.rank = rank
        self._dev = key

    def __call__(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """[B, S, H] bf16 -> routed + shared output [B, S, H] (layers/moe.py:156-192)."""
        dev = hidden_states.device
        self._prepare(dev)
        H = self.hidden_size
        x = hidden_states.reshape(-1, H).contiguous()
        N = x.shape[0]
        tk_w, tk_i = self.gate(x)
        out = torch.zeros(N, H, dtype=torch.bfloat16, device=dev)
        comm = None if self.mesh is None or not hasattr(self.mesh, "comm_moe") else \
            self.mesh.comm_moe(K.MAX_DECODE_TOKENS, H)
        Kk = self.num_experts_per_tok
        ws = K.moe_workspace(min(N, 32), Kk, self.num_experts, H, self.w_gu.shape[1] // 2, dev)
        routed = torch.empty(N, H, dtype=torch.bfloat16, device=dev)
        for n0 in range(0, N, 32):
            n1 = min(N, n0 + 32)
            K.moe_experts(x[n0:n1], tk_w[n0:n1].contiguous(), tk_i[n0:n1].contiguous(), self.w_gu, self.w_d,
                          routed[n0:n1], ws, owner=self.owner, rank=self.rank)
        act = torch.empty(N, self.s_gu.shape[0] // 2, dtype=torch.bfloat16, device=dev)
        for n0 in range(0, N, K.MAX_DECODE_TOKENS):
            n1 = min(N, n0 + K.MAX_DECODE_TOKENS)
            K.gate_up_swiglu(x[n0:n1], None, 0.0, self.s_gu, act[n0:n1])
            K.row_linear_allreduce_add(comm, act[n0:n1], self.s_d, routed[n0:n1], out[n0:n1])
        return out.reshape(hidden_states.shape)


class DenseMLP:
    """layers/moe.py:270-300: down(silu(gate(x)) * up(x)) for the first_k_dense_replace
    layers of GLM-4.7-Flash, gate/up column-parallel and down row-parallel over the
    tensor axis like GLM-4-9B's MLP: jsx_gate_up_swiglu on this rank's gate/up slice,
    then the down projection with its fused all-reduce."""

    def __init__(self, hidden_size: int, intermediate_size: int, mesh, dtype=torch.bfloat16):
        self.hidden_size = hidden_size
        self.gate_proj = LinearBase(hidden_size, intermediate_size, mesh, params_dtype=dtype,
                                    kernel_axes=(None, "tensor"))
        self.up_proj = LinearBase(hidden_size, intermediate_size, mesh, params_dtype=dtype,
                                  kernel_axes=(None, "tensor"))
        self.down_proj = LinearBase(intermediate_size, hidden_size, mesh, params_dtype=dtype,
                                    kernel_axes=("tensor", None))
        self._key = None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        dev = x.device
        key = (id(self.gate_proj.weight.value), id(self.up_proj.weight.value), str(dev))
        if self._key != key:
            self.w_gu = K.pack_gate_up(self.gate_proj.local_weight(dev), self.up_proj.local_weight(dev))
            self._key = key
        H = self.hidden_size
        x2 = x.reshape(-1, H).contiguous()
        act = torch.empty(x2.shape[0], self.w_gu.shape[0] // 2, dtype=torch.bfloat16, device=dev)
        for m0 in range(0, x2.shape[0], K.MAX_DECODE_TOKENS):
            m1 = min(x2.shape[0], m0 + K.MAX_DECODE_TOKENS)
            K.gate_up_swiglu(x2[m0:m1], None, 0.0, self.w_gu, act[m0:m1])
        return self.down_proj(act).reshape(x.shape)
