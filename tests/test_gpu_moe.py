"""MoE experts and the MoE layer (GLM-4.7-Flash, layers/moe.py) against the oracle
(oracle/glm4_ref.py moe_experts / moe_layer, pinned to the reference's MoELayer by
tests/test_oracle_pin.py::test_moe_layer).

The expert GEMVs accumulate in fp32 in another order than numpy's einsum and round
to bf16 at the reference's points, so outputs agree to about one bf16 ulp: max
relative error <= 1e-2, cosine >= 0.9999, most elements bit-identical.  The layer
test uses the model-level tolerance (2e-2, cosine 0.999) because its router computes
its own logits; router ids on identical logits are checked bit-exact in
tests/test_gpu_ops.py."""

import importlib

import numpy as np
import pytest
import torch

from test_gpu_ops import bf, close, npf, rand_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture
def rng():
    return np.random.default_rng(77)


def packed_experts(K, eg, eu, ed, dev):
    E = eg.shape[0]
    w_gu = torch.stack([K.pack_gate_up(bf(eg[e], dev), bf(eu[e], dev)) for e in range(E)]).contiguous()
    w_d = torch.stack([K.pack_transpose(bf(ed[e], dev)) for e in range(E)]).contiguous()
    return w_gu, w_d


@pytest.mark.parametrize("N,E,H,I,k", [(1, 64, 2048, 1536, 4), (8, 64, 2048, 1536, 4), (13, 16, 256, 96, 4),
                                        (32, 8, 128, 64, 2)])
def test_moe_experts_match_oracle(jsx, ref, cuda, rng, N, E, H, I, k):
    K = jsx.kernels
    x = rand_bf16(ref, rng, (N, H))
    eg = rand_bf16(ref, rng, (E, H, I), 0.05)
    eu = rand_bf16(ref, rng, (E, H, I), 0.05)
    ed = rand_bf16(ref, rng, (E, I, H), 0.05)
    # routing: distinct experts per token, some experts shared by several tokens
    ids = np.stack([rng.choice(min(E, 8 + N // 2), size=k, replace=False) for _ in range(N)]).astype(np.int32)
    w = ref.bf16(rng.random((N, k), dtype=np.float32))
    want = ref.moe_experts(x, w, ids, eg, eu, ed)
    w_gu, w_d = packed_experts(K, eg, eu, ed, cuda)
    out = torch.empty(N, H, dtype=torch.bfloat16, device=cuda)
    ws = K.moe_workspace(N, k, E, H, I, cuda)
    K.moe_experts(bf(x, cuda), bf(w, cuda), torch.from_numpy(ids).to(cuda), w_gu, w_d, out, ws)
    close(npf(out), want, exact_min=0.9)
    # an owner table that keeps only even experts on this rank: the partial sums just those
    owner = torch.tensor([e % 2 for e in range(E)], dtype=torch.int32, device=cuda)
    out0 = torch.empty_like(out)
    K.moe_experts(bf(x, cuda), bf(w, cuda), torch.from_numpy(ids).to(cuda), w_gu, w_d, out0, ws, owner=owner,
                  rank=0)
    w_even = np.where(ids % 2 == 0, np.asarray(w, np.float32), np.float32(0))
    close(npf(out0), ref.moe_experts(x, ref.bf16(w_even), ids, eg, eu, ed), exact_min=0.9)


def test_moe_layer_matches_reference_golden(jsx, ref, cuda):
    """The reference's own MoELayer output (tests/golden, 8 experts, top-4, shared expert)."""
    g = np.load(importlib.import_module("os").path.join(
        importlib.import_module("os").path.dirname(__file__), "golden", "reference_golden.npz"))
    moe_mod = importlib.import_module("e2e-jaxscale_b200.layers.moe")
    E, H, I, Is = 8, 128, 64, 64
    layer = moe_mod.MoELayer(H, I, Is, E, 4, 1.8, True, None)
    layer.gate.weight.weight.value = g["moel_router"]
    layer.gate.e_score_correction_bias.value = g["moel_bias"]
    layer.expert_gate_weight.value = g["moel_eg"]
    layer.expert_up_weight.value = g["moel_eu"]
    layer.expert_down_weight.value = g["moel_ed"]
    layer.shared_experts.gate_proj.weight.value = g["moel_sg"]
    layer.shared_experts.up_proj.weight.value = g["moel_su"]
    layer.shared_experts.down_proj.weight.value = g["moel_sd"]
    y = layer(bf(g["moel_x"], cuda))
    want = g["moel_y"]
    got = npf(y)
    err = np.max(np.abs(got - want)) / np.max(np.abs(want))
    cos = float(np.sum(got * want) / (np.linalg.norm(got) * np.linalg.norm(want)))
    assert err <= 2e-2 and cos >= 0.999, (err, cos)


@pytest.mark.parametrize("N", [1, 12])
def test_moe_layer_flash_shapes(jsx, ref, cuda, rng, N):
    """GLM-4.7-Flash widths (H 2048, 64 experts of 1536, top-4, shared 1536) against the oracle."""
    moe_mod = importlib.import_module("e2e-jaxscale_b200.layers.moe")
    E, H, I, Is = 64, 2048, 1536, 1536
    layer = moe_mod.MoELayer(H, I, Is, E, 4, 1.8, True, None)
    p = dict(router=rand_bf16(ref, rng, (H, E), 0.02), eg=rand_bf16(ref, rng, (E, H, I), 0.02),
             eu=rand_bf16(ref, rng, (E, H, I), 0.02), ed=rand_bf16(ref, rng, (E, I, H), 0.02),
             sg=rand_bf16(ref, rng, (H, Is), 0.02), su=rand_bf16(ref, rng, (H, Is), 0.02),
             sd=rand_bf16(ref, rng, (Is, H), 0.02))
    layer.gate.weight.weight.value = p["router"]
    layer.expert_gate_weight.value = p["eg"]
    layer.expert_up_weight.value = p["eu"]
    layer.expert_down_weight.value = p["ed"]
    layer.shared_experts.gate_proj.weight.value = p["sg"]
    layer.shared_experts.up_proj.weight.value = p["su"]
    layer.shared_experts.down_proj.weight.value = p["sd"]
    x = rand_bf16(ref, rng, (1, N, H))
    y = npf(layer(bf(x, cuda)))
    want = ref.moe_layer(x, p["router"], None, 4, 1.8, True, p["eg"], p["eu"], p["ed"], p["sg"], p["su"], p["sd"])
    err = np.max(np.abs(y - want)) / np.max(np.abs(want))
    cos = float(np.sum(y * want) / (np.linalg.norm(y) * np.linalg.norm(want)))
    assert err <= 2e-2 and cos >= 0.999, (err, cos)
