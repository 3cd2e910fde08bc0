"""Options of the whole-step decode kernel that change how it moves data, not
what it computes: the attention's split merge done by the o_proj staging
(JSX_STEP_CMERGE) or by every split merging a share of the heads
(JSX_STEP_DMERGE=1, instead of the last split merging them all), the L2 prefetch of the next projection's rows
(l2_next_bytes / l2_attn_bytes) and the traces (trace_ar, trace_phase).  Each must
give bit-identical logits and ids to the default kernel on the same inputs.
The options are read per launch, so one process compares them."""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(jsx, model, prompt, steps, L, setup=None):
    st = jsx.DecodeState(model, prompt.shape[0], L, want_logits=True)
    if setup is not None:
        setup(st)
    out = []
    for s in range(prompt.shape[1]):
        st.ids.copy_(torch.from_numpy(prompt[:, s].astype(np.int32)))
        model.step(st, head=(s == prompt.shape[1] - 1))
    out.append((st.logits.float().cpu().numpy(), st.ids.cpu().numpy()))
    for _ in range(steps):
        model.step(st, head=True)
        out.append((st.logits.float().cpu().numpy(), st.ids.cpu().numpy()))
    return out


@pytest.fixture(scope="module")
def glm_2layer(jsx, cuda):
    """GLM-4-9B widths (K = 4096 and 13696: several weight batches per row pair), 2 layers."""
    cfg = jsx.ModelConfig(num_hidden_layers=2, vocab_size=8192)
    model = jsx.GLM4ForCausalLM(cfg, jsx.create_mesh(1))
    model.load_state(jsx.weights.random_reference_params(cfg, seed=3))
    return model


@pytest.mark.parametrize("B", [1, 2])
def test_step_options_bit_identical(jsx, cuda, glm_2layer, B):
    model = glm_2layer
    nl = model.config.num_hidden_layers
    prompt = np.random.default_rng(8).integers(0, model.config.vocab_size, (B, 70))  # two attention splits
    L = 80
    base = _run(jsx, model, prompt, 6, L)
    tar = torch.zeros(4 * nl, dtype=torch.int64, device=cuda)
    tph = torch.zeros(15 * nl, dtype=torch.int64, device=cuda)

    def with_l2_and_trace(st):
        st.step_args.l2_next_bytes = 16384
        st.step_args.l2_attn_bytes = 16384
        st.step_args.trace_ar = tar.data_ptr()
        st.step_args.trace_phase = tph.data_ptr()

    variants = [("JSX_STEP_CMERGE", "1", None), ("JSX_STEP_DMERGE", "1", None), (None, None, with_l2_and_trace)]
    for env, val, setup in variants:
        if env:
            os.environ[env] = val
        try:
            got = _run(jsx, model, prompt, 6, L, setup)
        finally:
            if env:
                del os.environ[env]
        for (lg0, id0), (lg1, id1) in zip(base, got):
            assert np.array_equal(lg0, lg1), (env, setup)
            assert np.array_equal(id0, id1), (env, setup)
    # the exchange stamps were written (one rank: the exchange part is empty, so both
    # stamps of a phase come from the same barrier-free point)
    assert int(tar.cpu().numpy().min()) > 0
    # every phase point of every layer was stamped, in order within each phase
    pts = tph.cpu().numpy().reshape(nl, 5, 3)
    assert int(pts.min()) > 0
    assert np.all(np.diff(pts, axis=2) >= 0)


def test_qkv_split_matches_per_op(jsx, cuda):
    """hidden 4096 with 8 query heads: 768 q/k/v rows are few enough that the
    whole-step kernel splits their K over warp pairs (both halves prefetched at
    the barrier), as it does at tensor parallelism >= 2 with the GLM-4-9B shape;
    the per-op GEMV keeps one warp per row pair.  The two differ only in the fp32
    summation order of the projection, so teacher-forced logits agree to within
    bf16 rounding."""
    cfg = jsx.ModelConfig(hidden_size=4096, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                          head_dim=128, intermediate_size=2048, vocab_size=4096)
    model = jsx.GLM4ForCausalLM(cfg, jsx.create_mesh(1))
    model.load_state(jsx.weights.random_reference_params(cfg, seed=5))
    prompt = np.random.default_rng(9).integers(0, cfg.vocab_size, (1, 12))
    logits = {}
    for fused in (False, True):
        model.fused_step = fused
        st = jsx.DecodeState(model, 1, 16, want_logits=True)
        out = []
        for s in range(prompt.shape[1]):
            st.ids.copy_(torch.from_numpy(prompt[:, s].astype(np.int32)))
            model.step(st, head=True)
            out.append(st.logits.float().cpu().numpy().copy())
        logits[fused] = np.stack(out)
    model.fused_step = True
    a, b = logits[False], logits[True]
    assert np.all(np.isfinite(b))
    scale = float(np.abs(a).max())
    assert float(np.abs(a - b).max()) <= 0.02 * scale
    cos = (a * b).sum(-1) / (np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1))
    assert float(cos.min()) > 0.9999
    status = __import__("ctypes").c_int(-1)
    jsx._lib.call("jsx_device_error", __import__("ctypes").byref(status))
    assert status.value == 0
