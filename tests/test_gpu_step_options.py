"""Options of the whole-step decode kernel that change how it moves data, not
what it computes: the attention's split merge done by the o_proj staging
(JSX_STEP_CMERGE) or by the last split alone (JSX_STEP_DMERGE=0, instead of
every split merging a share of the heads), the L2 prefetch of the next projection's rows
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

    variants = [("JSX_STEP_CMERGE", "1", None), ("JSX_STEP_DMERGE", "0", None), (None, None, with_l2_and_trace)]
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
