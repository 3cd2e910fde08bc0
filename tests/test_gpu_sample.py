"""Sampling (jsx_sample: repetition penalty, temperature, top-k, top-p, categorical
draw, runner.py:315-359) against the oracle's restatement (oracle/glm4_ref.py
sample_tokens) with the same Gumbel noise: token ids bit-exact, at the GLM-4
vocabulary and on a coarse-valued vocabulary with many tied logits.  Rows whose
top-p boundary lies within 1e-5 of a candidate's preceding mass are near-ties of
the fp32 softmax sums and are reported, not compared."""

import numpy as np
import pytest
import torch

from test_gpu_ops import bf

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("V,rp,T,top_k,top_p,coarse", [
    (151552, 1.1, 0.7, 0, 0.9, False),
    (151552, 1.3, 1.0, 50, 1.0, False),
    (151552, 1.0, 1.5, 256, 0.5, False),
    (4096, 1.1, 0.8, 0, 0.95, True),
    (777, 1.2, 1.0, 7, 1.0, True),
])
def test_sample_matches_oracle(jsx, ref, cuda, V, rp, T, top_k, top_p, coarse):
    rng = np.random.default_rng(V + top_k)
    B = 6
    lg = rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)
    if coarse:
        lg = np.round(lg * 2) / 2  # many equal logits: the lower index must win ties
    pres = rng.random((B, V)) < 0.02
    k = top_k if top_k > 0 else 200
    g = ref.bf16(-np.log(-np.log(rng.random((B, k))))).astype(np.float32)
    want, margins = ref.sample_tokens(lg, pres, g, rp, T, top_k, top_p)
    got = jsx.kernels.sample(bf(lg, cuda), bf(g, cuda), presence=torch.from_numpy(pres).to(cuda),
                             repetition_penalty=rp, temperature=T, top_k=top_k, top_p=top_p).cpu().numpy()
    sure = margins > 1e-5
    assert sure.sum() >= B - 1
    assert np.array_equal(got[sure], want[sure]), (got, want, margins)


def test_sample_greedy_limit(jsx, ref, cuda):
    """Zero noise, no penalty, temperature 1, top-p 1: the draw is the argmax (runner.py:297)."""
    rng = np.random.default_rng(3)
    lg = ref.bf16(rng.standard_normal((4, 151552), dtype=np.float32) * np.float32(2.0))
    got = jsx.kernels.sample(bf(lg, cuda), torch.zeros(4, 200, dtype=torch.bfloat16, device=cuda)).cpu().numpy()
    assert np.array_equal(got, ref.argmax_first(lg))


@pytest.mark.parametrize("S", [5, 40])
def test_sample_generate_top1_is_greedy(jsx, ref, cuda, S):
    """runner.sample_generate with one candidate (top_k 1), no penalty and temperature 1
    reproduces greedy_generate, with the prompt token by token (S = 5) and in one pass
    (2 x 40 tokens)."""
    from test_gpu_model import small_cfg, to_model_config
    rc = small_cfg(ref)
    params = ref.init_params(rc, seed=15)
    model = jsx.GLM4ForCausalLM(to_model_config(jsx, rc), jsx.create_mesh(1))
    model.load_state(params)
    prompt = np.random.default_rng(16).integers(0, rc.vocab_size, (2, S))
    a = jsx.sample_generate(model, prompt, max_new_tokens=5, max_cache_len=S + 8, temperature=1.0, top_k=1,
                            top_p=1.0, repetition_penalty=1.0).numpy()
    b = jsx.greedy_generate(model, prompt, max_new_tokens=5, max_cache_len=S + 8).numpy()
    assert np.array_equal(a, b), (a, b)
