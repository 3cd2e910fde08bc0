"""Causal prefill attention (jsx_attn_prefill) against the oracle's SDPA with the
reference's prefill mask (oracle/glm4_ref.py sdpa + make_prefill_mask, pinned to
GQAAttention by tests/test_oracle_pin.py), on seeded inputs: from an empty cache
(start 0), after an earlier prefix (start > 0), ragged query blocks and GQA
group sizes 2 and 16.

The kernel keeps an online fp32 softmax and rounds the unnormalised
probabilities to bf16 for the P.V product (the reference rounds the normalised
ones), so the bar is the decode attention tests' one: max relative error
<= 2e-2, cosine >= 0.999, at least half of the elements bit-identical."""

import numpy as np
import pytest
import torch

from test_gpu_ops import bf, close, npf, rand_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,S,start,nq,nkv,L", [(2, 300, 0, 4, 2, 320), (1, 130, 50, 32, 2, 256),
                                                (3, 64, 0, 2, 1, 64), (1, 1, 77, 16, 1, 100),
                                                (2, 1024, 0, 2, 1, 1024)])
def test_attn_prefill_matches_oracle(jsx, ref, cuda, B, S, start, nq, nkv, L):
    rng = np.random.default_rng(5 + S + start)
    hd = 128
    q = rand_bf16(ref, rng, (B, S, nq, hd))
    kc = np.zeros((B, L, nkv, hd), np.float32)
    vc = np.zeros((B, L, nkv, hd), np.float32)
    kc[:, :start + S] = rand_bf16(ref, rng, (B, start + S, nkv, hd))
    vc[:, :start + S] = rand_bf16(ref, rng, (B, start + S, nkv, hd))
    kc[:, start + S:] = np.nan  # rows past the prefill are never read
    vc[:, start + S:] = np.nan
    # additive mask: query i sees rows [0, start + i]
    mask = np.where(np.arange(L)[None, :] <= start + np.arange(S)[:, None], 0.0, ref.NEG).astype(np.float32)
    want = ref.sdpa(q, np.nan_to_num(kc), np.nan_to_num(vc), mask[None, None], hd ** -0.5)
    out = jsx.kernels.attn_prefill(bf(q.reshape(B * S, nq * hd), cuda), bf(kc, cuda), bf(vc, cuda), nq, nkv, hd, S,
                                   start_pos=start)
    close(npf(out).reshape(B, S, nq, hd), want, rel=2e-2, cos_min=0.999, exact_min=0.5)


def test_attn_prefill_matches_reference_prefill_mask(jsx, ref, cuda):
    """From an empty cache the mask is exactly the reference's make_prefill_mask."""
    rng = np.random.default_rng(11)
    B, S, L, nq, nkv, hd = 2, 96, 128, 32, 2, 128
    q = rand_bf16(ref, rng, (B, S, nq, hd))
    kc = np.zeros((B, L, nkv, hd), np.float32)
    vc = np.zeros((B, L, nkv, hd), np.float32)
    kc[:, :S] = rand_bf16(ref, rng, (B, S, nkv, hd))
    vc[:, :S] = rand_bf16(ref, rng, (B, S, nkv, hd))
    want = ref.sdpa(q, kc, vc, ref.make_prefill_mask(S, L), hd ** -0.5)
    out = jsx.kernels.attn_prefill(bf(q.reshape(B * S, nq * hd), cuda), bf(kc, cuda), bf(vc, cuda), nq, nkv, hd, S)
    close(npf(out).reshape(B, S, nq, hd), want, rel=2e-2, cos_min=0.999, exact_min=0.5)


def test_attn_prefill_rejects_other_head_dims(jsx, cuda):
    q = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    kc = torch.zeros(1, 8, 1, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(jsx._lib.JsxError) as e:
        jsx.kernels.attn_prefill(q, kc, kc, 1, 1, 64, 4)
    assert e.value.status == jsx._lib.JSX_ENOTSUP
