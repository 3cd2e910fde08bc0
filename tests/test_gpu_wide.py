"""Parity of the wide tensor-core projections (jsx_wide_*, 128 x 256 tcgen05
tiles for prefill and many-token products) against the oracle
(oracle/glm4_ref.py) on the same seeded inputs, including ragged M / N / K
edges (TMA zero fill past every edge) and several token and weight tiles.

Tolerances as for the other projection kernels: fp32 accumulation in another
order than numpy, bf16 rounding at the reference's points, so
max |a - b| / max |b| <= 1e-2, cosine >= 0.9999 and most elements
bit-identical."""

import numpy as np
import pytest
import torch

from test_gpu_ops import bf, close, npf, rand_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture
def rng():
    return np.random.default_rng(9876)


@pytest.mark.parametrize("M,K,N", [(256, 4096, 4096), (300, 520, 130), (1, 64, 2), (2049, 1024, 640),
                                   (700, 13696, 256)])
def test_wide_linear_matches_oracle(jsx, ref, cuda, rng, M, K, N):
    x = rand_bf16(ref, rng, (M, K))
    w = rand_bf16(ref, rng, (K, N), 0.02)
    b = rand_bf16(ref, rng, (N,), 0.02)
    Kx = jsx.kernels
    wt = Kx.pack_transpose(bf(w, cuda))
    ws = Kx.wide_workspace(M, [(K, N)], cuda)
    y = Kx.wide_linear(bf(x, cuda), wt, ws, bias=bf(b, cuda))
    close(npf(y), ref.linear(x, w, b), exact_min=0.98)
    y0 = Kx.wide_linear(bf(x, cuda), wt, ws)
    close(npf(y0), ref.linear(x, w), exact_min=0.98)


def test_wide_linear_matches_cublas(jsx, ref, cuda, rng):
    """M = 4096 tokens (16 token tiles, two tile groups) against torch.matmul."""
    M, K, N = 4096, 4096, 1024
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) * 0.02).to(torch.bfloat16)
    Kx = jsx.kernels
    y = Kx.wide_linear(x, w, Kx.wide_workspace(M, [(K, N)], cuda, norm=False))
    want = (x.float() @ w.float().t()).to(torch.bfloat16).float()
    got = y.float()
    err = float((got - want).abs().max() / want.abs().max())
    assert err <= 1e-2, err
    assert float((got == want).float().mean()) >= 0.95


@pytest.mark.parametrize("M,K", [(512, 4096), (37, 256)])
def test_wide_linear_rmsnorm_prologue(jsx, ref, cuda, rng, M, K):
    N, eps = 192, 1.5625e-7
    x = rand_bf16(ref, rng, (M, K), 3.0)
    g = rand_bf16(ref, rng, (K,), 1.0)
    w = rand_bf16(ref, rng, (K, N), 0.02)
    Kx = jsx.kernels
    ws = Kx.wide_workspace(M, [(K, N)], cuda)
    y = Kx.wide_linear(bf(x, cuda), Kx.pack_transpose(bf(w, cuda)), ws, gamma=bf(g, cuda), eps=eps)
    close(npf(y), ref.linear(ref.rmsnorm(x, g, eps), w), exact_min=0.95)


@pytest.mark.parametrize("M,H,I", [(600, 512, 384), (257, 4096, 1712)])
def test_wide_gate_up_swiglu(jsx, ref, cuda, rng, M, H, I):
    eps = 1.5625e-7
    h = rand_bf16(ref, rng, (M, H), 1.0)
    g = rand_bf16(ref, rng, (H,), 1.0)
    wg = rand_bf16(ref, rng, (H, I), 0.05)
    wu = rand_bf16(ref, rng, (H, I), 0.05)
    Kx = jsx.kernels
    act = torch.empty(M, I, dtype=torch.bfloat16, device=cuda)
    ws = Kx.wide_workspace(M, [(H, 2 * I)], cuda)
    Kx.wide_gate_up_swiglu(bf(h, cuda), bf(g, cuda), eps, Kx.pack_gate_up(bf(wg, cuda), bf(wu, cuda)), act, ws)
    xn = ref.rmsnorm(h, g, eps)
    want = ref.bf16(ref.silu(ref.linear(xn, wg)) * ref.linear(xn, wu))
    close(npf(act), want)


@pytest.mark.parametrize("nq,nkv,hd,B,S", [(32, 2, 128, 2, 300), (4, 2, 128, 3, 100), (2, 1, 64, 1, 513)])
def test_wide_qkv_rope_cache_prefill(jsx, ref, cuda, rng, nq, nkv, hd, B, S):
    """A prefill block: B sequences of S consecutive positions from 0."""
    H, eps = 512, 1.5625e-7
    M, L = B * S, S + 16
    pos = np.tile(np.arange(S), B)
    h = rand_bf16(ref, rng, (M, H), 1.0)
    g = rand_bf16(ref, rng, (H,), 1.0)
    wq = rand_bf16(ref, rng, (H, nq * hd), 0.05)
    wk = rand_bf16(ref, rng, (H, nkv * hd), 0.05)
    wv = rand_bf16(ref, rng, (H, nkv * hd), 0.05)
    bq, bk, bv = (rand_bf16(ref, rng, (n * hd,), 0.05) for n in (nq, nkv, nkv))
    rot = hd // 2
    Kx = jsx.kernels
    w_qkv = Kx.pack_qkv(bf(wq, cuda), bf(wk, cuda), bf(wv, cuda), nq, nkv, hd, rot)
    b_qkv = bf(np.concatenate([bq, bk, bv]), cuda)
    inv = ref.rope_inv_freq(hd)
    positions = torch.tensor(pos, dtype=torch.int32, device=cuda)
    q_out = torch.zeros(M, nq * hd, dtype=torch.bfloat16, device=cuda)
    kc = torch.zeros(B, L, nkv, hd, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    ws = Kx.wide_workspace(M, [(H, w_qkv.shape[0])], cuda)
    Kx.wide_qkv_rope_cache(bf(h, cuda), bf(g, cuda), eps, w_qkv, b_qkv, torch.from_numpy(inv).to(cuda),
                           positions, q_out, kc, vc, nq, nkv, hd, rot, ws, tokens_per_seq=S)
    xn = ref.rmsnorm(h, g, eps)
    q = ref.linear(xn, wq, bq).reshape(M, nq, hd)
    k = ref.linear(xn, wk, bk).reshape(M, nkv, hd)
    v = ref.linear(xn, wv, bv).reshape(M, nkv, hd)
    qr, kr = ref.rope(pos, q, k, inv)
    close(npf(q_out).reshape(M, nq, hd), qr)
    kcn, vcn = npf(kc), npf(vc)
    close(kcn[:, :S].reshape(M, nkv, hd), kr)
    close(vcn[:, :S].reshape(M, nkv, hd), v)
    assert np.all(kcn[:, S:] == 0) and np.all(vcn[:, S:] == 0)


@pytest.mark.parametrize("M,K,N", [(4096, 4096, 256), (257, 13696, 128), (64, 520, 64)])
def test_wide_row_linear_residual(jsx, ref, cuda, rng, M, K, N):
    x = rand_bf16(ref, rng, (M, K))
    w = rand_bf16(ref, rng, (K, N), 0.02)
    h0 = rand_bf16(ref, rng, (M, N))
    h = bf(h0, cuda)
    Kx = jsx.kernels
    Kx.wide_row_linear_allreduce(None, bf(x, cuda), Kx.pack_transpose(bf(w, cuda)), h,
                                 Kx.wide_workspace(M, [(K, N)], cuda, norm=False))
    close(npf(h), ref.bf16(h0 + ref.linear(x, w)), exact_min=0.98)


def test_wide_device_error_clear(jsx, cuda):
    import ctypes
    status = ctypes.c_int(-1)
    jsx._lib.call("jsx_device_error", ctypes.byref(status))
    assert status.value == 0
