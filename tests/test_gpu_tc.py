"""Parity of the tensor-core projections (jsx_tc_*, tcgen05 + TMA) against the
oracle (oracle/glm4_ref.py) on the same seeded inputs, and against the GEMV
entry points where both apply (M <= 8).

Tolerances as for the GEMV kernels (tests/test_gpu_ops.py): fp32 accumulation
in another order than numpy, bf16 rounding at the reference's points, so
max |a - b| / max |b| <= 1e-2, cosine >= 0.9999 and most elements
bit-identical.  Token ids are compared exactly against the argmax of the
kernel's own logits.
"""

import numpy as np
import pytest
import torch

from test_gpu_ops import bf, close, npf, rand_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture
def rng():
    return np.random.default_rng(4321)


@pytest.mark.parametrize("M,K,N", [(32, 4096, 4608), (9, 4096, 4096), (16, 256, 130), (32, 1712, 256),
                                   (12, 520, 34), (1, 64, 2), (25, 13696, 128)])
def test_tc_linear_matches_oracle(jsx, ref, cuda, rng, M, K, N):
    x = rand_bf16(ref, rng, (M, K))
    w = rand_bf16(ref, rng, (K, N), 0.02)
    b = rand_bf16(ref, rng, (N,), 0.02)
    Kx = jsx.kernels
    wt = Kx.pack_transpose(bf(w, cuda))
    ws = Kx.tc_workspace(M, [(K, N)], cuda)
    y = Kx.tc_linear(bf(x, cuda), wt, ws, bias=bf(b, cuda))
    close(npf(y), ref.linear(x, w, b), exact_min=0.98)
    y0 = Kx.tc_linear(bf(x, cuda), wt, ws)
    close(npf(y0), ref.linear(x, w), exact_min=0.98)


@pytest.mark.parametrize("M,K", [(32, 4096), (11, 256)])
def test_tc_linear_rmsnorm_prologue(jsx, ref, cuda, rng, M, K):
    N, eps = 192, 1.5625e-7
    x = rand_bf16(ref, rng, (M, K), 3.0)
    g = rand_bf16(ref, rng, (K,), 1.0)
    w = rand_bf16(ref, rng, (K, N), 0.02)
    Kx = jsx.kernels
    ws = Kx.tc_workspace(M, [(K, N)], cuda)
    y = Kx.tc_linear(bf(x, cuda), Kx.pack_transpose(bf(w, cuda)), ws, gamma=bf(g, cuda), eps=eps)
    close(npf(y), ref.linear(ref.rmsnorm(x, g, eps), w), exact_min=0.95)


def test_tc_matches_gemv_at_small_m(jsx, ref, cuda, rng):
    """Both paths take M <= 8; they agree to fp32 rounding of the dot products."""
    M, K, N = 8, 4096, 512
    x = rand_bf16(ref, rng, (M, K))
    w = rand_bf16(ref, rng, (K, N), 0.02)
    Kx = jsx.kernels
    wt = Kx.pack_transpose(bf(w, cuda))
    a = npf(Kx.linear(bf(x, cuda), wt))
    b = npf(Kx.tc_linear(bf(x, cuda), wt, Kx.tc_workspace(M, [(K, N)], cuda)))
    close(b, a, exact_min=0.98)


@pytest.mark.parametrize("nq,nkv,hd,M,tps", [(32, 2, 128, 32, 1), (4, 2, 128, 12, 3), (2, 1, 64, 20, 1)])
def test_tc_qkv_rope_cache(jsx, ref, cuda, rng, nq, nkv, hd, M, tps):
    H, eps = 512, 1.5625e-7
    B = M // tps
    pos = (np.arange(M) * 37 + 5) % 700
    if tps > 1:  # consecutive positions within a sequence
        pos = np.repeat(np.arange(B) * 50, tps) + np.tile(np.arange(tps), B)
    L = max(512, int(pos.max()) + 1)
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
    ws = Kx.tc_workspace(M, [(H, w_qkv.shape[0])], cuda)
    Kx.tc_qkv_rope_cache(bf(h, cuda), bf(g, cuda), eps, w_qkv, b_qkv, torch.from_numpy(inv).to(cuda),
                         positions, q_out, kc, vc, nq, nkv, hd, rot, ws, tokens_per_seq=tps)
    xn = ref.rmsnorm(h, g, eps)
    q = ref.linear(xn, wq, bq).reshape(M, nq, hd)
    k = ref.linear(xn, wk, bk).reshape(M, nkv, hd)
    v = ref.linear(xn, wv, bv).reshape(M, nkv, hd)
    qr, kr = ref.rope(pos, q, k, inv)
    close(npf(q_out).reshape(M, nq, hd), qr)
    kcn, vcn = npf(kc), npf(vc)
    for m, p in enumerate(pos):
        close(kcn[m // tps, p], kr[m])
        close(vcn[m // tps, p], v[m])
    written = np.zeros((B, L), bool)
    written[np.arange(M) // tps, pos] = True
    assert np.all(kcn[~written] == 0) and np.all(vcn[~written] == 0)


@pytest.mark.parametrize("M,H,I", [(32, 4096, 1712), (20, 256, 96), (9, 512, 2)])
def test_tc_gate_up_swiglu(jsx, ref, cuda, rng, M, H, I):
    eps = 1.5625e-7
    h = rand_bf16(ref, rng, (M, H), 1.0)
    g = rand_bf16(ref, rng, (H,), 1.0)
    wg = rand_bf16(ref, rng, (H, I), 0.05)
    wu = rand_bf16(ref, rng, (H, I), 0.05)
    Kx = jsx.kernels
    act = torch.empty(M, I, dtype=torch.bfloat16, device=cuda)
    ws = Kx.tc_workspace(M, [(H, 2 * I)], cuda)
    Kx.tc_gate_up_swiglu(bf(h, cuda), bf(g, cuda), eps, Kx.pack_gate_up(bf(wg, cuda), bf(wu, cuda)), act, ws)
    xn = ref.rmsnorm(h, g, eps)
    want = ref.bf16(ref.silu(ref.linear(xn, wg)) * ref.linear(xn, wu))
    close(npf(act), want)


@pytest.mark.parametrize("M,K,N", [(32, 13696, 4096), (9, 4096, 256), (17, 520, 64)])
def test_tc_row_linear_single_rank(jsx, ref, cuda, rng, M, K, N):
    x = rand_bf16(ref, rng, (M, K))
    w = rand_bf16(ref, rng, (K, N), 0.02)
    h0 = rand_bf16(ref, rng, (M, N))
    h = bf(h0, cuda)
    Kx = jsx.kernels
    Kx.tc_row_linear_allreduce(None, bf(x, cuda), Kx.pack_transpose(bf(w, cuda)), h,
                               Kx.tc_workspace(M, [(K, N)], cuda))
    close(npf(h), ref.bf16(h0 + ref.linear(x, w)), exact_min=0.98)


@pytest.mark.parametrize("M,H,V", [(32, 4096, 151552 // 8), (17, 256, 1000), (10, 128, 66)])
def test_tc_lmhead_argmax(jsx, ref, cuda, rng, M, H, V):
    h = rand_bf16(ref, rng, (M, H), 2.0)
    g = np.ones(H, np.float32)
    w = rand_bf16(ref, rng, (V, H), 0.02)
    Kx = jsx.kernels
    ids = torch.empty(M, dtype=torch.int32, device=cuda)
    logits = torch.empty(M, V, dtype=torch.bfloat16, device=cuda)
    ws = Kx.tc_workspace(M, [(H, V)], cuda)
    for _ in range(2):
        Kx.tc_lmhead_argmax(None, bf(h, cuda), bf(g, cuda), 1.5625e-7, bf(w, cuda), 0, ids, ws, logits)
        lg = npf(logits)
        close(lg, ref.bf16(ref.rmsnorm(h, g, 1.5625e-7) @ w.T))
        assert np.array_equal(npf(ids.float()).astype(np.int64), np.argmax(lg, axis=-1))
        assert int(ws[:512].sum()) == 0, "argmax header not left zeroed"


def test_tc_lmhead_ties_pick_lowest_index(jsx, ref, cuda):
    H, V, M = 64, 300, 12
    h = np.zeros((M, H), np.float32)
    h[:, 0] = 1.0
    w = np.zeros((V, H), np.float32)
    w[:, 0] = -1.0
    for r in (7, 100, 250):
        w[r, 0] = 2.0
    Kx = jsx.kernels
    ids = torch.empty(M, dtype=torch.int32, device=cuda)
    ws = Kx.tc_workspace(M, [(H, V)], cuda)
    Kx.tc_lmhead_argmax(None, bf(h, cuda), None, 0.0, bf(w, cuda), 40, ids, ws)
    assert ids.tolist() == [47] * M


def test_tc_device_error_clear(jsx, cuda):
    import ctypes
    status = ctypes.c_int(-1)
    jsx._lib.call("jsx_device_error", ctypes.byref(status))
    assert status.value == 0


@pytest.mark.parametrize("B", [12, 32, 40])
def test_tc_model_teacher_forced(jsx, ref, cuda, B):
    """Batches above 8 take the tensor-core projections (40 = one 32-token call + one of 8)."""
    from test_gpu_model import check_steps, run_teacher_forced, small_cfg
    rc = small_cfg(ref)
    params = ref.init_params(rc, seed=21)
    prompt = np.random.default_rng(22).integers(0, rc.vocab_size, (B, 5))
    got, record = run_teacher_forced(jsx, ref, rc, params, prompt, steps=4, L=16)
    check_steps(ref, got, record)
