"""Per-kernel parity: each jsx_* entry point against the CPU oracle (oracle/glm4_ref.py)
on the same seeded inputs.

Tolerances: the kernels accumulate in fp32 in a different order from numpy and
round to bf16 at the same points as the reference, so outputs agree to about
one bf16 ulp.  Checked: max |a - b| / max |b| <= 1e-2, cosine >= 0.9999, and
at least 95 % of elements bit-identical (99 % when no normalisation precedes
the product).  Integer outputs (token ids, expert ids) are compared exactly.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def bf(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev).to(torch.bfloat16)


def npf(t):
    return t.float().cpu().numpy()


def close(a, b, rel=1e-2, cos_min=0.9999, exact_min=0.95):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    assert np.all(np.isfinite(a)), "non-finite output"
    err = np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30)
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
    exact = float(np.mean(a == b))
    assert err <= rel, f"max rel err {err:.3e} > {rel}"
    assert cos >= cos_min, f"cosine {cos:.6f} < {cos_min}"
    assert exact >= exact_min, f"bit-exact fraction {exact:.4f} < {exact_min}"


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def rand_bf16(ref, rng, shape, std=1.0):
    return ref.bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4608), (3, 1712, 130), (8, 256, 64), (5, 13696, 34),
                                   (2, 64, 2)])
def test_linear_matches_oracle(jsx, ref, cuda, rng, M, K, N):
    x = rand_bf16(ref, rng, (M, K))
    w = rand_bf16(ref, rng, (K, N), 0.02)
    b = rand_bf16(ref, rng, (N,), 0.02)
    wt = jsx.kernels.pack_transpose(bf(w, cuda))
    y = jsx.kernels.linear(bf(x, cuda), wt, bias=bf(b, cuda))
    close(npf(y), ref.linear(x, w, b), exact_min=0.99)
    y0 = jsx.kernels.linear(bf(x, cuda), wt)
    close(npf(y0), ref.linear(x, w), exact_min=0.99)


def test_pack_transpose_exact(jsx, ref, cuda, rng):
    w = rand_bf16(ref, rng, (100, 37))
    t = jsx.kernels.pack_transpose(bf(w, cuda))
    assert np.array_equal(npf(t), w.T)


@pytest.mark.parametrize("M,K", [(1, 4096), (4, 256), (8, 1024)])
def test_linear_with_rmsnorm_prologue(jsx, ref, cuda, rng, M, K):
    x = rand_bf16(ref, rng, (M, K), 3.0)
    g = rand_bf16(ref, rng, (K,), 1.0)
    w = rand_bf16(ref, rng, (K, 96), 0.02)
    y = jsx.kernels.linear(bf(x, cuda), jsx.kernels.pack_transpose(bf(w, cuda)), gamma=bf(g, cuda),
                           eps=1.5625e-7)
    close(npf(y), ref.linear(ref.rmsnorm(x, g, 1.5625e-7), w))


def test_rmsnorm(jsx, ref, cuda, rng):
    x = rand_bf16(ref, rng, (5, 4096), 2.0)
    g = rand_bf16(ref, rng, (4096,), 1.0)
    y = jsx.kernels.rmsnorm(bf(x, cuda), bf(g, cuda), 1.5625e-7)
    close(npf(y), ref.rmsnorm(x, g, 1.5625e-7), exact_min=0.99)


@pytest.mark.parametrize("nq,nkv,hd,M,pos", [
    (4, 2, 128, 3, [5, 17, 300]),
    (16, 1, 128, 1, [1023]),
    (2, 1, 64, 8, [0, 1, 2, 3, 100, 101, 511, 7]),
])
def test_qkv_rope_cache(jsx, ref, cuda, rng, nq, nkv, hd, M, pos):
    H, eps = 256, 1.5625e-7
    L = max(512, max(pos) + 1)
    h = rand_bf16(ref, rng, (M, H), 1.0)
    g = np.ones(H, np.float32)
    wq = rand_bf16(ref, rng, (H, nq * hd), 0.05)
    wk = rand_bf16(ref, rng, (H, nkv * hd), 0.05)
    wv = rand_bf16(ref, rng, (H, nkv * hd), 0.05)
    bq, bk, bv = (rand_bf16(ref, rng, (n * hd,), 0.05) for n in (nq, nkv, nkv))
    rot = hd // 2
    K = jsx.kernels
    w_qkv = K.pack_qkv(bf(wq, cuda), bf(wk, cuda), bf(wv, cuda), nq, nkv, hd, rot)
    b_qkv = bf(np.concatenate([bq, bk, bv]), cuda)
    inv = ref.rope_inv_freq(hd)
    positions = torch.tensor(pos, dtype=torch.int32, device=cuda)
    q_out = torch.zeros(M, nq * hd, dtype=torch.bfloat16, device=cuda)
    kc = torch.zeros(M, L, nkv, hd, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    K.qkv_rope_cache(bf(h, cuda), bf(g, cuda), eps, w_qkv, b_qkv, torch.from_numpy(inv).to(cuda),
                     positions, q_out, kc, vc, nq, nkv, hd, rot)
    xn = ref.rmsnorm(h, g, eps)
    q = ref.linear(xn, wq, bq).reshape(M, nq, hd)
    k = ref.linear(xn, wk, bk).reshape(M, nkv, hd)
    v = ref.linear(xn, wv, bv).reshape(M, nkv, hd)
    qr, kr = ref.rope(np.array(pos), q, k, inv)
    close(npf(q_out).reshape(M, nq, hd), qr)
    kcn, vcn = npf(kc), npf(vc)
    for m, p in enumerate(pos):
        close(kcn[m, p], kr[m])
        close(vcn[m, p], v[m])
    # only the addressed rows were written
    mask = np.ones((M, L), bool)
    mask[np.arange(M), pos] = False
    assert np.all(kcn[mask] == 0) and np.all(vcn[mask] == 0)


@pytest.mark.parametrize("M,H,I", [(1, 4096, 1712), (5, 256, 96), (8, 512, 2)])
def test_gate_up_swiglu(jsx, ref, cuda, rng, M, H, I):
    h = rand_bf16(ref, rng, (M, H), 1.0)
    g = rand_bf16(ref, rng, (H,), 1.0)
    wg = rand_bf16(ref, rng, (H, I), 0.05)
    wu = rand_bf16(ref, rng, (H, I), 0.05)
    K = jsx.kernels
    act = torch.empty(M, I, dtype=torch.bfloat16, device=cuda)
    K.gate_up_swiglu(bf(h, cuda), bf(g, cuda), 1.5625e-7, K.pack_gate_up(bf(wg, cuda), bf(wu, cuda)), act)
    xn = ref.rmsnorm(h, g, 1.5625e-7)
    want = ref.bf16(ref.silu(ref.linear(xn, wg)) * ref.linear(xn, wu))
    close(npf(act), want)


@pytest.mark.parametrize("B,nq,nkv,hd,L,pos", [
    (3, 8, 2, 128, 200, [0, 37, 199]),
    (1, 32, 2, 128, 1100, [1024]),
    (2, 4, 1, 128, 64, [31, 32]),
    (1, 20, 20, 256, 100, [63]),
    # 16-head groups of many sequences: the records do not fit shared memory and the
    # splits are merged by the separate merge launch
    (32, 32, 2, 128, 1100, [1024 - 31 * i for i in range(32)]),
    (8, 16, 1, 128, 600, [599, 0, 64, 63, 300, 1, 128, 511]),
])
def test_attn_decode(jsx, ref, cuda, rng, B, nq, nkv, hd, L, pos):
    q = rand_bf16(ref, rng, (B, nq, hd))
    kc = rand_bf16(ref, rng, (B, L, nkv, hd))
    vc = rand_bf16(ref, rng, (B, L, nkv, hd))
    K = jsx.kernels
    out = torch.empty(B, nq * hd, dtype=torch.bfloat16, device=cuda)
    ws = K.attn_workspace(B, nq, nkv, hd, L, cuda)
    positions = torch.tensor(pos, dtype=torch.int32, device=cuda)
    for _ in range(2):  # the workspace must come back clean for a second call
        K.attn_decode(bf(q, cuda), bf(kc, cuda), bf(vc, cuda), out, positions, hd ** -0.5, ws)
        for b in range(B):
            mask = ref.make_decode_mask(pos[b], L)
            want = ref.sdpa(q[b:b + 1, None], kc[b:b + 1], vc[b:b + 1], mask, hd ** -0.5)
            # probabilities rounded per split here vs after normalisation in the reference: the
            # bar is the tolerance, the bit-identical share is not (about half at 16-head groups)
            close(npf(out[b]), want.reshape(-1), rel=2e-2, cos_min=0.999, exact_min=0.3)


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (4, 13696, 256), (8, 512, 64)])
def test_row_linear_single_rank(jsx, ref, cuda, rng, M, K, N):
    x = rand_bf16(ref, rng, (M, K))
    w = rand_bf16(ref, rng, (K, N), 0.02)
    h0 = rand_bf16(ref, rng, (M, N))
    h = bf(h0, cuda)
    jsx.kernels.row_linear_allreduce(None, bf(x, cuda), jsx.kernels.pack_transpose(bf(w, cuda)), h)
    close(npf(h), ref.bf16(h0 + ref.linear(x, w)), exact_min=0.99)


@pytest.mark.parametrize("M,H,V", [(1, 4096, 151552 // 8), (4, 256, 1000), (8, 128, 66)])
def test_lmhead_argmax(jsx, ref, cuda, rng, M, H, V):
    h = rand_bf16(ref, rng, (M, H), 2.0)
    g = np.ones(H, np.float32)
    w = rand_bf16(ref, rng, (V, H), 0.02)
    K = jsx.kernels
    ids = torch.empty(M, dtype=torch.int32, device=cuda)
    logits = torch.empty(M, V, dtype=torch.bfloat16, device=cuda)
    ws = K.lmhead_workspace(M, cuda)
    for _ in range(2):
        K.lmhead_argmax(None, bf(h, cuda), bf(g, cuda), 1.5625e-7, bf(w, cuda), 0, ids, ws, logits)
        lg = npf(logits)
        want = ref.bf16(ref.rmsnorm(h, g, 1.5625e-7) @ w.T)
        close(lg, want)
        # ids are exactly the first argmax of the kernel's own bf16 logits
        assert np.array_equal(npf(ids.float()).astype(np.int64), np.argmax(lg, axis=-1))
        assert int(ws.sum()) == 0, "workspace not left zeroed"


def test_lmhead_ties_pick_lowest_index(jsx, ref, cuda):
    H, V = 64, 300
    h = np.zeros((2, H), np.float32)
    h[:, 0] = 1.0
    w = np.full((V, H), 0.0, np.float32)
    w[:, 0] = -1.0
    for r in (7, 100, 250):
        w[r, 0] = 2.0  # three equal maxima
    w[3, 0] = -0.0
    K = jsx.kernels
    ids = torch.empty(2, dtype=torch.int32, device=cuda)
    K.lmhead_argmax(None, bf(h, cuda), None, 0.0, bf(w, cuda), 40, ids, K.lmhead_workspace(2, cuda))
    assert ids.tolist() == [47, 47]  # row 7 + vocab_offset 40


def test_embed_and_out_of_range(jsx, ref, cuda, rng):
    table = rand_bf16(ref, rng, (50, 64))
    ids = torch.tensor([3, 49, 0, 50, -1], dtype=torch.int32, device=cuda)
    out = npf(jsx.kernels.embed(ids, bf(table, cuda)))
    assert np.array_equal(out[:3], table[[3, 49, 0]])
    assert np.all(np.isnan(out[3:]))  # jnp.take fills out-of-bounds rows with NaN


@pytest.mark.parametrize("bias_std", [0.0, 1e-3])
def test_moe_gate_same_logits(jsx, ref, cuda, rng, bias_std):
    N, E, k = 33, 64, 4
    logits = rand_bf16(ref, rng, (N, E), 1.0)
    bias = (rng.standard_normal(E).astype(np.float32) * np.float32(bias_std)) if bias_std else None
    w, i = jsx.kernels.moe_gate(bf(logits, cuda), None, k, 1.8, True,
                                None if bias is None else torch.from_numpy(bias).to(cuda),
                                logits_given=True)
    # oracle on the same logits: identity weight so linear() returns the logits unchanged
    want_w, want_i = ref.moe_gate(logits, np.eye(E, dtype=np.float32), k, 1.8, True, bias)
    assert np.array_equal(i.cpu().numpy(), want_i), "expert ids differ"
    close(npf(w), want_w, rel=1e-2, cos_min=0.9999, exact_min=0.9)


def test_moe_gate_from_hidden(jsx, ref, cuda, rng):
    N, H, E, k = 16, 2048, 64, 4
    x = rand_bf16(ref, rng, (N, H))
    wg = rand_bf16(ref, rng, (H, E), 0.02)
    K = jsx.kernels
    w, i = K.moe_gate(bf(x, cuda), K.pack_transpose(bf(wg, cuda)), k, 1.8, True)
    want_w, want_i = ref.moe_gate(x, wg, k, 1.8, True)
    got_i = i.cpu().numpy()
    logits = ref.linear(x, wg)
    for t in range(N):
        if not np.array_equal(got_i[t], want_i[t]):
            # only acceptable when the reference's own k-th/k+1-th logits are within one bf16 ulp
            srt = np.sort(logits[t])[::-1]
            assert srt[k - 1] - srt[k] <= abs(srt[k - 1]) * 2 ** -7, f"token {t}: ids differ"


def test_invalid_arguments_raise(jsx, cuda):
    K = jsx.kernels
    x = torch.zeros(9, 64, dtype=torch.bfloat16, device=cuda)
    w = torch.zeros(8, 64, dtype=torch.bfloat16, device=cuda)
    from importlib import import_module
    lib = import_module("e2e-jaxscale_b200._lib")
    with pytest.raises(lib.JsxError) as e:
        lib.call("jsx_linear", x.data_ptr(), None, 0.0, w.data_ptr(), None, x.data_ptr(), 9, 64, 8, None)
    assert e.value.status in (lib.JSX_EINVAL, lib.JSX_ENOTSUP)
    with pytest.raises(lib.JsxError):
        lib.call("jsx_linear", x.data_ptr(), None, 0.0, w.data_ptr(), None, x.data_ptr(), 1, 60, 8, None)
