"""jsx_attn_decode_noalloc — decode attention for callers that cannot allocate
device memory (graph-capture regions of allocators that forbid it, fixed-budget
embedded runtimes, FFI hosts that pass only inputs and outputs).  It must give
the same result as jsx_attn_decode with a caller workspace, on two consecutive
calls (the shared static scratch keeps the previous call's contents, so the
second call checks that the entry point clears what must start at zero).

Collected last (file name) so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("B,nq,nkv,hd,L,pos", [
    (1, 32, 2, 128, 1100, [1024]),
    (3, 8, 2, 128, 200, [0, 37, 199]),
])
def test_noalloc_matches_workspace_entry_point(jsx, cuda, B, nq, nkv, hd, L, pos):
    lib = jsx._lib
    fn = lib.lib.jsx_attn_decode_noalloc
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    g = torch.Generator(device=cuda).manual_seed(11)
    q = torch.randn(B, nq, hd, generator=g, device=cuda).to(torch.bfloat16)
    kc = torch.randn(B, L, nkv, hd, generator=g, device=cuda).to(torch.bfloat16)
    vc = torch.randn(B, L, nkv, hd, generator=g, device=cuda).to(torch.bfloat16)
    positions = torch.tensor(pos, dtype=torch.int32, device=cuda)
    scale = hd ** -0.5
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    want = torch.empty(B, nq * hd, dtype=torch.bfloat16, device=cuda)
    ws = jsx.kernels.attn_workspace(B, nq, nkv, hd, L, cuda)
    lib.call("jsx_attn_decode", _ptr(q), _ptr(kc), _ptr(vc), _ptr(want), _ptr(positions), B, nq, nkv,
             hd, L, ctypes.c_float(scale), _ptr(ws), ws.numel(), stream)

    for _ in range(2):
        got = torch.full((B, nq * hd), float("nan"), dtype=torch.bfloat16, device=cuda)
        st = fn(_ptr(q), _ptr(kc), _ptr(vc), _ptr(got), _ptr(positions), B, nq, nkv, hd, L, scale, stream)
        assert st == 0, lib.last_error()
        torch.cuda.synchronize()
        a = got.float().cpu().numpy()
        b = want.float().cpu().numpy()
        assert np.all(np.isfinite(a))
        # same kernel and reduction order: within the attention tests' tolerance, in fact identical
        assert np.max(np.abs(a - b)) <= 2e-2 * np.max(np.abs(b))
        assert np.array_equal(a, b)


def test_noalloc_rejects_shapes_beyond_the_static_scratch(jsx, cuda):
    lib = jsx._lib
    fn = lib.lib.jsx_attn_decode_noalloc
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    dummy = torch.zeros(16, dtype=torch.bfloat16, device=cuda)
    pos = torch.zeros(64, dtype=torch.int32, device=cuda)
    # 64 sequences x 2 kv heads x 512 splits of 16 heads x 128 dims is far beyond 16 MiB
    st = fn(_ptr(dummy), _ptr(dummy), _ptr(dummy), _ptr(dummy), _ptr(pos), 64, 32, 2, 128, 32768, 0.1,
            None)
    assert st == lib.JSX_EINVAL
    assert "static scratch" in lib.last_error()
