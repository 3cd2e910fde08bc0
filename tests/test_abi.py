"""The C ABI library loads and exports every entry point declared in
include/jsx.h; argument validation answers without touching a GPU."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "jsx.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(jsx_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("jsx_linear", "jsx_qkv_rope_cache", "jsx_gate_up_swiglu", "jsx_attn_decode",
              "jsx_row_linear_allreduce", "jsx_lmhead_argmax", "jsx_moe_gate", "jsx_comm_create"):
        assert n in names


def test_library_exports_every_declared_symbol(jsx):
    lib = ctypes.CDLL(jsx._lib.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(jsx._lib.SIGNATURES) | {"jsx_last_error"} >= set(declared_functions())


def test_abi_version(jsx):
    assert jsx._lib.lib.jsx_abi_version() == 1


@pytest.mark.parametrize("call,args", [
    ("jsx_linear", (None, None, 0.0, None, None, None, 1, 64, 8, None)),
    ("jsx_comm_create", (0, 9, 8, 4096, 0, None)),
    ("jsx_comm_create", (2, 2, 8, 4096, 0, None)),
    ("jsx_moe_gate", (None, None, None, None, None, 1, 8, 512, 4, 1.0, 1, None)),
    ("jsx_set_launch_flags", (0x10,)),
    ("jsx_tc_linear", (None, None, 0.0, None, None, None, 16, 64, 8, None, 0, None)),
    ("jsx_tc_workspace_size", (33, 4096, 4096, None)),
    ("jsx_sample", (256, None, 256, 256, 1, 1000, 1.0, 1.0, 300, 1.0, None)),    # k above 256
    ("jsx_sample", (256, None, 256, 256, 1, 1000, 1.0, 0.0, 0, 1.0, None)),      # temperature 0
    ("jsx_attn_prefill", (256, 256, 256, 256, 1, 8, 4, 4, 2, 128, 10, 0.1, None)),  # start + S > max_seq
    ("jsx_comm_create_tiles", (0, 9, 4096, 4096, 0, None)),
    ("jsx_wide_row_linear_allreduce", (None, 256, 256, 256, 64, 4096, 33, 256, 1 << 20, None)),  # odd N
])
def test_invalid_arguments_are_rejected_on_the_host(jsx, call, args):
    lib = jsx._lib
    with pytest.raises(lib.JsxError) as e:
        lib.call(call, *args)
    assert e.value.status == lib.JSX_EINVAL
    assert lib.last_error()


def test_workspace_size_queries(jsx):
    lib = jsx._lib
    n = ctypes.c_size_t(0)
    lib.call("jsx_attn_decode_workspace_size", 1, 32, 2, 128, 1152, ctypes.byref(n))
    splits = (1152 + 63) // 64           # 64 cache rows per split
    # batch 1 leaves the GPU mostly idle, so each kv head's 16 query heads are split in 4 groups
    groups, heads = 1 * 2 * 4, 4
    record = heads * 128 + 8             # accumulator tile + (m, l) per head, padded to 16 bytes
    assert n.value >= groups * splits * record * 4
    lib.call("jsx_lmhead_workspace_size", 8, ctypes.byref(n))
    assert n.value >= 256 + 8 * 8
    with pytest.raises(lib.JsxError):
        lib.call("jsx_lmhead_workspace_size", 9, ctypes.byref(n))


def test_tc_workspace_size(jsx):
    """256 B done counter + argmax keys, the normalised activations [32][K] bf16
    (from byte 1024, rounded to 1 KB), then the rank-local fp32 rows [M][N]."""
    lib = jsx._lib
    n = ctypes.c_size_t(0)
    lib.call("jsx_tc_workspace_size", 32, 4096, 4608, ctypes.byref(n))
    assert n.value == 1024 + 32 * 4096 * 2 + 32 * 4608 * 4
    lib.call("jsx_tc_workspace_size", 9, 13696, 4096, ctypes.byref(n))
    assert n.value == 1024 + 32 * 13696 * 2 + 9 * 4096 * 4
    lib.call("jsx_tc_workspace_size", 3, 100, 8, ctypes.byref(n))
    assert n.value == 1024 + 7168 + 3 * 8 * 4      # 32 x 100 x 2 = 6400 -> 7168
    with pytest.raises(lib.JsxError):
        lib.call("jsx_tc_workspace_size", 0, 64, 64, ctypes.byref(n))


def test_wide_workspace_size(jsx):
    """1 KB header, then (with a gain) the normalised activations [M][K] bf16
    rounded to 1 KB."""
    lib = jsx._lib
    n = ctypes.c_size_t(0)
    lib.call("jsx_wide_workspace_size", 4096, 4096, 4608, 1, ctypes.byref(n))
    assert n.value == 1024 + 4096 * 4096 * 2
    lib.call("jsx_wide_workspace_size", 300, 100, 8, 1, ctypes.byref(n))
    assert n.value == 1024 + 60416                 # 300 x 100 x 2 = 60000 -> 60416
    lib.call("jsx_wide_workspace_size", 300, 100, 8, 0, ctypes.byref(n))
    assert n.value == 1024
    with pytest.raises(lib.JsxError):
        lib.call("jsx_wide_workspace_size", 0, 64, 64, 1, ctypes.byref(n))
    with pytest.raises(lib.JsxError) as e:         # K not a multiple of 8, checked before any launch
        lib.call("jsx_wide_linear", 1, None, 0.0, 1, None, 1, 256, 100, 64, 1, 1 << 20, None)
    assert e.value.status == lib.JSX_EINVAL


def test_moe_experts_workspace_and_limits(jsx):
    lib = jsx._lib
    n = ctypes.c_size_t(0)
    lib.call("jsx_moe_experts_workspace_size", 32, 4, 64, 2048, 1536, ctypes.byref(n))
    P = 32 * 4
    assert n.value >= 65 * 4 + 3 * P * 4 + P * 1536 * 2 + P * 2048 * 2
    with pytest.raises(lib.JsxError):   # 33 tokens per call
        lib.call("jsx_moe_experts", 1, 1, 1, None, 0, 33, 4, 64, 2048, 1536, 1, 1, 1, 1, 1 << 30, None)


def test_unsupported_shapes_answer_enotsup(jsx):
    """The prefill attention kernel takes head_dim 128; others are refused before any launch."""
    lib = jsx._lib
    with pytest.raises(lib.JsxError) as e:
        lib.call("jsx_attn_prefill", 256, 256, 256, 256, 1, 8, 0, 4, 2, 64, 16, 0.1, None)
    assert e.value.status == lib.JSX_ENOTSUP
