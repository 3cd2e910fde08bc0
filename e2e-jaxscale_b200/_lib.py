"""ctypes binding of libjsx.so (the C ABI declared in include/jsx.h).

The library is the only compute path: if it is missing this module raises at
import, and every op raises JsxError on a non-zero status.  There is no
Python, torch or CPU fallback for any kernel.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libjsx.so")

JSX_OK, JSX_EINVAL, JSX_ECUDA, JSX_ETIMEDOUT, JSX_ENOTSUP, JSX_ENOMEM = range(6)
JSX_LAUNCH_PDL = 1

_STATUS_NAMES = {
    JSX_EINVAL: "JSX_EINVAL", JSX_ECUDA: "JSX_ECUDA", JSX_ETIMEDOUT: "JSX_ETIMEDOUT",
    JSX_ENOTSUP: "JSX_ENOTSUP", JSX_ENOMEM: "JSX_ENOMEM",
}


class JsxError(RuntimeError):
    def __init__(self, status: int, fn: str, msg: str):
        super().__init__(f"{fn}: {_STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
SZ = ctypes.c_size_t
U64 = ctypes.c_uint64

# name -> argtypes (every function returns int)
SIGNATURES = {
    "jsx_abi_version": [],
    "jsx_device_sm_count": [P],
    "jsx_set_launch_flags": [I],
    "jsx_get_launch_flags": [],
    "jsx_device_error": [P],
    "jsx_pack_transpose": [P, P, I, I, P],
    "jsx_pack_qkv": [P, P, P, P, I, I, I, I, I, P],
    "jsx_pack_gate_up": [P, P, P, I, I, P],
    "jsx_rmsnorm": [P, P, P, I, I, F, P],
    "jsx_embed": [P, P, P, I, I, I, P],
    "jsx_linear": [P, P, F, P, P, P, I, I, I, P],
    "jsx_qkv_rope_cache": [P, P, F, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, P],
    "jsx_gate_up_swiglu": [P, P, F, P, P, I, I, I, P],
    "jsx_attn_decode_workspace_size": [I, I, I, I, I, P],
    "jsx_attn_decode": [P, P, P, P, P, I, I, I, I, I, F, P, SZ, P],
    "jsx_attn_decode_noalloc": [P, P, P, P, P, I, I, I, I, I, F, P],
    "jsx_row_linear_allreduce": [P, P, P, P, I, I, I, P],
    "jsx_lmhead_workspace_size": [I, P],
    "jsx_lmhead_argmax": [P, P, P, F, P, I, I, I, I, P, P, P, SZ, P],
    "jsx_tc_workspace_size": [I, I, I, P],
    "jsx_tc_set_trace": [P],
    "jsx_tc_linear": [P, P, F, P, P, P, I, I, I, P, SZ, P],
    "jsx_tc_qkv_rope_cache": [P, P, F, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, P, SZ, P],
    "jsx_tc_gate_up_swiglu": [P, P, F, P, P, I, I, I, P, SZ, P],
    "jsx_tc_row_linear_allreduce": [P, P, P, P, I, I, I, P, SZ, P],
    "jsx_tc_lmhead_argmax": [P, P, P, F, P, I, I, I, I, P, P, P, SZ, P],
    "jsx_wide_workspace_size": [I, I, I, I, P],
    "jsx_attn_prefill": [P, P, P, P, I, I, I, I, I, I, I, F, P],
    "jsx_sample": [P, P, P, P, I, I, F, F, I, F, P],
    "jsx_wide_linear": [P, P, F, P, P, P, I, I, I, P, SZ, P],
    "jsx_wide_qkv_rope_cache": [P, P, F, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, P, SZ, P],
    "jsx_wide_gate_up_swiglu": [P, P, F, P, P, I, I, I, P, SZ, P],
    "jsx_wide_row_linear_allreduce": [P, P, P, P, I, I, I, P, SZ, P],
    "jsx_moe_gate": [P, P, P, P, P, I, I, I, I, F, I, P],
    "jsx_mla_rope_cache": [P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, P],
    "jsx_mla_latent_cache": [P, P, P, P, P, P, P, I, I, I, I, I, I, I, P],
    "jsx_mla_absorb": [P, I, I, P, P, I, I, I, I, P],
    "jsx_mla_decode_workspace_size": [I, I, I, I, P],
    "jsx_mla_decode": [P, P, P, P, P, I, I, I, I, I, F, P, SZ, P],
    "jsx_moe_experts_workspace_size": [I, I, I, I, I, P],
    "jsx_moe_experts": [P, P, P, P, I, I, I, I, I, I, P, P, P, P, SZ, P],
    "jsx_row_linear_allreduce_add": [P, P, P, P, P, I, I, I, P],
    "jsx_decode_step_workspace_size": [P, P],
    "jsx_decode_step": [P, P, P],
    "jsx_comm_create": [I, I, I, I, U64, P],
    "jsx_comm_create_tiles": [I, I, I, I, U64, P],
    "jsx_comm_ipc_handle": [P, P],
    "jsx_comm_open_peers": [P, P],
    "jsx_comm_check": [P, P],
    "jsx_comm_destroy": [P],
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python e2e-jaxscale_b200/build.py` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    lib.jsx_last_error.argtypes = []
    lib.jsx_last_error.restype = ctypes.c_char_p
    return lib


lib = _load()


def call(name: str, *args) -> None:
    """Call a jsx_* entry point and raise JsxError on a non-zero status."""
    st = getattr(lib, name)(*args)
    if st != JSX_OK:
        raise JsxError(st, name, (lib.jsx_last_error() or b"").decode(errors="replace"))


def last_error() -> str:
    return (lib.jsx_last_error() or b"").decode(errors="replace")
