"""Builds libjsx.so (the C-ABI kernel library) in-tree for sm_100a with nvcc.

Usage: python e2e-jaxscale_b200/build.py [--debug]
The library lands next to this file; it is git-ignored but travels with the
repository snapshot to the GPU host.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libjsx.so")

SOURCES = ["lib.cu", "gemv.cu", "attention.cu", "misc.cu", "comm.cu", "noalloc.cu", "decode_step.cu", "tc_gemm.cu", "tc_wide.cu", "attn_prefill.cu", "sample.cu", "moe.cu", "mla.cu", "mla_absorbed.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(debug: bool = False, verbose: bool = False) -> str:
    objs = []
    os.makedirs(os.path.join(HERE, "_build"), exist_ok=True)
    flags = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC,
             "--expt-relaxed-constexpr"] + ARCH
    if debug:
        flags += ["-DJSX_DEBUG"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    newest_dep = max(os.path.getmtime(os.path.join(CSRC, f)) for f in os.listdir(CSRC))
    newest_dep = max(newest_dep, os.path.getmtime(os.path.join(INCLUDE, "jsx.h")))
    for src in SOURCES:
        obj = os.path.join(HERE, "_build", src.replace(".cu", ".o"))
        objs.append(obj)
        if os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep and not verbose:
            continue
        cmd = [nvcc(), "-c", os.path.join(CSRC, src), "-o", obj] + flags
        subprocess.run(cmd, check=True)
    cmd = [nvcc(), "-shared", "-o", LIB] + objs + ARCH + ["-lcudart"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="pass -Xptxas -v")
    args = ap.parse_args()
    print(build(args.debug, args.verbose))
    sys.exit(0)
