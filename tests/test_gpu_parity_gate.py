"""The decode parity gate that bench.py runs before timing, on one GPU: a
GLM-4-9B-shaped 2-layer model (vocabulary 8192, host-seeded weights) run
teacher-forced through the whole-step kernel (batch 1) and the tensor-core
chain (batch 32), compared with the oracle's outputs stored in
tests/golden/tp_parity.npz.  The same gate runs at TP = 2, 4, 8 inside
tests/test_gpu_tp.py."""

import importlib
import os
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_parity_gate_one_gpu(jsx, cuda):
    sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")
    mesh = jsx.create_mesh(tp=1)
    res = bench.parity_gate(jsx, mesh, cuda, 1)
    assert res["ok"], res
    assert res["steps"] == 9 + 5
    assert res["max_rel"] <= 2e-2 and res["min_cos"] >= 0.999
    assert res["ids"] == 9 + 5 * 32
