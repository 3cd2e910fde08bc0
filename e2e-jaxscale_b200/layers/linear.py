"""LinearBase (layers/linear.py:13-82): y = x @ W (+ b), W is [in, out].

kernel_axes (None, "tensor") = column-parallel: this rank computes its output
shard; ("tensor", None) = row-parallel: this rank holds an input shard and the
result is all-reduced over the tensor axis (the XLA all-reduce implied by the
replicated output constraint at layers/linear.py:72-78) inside the fused
row-parallel kernels: up to 8 tokens the CUDA-core GEMV with the LL-word
all-reduce (jsx_row_linear_allreduce), up to 32 the tensor-core product
(jsx_tc_row_linear_allreduce), beyond that the wide tensor-core GEMM with its
in-epilogue tile exchange (jsx_wide_row_linear_allreduce).  A row-parallel bias
(replicated, layers/linear.py:80-81) is added after the all-reduce: the output
rows start as the bias and the kernels add bf16(sum of the partials), which is
the reference's bf16(bf16(x @ W) + b).
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from .. import kernels as K
from ._param import Param, to_device


class LinearBase:
    def __init__(self, input_size: int, output_size: int, mesh, use_bias: bool = False,
                 params_dtype=torch.bfloat16, kernel_axes: Sequence[str | None] | None = None):
        self.input_size = input_size
        self.output_size = output_size
        self.mesh = mesh
        self.params_dtype = params_dtype
        self.kernel_axes = tuple(kernel_axes or (None, None))
        self.weight = Param(None)
        self.bias = Param(None) if use_bias else None
        self._packed = None
        self._key = None
        self._ws = {}

    # --- sharding (utils/weight_utils.py:248-265) ---
    @property
    def tp(self) -> int:
        return 1 if self.mesh is None else self.mesh.shape.get("tensor", 1)

    @property
    def tp_rank(self) -> int:
        return 0 if self.mesh is None else self.mesh.tp_rank

    @property
    def is_row_parallel(self) -> bool:
        return self.kernel_axes[0] == "tensor" and self.tp > 1

    @property
    def is_column_parallel(self) -> bool:
        return self.kernel_axes[1] == "tensor" and self.tp > 1

    def local_weight(self, device) -> torch.Tensor:
        w = to_device(self.weight.value, device)
        t, r = self.tp, self.tp_rank
        if self.is_column_parallel:
            n = w.shape[1] // t
            w = w[:, r * n:(r + 1) * n]
        elif self.is_row_parallel:
            k = w.shape[0] // t
            w = w[r * k:(r + 1) * k]
        return w.contiguous()

    def local_bias(self, device):
        if self.bias is None or self.bias.value is None:
            return None
        b = to_device(self.bias.value, device)
        if self.is_column_parallel:
            n = b.shape[0] // self.tp
            b = b[self.tp_rank * n:(self.tp_rank + 1) * n]
        return b.contiguous()

    def _ensure_packed(self, device):
        key = (id(self.weight.value), None if self.bias is None else id(self.bias.value), str(device))
        if self._key != key:
            self._packed = (K.pack_transpose(self.local_weight(device)), self.local_bias(device))
            self._key = key
        return self._packed

    def _workspace(self, kind: str, M: int, K_: int, N: int, device) -> torch.Tensor:
        key = (kind, M, str(device))
        if key not in self._ws:
            self._ws[key] = (K.tc_workspace(M, [(K_, N)], device) if kind == "tc"
                             else K.wide_workspace(M, [(K_, N)], device, norm=False))
        return self._ws[key]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        w_nk, b = self._ensure_packed(x.device)
        if self.is_row_parallel:
            N, K_ = w_nk.shape
            x2 = x.reshape(-1, K_).contiguous()
            M = x2.shape[0]
            if b is not None:
                y = b.reshape(1, N).expand(M, N).contiguous()
            else:
                y = torch.zeros((M, N), dtype=torch.bfloat16, device=x.device)
            if M <= K.MAX_DECODE_TOKENS:
                K.row_linear_allreduce(self.mesh.comm(K.TC_MAX_TOKENS, N), x2, w_nk, y)
            elif M <= K.TC_MAX_TOKENS:
                K.tc_row_linear_allreduce(self.mesh.comm(K.TC_MAX_TOKENS, N), x2, w_nk, y,
                                          self._workspace("tc", M, K_, N, x.device))
            else:
                K.wide_row_linear_allreduce(self.mesh.comm_tiles(M, N), x2, w_nk, y,
                                            self._workspace("wide", M, K_, N, x.device))
            return y.reshape(*x.shape[:-1], N)
        return K.linear(x.contiguous(), w_nk, bias=b)
