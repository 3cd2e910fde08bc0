"""RMSNorm (layers/normalization.py:10-37).  GLM-4 builds it with bf16 gains
(models/glm4.py:86-95); the kernel takes bf16 gains."""

from __future__ import annotations

import torch

from .. import kernels as K
from ._param import Param, to_device


class RMSNorm:
    def __init__(self, hidden_size: int, epsilon: float = 1e-6, param_dtype=torch.bfloat16):
        self.hidden_size = hidden_size
        self.epsilon = epsilon
        self.param_dtype = param_dtype
        self.scale = Param(torch.ones(hidden_size, dtype=torch.float32))
        self._gain = None
        self._key = None

    def gain(self, device) -> torch.Tensor:
        """The gain on `device` (bf16), converted once per assigned value."""
        key = (id(self.scale.value), str(device))
        if self._key != key:
            self._gain = to_device(self.scale.value, device)
            self._key = key
        return self._gain

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return K.rmsnorm(x.contiguous(), self.gain(x.device), self.epsilon)
