"""Parameter holder and host->device conversion shared by the layers."""

from __future__ import annotations

import numpy as np
import torch


class Param:
    """Stand-in for flax.nnx.Param: a mutable `.value` (torch tensor or numpy array)."""

    def __init__(self, value=None):
        self.value = value


def to_device(value, device, dtype=torch.bfloat16) -> torch.Tensor:
    """numpy (float32 holding bf16 values, or ml_dtypes.bfloat16) / torch -> contiguous device tensor."""
    if isinstance(value, torch.Tensor):
        t = value
    else:
        arr = np.asarray(value)
        if arr.dtype.name == "bfloat16":
            t = torch.from_numpy(arr.view(np.uint16).astype(np.int16)).view(torch.bfloat16)
        else:
            t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32))
    return t.to(device=device, dtype=dtype).contiguous()
