"""RotaryEmbedding (layers/rotary.py:8-93): neox half-split rotation of the first
rotary_dim = head_dim * partial_rotary_factor dims.  The rotation itself is
fused into jsx_qkv_rope_cache; this class owns the frequency table, computed
exactly as the reference does (numpy float32)."""

from __future__ import annotations

import numpy as np
import torch


class RotaryEmbedding:
    def __init__(self, head_dim: int, max_position_embeddings: int = 131072,
                 rope_theta: float = 10000.0, dtype=torch.bfloat16, partial_rotary_factor: float = 0.5):
        self.head_dim = head_dim
        self.rotary_dim = int(head_dim * partial_rotary_factor)
        self.max_position_embeddings = max_position_embeddings
        self.rope_theta = rope_theta
        self.dtype = dtype
        self._inv_freq = 1.0 / (
            rope_theta ** (np.arange(0, self.rotary_dim, 2, dtype=np.float32) / self.rotary_dim))
        self._dev = {}

    def inv_freq(self, device) -> torch.Tensor:
        key = str(device)
        if key not in self._dev:
            self._dev[key] = torch.from_numpy(np.asarray(self._inv_freq, np.float32)).to(device)
        return self._dev[key]
