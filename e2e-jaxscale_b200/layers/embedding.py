"""Embed and ParallelLMHead (layers/embedding.py:10-96).

The reference replicates both tables on every TP rank.  Here the LM head is
vocabulary-sharded ([V/tp, H] per rank) and the greedy argmax is reduced
across ranks inside jsx_lmhead_argmax; ParallelLMHead.__call__ (full logits)
gathers the shards with torch.distributed for callers that need every logit.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import kernels as K
from ._param import Param, to_device


class Embed:
    def __init__(self, num_embeddings: int, features: int, dtype=torch.bfloat16, mesh=None):
        self.num_embeddings = num_embeddings
        self.features = features
        self.dtype = dtype
        self.mesh = mesh
        self.embedding = Param(None)
        self._dev = None
        self._key = None

    def table(self, device) -> torch.Tensor:
        key = (id(self.embedding.value), str(device))
        if self._key != key:
            self._dev = to_device(self.embedding.value, device)
            self._key = key
        return self._dev

    def __call__(self, input_ids: torch.Tensor) -> torch.Tensor:
        dev = self.mesh.device if self.mesh is not None and self.mesh.device is not None else "cuda"
        ids = input_ids.to(device=dev, dtype=torch.int32).contiguous()
        out = K.embed(ids.reshape(-1), self.table(dev))
        return out.reshape(*input_ids.shape, self.features)


class ParallelLMHead:
    def __init__(self, vocab_size: int, hidden_size: int, dtype=torch.bfloat16, mesh=None):
        self.vocab_size = vocab_size
        self.hidden_size = hidden_size
        self.dtype = dtype
        self.mesh = mesh
        self.embedding = Param(None)  # [V, H]
        self._dev = None
        self._key = None

    @property
    def tp(self) -> int:
        return 1 if self.mesh is None else self.mesh.shape.get("tensor", 1)

    def shard(self, device) -> tuple[torch.Tensor, int]:
        """(this rank's [V/tp, H] rows, vocab offset)."""
        key = (id(self.embedding.value), str(device))
        if self._key != key:
            w = to_device(self.embedding.value, device)
            if self.tp > 1:
                n = self.vocab_size // self.tp
                r = self.mesh.tp_rank
                w = w[r * n:(r + 1) * n].contiguous()
            self._dev = w
            self._key = key
        off = 0 if self.tp == 1 else self.mesh.tp_rank * (self.vocab_size // self.tp)
        return self._dev, off

    def __call__(self, hidden_states: torch.Tensor) -> torch.Tensor:
        w, _ = self.shard(hidden_states.device)
        logits = K.linear(hidden_states.contiguous(), w)
        if self.tp > 1:
            parts = [torch.empty_like(logits) for _ in range(self.tp)]
            dist.all_gather(parts, logits, group=self.mesh.group("tensor"))
            logits = torch.cat(parts, dim=-1)
        return logits
