"""Static KV cache (layers/kv_cache.py:16-61): per layer k, v of shape
[batch, max_seq_len, kv_heads_on_this_rank, head_dim], zero-initialised and
updated in place (the reference donates the cache to jit, runner.py:141).

Tensor parallelism: the reference shards the KV-head axis over "tensor"
(P(None, None, "tensor", None)); with 2 KV heads that only divides at TP <= 2.
At TP > 2 each rank keeps the one KV head its query heads use (replicated
across the ranks that share it), so TP = 4 and 8 work.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class KVCache:
    k: torch.Tensor
    v: torch.Tensor


def local_kv_heads(num_heads: int, num_kv_heads: int, tp: int, rank: int) -> tuple[int, int]:
    """(first KV head, count) held by `rank`."""
    if tp <= num_kv_heads:
        n = num_kv_heads // tp
        return rank * n, n
    q_per_rank = num_heads // tp
    group = num_heads // num_kv_heads
    return (rank * q_per_rank) // group, 1


def init_kv_caches(batch_size: int, max_seq_len: int, num_layers: int, num_kv_heads: int,
                   head_dim: int, dtype=torch.bfloat16, mesh=None, num_heads: int | None = None,
                   device=None) -> list[KVCache]:
    tp = 1 if mesh is None else mesh.shape.get("tensor", 1)
    rank = 0 if mesh is None else mesh.tp_rank
    if device is None:
        device = mesh.device if mesh is not None and mesh.device is not None else "cuda"
    nq = num_heads if num_heads is not None else num_kv_heads
    _, n_local = local_kv_heads(nq, num_kv_heads, tp, rank) if tp > 1 else (0, num_kv_heads)
    shape = (batch_size, max_seq_len, n_local, head_dim)
    return [KVCache(k=torch.zeros(shape, dtype=dtype, device=device),
                    v=torch.zeros(shape, dtype=dtype, device=device)) for _ in range(num_layers)]
