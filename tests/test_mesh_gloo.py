"""Host-side tensor-parallel logic on CPU ranks (gloo, world size 2 and 4):
mesh coordinates and groups, per-rank weight shards and KV-head assignment,
the row-parallel exchange the fused kernel performs, emulated with a gloo
all-reduce of the per-rank fp32 partials, and the vocabulary-shard gather of
the sampling loop (runner._full_logits)."""

import importlib
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, tp, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        jsx = importlib.import_module("e2e-jaxscale_b200")
        ref = importlib.import_module("oracle.glm4_ref")
        import torch
        mesh = jsx.mesh.Mesh(tp=tp, dp=world // tp, rank=rank, world=world)
        tg = mesh.group("tensor")
        out = {"coords": dict(mesh.coords), "tensor_ranks": mesh.axis_ranks("tensor")}
        # row-parallel o_proj: this rank's input shard times its weight rows, summed over ranks
        rng = np.random.default_rng(0)
        x = ref.bf16(rng.standard_normal((2, 256)))
        w = ref.bf16(rng.standard_normal((256, 32)) * 0.02)
        r = mesh.tp_rank
        part = np.asarray(ref.shard_columns(x, tp, r), np.float32) @ np.asarray(ref.shard_rows(w, tp, r), np.float32)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t, group=tg)
        y = ref.bf16(t.numpy())
        out["row_parallel_err"] = float(np.max(np.abs(y - ref.linear(x, w))))
        out["kv_heads"] = jsx.layers.kv_cache.local_kv_heads(32, 2, tp, r)
        # the sampling loop's full-vocabulary logits: the tensor ranks' vocab shards in rank order
        V = 40

        class _Model:  # the two attributes runner._full_logits reads
            pass
        m = _Model()
        m.tp, m.mesh = tp, mesh
        local = torch.arange(V // tp, dtype=torch.float32)[None].repeat(3, 1) + r * (V // tp)
        full = jsx.runner._full_logits(m, local)
        out["gathered_ok"] = bool(torch.equal(full, torch.arange(V, dtype=torch.float32)[None].repeat(3, 1)))
        q.put((rank, out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        q.put((rank, {"error": repr(e)}))


@pytest.mark.parametrize("world,tp", [(2, 2), (4, 2), (4, 4)])
def test_mesh_and_row_parallel_on_cpu_ranks(world, tp):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tp, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert "error" not in res[r], res[r]
        assert res[r]["coords"] == {"data": r // tp, "tensor": r % tp}
        assert res[r]["tensor_ranks"] == [(r // tp) * tp + i for i in range(tp)]
        assert res[r]["row_parallel_err"] <= 0.01
        assert res[r]["gathered_ok"]
        first, n = res[r]["kv_heads"]
        if tp <= 2:
            assert (first, n) == (r % tp * (2 // tp), 2 // tp)
        else:
            # query heads [r*32/tp, (r+1)*32/tp) all read kv head (r*32/tp)//16
            assert n == 1 and first == ((r % tp) * (32 // tp)) // 16
