"""bench.py's configuration runs (row-parallel op, prefill, Flash slice) after the
decode measurement: a configuration that raises is reported in the JSON line's
`configs` as `<name>_error`, the later ones are skipped on every rank, and the
run goes on to print its line.  The measurements are replaced by host fakes; the
two-rank case runs as gloo ranks on CPU."""

import importlib
import os
import socket
import sys
import types

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    sys.path.insert(0, ROOT)
    return importlib.import_module("bench")


class _FakeMesh:
    closed = 0

    def close(self):
        _FakeMesh.closed += 1


_fake_jsx = types.SimpleNamespace(create_mesh=lambda tp, ep: _FakeMesh())
_args = types.SimpleNamespace(ctx=64, seed=0, vocab=1024)
_row = {"op": "o_proj", "M": 1, "fused_us": 10.0, "gemm_nccl_us": 20.0, "rel_err": 1e-3}


def _patch(bench, rowpar=None, prefill=None, flash=None, calls=None, setattr_=setattr):
    def wrap(name, fn):
        def f(*a, **k):
            if calls is not None:
                calls.append(name)
            return fn()
        return f
    setattr_(bench, "measure_rowpar", wrap("rowpar", rowpar or (lambda: [_row])))
    setattr_(bench, "measure_prefill", wrap("prefill", prefill or (lambda: {
        "value": 1.0, "ms_per_prefill": 2.0, "mfu": 0.5, "achieved_tflops_per_gpu": 3.0})))
    setattr_(bench, "measure_flash", wrap("flash", flash or (lambda: {"expanded_batch_1": {"value": 5.0}})))


def _raise():
    raise RuntimeError("no room for the exchange slots")


def test_configs_all_measured(monkeypatch):
    bench = _bench()
    _patch(bench, setattr_=monkeypatch.setattr)
    out = bench.run_configs(_fake_jsx, None, None, torch.device("cpu"), 1, 0, _args)
    assert out["rowpar_us"] == {"o_proj_M1": [10.0, 20.0]}
    assert out["prefill_32x1024"]["tok_s"] == 1.0
    assert out["flash_tok_s"] == {"expanded_batch_1": 5.0} and out["flash_mesh"] == "tp1xep1"
    assert not any(k.endswith("_error") for k in out)


def test_config_error_skips_the_rest(monkeypatch):
    bench = _bench()
    calls = []
    _patch(bench, rowpar=_raise, calls=calls, setattr_=monkeypatch.setattr)
    out = bench.run_configs(_fake_jsx, None, None, torch.device("cpu"), 1, 0, _args)
    assert calls == ["rowpar"]
    assert out["rowpar_error"].startswith("RuntimeError: no room")
    assert "prefill_32x1024" not in out and "flash_tok_s" not in out


def test_flash_error_closes_its_mesh(monkeypatch):
    bench = _bench()
    before = _FakeMesh.closed
    _patch(bench, flash=_raise, setattr_=monkeypatch.setattr)
    out = bench.run_configs(_fake_jsx, None, None, torch.device("cpu"), 1, 0, _args)
    assert "rowpar_us" in out and "prefill_32x1024" in out
    assert out["flash_error"].startswith("RuntimeError") and "flash_tok_s" not in out
    assert _FakeMesh.closed == before + 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        bench = _bench()
        calls = []
        # only rank 1's row-parallel measurement fails
        _patch(bench, rowpar=_raise if rank == 1 else None, calls=calls)
        out = bench.run_configs(_fake_jsx, None, None, torch.device("cpu"), world, rank, _args)
        q.put((rank, calls, out))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, "error", repr(e)))


def test_config_error_on_one_rank_stops_every_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, calls, out = q.get(timeout=120)
        res[rank] = (calls, out)
    for p in procs:
        p.join(timeout=60)
    assert all(calls != "error" for calls, _ in res.values()), res
    for rank, (calls, out) in res.items():
        assert calls == ["rowpar"], (rank, calls)
        assert "prefill_32x1024" not in out
    assert res[1][1]["rowpar_error"].startswith("RuntimeError")
    assert res[0][1]["rowpar_error"] == "failed on another rank"
    assert "rowpar_us" in res[0][1]
