#!/usr/bin/env python
"""GLM-4-9B decode benchmark: tok/s and HBM-roofline MBU on 1..8 B200s (TP=N).

Workload: the full GLM-4-9B-shaped dense model (40 layers, hidden 4096,
32 q / 2 kv heads, head_dim 128, SwiGLU 13696, vocab 151552), random-init
bf16 weights generated on the device (seed 0), KV cache pre-filled by running
the seeded uniform-random prompt (context 1024) through the model, then greedy
decode steps at batch B (default 1; batch 32 is measured in the same run and
reported as "batch_32").  One step = one token per sequence.

    python bench.py [--gpus N --steps K --warmup W --batch B --ctx C --also-batch 32]
    torchrun --nproc-per-node N bench.py --gpus N ...        (TP = N, one rank per GPU)
    python bench.py --impl reference                          (CPU arm, see below)

value:  B / step time, whole job (the TP ranks cooperate on the same tokens:
        total work is fixed as N grows, scaling "strong"); step time is the
        CUDA-event time of K CUDA-graph replays with device-resident inputs,
        max over ranks.
e2e:    the same metric through the public API with host buffers: every step
        copies the fed token ids from pinned host memory, replays the step and
        reads the greedy ids back (the reference's per-step host sync).
configs: after the decode measurement the same ranks time short versions of
        configuration 2 (isolated row-parallel op, fused vs cuBLAS + NCCL),
        configuration 3 (32 x 1024-token prefill, MFU) and configuration 4 (the
        GLM-4.7-Flash slice in both MLA forms, TP = min(2, N) x EP = N / TP),
        reported compactly under "configs" (--no-configs skips them).
exposed_comm_us: per layer, the row-parallel exchanges' time on the critical
        path beyond their products (whole-step kernel stamps, max over ranks).
parity: before timing, at every GPU count, a 2-layer GLM-4-9B-shaped model
        (vocabulary 8192, host-seeded weights) runs teacher-forced through the
        same kernels (whole-step kernel at batch 1, tensor-core chain at batch
        32) and its logits, hidden states and greedy ids are compared with the
        oracle's outputs stored in tests/golden/tp_parity.npz (max relative
        error <= 2e-2, cosine >= 0.999, ids equal unless the oracle's own
        top-1/top-2 margin is within twice the measured logit error).  The
        run exits non-zero, after its JSON line, when the gate fails, when a
        peer wait timed out, or when the ranks' greedy ids disagree.
--impl reference: the reference's algorithm on the host cores.  JAX/Flax (the
        reference's runtime) is not installable on this image, so this times
        the numpy restatement under oracle/ (kind "port") on a bounded sample
        (whole 40-layer decode steps at context C, one layer's weights shared
        by the 40 layers), rank 0 only, on every host core.
"""

from __future__ import annotations

import argparse
import datetime
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "GLM-4-9B decode tok/s & HBM-roofline MBU at TP=1/2/4/8, batch 1 and 32"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--also-batch", type=lambda v: [int(x) for x in v.split(",") if x], default=[32],
                    help="further batches measured in the same run and reported as batch_<B> (default 32; '' for none)")
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--impl", choices=["jsx", "reference"], default="jsx")
    ap.add_argument("--rowpar", action="store_true",
                    help="isolated row-parallel projection: fused vs cuBLAS + NCCL (configuration 2)")
    ap.add_argument("--prefill", action="store_true",
                    help="prefill of --batch x --seq prompt tokens in one pass (configuration 3)")
    ap.add_argument("--seq", type=int, default=1024, help="prompt length of --prefill")
    ap.add_argument("--flash", action="store_true",
                    help="GLM-4.7-Flash-shaped MoE + MLA decode, 4-layer slice (configuration 4)")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch without programmatic dependent launch (on by default)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the short runs of configurations 2-4 that follow the decode measurement")
    # profiling-only shape overrides (a smaller device footprint for ncu captures)
    ap.add_argument("--layers", type=int, default=40, help=argparse.SUPPRESS)
    ap.add_argument("--vocab", type=int, default=151552, help=argparse.SUPPRESS)
    # profiling only: build the model, set the positions to --ctx (cache rows of zeros; the
    # kernels read the same bytes) and run this many eager decode steps at --batch, nothing else
    ap.add_argument("--profile-steps", type=int, default=0, help=argparse.SUPPRESS)
    return ap.parse_args()


# ---------------------------------------------------------------------------
# CPU arm (oracle restatement, host cores)
# ---------------------------------------------------------------------------

def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:
        return 1


def cpu_decode_sample(ctx: int, steps: int = 3) -> dict:
    """Whole GLM-4-9B decode steps at batch 1 on the host cores with the oracle:
    embedding, 40 decoder layers (each with its own KV cache of ctx rows), final
    norm, LM head and argmax.  The 40 layers share one layer's weights (40 distinct
    layers would need 72 GB of float32 host arrays; 1.8 GB per layer already
    streams past the host caches, so the work per layer is the same).  BLAS uses
    every core this process may run on, whatever OMP_NUM_THREADS says (torchrun
    sets it to 1), so the figure is the same at every GPU count."""
    from threadpoolctl import threadpool_limits
    cores = host_cores()
    ref = importlib.import_module("oracle.glm4_ref")
    cfg = ref.GLMConfig(num_hidden_layers=1)
    p = ref.init_params(ref.GLMConfig(num_hidden_layers=1, vocab_size=8), seed=0)  # one layer's shapes
    lp = p.layers[0]
    rng = np.random.default_rng(0)
    embed = ref.bf16(rng.standard_normal((cfg.vocab_size, cfg.hidden_size), dtype=np.float32) * 0.02)
    lm_head = ref.bf16(rng.standard_normal((cfg.vocab_size, cfg.hidden_size), dtype=np.float32) * 0.02)
    norm = np.ones(cfg.hidden_size, np.float32)
    L = ctx + steps + 2
    nl = 40
    caches = [(ref.bf16(rng.standard_normal((1, L, cfg.num_key_value_heads, cfg.head_dim), dtype=np.float32)),
               ref.bf16(rng.standard_normal((1, L, cfg.num_key_value_heads, cfg.head_dim), dtype=np.float32)))
              for _ in range(nl)]
    inv = ref.rope_inv_freq(cfg.head_dim)
    tok = np.array([[1]], np.int64)
    times = []
    with threadpool_limits(limits=cores, user_api="blas"):
        for s_ in range(steps + 1):  # the first step is a warm-up
            cur = ctx + s_
            pos = np.full((1, 1), cur, np.int32)
            mask = ref.make_decode_mask(cur, L)
            t0 = time.perf_counter()
            h = embed[tok]
            for i in range(nl):
                h = ref.decoder_layer(lp, cfg, h, pos, mask, caches[i], np.array([cur]), inv)
            logits = ref.bf16(ref.rmsnorm(h, norm, cfg.rms_norm_eps) @ lm_head.T)
            tok = ref.argmax_first(logits[:, -1])[:, None]
            t1 = time.perf_counter()
            if s_ > 0:
                times.append(t1 - t0)
        threads = blas_threads()
    per_tok = statistics.median(times)
    return {"value": 1.0 / per_tok, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"numpy oracle (oracle/glm4_ref.py) on {threads} BLAS threads ({cores} cores available), "
                       f"batch 1: {steps} whole decode steps (embedding, 40 decoder layers sharing one layer's "
                       f"weights, KV caches of {ctx}+ rows, final norm, LM head, argmax), median "
                       f"{per_tok * 1e3:.0f} ms; the reference's JAX runtime is not installable here")}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cb = cpu_decode_sample(args.ctx)
    v = cb["value"]
    line = {
        "metric": METRIC, "impl": "reference", "value": v, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / v, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(args),
        "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args) -> dict:
    return {"workload": (f"GLM-4-9B-shaped dense decode (40 layers, random-init bf16), batch {args.batch}, "
                         f"KV cache pre-filled to context {args.ctx}, TP={args.gpus}"),
            "batch": args.batch, "context": args.ctx, "tp": args.gpus, "parallelism": f"tp{args.gpus}",
            "l2": "inputs larger than L2: every step streams all weights (>= 2.2 GB per GPU)"}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASON_NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    def __init__(self, device_index):
        import torch
        self.path = tempfile.mktemp(prefix="jsx_clocks_", suffix=".csv")
        sel = str(device_index)
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            sel = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            pass
        self.proc = None
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", sel], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(REASON_NAMES, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def measured_hbm_peak() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(key: str, layers: int, lm_head_bytes: int):
    """DRAM bytes of one step from the ncu fit in profiles/ncu_traffic.json (captured at 2 and
    4 layers with a 16384-entry vocabulary, TP=1): per_layer * layers + fixed, the captured
    LM head replaced by this run's.  None where no capture exists (TP > 1: ncu does not run
    on multi-rank commands)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            e = json.load(f).get(key)
        if not e:
            return None
        return e["per_layer"] * layers + e["fixed"] - e["lm_head_capture"] + lm_head_bytes
    except Exception:
        return None


PARITY_FIXTURE = os.path.join(ROOT, "tests", "golden", "tp_parity.npz")
PARITY_REL, PARITY_COS = 2e-2, 0.999


def _bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def parity_gate(jsx, mesh, dev, world: int) -> dict:
    """Teacher-forced decode of the stored parity model on this mesh (TP = world),
    compared with the oracle's outputs in tests/golden/tp_parity.npz (written by
    tests/golden/make_tp_parity.py).  Batch 1 runs the whole-step kernel, batch
    32 the tensor-core chain with its separate all-reduce kernel.  Every rank
    runs the same calls; logits are gathered over the tensor ranks."""
    import torch
    import torch.distributed as dist

    K = jsx.kernels
    fx = np.load(PARITY_FIXTURE)
    V, nl = int(fx["vocab"]), int(fx["layers"])
    cfg = jsx.ModelConfig(num_hidden_layers=nl, vocab_size=V)
    params = jsx.weights.random_reference_params(cfg, seed=int(fx["seed"]))
    model = jsx.GLM4ForCausalLM(cfg, mesh)
    model.load_state(params)
    del params
    group = mesh.group("tensor")

    def gather_logits(st, rows):
        local = st.logits[:rows].float().contiguous()
        if world == 1:
            return local.cpu().numpy().astype(np.float64)
        if dist.get_backend(group) == "gloo":  # CPU process groups (the multi-GPU tests)
            local = local.cpu()
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local, group=group)
        return torch.cat(parts, dim=-1).cpu().numpy().astype(np.float64)

    res = {"max_rel": 0.0, "min_cos": 1.0, "ids": 0, "ids_equal": 0, "flips": [], "steps": 0}

    def compare(name, a, b):
        err = float(np.max(np.abs(a - b)) / np.max(np.abs(b)))
        cos = float(np.sum(a * b) / (np.linalg.norm(a) * np.linalg.norm(b)))
        res["max_rel"] = max(res["max_rel"], err)
        res["min_cos"] = min(res["min_cos"], cos)
        return err <= PARITY_REL and cos >= PARITY_COS

    ok = True
    for case, B in (("b1", 1), ("b32", 32)):
        prompt, toks = fx[f"{case}_prompt"], fx[f"{case}_tokens"]
        S, T = prompt.shape[1], toks.shape[1]
        want_lg = _bf16_bits_to_f32(fx[f"{case}_logits"]).astype(np.float64)
        st = jsx.DecodeState(model, B, S + T, want_logits=True)
        for s_ in range(S):
            st.ids.copy_(torch.from_numpy(prompt[:, s_]).to(dev))
            model.step(st, head=(s_ == S - 1))
        for t in range(T):
            if t > 0:
                st.ids.copy_(torch.from_numpy(toks[:, t - 1]).to(dev))
                model.step(st, head=True)
            ids = st.ids.cpu().numpy()
            if case == "b1":
                lg = gather_logits(st, 1)
                ok &= compare("logits", lg[0], want_lg[t])
                ok &= compare("hidden", st.h[0].float().cpu().numpy().astype(np.float64),
                              _bf16_bits_to_f32(fx["b1_hidden"][t]).astype(np.float64))
                srt = np.sort(want_lg[t])
                margins = np.array([srt[-1] - srt[-2]])
                bound = float(np.max(np.abs(lg[0] - want_lg[t])))
            else:
                nchk = want_lg.shape[1]
                lg = gather_logits(st, nchk)
                for b in range(nchk):
                    ok &= compare("logits", lg[b], want_lg[t, b])
                margins = fx["b32_margin"][t]
                bound = float(np.max(np.abs(lg - want_lg[t])))
            want_ids = toks[:, t]
            res["ids"] += len(ids)
            res["ids_equal"] += int(np.sum(ids == want_ids))
            for b in np.nonzero(ids != want_ids)[0]:
                res["flips"].append({"case": case, "step": t, "seq": int(b), "margin": float(margins[b]),
                                     "logit_err": bound})
                ok &= bool(margins[b] <= 2 * bound)
            res["steps"] += 1
        del st
    torch.cuda.synchronize()
    if model.comm is not None:
        try:
            model.comm.check()
        except jsx._lib.JsxError:
            ok = False
            res["timeout"] = True
    ok &= K.device_error() == 0
    del model
    torch.cuda.synchronize()
    res["ok"] = bool(ok)
    res["tolerance"] = f"max rel {PARITY_REL}, cosine {PARITY_COS}, ids equal outside the margin rule"
    res["model"] = (f"GLM-4-9B-shaped, {nl} layers, vocabulary {V}, host-seeded weights; batch 1 (whole-step "
                    f"kernel) and 32 (tensor-core chain), teacher-forced against the oracle's stored outputs")
    return res


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    jsx = importlib.import_module("e2e-jaxscale_b200")
    K = jsx.kernels
    K.set_pdl(not args.no_pdl)
    dev = torch.device("cuda", local)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    mesh = jsx.create_mesh(tp=args.gpus)
    if args.profile_steps:
        cfg = jsx.ModelConfig(num_hidden_layers=args.layers, vocab_size=args.vocab)
        model = jsx.GLM4ForCausalLM(cfg, mesh)
        model.init_random(seed=args.seed)
        st = jsx.DecodeState(model, args.batch, args.ctx + args.profile_steps + 1)
        st.pos.fill_(args.ctx)
        for _ in range(args.profile_steps):
            model.step(st, head=True)
        torch.cuda.synchronize()
        print(json.dumps({"mode": "profile", "steps": args.profile_steps, "batch": args.batch,
                          "layers": args.layers, "vocab": args.vocab,
                          "kernels_per_step": model.kernels_per_step(args.batch),
                          "weight_bytes": model.weight_bytes()}), flush=True)
        mesh.close()
        return
    # correctness first: the same kernels on the stored parity model, at this TP
    parity = parity_gate(jsx, mesh, dev, world)
    failures = [] if parity["ok"] else ["parity gate"]
    cfg = jsx.ModelConfig(num_hidden_layers=args.layers, vocab_size=args.vocab)
    model = jsx.GLM4ForCausalLM(cfg, mesh)
    model.init_random(seed=args.seed)
    peak, peak_kind = measured_hbm_peak()

    def run_checks(st) -> dict:
        """After a timed run, on every rank: no peer or barrier wait timed out, and the
        greedy ids are identical on every rank."""
        out = {"timeout": False, "ids_agree": True}
        torch.cuda.synchronize()
        if model.comm is not None:
            try:
                model.comm.check()
            except jsx._lib.JsxError:
                out["timeout"] = True
        if K.device_error() != 0:
            out["timeout"] = True
        if world > 1:
            ids = st.ids.clone()
            parts = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(parts, ids)
            out["ids_agree"] = all(torch.equal(parts[0], x) for x in parts)
            flag = torch.tensor([1.0 if out["timeout"] else 0.0], device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
            out["timeout"] = bool(flag.item() > 0)
        return out
    stream = torch.cuda.current_stream()
    c = cfg

    def measure(B: int, with_clocks: bool) -> dict:
        """Prefill the context at batch B, then time K decode steps (device) and
        K/2 end-to-end steps (host ids in, greedy ids out)."""
        C = args.ctx
        e2e_steps = max(16, args.steps // 2)
        L = C + 2 * args.warmup + args.steps + e2e_steps + 24
        st = jsx.DecodeState(model, B, L)
        graph = jsx.DecodeGraph(model, st)
        barrier()
        # prefill the context with seeded uniform prompt ids (one graph replay per position)
        prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, (B, C)).astype(np.int32)
        prompt_dev = torch.from_numpy(prompt).to(dev)
        st.pos.zero_()
        for s_ in range(C):
            st.ids.copy_(prompt_dev[:, s_])
            if s_ < C - 1:
                graph.prefill()
            else:
                graph.decode()
        for _ in range(args.warmup):
            graph.decode()
        torch.cuda.synchronize()
        barrier()

        clocks = ClockSampler(local) if with_clocks else None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            graph.decode()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

        # end to end through the public API, host buffers
        host_in = torch.empty(B, dtype=torch.int32).pin_memory()
        host_out = torch.empty(B, dtype=torch.int32).pin_memory()
        host_in.copy_(st.ids.cpu())
        for _ in range(args.warmup):
            st.ids.copy_(host_in, non_blocking=True)
            graph.decode()
            host_out.copy_(st.ids, non_blocking=True)
            stream.synchronize()
            host_in.copy_(host_out)
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            st.ids.copy_(host_in, non_blocking=True)
            graph.decode()
            host_out.copy_(st.ids, non_blocking=True)
            stream.synchronize()
            host_in.copy_(host_out)
        t1 = time.perf_counter()
        barrier()
        e2e_ms = max_over_ranks((t1 - t0) * 1e3 / e2e_steps)
        clk = clocks.stop() if clocks else None
        checks = run_checks(st)

        # step bytes: weights streamed + KV rows read/written + embedding rows
        kv_bytes = B * c.num_hidden_layers * 2 * (C + args.warmup + args.steps) * model.nkv_l * c.head_dim * 2
        step_bytes = model.weight_bytes() + kv_bytes + B * c.hidden_size * 2
        mbu = step_bytes / (ms * 1e-3) / (peak * 1e9)
        ref_model_bytes = 2 * (c.num_hidden_layers * (
            c.hidden_size * c.num_attention_heads * c.head_dim * 2
            + c.hidden_size * c.num_key_value_heads * c.head_dim * 2
            + c.num_attention_heads * c.head_dim + 2 * c.num_key_value_heads * c.head_dim
            + 3 * c.hidden_size * c.intermediate_size + 2 * c.hidden_size)
            + 2 * c.vocab_size * c.hidden_size + c.hidden_size)
        mbu_ref = ref_model_bytes / (ms * 1e-3) / (peak * 1e9 * args.gpus)

        fused = model.fused_step and st.step_args is not None
        phase_us, exposed = None, None
        lm_bytes = model.lm_head.numel() * 2
        traffic = ncu_traffic(f"decode_step_tp{args.gpus}_b{B}", c.num_hidden_layers, lm_bytes)
        if fused:
            # the whole step is one kernel launch: its duration is the timed step
            kern_name = "jsx_decode_step (k_decode_step<M>): the whole decode step, one launch per step"
            kern_ms, kern_bytes = ms, step_bytes
            # per-phase breakdown from the kernel's %globaltimer trace (CTA 0, after each grid barrier)
            nl = c.num_hidden_layers
            tr = torch.zeros(2 + 13 * nl, dtype=torch.int64, device=dev)
            tar = torch.zeros(4 * nl, dtype=torch.int64, device=dev)
            tph = torch.zeros(15 * nl, dtype=torch.int64, device=dev)
            st.step_args.trace = tr.data_ptr()
            st.step_args.trace_ar = tar.data_ptr()
            acc, sub, exp_, pts = None, None, None, None
            for i in range(12):
                # steps 8-11 add the per-phase points (a block synchronisation each) and
                # feed only the points
                tar.zero_()
                tph.zero_()
                st.step_args.trace_phase = tph.data_ptr() if i >= 8 else None
                model.step(st, head=True)
                t = tr.cpu().numpy().astype(np.float64)
                if i >= 8:
                    # latest CTA at each point of each phase, from the phase's start
                    pstart = t[:5 * nl].reshape(nl, 5)
                    pp = (tph.cpu().numpy().astype(np.float64).reshape(nl, 5, 3) - pstart[:, :, None]) / 1e3
                    pts = pp if pts is None else pts + pp
                    continue
                ta = tar.cpu().numpy().astype(np.float64).reshape(nl, 2, 2)
                e_ = (ta[:, :, 1] - ta[:, :, 0]) / 1e3  # [layer][o_proj, down]
                exp_ = e_ if exp_ is None else exp_ + e_
                d = np.diff(t[:2 + 5 * nl]) / 1e3
                acc = d if acc is None else acc + d
                # attention of head group 0, relative to the start of the attention phase
                start = t[1:1 + 5 * nl:5]
                s5 = (t[2 + 5 * nl:].reshape(nl, 8) - start[:, None]) / 1e3
                sub = s5 if sub is None else sub + s5
            st.step_args.trace = None
            st.step_args.trace_ar = None
            st.step_args.trace_phase = None
            acc /= 8
            sub /= 8
            exp_ /= 8
            pts /= 4
            exposed = {"per_layer_us": max_over_ranks(float(exp_.sum(axis=1).mean())),
                       "o_proj_us": max_over_ranks(float(exp_[:, 0].mean())),
                       "down_us": max_over_ranks(float(exp_[:, 1].mean())),
                       "definition": ("per row-parallel phase: latest time any CTA finished its rank-ordered "
                                      "sums minus the latest time any CTA had pushed its partials (the phase's "
                                      "critical path beyond its own product: what a local no-op exchange would "
                                      "remove); mean over layers of o_proj + down, 8 traced eager steps, max "
                                      "over ranks")}
            per = acc[:5 * nl].reshape(nl, 5)
            names = ["qkv", "attention", "o_proj_allreduce", "gate_up", "down_allreduce"]
            phase_us = {n: float(per[:, i].mean()) for i, n in enumerate(names)}
            phase_us["lm_head"] = float(acc[5 * nl])
            # from 4 further steps (the points' block synchronisations stay out of the times above)
            phase_us["points_us"] = {n: [round(float(pts[:, i, k].mean()), 2) for k in range(3)]
                                     for i, n in enumerate(names)}
            # stamps an item never writes (the split merge runs in the o_proj staging when the
            # records are small) stay zero and are left out
            phase_us["attention_group0_us"] = {k: float(sub[:, i].mean()) for i, k in enumerate(
                ["split0_start", "split0_staged", "split0_scored", "split0_softmax", "split0_pv_done",
                 "split0_counted", "merge_done", "merge_start"]) if np.all(t[2 + 5 * nl:].reshape(nl, 8)[:, i] > 0)}
            phase_us["note"] = ("mean us per layer (lm_head: once per step) between grid barriers, each "
                                "phase including its barrier; CTA 0 %globaltimer over 8 eager steps; "
                                "attention_group0_us: head group 0 from the start of the attention phase; "
                                "points_us: per phase, from its start, the latest CTA to have staged its "
                                "input, finished its product (row-parallel: pushed its partials) and "
                                "finished the phase; 4 more traced steps")
        else:
            # the tensor-core chain: the step is one CUDA graph of its launches; its algorithmic
            # bytes over its time
            kern_name = (f"the batch-{B} step: {model.kernels_per_step(B)} launches (RMSNorm, tcgen05 GEMMs "
                         "k_tc_gemm<EPI>, decode attention, two-shot exchanges at TP > 1) in one CUDA graph")
            kern_ms, kern_bytes = ms, step_bytes
        achieved = kern_bytes / (kern_ms * 1e-3) / 1e9
        graph.release()
        del st, graph
        torch.cuda.synchronize()
        return {
            "B": B, "ms": ms, "e2e_ms": e2e_ms, "clocks": clk, "mbu": mbu, "mbu_ref": mbu_ref,
            "step_bytes": step_bytes, "phase_us": phase_us, "exposed": exposed, "checks": checks,
            "roofline": {"bound": "hbm", "kernel": kern_name,
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} hbm_gbs (burst)",
                         "traffic": traffic, "algorithmic_bytes_per_launch": kern_bytes,
                         "launch_ms": kern_ms},
            "launches": model.kernels_per_step(B, head=True) * args.steps,
        }

    main_res = measure(args.batch, with_clocks=True)
    extra = {}
    for b in args.also_batch:
        if b != args.batch:
            extra[b] = measure(b, with_clocks=False)
    configs = None
    if not args.no_configs:
        configs = run_configs(jsx, model, mesh, dev, world, rank, args)
    cpu = cpu_decode_sample(args.ctx) if (rank == 0 and world == 1) else None

    for b, x in [(args.batch, main_res)] + list(extra.items()):
        if x["checks"]["timeout"]:
            failures.append(f"batch {b}: a peer or grid-barrier wait timed out")
        if not x["checks"]["ids_agree"]:
            failures.append(f"batch {b}: greedy ids differ across ranks")

    if rank == 0:
        r = main_res
        B = r["B"]
        line = {
            "metric": METRIC, "value": B / (r["ms"] * 1e-3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init N(0,0.02) bf16 weights (device RNG seed 0), uniform prompt ids seed 1",
            "config": workload_config(args),
            "mbu": r["mbu"], "bytes_per_step_per_gpu": r["step_bytes"],
            "mbu_reference_formula": r["mbu_ref"],
            "roofline": r["roofline"],
            "cpu_baseline": cpu,
            "e2e": {"value": B / (r["e2e_ms"] * 1e-3), "unit": "tok/s", "ms_per_step": r["e2e_ms"],
                    "h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * 4},
            "gpu_launches": r["launches"],
            "pdl": K.pdl_enabled(),
            "clocks": r["clocks"],
        }
        for b, x in extra.items():
            line[f"batch_{b}"] = {
                "value": b / (x["ms"] * 1e-3), "unit": "tok/s", "ms_per_step": x["ms"], "mbu": x["mbu"],
                "bytes_per_step_per_gpu": x["step_bytes"],
                "e2e": {"value": b / (x["e2e_ms"] * 1e-3), "unit": "tok/s", "ms_per_step": x["e2e_ms"],
                        "h2d_bytes_per_step": b * 4, "d2h_bytes_per_step": b * 4},
                "roofline": x["roofline"], "gpu_launches": x["launches"], "checks": x["checks"],
                "note": "same workload and timing at this batch, measured after the headline batch in the same run",
            }
        if configs is not None:
            line["configs"] = configs
        # last and compact, so they stay in view at the end of the line
        if r["phase_us"] is not None:
            line["phase_us"] = {k: (round(v, 2) if isinstance(v, float) else
                                    {kk: (round(vv, 2) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                                    if isinstance(v, dict) else v)
                                for k, v in r["phase_us"].items() if k != "note"}
        if r["exposed"] is not None:
            line["exposed_comm_us"] = {k: round(v, 2) for k, v in r["exposed"].items() if k != "definition"}
        line["checks"] = r["checks"]
        line["parity"] = {"ok": parity["ok"], "tp": world, "max_rel": round(parity["max_rel"], 4),
                          "min_cos": round(parity["min_cos"], 6),
                          "ids_equal": f"{parity['ids_equal']}/{parity['ids']}",
                          "flips_within_margin": len(parity["flips"]), "steps": parity["steps"]}
        line["failures"] = failures
        print(json.dumps(line), flush=True)
    barrier()
    mesh.close()
    if world > 1:
        dist.destroy_process_group()
    if failures:
        print("bench: FAILED: " + "; ".join(failures), file=sys.stderr, flush=True)
        raise SystemExit(1)


def measure_rowpar(jsx, mesh, dev, world: int, rank: int, steps: int, warmup: int,
                   Ms=(1, 8, 32, 256, 4096)) -> list:
    """Configuration 2 on `mesh` (TP = world): o_proj W[4096 x 4096] and down_proj
    W[13696 x 4096] (bf16 N(0, 0.02)), activations N(0, 1), K split over the ranks: this
    library's fused product + NVLink all-reduce + residual against cuBLAS (torch.matmul)
    then NCCL all_reduce and the residual add.  Time per call = CUDA events over `steps`
    back-to-back calls after `warmup`, max over ranks; rel_err compares the two results."""
    import torch
    import torch.distributed as dist

    K = jsx.kernels
    comm = mesh.comm(K.TC_MAX_TOKENS, 4096)
    comm_t = mesh.comm_tiles(max(Ms), 4096) if any(M > K.TC_MAX_TOKENS for M in Ms) else None
    stream = torch.cuda.current_stream()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn) -> float:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(b) * 1e3 / steps)

    g = torch.Generator(device=dev).manual_seed(1234)
    results = []
    for name, Kfull in (("o_proj", 4096), ("down_proj", 13696)):
        N = 4096
        kl = Kfull // world
        w_full = (torch.randn(N, Kfull, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w = w_full[:, rank * kl:(rank + 1) * kl].contiguous()          # this rank's [N, K/t]
        del w_full
        for M in Ms:
            x_full = torch.randn(M, Kfull, generator=g, device=dev).to(torch.bfloat16)
            x = x_full[:, rank * kl:(rank + 1) * kl].contiguous()
            h0 = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
            h_f = h0.clone()
            if M <= K.MAX_DECODE_TOKENS:
                fused = lambda: K.row_linear_allreduce(comm, x, w, h_f)
                path = "gemv"
            elif M <= K.TC_MAX_TOKENS:
                ws = K.tc_workspace(M, [(kl, N)], dev)
                fused = lambda: K.tc_row_linear_allreduce(comm, x, w, h_f, ws)
                path = "tcgen05"
            else:
                ws = K.wide_workspace(M, [(kl, N)], dev, norm=False)
                fused = lambda: K.wide_row_linear_allreduce(comm_t, x, w, h_f, ws)
                path = "tcgen05-wide+tile-exchange"
            h_b = h0.clone()

            def unfused():
                y = torch.matmul(x, w.t())
                if world > 1:
                    dist.all_reduce(y)
                h_b.add_(y)

            # one call each from the same residual for the parity check
            h_f.copy_(h0)
            fused()
            h_b.copy_(h0)
            unfused()
            torch.cuda.synchronize()
            ref_ = h_b.float()
            err = float((h_f.float() - ref_).abs().max() / ref_.abs().max())
            t_f = timed(fused)
            t_u = timed(unfused)
            r_ = {"op": name, "M": M, "fused_us": t_f, "gemm_nccl_us": t_u, "speedup": t_u / t_f,
                  "rel_err": err, "fused_path": path}
            if world > 1 and M > K.TC_MAX_TOKENS:
                # how much of the exchange the tile pipeline hides: the same product without
                # the exchange (one rank's local shard), and NCCL's all-reduce of the result alone
                h_l = h0.clone()
                t_g = timed(lambda: K.wide_row_linear_allreduce(None, x, w, h_l, ws))
                y_ = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
                t_ar = timed(lambda: dist.all_reduce(y_))
                r_.update({"gemm_only_us": t_g, "nccl_allreduce_us": t_ar,
                           "hidden_frac": max(0.0, 1.0 - (t_f - t_g) / t_ar)})
            results.append(r_)
    for c_ in (comm, comm_t):
        if c_ is not None:
            c_.check()
    return results


def run_configs(jsx, model, mesh, dev, world: int, rank: int, args) -> dict:
    """Short runs of configurations 2, 3 and 4 at this GPU count after the decode
    measurement (same processes, same mesh for 2 and 3; TP = min(2, N) x EP = N / TP for
    4), summarised compactly for the JSON line.  A configuration that raises is recorded
    as `<name>_error` and the ones after it are skipped (every rank agrees first); the
    decode measurement, already taken, stands."""
    import torch
    import torch.distributed as dist

    out = {}

    def rowpar():
        rp = measure_rowpar(jsx, mesh, dev, world, rank, steps=20, warmup=3)
        out["rowpar_us"] = {f"{r['op']}_M{r['M']}": [round(r["fused_us"], 1), round(r["gemm_nccl_us"], 1)]
                            + ([round(r["gemm_only_us"], 1), round(r["nccl_allreduce_us"], 1)]
                               if "gemm_only_us" in r else []) for r in rp}
        out["rowpar_note"] = ("[fused, cuBLAS+NCCL(, fused product without the exchange, NCCL all-reduce "
                              "alone)] us per call, configuration 2, K split over the N ranks")
        hid = {f"{r['op']}_M{r['M']}": round(r["hidden_frac"], 3) for r in rp if "hidden_frac" in r}
        if hid:
            out["allreduce_hidden_frac"] = hid
        out["rowpar_max_rel_err"] = round(max(r["rel_err"] for r in rp), 5)

    def prefill():
        pf = measure_prefill(jsx, model, dev, world, 32, 1024, steps=2, warmup=1)
        out["prefill_32x1024"] = {"tok_s": round(pf["value"], 1), "ms": round(pf["ms_per_prefill"], 2),
                                  "mfu": round(pf["mfu"], 4), "tflops_per_gpu": round(pf["achieved_tflops_per_gpu"], 1)}

    def flash():
        tp = min(2, world)
        out["flash_mesh"] = f"tp{tp}xep{world // tp}"
        fmesh = jsx.create_mesh(tp=tp, ep=world // tp)
        try:
            fl = measure_flash(jsx, fmesh, dev, world, args.ctx, steps=20, warmup=3, seed=args.seed,
                               vocab=args.vocab)
        finally:
            fmesh.close()
        out["flash_tok_s"] = {k: round(v["value"], 1) for k, v in fl.items()}

    for name, fn in (("rowpar", rowpar), ("prefill", prefill), ("flash", flash)):
        err = None
        try:
            fn()
        except Exception as e:  # noqa: BLE001 - reported in the line; the decode numbers stand
            err = f"{type(e).__name__}: {e}"[:300]
            out[f"{name}_error"] = err
        torch.cuda.empty_cache()
        failed = torch.tensor([1.0 if err else 0.0], device=dev)
        if world > 1:
            dist.all_reduce(failed)
        if failed.item() > 0:
            if err is None:
                out[f"{name}_error"] = "failed on another rank"
            break
    return out


def run_rowpar(args) -> None:
    """Isolated row-parallel projection (configuration 2): measure_rowpar on TP = N ranks."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    jsx = importlib.import_module("e2e-jaxscale_b200")
    mesh = jsx.create_mesh(tp=world)
    results = measure_rowpar(jsx, mesh, dev, world, rank, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps({"mode": "rowpar", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "dtype": "bf16", "data": "synthetic N(0,0.02) weights, N(0,1) activations (seed 1234)",
                          "baseline": "torch.matmul (cuBLAS) + torch.distributed all_reduce (NCCL) + residual add",
                          "results": results}), flush=True)
    mesh.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def prefill_peak() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["bf16_tflops_sustained"]), "measured bf16_tflops_sustained (cuBLAS, long loop)"
    except Exception:
        return 1400.0, "fallback sustained bf16"


def measure_prefill(jsx, model, dev, world: int, B: int, S: int, steps: int, warmup: int) -> dict:
    """Configuration 3 on the model's mesh: B x S seeded uniform prompt ids prefilled in one
    pass per rank (GLM4ForCausalLM.prefill: wide tcgen05 projections, prefill attention,
    row-parallel products with the in-epilogue tile exchange at TP > 1, the greedy token of
    every sequence's last position).  Time per prefill = CUDA events over `steps` prefills
    after `warmup`, max over ranks.  MFU counts the matmul flops of every position without
    the all-position LM head (this path computes last-position logits only; the reference
    all of them), the causal attention flops and the last-position LM head.  The share of
    the all-reduce hidden behind the GEMM is measured on the row-parallel products alone
    (measure_rowpar, M = 4096: hidden_frac)."""
    import torch
    import torch.distributed as dist

    cfg = model.config
    ps = jsx.PrefillState(model, B, S, S)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g, dtype=torch.int32).to(dev)
    for _ in range(max(warmup, 1)):
        model.prefill(ps, ids)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    steps = max(steps, 1)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        model.prefill(ps, ids)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if ps.comm is not None:
        ps.comm.check()
    H, I, nq, hd, L = cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads, cfg.head_dim, \
        cfg.num_hidden_layers
    qkv_rows = (nq + 2 * cfg.num_key_value_heads) * hd
    mm_per_tok = 2.0 * L * H * (qkv_rows + H + 3 * I)
    attn = 4.0 * nq * hd * (S + 1) / 2 * L
    flops = B * S * (mm_per_tok + attn) + 2.0 * B * H * cfg.vocab_size
    peak, peak_src = prefill_peak()
    tflops = flops / (ms * 1e-3) / 1e12
    del ps
    torch.cuda.synchronize()
    return {"value": B * S / (ms * 1e-3), "unit": "tok/s", "ms_per_prefill": ms, "batch": B, "seq": S,
            "flops_per_prefill": flops, "achieved_tflops_per_gpu": tflops / world, "mfu": tflops / world / peak,
            "peak_tflops": peak, "peak_source": peak_src}


def run_prefill(args) -> None:
    """Configuration 3: GLM-4-9B-shaped prefill of --batch x --seq seeded uniform prompt ids
    (random-init bf16 weights, causal, cache length --seq), measure_prefill on TP = N ranks."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    jsx = importlib.import_module("e2e-jaxscale_b200")
    K = jsx.kernels
    K.set_pdl(not args.no_pdl)
    mesh = jsx.create_mesh(tp=world)
    cfg = jsx.ModelConfig(num_hidden_layers=args.layers, vocab_size=args.vocab)
    model = jsx.GLM4ForCausalLM(cfg, mesh)
    model.init_random(seed=args.seed)
    B = args.batch if args.batch > 1 else 32
    S = args.seq
    clocks = ClockSampler(local)
    res = measure_prefill(jsx, model, dev, world, B, S, args.steps, args.warmup)
    clk = clocks.stop()
    if rank == 0:
        print(json.dumps({
            "mode": "prefill", "metric": "GLM-4-9B prefill tok/s and MFU (configuration 3)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic: random-init N(0,0.02) bf16 weights (device RNG), uniform prompt ids seed 1",
            "config": {"workload": f"GLM-4-9B-shaped prefill, batch {B} x {S} tokens, causal, cache {S}, "
                                   f"{args.layers} layers, TP={world}", "batch": B, "seq": S, "tp": world,
                       "parallelism": f"tp{world}"},
            **res,
            "flops_note": "matmul flops of every position without the all-position LM head, causal attention "
                          "flops, and the last-position LM head",
            "clocks": clk}), flush=True)
    mesh.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def flash_config(jsx, vocab: int):
    """GLM-4.7-Flash-shaped 4-layer slice (configuration 4)."""
    return jsx.ModelConfig(hidden_size=2048, num_hidden_layers=4, num_attention_heads=20, num_key_value_heads=20,
                           intermediate_size=10240, vocab_size=vocab, rms_norm_eps=1e-5,
                           rope_theta=1000000.0, n_routed_experts=64, n_shared_experts=1, num_experts_per_tok=4,
                           moe_intermediate_size=1536, routed_scaling_factor=1.8, norm_topk_prob=True,
                           first_k_dense_replace=1, q_lora_rank=768, kv_lora_rank=512, qk_nope_head_dim=192,
                           qk_rope_head_dim=64, v_head_dim=256, attention_bias=False, partial_rotary_factor=1.0)


def measure_flash(jsx, mesh, dev, world: int, ctx: int, steps: int, warmup: int, seed: int, vocab: int,
                  batches=(1, 32)) -> dict:
    """Decode steps of the configuration-4 slice on `mesh` for both MLA forms (the
    reference's expanded per-head cache, and the absorbed-weight latent cache), each a
    CUDA graph of one step replayed `steps` times; ms per step = max over ranks."""
    import torch
    import torch.distributed as dist

    cfg = flash_config(jsx, vocab)
    out = {}
    for absorbed in (False, True):
        model = jsx.GLM4FlashForCausalLM(cfg, mesh, absorbed_mla=absorbed)
        model.init_random(seed=seed)
        form = "latent" if absorbed else "expanded"
        for B in batches:
            L = ctx + warmup + max(steps, 1) + 1
            caches = model.init_kv_caches(B, L)
            g = torch.Generator(device=dev).manual_seed(7)
            for c_ in caches:
                c_.k[:, :ctx].normal_(generator=g)
                if c_.v.numel():
                    c_.v[:, :ctx].normal_(generator=g)
            ids = torch.from_numpy(np.random.default_rng(1).integers(0, cfg.vocab_size, (B, 1))
                                   .astype(np.int32)).to(dev)
            pos = torch.full((B, 1), ctx, dtype=torch.int32, device=dev)

            def step():
                model(ids, pos, None, kv_caches=caches, cache_position=None)
                pos.add_(1)

            for _ in range(max(warmup, 1)):  # eager: creates every lazily built resource
                step()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            pos.fill_(ctx + max(warmup, 1))
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(max(steps, 1)):
                graph.replay()
            b.record()
            torch.cuda.synchronize()
            del graph
            ms = a.elapsed_time(b) / max(steps, 1)
            if world > 1:
                t = torch.tensor([ms], dtype=torch.float64, device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            cache_bytes = sum(c_.k.numel() + c_.v.numel() for c_ in caches) * 2 * (ctx + 1) // L
            out[f"{form}_batch_{B}"] = {"value": B / (ms * 1e-3), "unit": "tok/s", "ms_per_step": ms,
                                        "cache_bytes_read_per_step": cache_bytes}
            del caches
        del model
        torch.cuda.synchronize()
    return out


def run_flash(args) -> None:
    """Configuration 4: GLM-4.7-Flash-shaped MoE decode on a 4-layer slice (hidden 2048, MLA with
    q_lora 768 / kv_lora 512 / nope 192 / rope 64 / v 256 / 20 heads, 64 routed experts of 1536
    with top-4 softmax routing and one shared expert of 1536, a dense SwiGLU MLP of 10240 in
    layer 0), random-init bf16 weights N(0, 0.02), batch 1 and 32 at context 1024 (the cache
    rows before the position hold seeded random values), both MLA forms.  Each step is the
    reference-signature forward of one token per sequence through GLM4FlashForCausalLM on
    device-resident ids and positions, captured once in a CUDA graph (the position advances
    inside the graph) and replayed; time per step = CUDA events over --steps replays after
    --warmup, max over ranks.  Mesh: TP = min(2, N), EP = N / TP."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    jsx = importlib.import_module("e2e-jaxscale_b200")
    K = jsx.kernels
    K.set_pdl(not args.no_pdl)
    tp = min(2, world)
    mesh = jsx.create_mesh(tp=tp, ep=world // tp)
    ctx = args.ctx
    out = measure_flash(jsx, mesh, dev, world, ctx, args.steps, args.warmup, args.seed, args.vocab)
    if rank == 0:
        print(json.dumps({"mode": "flash", "metric": "GLM-4.7-Flash-shaped MoE decode tok/s (configuration 4)",
                          "n_gpus": world, "mesh": {"tensor": tp, "expert": world // tp}, "steps": args.steps,
                          "warmup": args.warmup, "dtype": "bf16", "context": ctx,
                          "data": "synthetic: random-init N(0,0.02) bf16 weights, random cache rows, seeded ids",
                          "config": {"workload": "GLM-4.7-Flash-shaped 4-layer slice, decode, context "
                                                 f"{ctx}, TP={tp} x EP={world // tp}"},
                          "note": ("one decode step captured in a CUDA graph and replayed; expanded = the "
                                   "reference's per-head MLA cache, latent = the absorbed-weight form"),
                          **out}), flush=True)
    mesh.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.rowpar:
        run_rowpar(args)
    elif args.prefill:
        run_prefill(args)
    elif args.flash:
        run_flash(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
