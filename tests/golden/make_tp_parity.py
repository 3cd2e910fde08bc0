"""Generates tests/golden/tp_parity.npz: the oracle's outputs for the decode
parity gate that bench.py runs at every GPU count before it times anything.

Model: the GLM-4-9B architecture (hidden 4096, 32 query / 2 kv heads of 128,
SwiGLU 13696, RMSNorm eps 1.5625e-7, RoPE theta 10000 on half of each head)
truncated to 2 decoder layers with a 8192-entry vocabulary (so the stored
logits stay small; every TP size 1/2/4/8 divides it).  Weights: the package's
random_reference_params(cfg, seed=0) — N(0, 0.02) bf16 from torch's CPU
generator, identical on every host with the same torch build — converted to
the oracle's float32 arrays.

Cases (oracle.glm4_ref.greedy_generate, whose tokens are fed back to the GPU
run: teacher forcing like benchmarks/verify_kvcache.py:111-166):
  b1:  batch 1, prompt of 8 ids (seed 1), 8 further tokens: logits [9][V] and
       the last-layer hidden state [9][H] of every produced token;
  b32: batch 32, prompt of 8 ids (seed 2), 4 further tokens: logits of
       sequences 0..3 [5][4][V], every sequence's greedy id and top-1/top-2
       margin [5][32].
Logits and hidden states are stored as bf16 bit patterns (uint16).

    python tests/golden/make_tp_parity.py [--out PATH]
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

VOCAB = 8192
LAYERS = 2
PROMPT = 8
STEPS_B1 = 8
STEPS_B32 = 4
CHECK_SEQS = 4


def bf16_bits(x) -> np.ndarray:
    import ml_dtypes
    return np.asarray(x, np.float32).astype(ml_dtypes.bfloat16).view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "tp_parity.npz"))
    args = ap.parse_args()
    sys.path.insert(0, ROOT)
    import torch

    jsx = importlib.import_module("e2e-jaxscale_b200")
    weights = importlib.import_module("e2e-jaxscale_b200.weights")
    ref = importlib.import_module("oracle.glm4_ref")

    cfg = jsx.ModelConfig(num_hidden_layers=LAYERS, vocab_size=VOCAB)
    tp = weights.random_reference_params(cfg, seed=0)
    f32 = lambda t: t.to(torch.float32).numpy()
    rc = ref.GLMConfig(num_hidden_layers=LAYERS, vocab_size=VOCAB)
    for name in ("hidden_size", "num_attention_heads", "num_key_value_heads", "head_dim", "intermediate_size",
                 "rms_norm_eps", "rope_theta"):
        assert getattr(rc, name) == getattr(cfg, name), name
    p = ref.ModelParams(cfg=rc, embed=f32(tp["embed"]))
    for lp in tp["layers"]:
        p.layers.append(ref.LayerParams(**{k: f32(v) for k, v in lp.items()}))
    p.norm = f32(tp["norm"])
    p.lm_head = f32(tp["lm_head"])

    out = {"vocab": np.int32(VOCAB), "layers": np.int32(LAYERS), "seed": np.int32(0)}
    prompt1 = np.random.default_rng(1).integers(0, VOCAB, (1, PROMPT)).astype(np.int32)
    rec = []
    toks = ref.greedy_generate(p, prompt1, STEPS_B1 + 1, max_cache_len=PROMPT + STEPS_B1 + 1, record=rec)
    out["b1_prompt"] = prompt1
    out["b1_tokens"] = toks[:, PROMPT:].astype(np.int32)            # [1][9]: fed back one by one
    out["b1_logits"] = bf16_bits(np.stack([r[0][0] for r in rec]))  # [9][V]
    out["b1_hidden"] = bf16_bits(np.stack([r[1][0] for r in rec]))  # [9][H]

    prompt32 = np.random.default_rng(2).integers(0, VOCAB, (32, PROMPT)).astype(np.int32)
    rec = []
    toks = ref.greedy_generate(p, prompt32, STEPS_B32 + 1, max_cache_len=PROMPT + STEPS_B32 + 1, record=rec)
    out["b32_prompt"] = prompt32
    out["b32_tokens"] = toks[:, PROMPT:].astype(np.int32)           # [32][5]
    out["b32_logits"] = bf16_bits(np.stack([r[0][:CHECK_SEQS] for r in rec]))  # [5][4][V]
    margins = []
    for r in rec:
        srt = np.sort(np.asarray(r[0], np.float64), axis=-1)
        margins.append(srt[:, -1] - srt[:, -2])
    out["b32_margin"] = np.stack(margins).astype(np.float32)          # [5][32]
    np.savez_compressed(args.out, **out)
    print(args.out, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
