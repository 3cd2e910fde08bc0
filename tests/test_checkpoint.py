"""HF safetensors loading (e2e-jaxscale_b200/checkpoint.py) against the mapping of
the reference's loader (models/glm4.py:277-358, utils/weight_utils.py:61-161):
a small GLM-4-shaped checkpoint written in HF naming (BF16 matrices, fused
gate_up_proj, an F32 norm, two shard files) must come back as the reference
layout: [in, out] matrices, gate/up split from the fused rows, biases, gains."""

import json
import os
import struct

import ml_dtypes
import numpy as np
import pytest
import torch


def write_safetensors(path, tensors):
    """name -> numpy array (ml_dtypes.bfloat16, float16 or float32)."""
    header, blobs, off = {}, [], 0
    codes = {np.dtype(ml_dtypes.bfloat16): "BF16", np.dtype(np.float16): "F16", np.dtype(np.float32): "F32"}
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        header[name] = {"dtype": codes[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def hf_checkpoint(ref, tmp_path, rc, p):
    """The oracle parameters p written as a 2-file HF checkpoint; returns the directory."""
    bf = lambda a: np.asarray(a, np.float32).astype(ml_dtypes.bfloat16)
    t0 = {"model.embed_tokens.weight": bf(p.embed), "model.norm.weight": np.asarray(p.norm, np.float32),
          "lm_head.weight": bf(p.lm_head)}
    t1 = {}
    for i, lp in enumerate(p.layers):
        d = t0 if i % 2 == 0 else t1
        q = f"model.layers.{i}"
        d[f"{q}.input_layernorm.weight"] = bf(lp.ln1)
        d[f"{q}.post_attention_layernorm.weight"] = bf(lp.ln2)
        for n, w, b in (("q", lp.wq, lp.bq), ("k", lp.wk, lp.bk), ("v", lp.wv, lp.bv)):
            d[f"{q}.self_attn.{n}_proj.weight"] = bf(np.asarray(w).T)
            d[f"{q}.self_attn.{n}_proj.bias"] = bf(b)
        d[f"{q}.self_attn.o_proj.weight"] = bf(np.asarray(lp.wo).T)
        d[f"{q}.mlp.gate_up_proj.weight"] = bf(np.concatenate([np.asarray(lp.wg).T, np.asarray(lp.wu).T], axis=0))
        d[f"{q}.mlp.down_proj.weight"] = bf(np.asarray(lp.wd).T)
    write_safetensors(os.path.join(tmp_path, "model-00001-of-00002.safetensors"), t0)
    write_safetensors(os.path.join(tmp_path, "model-00002-of-00002.safetensors"), t1)
    return str(tmp_path)


def small(ref):
    return ref.GLMConfig(hidden_size=64, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=16, intermediate_size=48, vocab_size=50)


def test_reference_layout_from_hf_names(jsx, ref, tmp_path):
    import importlib
    ckpt = importlib.import_module("e2e-jaxscale_b200.checkpoint")
    rc = small(ref)
    p = ref.init_params(rc, seed=4)
    path = hf_checkpoint(ref, tmp_path, rc, p)
    cfg = jsx.ModelConfig(hidden_size=64, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
                          head_dim=16, intermediate_size=48, vocab_size=50, model_path=path)
    ck = ckpt.Checkpoint(path)
    try:
        got = ckpt.GLM4Params(ck, cfg)
        f = lambda t: t.float().numpy()
        assert np.array_equal(f(got.embed), p.embed)
        assert np.array_equal(f(got.norm), p.norm) and got.norm.dtype == torch.float32
        assert np.array_equal(f(got.lm_head), p.lm_head)
        for lg, lp in zip(got.layers, p.layers):
            for n in ("ln1", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "ln2", "wg", "wu", "wd"):
                t = getattr(lg, n)
                assert t.dtype == torch.bfloat16 and np.array_equal(f(t), getattr(lp, n)), n
    finally:
        ck.close()


def test_tied_embeddings_and_errors(jsx, ref, tmp_path):
    import importlib
    ckpt = importlib.import_module("e2e-jaxscale_b200.checkpoint")
    emb = np.arange(12, dtype=np.float32).reshape(3, 4).astype(ml_dtypes.bfloat16)
    write_safetensors(os.path.join(tmp_path, "a.safetensors"), {"model.embed_tokens.weight": emb,
                                                                 "model.norm.weight": np.ones(4, np.float16)})
    cfg = jsx.ModelConfig(hidden_size=4, num_hidden_layers=0, num_attention_heads=1, num_key_value_heads=1,
                          head_dim=4, intermediate_size=4, vocab_size=3, tie_word_embeddings=True)
    ck = ckpt.Checkpoint(str(tmp_path))
    try:
        prm = ckpt.GLM4Params(ck, cfg)
        assert np.array_equal(prm.lm_head.float().numpy(), emb.astype(np.float32))
        assert prm.norm.dtype == torch.float16
        with pytest.raises(KeyError):
            ck.get("model.layers.0.mlp.down_proj.weight")
    finally:
        ck.close()
    with pytest.raises(FileNotFoundError):
        ckpt.Checkpoint(str(tmp_path / "empty"))
    bad = tmp_path / "bad"
    bad.mkdir()
    with open(bad / "x.safetensors", "wb") as fh:
        fh.write(struct.pack("<Q", 1 << 40))
    with pytest.raises(ValueError):
        ckpt.Checkpoint(str(bad))
