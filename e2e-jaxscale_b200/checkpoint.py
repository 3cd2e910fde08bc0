"""HF safetensors checkpoints of GLM-4-9B (utils/weight_utils.py:61-161 with the
mapping of models/glm4.py:277-358) into the reference-layout parameters that
GLM4ForCausalLM.load_state packs per rank.

Mapping (HF [out, in] matrices are transposed to the reference's [in, out]):

    model.embed_tokens.weight                       -> embed       [V, H]
    model.norm.weight                               -> norm        [H]
    lm_head.weight                                  -> lm_head     [V, H]  (not transposed)
    model.layers.i.input_layernorm.weight           -> ln1
    model.layers.i.post_attention_layernorm.weight  -> ln2
    model.layers.i.self_attn.{q,k,v}_proj.weight    -> wq, wk, wv  (transposed)
    model.layers.i.self_attn.{q,k,v}_proj.bias      -> bq, bk, bv
    model.layers.i.self_attn.o_proj.weight          -> wo          (transposed)
    model.layers.i.mlp.gate_up_proj.weight          -> wg, wu      (rows split in two halves, transposed)
    model.layers.i.mlp.down_proj.weight             -> wd          (transposed)

The safetensors container is read directly (an 8-byte little-endian header
length, a JSON header of name -> dtype / shape / byte range, then the raw
little-endian data) through a memory map; a layer's tensors are read only when
the layer is packed, so host memory holds one layer at a time.  BF16, F16 and
F32 tensors are supported.
"""

from __future__ import annotations

import glob
import json
import mmap
import os
import struct

import numpy as np
import torch

_DTYPES = {"BF16": (np.uint16, torch.bfloat16), "F16": (np.float16, torch.float16),
           "F32": (np.float32, torch.float32)}


class SafetensorsFile:
    """Zero-copy view of one .safetensors file."""

    def __init__(self, path: str):
        self.path = path
        self._fh = open(path, "rb")
        self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ)
        (n,) = struct.unpack("<Q", self._mm[:8])
        if n <= 0 or 8 + n > len(self._mm):
            raise ValueError(f"{path}: bad safetensors header length {n}")
        self._header = json.loads(bytes(self._mm[8:8 + n]).decode("utf-8"))
        self._header.pop("__metadata__", None)
        self._base = 8 + n

    def keys(self):
        return self._header.keys()

    def get(self, name: str) -> torch.Tensor:
        """The tensor as a CPU torch tensor of its stored dtype (a copy)."""
        info = self._header[name]
        if info["dtype"] not in _DTYPES:
            raise ValueError(f"{self.path}: {name} has unsupported dtype {info['dtype']}")
        npt, tt = _DTYPES[info["dtype"]]
        b0, b1 = info["data_offsets"]
        shape = tuple(info["shape"])
        count = int(np.prod(shape)) if shape else 1
        if b1 - b0 != count * np.dtype(npt).itemsize:
            raise ValueError(f"{self.path}: {name}: byte range does not match shape {shape}")
        arr = np.frombuffer(self._mm, dtype=npt, count=count, offset=self._base + b0).reshape(shape)
        t = torch.from_numpy(arr.copy())
        return t.view(tt) if tt is torch.bfloat16 else t

    def close(self):
        self._mm.close()
        self._fh.close()


class Checkpoint:
    """Every *.safetensors file of a model directory, indexed by tensor name."""

    def __init__(self, model_path: str):
        files = sorted(glob.glob(os.path.join(model_path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"No .safetensors files found in {model_path}")
        self.files = [SafetensorsFile(f) for f in files]
        self.where = {}
        for f in self.files:
            for k in f.keys():
                self.where[k] = f

    def __contains__(self, name: str) -> bool:
        return name in self.where

    def get(self, name: str) -> torch.Tensor:
        if name not in self.where:
            raise KeyError(f"checkpoint has no tensor {name}")
        return self.where[name].get(name)

    def close(self):
        for f in self.files:
            f.close()


class _Layer:
    """Reference-layout parameters of decoder layer i, read on attribute access."""

    def __init__(self, ck: Checkpoint, i: int, bias: bool):
        self._ck, self._p, self._bias = ck, f"model.layers.{i}", bias
        self._gu = None

    def _t(self, name):
        return self._ck.get(f"{self._p}.{name}").t().contiguous()

    def _gate_up(self, half: int):
        if self._gu is None:
            self._gu = self._ck.get(f"{self._p}.mlp.gate_up_proj.weight")
        n = self._gu.shape[0] // 2
        w = self._gu[half * n:(half + 1) * n].t().contiguous()
        if half == 1:
            self._gu = None
        return w

    def __getattr__(self, name):
        if name.startswith("_"):
            raise AttributeError(name)
        p = self._p
        if name == "ln1":
            return self._ck.get(f"{p}.input_layernorm.weight")
        if name == "ln2":
            return self._ck.get(f"{p}.post_attention_layernorm.weight")
        if name in ("wq", "wk", "wv"):
            return self._t(f"self_attn.{name[1]}_proj.weight")
        if name in ("bq", "bk", "bv"):
            return self._ck.get(f"{p}.self_attn.{name[1]}_proj.bias") if self._bias else None
        if name == "wo":
            return self._t("self_attn.o_proj.weight")
        if name == "wg":
            return self._gate_up(0)
        if name == "wu":
            return self._gate_up(1)
        if name == "wd":
            return self._t("mlp.down_proj.weight")
        raise AttributeError(name)


class GLM4Params:
    """GLM4ForCausalLM.load_state input read lazily from a checkpoint: embed, norm,
    lm_head (the embedding when tie_word_embeddings), layers[i]."""

    def __init__(self, ck: Checkpoint, config):
        self._ck = ck
        self.layers = [_Layer(ck, i, config.attention_bias) for i in range(config.num_hidden_layers)]
        self._tie = config.tie_word_embeddings

    @property
    def embed(self):
        return self._ck.get("model.embed_tokens.weight")

    @property
    def norm(self):
        return self._ck.get("model.norm.weight")

    @property
    def lm_head(self):
        if self._tie or "lm_head.weight" not in self._ck:
            return self._ck.get("model.embed_tokens.weight")
        return self._ck.get("lm_head.weight")


def load_glm4(model, model_path: str | None = None) -> None:
    """Load a GLM-4 safetensors checkpoint into a GLM4ForCausalLM (models/glm4.py:262-274):
    this rank's shards are packed layer by layer from the memory-mapped files."""
    path = model_path or model.config.model_path
    ck = Checkpoint(path)
    try:
        model.load_state(GLM4Params(ck, model.config))
    finally:
        ck.close()
