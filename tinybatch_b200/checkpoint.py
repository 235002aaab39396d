"""Per-rank loading of a HuggingFace Qwen2 checkpoint (``config.json`` +
``*.safetensors``).

The reference loads every shard file whole into host memory and casts it
(``src/tinybatch/model.py:86-98``); a tensor-parallel rank then slices its
share (``src/tinybatch/tensor_parallel.py:35-61``).  Here each rank reads only
its own slice of every tensor from the memory-mapped files -- rows of the
column-parallel q/k/v weights and biases and gate/up weights, columns of the
row-parallel o/down weights, the replicated rest whole -- and moves it to its
GPU in the model dtype, one tensor at a time, so host memory never holds more
than one slice and a 72B checkpoint needs no host copy of the whole model.
"""
from __future__ import annotations

import glob
import json
import os

import torch

from .config import ModelConfig
from .tensor_parallel import COL_SUFFIXES, ROW_SUFFIXES


def resolve(model_id: str) -> str:
    """Local directory of a checkpoint: ``model_id`` itself, else the hub cache."""
    if os.path.isdir(model_id):
        return model_id
    from huggingface_hub import snapshot_download
    return snapshot_download(model_id, allow_patterns=["*.json", "*.safetensors"])


def load_config(path: str) -> ModelConfig:
    with open(os.path.join(path, "config.json")) as f:
        return ModelConfig.from_hf(json.load(f))


def split_of(name: str) -> int | None:
    """Dimension a tensor is split along across ranks (0 column-parallel, 1
    row-parallel), None when replicated -- the rule of ``shard_weights``."""
    if name.endswith(COL_SUFFIXES):
        return 0
    if name.endswith(ROW_SUFFIXES):
        return 1
    return None


def load_rank_weights(path: str, cfg: ModelConfig, rank: int = 0, world: int = 1,
                      device: torch.device | str = "cpu",
                      dtype: torch.dtype = torch.bfloat16) -> dict[str, torch.Tensor]:
    """This rank's weight dict, equal to ``shard_weights(full, cfg, rank,
    world)`` of the whole checkpoint cast to ``dtype``, read slice by slice.
    Raises ``AssertionError`` when heads, kv heads or d_ff do not divide the
    degree (as ``shard_weights``) and ``ValueError`` when a split dimension
    does not divide."""
    from safetensors import safe_open
    assert cfg.n_heads % world == 0, "q heads must divide tp degree"
    assert cfg.n_kv_heads % world == 0, "kv heads must divide tp degree"
    assert cfg.d_ff % world == 0, "d_ff must divide tp degree"
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no *.safetensors files under {path}")
    out: dict[str, torch.Tensor] = {}
    for fn in files:
        with safe_open(fn, framework="pt", device="cpu") as f:
            for name in f.keys():
                sl = f.get_slice(name)
                shape = sl.get_shape()
                dim = split_of(name)
                if dim is None or world == 1:
                    t = sl[:]
                else:
                    if shape[dim] % world:
                        raise ValueError(f"{name}: dimension {dim} of {shape} does not divide "
                                         f"by {world}")
                    n = shape[dim] // world
                    t = sl[rank * n:(rank + 1) * n] if dim == 0 else sl[:, rank * n:(rank + 1) * n]
                out[name] = t.to(device=device, dtype=dtype).contiguous()
    if cfg.tie_embeddings and "lm_head.weight" not in out:
        out["lm_head.weight"] = out["model.embed_tokens.weight"]
    return out
