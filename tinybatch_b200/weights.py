"""Seeded synthetic Qwen2 weights.

The benchmarks and parity tests never load a checkpoint: weights are drawn
N(0, std) from ``torch.Generator(device).manual_seed(seed)`` in fp32 (then
cast), q/k/v carry biases and every norm weight is 1.  The draw order is
fixed (below) so the CPU oracle and the GPU path see identical values for the
same seed when both draw on the CPU.
"""
from __future__ import annotations

import torch

from .config import ModelConfig


def weight_shapes(cfg: ModelConfig, bias: bool = True) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, kind) in draw order; kind is "randn" or "ones"."""
    qdim, kvdim = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    out = [("model.embed_tokens.weight", (cfg.vocab_size, cfg.d_model), "randn")]
    if not cfg.tie_embeddings:
        out.append(("lm_head.weight", (cfg.vocab_size, cfg.d_model), "randn"))
    out.append(("model.norm.weight", (cfg.d_model,), "ones"))
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (cfg.d_model,), "ones"),
            (p + "self_attn.q_proj.weight", (qdim, cfg.d_model), "randn"),
        ]
        if bias:
            out.append((p + "self_attn.q_proj.bias", (qdim,), "randn"))
        out.append((p + "self_attn.k_proj.weight", (kvdim, cfg.d_model), "randn"))
        if bias:
            out.append((p + "self_attn.k_proj.bias", (kvdim,), "randn"))
        out.append((p + "self_attn.v_proj.weight", (kvdim, cfg.d_model), "randn"))
        if bias:
            out.append((p + "self_attn.v_proj.bias", (kvdim,), "randn"))
        out += [
            (p + "self_attn.o_proj.weight", (cfg.d_model, qdim), "randn"),
            (p + "post_attention_layernorm.weight", (cfg.d_model,), "ones"),
            (p + "mlp.gate_proj.weight", (cfg.d_ff, cfg.d_model), "randn"),
            (p + "mlp.up_proj.weight", (cfg.d_ff, cfg.d_model), "randn"),
            (p + "mlp.down_proj.weight", (cfg.d_model, cfg.d_ff), "randn"),
        ]
    return out


def synthetic_weights(cfg: ModelConfig, seed: int, std: float = 0.02,
                      dtype: torch.dtype = torch.float32, device: str | torch.device = "cpu",
                      bias: bool = True, layers: range | None = None) -> dict[str, torch.Tensor]:
    """Draw the full weight dict.  With ``layers`` given, only those decoder
    layers (plus embeddings, head and final norm) are kept in the result, but
    the generator still advances over every tensor so the kept values equal
    the full draw's."""
    g = torch.Generator(device=device).manual_seed(seed)
    keep_layer = None if layers is None else set(layers)
    w: dict[str, torch.Tensor] = {}
    for name, shape, kind in weight_shapes(cfg, bias):
        if kind == "ones":
            t = torch.ones(shape, device=device, dtype=dtype)
        else:
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
            t = t.mul_(std).to(dtype)
        if keep_layer is not None and name.startswith("model.layers."):
            if int(name.split(".")[2]) not in keep_layer:
                continue
        w[name] = t
    if cfg.tie_embeddings:
        w["lm_head.weight"] = w["model.embed_tokens.weight"]
    return w


def synthetic_rank_weights(cfg: ModelConfig, seed: int, rank: int, world: int,
                           std: float = 0.02, dtype: torch.dtype = torch.bfloat16,
                           device: str | torch.device = "cpu",
                           bias: bool = True) -> dict[str, torch.Tensor]:
    """One tensor-parallel rank's slice of ``synthetic_weights(cfg, seed)``:
    the same draw, tensor by tensor on ``device``, keeping only the rows
    (column-parallel) or columns (row-parallel) of this rank -- the split of
    ``shard_weights`` -- so no device or host ever holds the whole model.
    Values equal ``shard_weights(synthetic_weights(cfg, seed, device=device),
    cfg, rank, world)`` cast to ``dtype``."""
    from .checkpoint import split_of
    assert cfg.n_heads % world == 0, "q heads must divide tp degree"
    assert cfg.n_kv_heads % world == 0, "kv heads must divide tp degree"
    assert cfg.d_ff % world == 0, "d_ff must divide tp degree"
    g = torch.Generator(device=device).manual_seed(seed)
    w: dict[str, torch.Tensor] = {}
    for name, shape, kind in weight_shapes(cfg, bias):
        if kind == "ones":
            full = torch.ones(shape, device=device, dtype=torch.float32)
        else:
            full = torch.randn(shape, generator=g, device=device, dtype=torch.float32).mul_(std)
        dim = split_of(name)
        if dim is not None and world > 1:
            n = shape[dim] // world
            full = full.narrow(dim, rank * n, n)
        w[name] = full.to(dtype).contiguous()
        del full
    if cfg.tie_embeddings:
        w["lm_head.weight"] = w["model.embed_tokens.weight"]
    return w


def reference_test_weights(cfg: ModelConfig, seed: int = 0) -> dict[str, torch.Tensor]:
    """The reference TP test's draw (``tests/test_tensor_parallel.py:21-45``):
    randn * 0.05, order embed, final norm, lm_head, then per layer
    norms, q, q-bias, k, k-bias, v, v-bias, o, gate, up, down."""
    g = torch.Generator().manual_seed(seed)

    def t(*shape):
        return torch.randn(*shape, generator=g) * 0.05

    w = {"model.embed_tokens.weight": t(cfg.vocab_size, cfg.d_model),
         "model.norm.weight": torch.ones(cfg.d_model),
         "lm_head.weight": t(cfg.vocab_size, cfg.d_model)}
    qdim, kvdim = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = torch.ones(cfg.d_model)
        w[p + "post_attention_layernorm.weight"] = torch.ones(cfg.d_model)
        for name, shape in (("self_attn.q_proj.weight", (qdim, cfg.d_model)),
                            ("self_attn.q_proj.bias", (qdim,)),
                            ("self_attn.k_proj.weight", (kvdim, cfg.d_model)),
                            ("self_attn.k_proj.bias", (kvdim,)),
                            ("self_attn.v_proj.weight", (kvdim, cfg.d_model)),
                            ("self_attn.v_proj.bias", (kvdim,)),
                            ("self_attn.o_proj.weight", (cfg.d_model, qdim)),
                            ("mlp.gate_proj.weight", (cfg.d_ff, cfg.d_model)),
                            ("mlp.up_proj.weight", (cfg.d_ff, cfg.d_model)),
                            ("mlp.down_proj.weight", (cfg.d_model, cfg.d_ff))):
            w[p + name] = t(*shape)
    return w


def fingerprint(w: dict[str, torch.Tensor]) -> dict[str, float]:
    """Per-tensor float64 sum of |values|: detects a changed draw."""
    return {k: float(v.detach().double().abs().sum()) for k, v in sorted(w.items())}
