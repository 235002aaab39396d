"""fp32 CPU restatement of the reference Qwen2 forward (test infrastructure).

Every function computes in float32 on the CPU whatever dtype its inputs come
in, which is the precision the reference's own tests and parity checks use
(``tests/test_tensor_parallel.py:57-65``, ``tests/test_correctness.py:32-54``).

Configuration objects are duck-typed: anything with the attributes of the
reference ``ModelConfig`` (``src/tinybatch/model.py:32-44``) works.
Weight dicts use the HF Qwen2 key names the reference uses.
"""
from __future__ import annotations

import math

import torch


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(device="cpu", dtype=torch.float32)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm in fp32: x * rsqrt(mean(x^2) + eps) * w.

    Follows ``src/tinybatch/model.py:65-69`` (weight applied in fp32 before
    any cast)."""
    x = _f32(x)
    inv = torch.rsqrt(x.square().mean(dim=-1, keepdim=True) + eps)
    return x * inv * _f32(weight)


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float):
    """cos/sin of pos * theta^(-2i/hd), i < hd/2, in fp32.

    Follows ``src/tinybatch/model.py:75-77``: the inverse frequencies are
    ``1 / theta ** (arange(0, hd, 2) / hd)`` and the angle is the fp32 product
    of position and inverse frequency."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    ang = positions.to(torch.float32)[:, None] * inv_freq[None, :]
    return ang.cos(), ang.sin()


def rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """NeoX half-split rotary embedding on ``x [T, heads, hd]``.

    Follows ``src/tinybatch/model.py:72-80``: with ``x = [x1 | x2]`` split at
    hd/2, the result is ``[x1*cos - x2*sin | x2*cos + x1*sin]``."""
    x = _f32(x)
    hd = x.shape[-1]
    cos, sin = rope_tables(positions, hd, theta)
    cos, sin = cos[:, None, :], sin[:, None, :]
    lo, hi = x[..., : hd // 2], x[..., hd // 2:]
    return torch.cat((lo * cos - hi * sin, hi * cos + lo * sin), dim=-1)


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T (+ b)`` in fp32, w in F.linear layout ``[out, in]``."""
    y = _f32(x) @ _f32(w).t()
    if b is not None:
        y = y + _f32(b)
    return y


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, first_pos: int,
              round_p: bool = False) -> torch.Tensor:
    """Causal GQA attention for one sequence.

    q ``[q_len, H, hd]``; k, v ``[ctx, KV, hd]``; query i (absolute position
    ``first_pos + i``) sees keys ``0 .. first_pos + i``.  Query head h uses
    kv head ``h // (H // KV)`` (``repeat_interleave`` in
    ``src/tinybatch/model.py:136-137``).  Scale ``1/sqrt(hd)``; the masks of
    ``src/tinybatch/model.py:139-146`` (``is_causal`` when q_len == ctx, else
    ``mask[i, :first_pos+i+1]``) are both this rule.

    ``round_p`` models a kernel that multiplies bf16 probabilities with V:
    ``exp(s - rowmax)`` is rounded to bf16 before the PV product while the
    normaliser sums the unrounded values."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    q_len, H, hd = q.shape
    ctx, KV, _ = k.shape
    rep = H // KV
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd)
    allowed = torch.arange(ctx)[None, :] <= (first_pos + torch.arange(q_len))[:, None]
    s = s.masked_fill(~allowed[None], float("-inf"))
    if not round_p:
        p = torch.softmax(s, dim=-1)
        return torch.einsum("hqk,khd->qhd", p, v)
    e = torch.exp(s - s.amax(dim=-1, keepdim=True))
    return torch.einsum("hqk,khd->qhd", _bf16(e), v) / e.sum(dim=-1).transpose(0, 1)[..., None]


# ----------------------------------------------------------------- paged KV

def new_pools(n_layers: int, num_blocks: int, block_size: int, n_kv: int, hd: int):
    """One zeroed fp32 pool per layer, ``[num_blocks, 2, n_kv, block_size, hd]``
    (``src/tinybatch/kv_cache.py:13-19``; K at index 0, V at 1)."""
    return [torch.zeros(num_blocks, 2, n_kv, block_size, hd) for _ in range(n_layers)]


def kv_write(pool, k, v, positions, seq_slices, block_tables, block_size: int) -> None:
    """Scatter: token at position p of a sequence goes to block
    ``table[p // bs]``, slot ``p % bs`` (``src/tinybatch/kv_cache.py:25-38``)."""
    for (s, e), table in zip(seq_slices, block_tables):
        for t in range(s, e):
            p = int(positions[t])
            blk, slot = table[p // block_size], p % block_size
            pool[blk, 0, :, slot] = _f32(k[t])
            pool[blk, 1, :, slot] = _f32(v[t])


def kv_gather(pool, table, ctx_len: int):
    """Contiguous ``[ctx, KV, hd]`` K and V of one sequence
    (``src/tinybatch/kv_cache.py:40-45``)."""
    blocks = pool[torch.tensor(table, dtype=torch.long)]        # [nb, 2, KV, bs, hd]
    kv = blocks.permute(1, 0, 3, 2, 4).reshape(2, -1, blocks.shape[2], blocks.shape[4])
    return kv[0, :ctx_len], kv[1, :ctx_len]


def slot_mapping(positions, seq_slices, block_tables, block_size: int) -> list[int]:
    """Flat pool slot ``block*bs + p%bs`` of every token (the index
    arithmetic of ``src/tinybatch/kv_cache.py:34-36``)."""
    out = [0] * len(positions)
    for (s, e), table in zip(seq_slices, block_tables):
        for t in range(s, e):
            p = int(positions[t])
            out[t] = table[p // block_size] * block_size + p % block_size
    return out


# ------------------------------------------------------------ full forwards

def _layer_qkv(cfg, w, p, x, n_heads, n_kv):
    q = linear(x, w[p + "self_attn.q_proj.weight"], w.get(p + "self_attn.q_proj.bias"))
    k = linear(x, w[p + "self_attn.k_proj.weight"], w.get(p + "self_attn.k_proj.bias"))
    v = linear(x, w[p + "self_attn.v_proj.weight"], w.get(p + "self_attn.v_proj.bias"))
    T = x.shape[0]
    return (q.view(T, n_heads, cfg.head_dim), k.view(T, n_kv, cfg.head_dim),
            v.view(T, n_kv, cfg.head_dim))


def _mlp(w, p, x):
    gate = linear(x, w[p + "mlp.gate_proj.weight"])
    up = linear(x, w[p + "mlp.up_proj.weight"])
    return torch.nn.functional.silu(gate) * up


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


# Tensors a bf16-storage forward rounds, by name:
#   gemm_in  the normed GEMM inputs bf16(h * g) of q/k/v and gate/up
#   head_in  the normed input of the LM head
#   q, kv    the rotated queries, and the keys/values stored in the pool
#   p        attention probabilities entering the PV product
#   attn     the attention output (o_proj input)
#   act      the SwiGLU output (down_proj input)
BF16_TENSORS = frozenset({"gemm_in", "head_in", "q", "kv", "p", "attn", "act"})
# ``emulate_bf16=True``: the stored activations (every name but ``p``)
BF16_STORED = frozenset(BF16_TENSORS - {"p"})


def _emu_set(emulate) -> frozenset:
    """``emulate_bf16`` argument -> set of tensor names to round."""
    if emulate is True:
        return BF16_STORED
    if not emulate:
        return frozenset()
    names = frozenset(emulate)
    unknown = names - BF16_TENSORS
    if unknown:
        raise ValueError(f"unknown bf16 tensors {sorted(unknown)}")
    return names


def _normed_linear(h, g, wt, b, eps, emulate):
    """``linear(rms_norm(h, g), wt, b)``.  With ``emulate`` the norm is
    applied the way the GPU path does it: the GEMM reads bf16(h * g) and its
    rows are scaled by rsqrt(mean(h^2) + eps) afterwards (same value in exact
    arithmetic, bf16 rounding at the GEMM input)."""
    if not emulate:
        return linear(rms_norm(h, g, eps), wt, b)
    h = _f32(h)
    s = torch.rsqrt(h.square().mean(dim=-1, keepdim=True) + eps)
    y = linear(_bf16(h * _f32(g)), wt) * s
    return y if b is None else y + _f32(b)


def paged_layer(cfg, w, layer: int, h, positions, seq_slices, block_tables, context_lens,
                pool, block_size: int, emulate_bf16=False):
    """One decoder layer of ``Qwen2Paged.forward`` (``src/tinybatch/model.py:114-154``):
    norm -> q/k/v (+bias) -> RoPE -> KV scatter -> per-sequence attention over
    the paged context -> o_proj + residual -> norm -> SwiGLU MLP + residual.

    ``emulate_bf16`` rounds to bf16 where a bf16-storage GPU forward does
    (``True``: every stored activation; or a set of ``BF16_TENSORS`` names)
    while keeping every sum in fp32 -- a model of a correct bf16 forward used
    to bound the kernels' own error and to attribute it to single tensors."""
    emu = _emu_set(emulate_bf16)
    p = f"model.layers.{layer}."
    T = h.shape[0]
    g_in = w[p + "input_layernorm.weight"]
    n_heads, n_kv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    gin = "gemm_in" in emu
    q = _normed_linear(h, g_in, w[p + "self_attn.q_proj.weight"],
                       w.get(p + "self_attn.q_proj.bias"), cfg.rms_eps, gin)
    k = _normed_linear(h, g_in, w[p + "self_attn.k_proj.weight"],
                       w.get(p + "self_attn.k_proj.bias"), cfg.rms_eps, gin)
    v = _normed_linear(h, g_in, w[p + "self_attn.v_proj.weight"],
                       w.get(p + "self_attn.v_proj.bias"), cfg.rms_eps, gin)
    q = rope(q.view(T, n_heads, hd), positions, cfg.rope_theta)
    k = rope(k.view(T, n_kv, hd), positions, cfg.rope_theta)
    v = v.view(T, n_kv, hd)
    if "q" in emu:
        q = _bf16(q)
    if "kv" in emu:
        k, v = _bf16(k), _bf16(v)
    kv_write(pool, k, v, positions, seq_slices, block_tables, block_size)
    attn = torch.empty(T, n_heads * hd)
    for (s, e), table, ctx in zip(seq_slices, block_tables, context_lens):
        keys, vals = kv_gather(pool, table, ctx)
        out = attention(q[s:e], keys, vals, first_pos=ctx - (e - s), round_p="p" in emu)
        attn[s:e] = out.reshape(e - s, -1)
    if "attn" in emu:
        attn = _bf16(attn)
    h = h + linear(attn, w[p + "self_attn.o_proj.weight"])
    g_post = w[p + "post_attention_layernorm.weight"]
    gate = _normed_linear(h, g_post, w[p + "mlp.gate_proj.weight"], None, cfg.rms_eps, gin)
    up = _normed_linear(h, g_post, w[p + "mlp.up_proj.weight"], None, cfg.rms_eps, gin)
    act = torch.nn.functional.silu(gate) * up
    if "act" in emu:
        act = _bf16(act)
    return h + linear(act, w[p + "mlp.down_proj.weight"])


def embed(w, token_ids):
    """Row gather of the embedding table (``src/tinybatch/model.py:112``)."""
    return _f32(w["model.embed_tokens.weight"])[torch.as_tensor(token_ids, dtype=torch.long)]


def lm_head_weight(cfg, w):
    """The tied head aliases the embedding (``src/tinybatch/model.py:97-98``)."""
    if "lm_head.weight" in w:
        return w["lm_head.weight"]
    return w["model.embed_tokens.weight"]


@torch.inference_mode()
def paged_forward(cfg, w, token_ids, positions, seq_slices, block_tables, context_lens,
                  pools, block_size: int, emulate_bf16=False) -> torch.Tensor:
    """``Qwen2Paged.forward`` (``src/tinybatch/model.py:100-158``): logits of the
    last token of every sequence, ``[n_seqs, vocab]`` fp32.  ``pools`` are
    updated in place, like the reference's ``PagedKVCache``.  See
    ``paged_layer`` for ``emulate_bf16``."""
    positions = torch.as_tensor(positions, dtype=torch.long)
    h = embed(w, token_ids)
    for layer in range(cfg.n_layers):
        h = paged_layer(cfg, w, layer, h, positions, seq_slices, block_tables, context_lens,
                        pools[layer], block_size, emulate_bf16)
    last = torch.tensor([e - 1 for _, e in seq_slices], dtype=torch.long)
    return _normed_linear(h[last], w["model.norm.weight"], lm_head_weight(cfg, w), None,
                          cfg.rms_eps, "head_in" in _emu_set(emulate_bf16))


def shard(w: dict, rank: int, world: int) -> dict:
    """Megatron split of ``src/tinybatch/tensor_parallel.py:45-60``: q/k/v
    weight+bias and gate/up split along dim 0, o/down along dim 1, the rest
    replicated."""
    col = ("q_proj.weight", "k_proj.weight", "v_proj.weight", "q_proj.bias",
           "k_proj.bias", "v_proj.bias", "gate_proj.weight", "up_proj.weight")
    row = ("o_proj.weight", "down_proj.weight")
    out = {}
    for k, v in w.items():
        if k.endswith(col):
            out[k] = v.chunk(world, dim=0)[rank].contiguous()
        elif k.endswith(row):
            out[k] = v.chunk(world, dim=1)[rank].contiguous()
        else:
            out[k] = v
    return out


@torch.inference_mode()
def tp_forward(cfg, w, token_ids, world: int = 1) -> torch.Tensor:
    """Cache-free causal prefill of ``tp_forward`` (``src/tinybatch/tensor_parallel.py:64-117``)
    with ``world`` ranks emulated in one process: every rank's row-parallel
    partial is computed from its own shard and the partials are summed in
    rank order (the all-reduce of ``:76-84``).  Returns ``[T, vocab]`` fp32."""
    shards = [shard(w, r, world) for r in range(world)]
    n_heads, n_kv = cfg.n_heads // world, cfg.n_kv_heads // world
    T = len(token_ids)
    positions = torch.arange(T)
    h = embed(w, token_ids)
    for layer in range(cfg.n_layers):
        p = f"model.layers.{layer}."
        x = rms_norm(h, w[p + "input_layernorm.weight"], cfg.rms_eps)
        part = torch.zeros_like(h)
        for sw in shards:
            q, k, v = _layer_qkv(cfg, sw, p, x, n_heads, n_kv)
            q = rope(q, positions, cfg.rope_theta)
            k = rope(k, positions, cfg.rope_theta)
            a = attention(q, k, v, first_pos=0).reshape(T, -1)
            part = part + linear(a, sw[p + "self_attn.o_proj.weight"])
        h = h + part
        x = rms_norm(h, w[p + "post_attention_layernorm.weight"], cfg.rms_eps)
        part = torch.zeros_like(h)
        for sw in shards:
            part = part + linear(_mlp(sw, p, x), sw[p + "mlp.down_proj.weight"])
        h = h + part
    h = rms_norm(h, w["model.norm.weight"], cfg.rms_eps)
    return linear(h, lm_head_weight(cfg, w))


# --------------------------------------------------- op-level (sweep config)

def row_gemm_allreduce_norm(x_shards, w_shards, residual, norm_w, eps: float):
    """The row-parallel block of ``src/tinybatch/tensor_parallel.py:108-110``
    in isolation: ``h = residual + sum_r x_r @ W_r`` (all-reduce SUM in rank
    order) then ``x = rms_norm(h)``.  ``w_shards[r]`` is in ``[K/t, N]``
    (the sweep's ``Y = X W`` orientation).  Returns (h, x) in fp32."""
    acc = None
    for xr, wr in zip(x_shards, w_shards):
        y = _f32(xr) @ _f32(wr)
        acc = y if acc is None else acc + y
    h = _f32(residual) + acc
    return h, rms_norm(h, norm_w, eps)
