"""Paged KV storage on the GPU.

Same layout and attributes as the reference ``PagedKVCache``
(``src/tinybatch/kv_cache.py:13-45``): one pool per layer shaped
``[num_blocks, 2, n_kv_heads, block_size, head_dim]`` (K at index 0, V at 1);
token position ``p`` of a sequence lives in block ``table[p // block_size]``,
slot ``p % block_size``.  Under tensor parallelism each rank builds its cache
with ``n_kv_heads / tp`` heads.

On the hot path nothing here runs: the fused QKV kernel writes K/V straight
into the pools and the attention kernel reads them through the block tables.
``write`` and ``gather`` keep the reference's methods for callers and tests;
they are plain device tensor indexing.
"""
from __future__ import annotations

import torch


class PagedKVCache:
    def __init__(self, n_layers: int, num_blocks: int, block_size: int, n_kv_heads: int,
                 head_dim: int, device: torch.device | str = "cuda",
                 dtype: torch.dtype = torch.bfloat16):
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.pools = [torch.zeros(num_blocks, 2, n_kv_heads, block_size, head_dim,
                                  device=device, dtype=dtype) for _ in range(n_layers)]

    def memory_bytes(self) -> int:
        return sum(p.numel() * p.element_size() for p in self.pools)

    def write(self, layer: int, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
              seq_slices: list[tuple[int, int]], block_tables: list[list[int]]) -> None:
        """Scatter ``k, v [n_tokens, n_kv_heads, head_dim]`` of a flat batch."""
        pool = self.pools[layer]
        pos = positions.to(pool.device, torch.long)
        for (s, e), table in zip(seq_slices, block_tables):
            tbl = torch.tensor(table, device=pool.device, dtype=torch.long)
            p = pos[s:e]
            blocks, slots = tbl[p // self.block_size], p % self.block_size
            pool[blocks, 0, :, slots] = k[s:e].to(pool.dtype)
            pool[blocks, 1, :, slots] = v[s:e].to(pool.dtype)

    def gather(self, layer: int, table: list[int], context_len: int):
        """Contiguous ``[context_len, n_kv_heads, head_dim]`` K and V of one sequence."""
        pool = self.pools[layer]
        blocks = pool[torch.tensor(table, device=pool.device, dtype=torch.long)]
        kv = blocks.permute(1, 0, 3, 2, 4).reshape(2, -1, blocks.shape[2], blocks.shape[4])
        return kv[0, :context_len], kv[1, :context_len]
