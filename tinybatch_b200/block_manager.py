"""Paged KV block bookkeeping (host side, unchanged behaviour).

The GPU path only consumes the block tables this class produces, so its
behaviour must be exactly the reference's ``BlockManager``
(``src/tinybatch/block_manager.py:43-175``): identical token streams must give
bit-identical tables, cached-token counts, free counts and hit statistics.
The rules, restated:

* ids are handed out from a free stack that starts as ``0..n-1`` and pops
  from the top (highest id first, ``:70``); freed unshared blocks are pushed
  back on top (``:170``);
* a full block is keyed by ``hash(tuple(tokens[0 : end of block]))``
  (``:38-40``); a prompt reuses cached blocks block by block until the first
  miss, after which nothing more can match (``:94-108``);
* cached blocks whose reference count drops to zero stay cached and become
  evictable in LRU order; a new block comes from the free stack first and
  only then by evicting the least recently released cached block (``:69-80``);
* ``append_slot`` is called before the new token is appended; crossing a
  block boundary takes a new block and publishes the block that just filled
  (``:127-145``), unless it is shared or its prefix is already cached
  (``:147-156``).

Nothing here touches the GPU.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field


class OutOfBlocks(Exception):
    """The pool cannot supply a block, even after evicting cached ones."""


@dataclass
class Block:
    block_id: int
    ref_count: int = 0
    prefix_hash: int | None = None          # set once the block is full and cached
    token_ids: list[int] = field(default_factory=list)


def hash_prefix(token_ids: list[int]) -> int:
    """Key of a full block: the hash of the whole prefix up to its end."""
    return hash(tuple(token_ids))


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, enable_prefix_caching: bool = True):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.enable_prefix_caching = enable_prefix_caching
        self.blocks: list[Block] = [Block(i) for i in range(num_blocks)]
        self.free_ids: list[int] = list(range(num_blocks))      # stack, top = end
        self.cache: dict[int, int] = {}                         # prefix hash -> block id
        self.evictable: OrderedDict[int, None] = OrderedDict()  # rc == 0 cached, LRU first
        self.prefix_hits = 0
        self.prefix_queries = 0

    # ------------------------------------------------------------ queries

    def num_free(self) -> int:
        return len(self.free_ids) + len(self.evictable)

    def blocks_needed(self, num_tokens: int) -> int:
        return -(-num_tokens // self.block_size)

    def hit_rate(self) -> float:
        return self.prefix_hits / self.prefix_queries if self.prefix_queries else 0.0

    # --------------------------------------------------------- allocation

    def _fresh_block(self) -> Block:
        """Top of the free stack, else the least recently released cached block."""
        if self.free_ids:
            return self.blocks[self.free_ids.pop()]
        if not self.evictable:
            raise OutOfBlocks(f"KV pool exhausted ({self.num_blocks} blocks)")
        bid, _ = self.evictable.popitem(last=False)
        blk = self.blocks[bid]
        if blk.prefix_hash is not None:
            self.cache.pop(blk.prefix_hash, None)
        blk.prefix_hash = None
        blk.token_ids = []
        return blk

    def _own(self, blk: Block, tokens: list[int]) -> Block:
        blk.ref_count = 1
        blk.token_ids = tokens
        return blk

    def allocate_prompt(self, token_ids: list[int]) -> tuple[list[int], int]:
        """Block table for a prompt, and how many leading tokens are already
        in the cache (whole blocks only)."""
        bs = self.block_size
        table: list[int] = []
        cached = 0
        still_matching = self.enable_prefix_caching
        for b in range(len(token_ids) // bs):
            end = (b + 1) * bs
            self.prefix_queries += 1
            key = hash_prefix(token_ids[:end])
            hit = self.cache.get(key) if still_matching else None
            if hit is None:
                still_matching = False
                blk = self._own(self._fresh_block(), token_ids[end - bs:end])
                if self.enable_prefix_caching:
                    blk.prefix_hash = key
                    self.cache[key] = blk.block_id
                table.append(blk.block_id)
                continue
            self.blocks[hit].ref_count += 1
            self.evictable.pop(hit, None)
            table.append(hit)
            cached += bs
            self.prefix_hits += 1
        tail = len(token_ids) % bs
        if tail:
            blk = self._own(self._fresh_block(), token_ids[len(token_ids) - tail:])
            table.append(blk.block_id)
        return table, cached

    def append_slot(self, table: list[int], seq_token_ids: list[int]) -> bool:
        """Make room for the token about to be appended at index
        ``len(seq_token_ids)``; True when a new block was added."""
        pos = len(seq_token_ids)
        bs = self.block_size
        if pos % bs:
            self.blocks[table[-1]].token_ids = seq_token_ids[(len(table) - 1) * bs:pos]
            return False
        blk = self._own(self._fresh_block(), [])
        table.append(blk.block_id)
        if self.enable_prefix_caching and len(table) >= 2:
            self._publish(table, len(table) - 2, seq_token_ids)
        return True

    def _publish(self, table: list[int], idx: int, seq_token_ids: list[int]) -> None:
        blk = self.blocks[table[idx]]
        if blk.prefix_hash is not None or blk.ref_count != 1:
            return
        end = (idx + 1) * self.block_size
        key = hash_prefix(seq_token_ids[:end])
        if key in self.cache:
            return
        blk.prefix_hash = key
        blk.token_ids = seq_token_ids[end - self.block_size:end]
        self.cache[key] = blk.block_id

    # ------------------------------------------------------------ release

    def free_table(self, table: list[int]) -> None:
        for bid in table:
            blk = self.blocks[bid]
            blk.ref_count -= 1
            assert blk.ref_count >= 0, "double free"
            if blk.ref_count:
                continue
            if blk.prefix_hash is None:
                blk.token_ids = []
                self.free_ids.append(bid)
            else:
                self.evictable[bid] = None
