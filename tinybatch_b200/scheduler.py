"""Continuous-batching scheduler (host side, unchanged behaviour).

Same policy as the reference ``Scheduler`` (``src/tinybatch/scheduler.py:72-154``):

1. every running sequence decodes one token; its slot is reserved with
   ``append_slot``; when the pool is exhausted the youngest running sequence
   is preempted (recompute policy: its blocks are freed, its output dropped,
   and it goes back to the head of the wait queue) (``:87-111``);
2. waiting requests are admitted first-come-first-served while the token
   budget, ``max_running`` and the free-block count allow (``:114-129``); a
   prompt that is entirely cached still recomputes its last token (``:123-124``).
"""
from __future__ import annotations

import itertools
import time
from dataclasses import dataclass, field
from enum import Enum

from .block_manager import BlockManager, OutOfBlocks
from .config import EngineConfig

_ids = itertools.count()


class Status(Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"


class TokenView:
    """Read-only sequence over ``prompt + outputs`` (optionally its first
    ``limit`` tokens) supporting ``len``, indexing and slicing; what the block
    manager reads of a sequence, without building the whole list every step."""

    __slots__ = ("_p", "_o", "_n")

    def __init__(self, prompt: list[int], outputs: list[int], limit: int | None = None):
        self._p, self._o = prompt, outputs
        total = len(prompt) + len(outputs)
        self._n = total if limit is None else max(0, min(limit, total))

    def __len__(self) -> int:
        return self._n

    def __getitem__(self, k):
        if isinstance(k, slice):
            a, b, step = k.indices(self._n)
            if step != 1:
                return list(self)[k]
            np_ = len(self._p)
            if b <= np_:
                return self._p[a:b]
            if a >= np_:
                return self._o[a - np_:b - np_]
            return self._p[a:] + self._o[:b - np_]
        if k < 0:
            k += self._n
        if not 0 <= k < self._n:
            raise IndexError(k)
        np_ = len(self._p)
        return self._p[k] if k < np_ else self._o[k - np_]

    def __iter__(self):
        return iter(self[0:self._n])


@dataclass
class Request:
    prompt_token_ids: list[int]
    max_new_tokens: int
    temperature: float = 0.0
    top_p: float = 1.0
    req_id: int = field(default_factory=lambda: next(_ids))
    arrival_time: float = field(default_factory=time.perf_counter)

    status: Status = Status.WAITING
    output_token_ids: list[int] = field(default_factory=list)
    block_table: list[int] = field(default_factory=list)
    num_cached_tokens: int = 0
    first_token_time: float | None = None
    finish_time: float | None = None
    preemptions: int = 0

    def all_token_ids(self) -> list[int]:
        return self.prompt_token_ids + self.output_token_ids

    def token_view(self, limit: int | None = None) -> "TokenView":
        """``all_token_ids()[:limit]`` as a read-only view (no copy of the
        whole sequence; slices are built on demand)."""
        return TokenView(self.prompt_token_ids, self.output_token_ids, limit)

    def context_len(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    def last_token_id(self) -> int:
        """``all_token_ids()[-1]`` without building the list."""
        return self.output_token_ids[-1] if self.output_token_ids else self.prompt_token_ids[-1]


@dataclass
class ScheduledBatch:
    prefill: list[Request]
    decode: list[Request]

    def is_empty(self) -> bool:
        return not (self.prefill or self.decode)


class Scheduler:
    def __init__(self, config: EngineConfig, block_manager: BlockManager):
        self.cfg = config
        self.bm = block_manager
        self.waiting: list[Request] = []
        self.running: list[Request] = []

    def add(self, req: Request) -> None:
        self.waiting.append(req)

    def has_work(self) -> bool:
        return bool(self.waiting) or bool(self.running)

    def _reserve_decode_slot(self, req: Request) -> bool:
        """Reserve one KV slot for ``req``; False if ``req`` got preempted."""
        try:
            self.bm.append_slot(req.block_table, req.token_view())
            return True
        except OutOfBlocks:
            pass
        if self._preempt_youngest() is req:
            return False
        try:
            self.bm.append_slot(req.block_table, req.token_view())
            return True
        except OutOfBlocks:
            self._preempt(req)
            return False

    def schedule(self) -> ScheduledBatch:
        budget = self.cfg.max_batch_tokens
        decode: list[Request] = []
        for req in list(self.running):
            if req.status is not Status.RUNNING:
                continue
            if self._reserve_decode_slot(req):
                decode.append(req)
                budget -= 1
        # a later preemption may have hit a request already listed
        decode = [r for r in decode if r.status is Status.RUNNING]

        prefill: list[Request] = []
        while self.waiting and len(self.running) < self.cfg.max_running:
            req = self.waiting[0]
            n = len(req.prompt_token_ids)
            if n > budget or self.bm.blocks_needed(n) > self.bm.num_free():
                break
            self.waiting.pop(0)
            req.block_table, req.num_cached_tokens = self.bm.allocate_prompt(req.prompt_token_ids)
            req.num_cached_tokens = min(req.num_cached_tokens, n - 1)
            req.status = Status.RUNNING
            self.running.append(req)
            prefill.append(req)
            budget -= n - req.num_cached_tokens
        return ScheduledBatch(prefill=prefill, decode=decode)

    def finish(self, req: Request) -> None:
        req.status = Status.FINISHED
        req.finish_time = time.perf_counter()
        self.running.remove(req)
        self.bm.free_table(req.block_table)
        req.block_table = []

    def _preempt(self, req: Request) -> None:
        req.preemptions += 1
        req.status = Status.WAITING
        self.running.remove(req)
        self.bm.free_table(req.block_table)
        req.block_table = []
        req.output_token_ids = []
        req.num_cached_tokens = 0
        self.waiting.insert(0, req)

    def _preempt_youngest(self) -> Request:
        victim = self.running[-1]
        self._preempt(victim)
        return victim
