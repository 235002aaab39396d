"""Continuous-batching engine over the B200 forward.

Same loop as the reference ``LLMEngine.step`` (``src/tinybatch/engine.py:94-143``):
schedule -> one flat batch (prefill suffixes first, then one token per
decoding sequence) -> forward -> sample -> append / finish.  Differences:

* the flat batch goes to the device as int32 metadata built with numpy
  (one pinned host->device copy per step) instead of per-sequence Python
  tensors;
* greedy sampling runs as an argmax kernel on the device and only the chosen
  token ids come back (4 bytes per sequence);
* requests can be given as token ids (``add_request_ids``); a tokenizer is
  only needed for text prompts;
* a prompt whose length is a multiple of the block size gets the block for
  its first decode token here.  The reference scheduler reserves the slot
  *after* the token being written (``append_slot`` sees the token list that
  already includes it), so such a prompt has no block for position
  ``len(prompt)`` and the reference's ``PagedKVCache.write`` indexes past the
  table.  The added block is taken through the unchanged ``BlockManager``
  (``append_slot`` on the list without the new token), so every table the
  reference can produce is produced identically.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .block_manager import BlockManager
from .config import EngineConfig
from .kv_cache import PagedKVCache
from .model import Qwen2Paged
from .runtime import DecodeGraph, StepMeta
from .scheduler import Request, Scheduler


@dataclass
class StepOutput:
    req_id: int
    token_id: int
    text_delta: str
    finished: bool
    request: Request = field(repr=False)


class LLMEngine:
    def __init__(self, config: EngineConfig | None = None, model: Qwen2Paged | None = None,
                 tokenizer=None, cuda_graphs: bool = True):
        self.cfg = config or EngineConfig()
        # decode-only greedy steps replay a CUDA graph captured per batch size
        self.cuda_graphs = cuda_graphs
        self._graphs: dict[int, DecodeGraph] = {}
        self._bt_width = -(-self.cfg.max_model_len // self.cfg.block_size) + 1
        self.device = torch.device(self.cfg.device)
        if model is None:
            model = Qwen2Paged(self.cfg.model_id, self.device, torch.bfloat16)
        self.model = model
        self.tokenizer = tokenizer
        if tokenizer is None and isinstance(self.cfg.model_id, str) and model is None:
            from transformers import AutoTokenizer
            self.tokenizer = AutoTokenizer.from_pretrained(self.cfg.model_id)
        self.kv_cache: PagedKVCache = model.make_kv_cache(self.cfg.num_blocks, self.cfg.block_size)
        self.block_manager = BlockManager(self.cfg.num_blocks, self.cfg.block_size,
                                          self.cfg.enable_prefix_caching)
        self.scheduler = Scheduler(self.cfg, self.block_manager)
        self.eos_ids = set(self.cfg.stop_token_ids)
        if self.tokenizer is not None:
            if self.tokenizer.eos_token_id is not None:
                self.eos_ids.add(self.tokenizer.eos_token_id)
            im_end = self.tokenizer.convert_tokens_to_ids("<|im_end|>")
            if im_end is not None:
                self.eos_ids.add(im_end)
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0

    # ------------------------------------------------------------- API

    def add_request_ids(self, ids: list[int], max_new_tokens: int | None = None,
                        temperature: float | None = None, top_p: float | None = None) -> Request:
        ids = list(ids)[: self.cfg.max_model_len - 1]
        req = Request(
            prompt_token_ids=ids,
            max_new_tokens=self.cfg.max_new_tokens if max_new_tokens is None else max_new_tokens,
            temperature=self.cfg.temperature if temperature is None else temperature,
            top_p=self.cfg.top_p if top_p is None else top_p,
        )
        self.scheduler.add(req)
        return req

    def add_request(self, prompt: str, *, chat: bool = True, max_new_tokens: int | None = None,
                    temperature: float | None = None, top_p: float | None = None) -> Request:
        if self.tokenizer is None:
            raise RuntimeError("text prompts need a tokenizer; use add_request_ids")
        if chat:
            ids = self.tokenizer.apply_chat_template([{"role": "user", "content": prompt}],
                                                     add_generation_prompt=True)
            if hasattr(ids, "keys"):
                ids = ids["input_ids"]
            if ids and isinstance(ids[0], list):
                ids = ids[0]
        else:
            ids = self.tokenizer.encode(prompt)
        return self.add_request_ids(ids, max_new_tokens, temperature, top_p)

    def generate(self, prompts: list, **kw) -> list:
        reqs = [self.add_request_ids(p, **kw) if isinstance(p, (list, tuple))
                else self.add_request(p, **kw) for p in prompts]
        while self.scheduler.has_work():
            self.step()
        if self.tokenizer is None:
            return [list(r.output_token_ids) for r in reqs]
        return [self.tokenizer.decode(r.output_token_ids, skip_special_tokens=True) for r in reqs]

    # ------------------------------------------------------------ step

    @staticmethod
    def _table(req) -> np.ndarray:
        """The request's block table as an int32 array, converted again only
        when the list changed (decode steps append a block every block_size
        tokens; preemption replaces the list)."""
        t = req.block_table
        cached = getattr(req, "_table_np", None)
        # the cache holds the list itself: tables only grow in place or are
        # replaced by a new list, so (same object, same length) means same content
        if cached is None or cached[0] is not t or cached[1] != len(t):
            cached = (t, len(t), np.asarray(t, dtype=np.int32))
            req._table_np = cached
        return cached[2]

    def build_batch(self, batch):
        bs = self.cfg.block_size
        ids: list[int] = []
        pos: list[int] = []
        slices: list[tuple[int, int]] = []
        tables: list[list[int]] = []
        ctx: list[int] = []
        for req in batch.prefill:
            s = len(ids)
            ids.extend(req.prompt_token_ids[req.num_cached_tokens:])
            pos.extend(range(req.num_cached_tokens, len(req.prompt_token_ids)))
            slices.append((s, len(ids)))
            tables.append(req.block_table)
            ctx.append(len(req.prompt_token_ids))
        for req in batch.decode:
            n = req.context_len()
            if len(req.block_table) * bs < n:
                self.block_manager.append_slot(req.block_table, req.token_view(n - 1))
            s = len(ids)
            ids.append(req.last_token_id())
            pos.append(n - 1)
            slices.append((s, s + 1))
            tables.append(self._table(req))
            ctx.append(n)
        return ids, pos, slices, tables, ctx

    def step(self, forced_tokens: list[int] | None = None) -> list[StepOutput]:
        """One engine iteration.  ``forced_tokens`` (one per scheduled
        sequence, prefill first) replaces the sampled tokens: teacher forcing
        for parity tests."""
        batch = self.scheduler.schedule()
        if batch.is_empty():
            return []
        ordered = batch.prefill + batch.decode
        ids, pos, slices, tables, ctx = self.build_batch(batch)
        greedy = all(r.temperature <= 0.0 for r in ordered)
        if self.cuda_graphs and greedy and not batch.prefill:
            g = self.decode_graph(len(ordered), sum(ctx))
            md = StepMeta(ids, pos, slices, tables, ctx, self.cfg.block_size,
                          self.model.cfg.n_heads // self.model.cfg.n_kv_heads, self.device,
                          bt_width=self._bt_width, dest=g.dest, staging=g.staging())
            g.run(md)
            logits = self.model.dm.logits[: len(ordered)]
        else:
            md = self.model.metadata(ids, pos, slices, tables, ctx, self.cfg.block_size)
            logits = self.model.forward_meta(md, self.kv_cache, sample=greedy)
        if greedy:
            next_ids = self.model.dm.next_ids[: len(ordered)].cpu().tolist()
            self.last_d2h_bytes = 4 * len(ordered)
        else:
            next_ids = self._sample(logits, ordered)
            self.last_d2h_bytes = 4 * len(ordered)
        self.last_h2d_bytes = md.h2d_bytes
        self.last_batch = (ids, pos, slices, tables, ctx)
        self.last_logits = logits
        if forced_tokens is not None:
            next_ids = list(forced_tokens)
        now = time.perf_counter()
        outputs: list[StepOutput] = []
        for req, tok in zip(ordered, next_ids):
            if req.first_token_time is None:
                req.first_token_time = now
            req.output_token_ids.append(tok)
            finished = (tok in self.eos_ids or len(req.output_token_ids) >= req.max_new_tokens
                        or req.context_len() >= self.cfg.max_model_len)
            delta = self.tokenizer.decode([tok], skip_special_tokens=True) if self.tokenizer else ""
            if finished:
                self.scheduler.finish(req)
            outputs.append(StepOutput(req.req_id, tok, delta, finished, req))
        return outputs

    def decode_graph(self, n: int, ctx_total: int | None = None) -> DecodeGraph:
        """The captured decode step for ``n`` sequences (captured on first
        use; its split-KV size is chosen for ``ctx_total``, by default the
        running requests' summed context length)."""
        g = self._graphs.get(n)
        if g is None or g.stale():
            if ctx_total is None:
                ctx_total = sum(r.context_len() for r in self.scheduler.running) or None
            g = DecodeGraph(self.model.dm, self.kv_cache.pools, n, self._bt_width,
                            self.cfg.max_model_len, self.cfg.block_size, ctx_total=ctx_total)
            self._graphs[n] = g
        return g

    def _sample(self, logits: torch.Tensor, reqs: list[Request]) -> list[int]:
        """Per-row sampling for non-greedy requests (``src/tinybatch/engine.py:145-159``)."""
        out: list[int] = []
        greedy_rows = torch.argmax(logits, dim=-1)
        for i, req in enumerate(reqs):
            if req.temperature <= 0.0:
                out.append(int(greedy_rows[i]))
                continue
            probs = torch.softmax(logits[i] / req.temperature, dim=-1)
            if req.top_p < 1.0:
                sp, idx = probs.sort(descending=True)
                keep = sp.cumsum(0) - sp < req.top_p
                probs = torch.zeros_like(probs).scatter(0, idx[keep], sp[keep])
                probs = probs / probs.sum()
            out.append(int(torch.multinomial(probs, 1)))
        return out

    def stats(self) -> dict:
        bm = self.block_manager
        return {
            "kv_pool_mb": round(self.kv_cache.memory_bytes() / 2**20, 1),
            "free_blocks": bm.num_free(),
            "prefix_hit_rate": round(bm.hit_rate(), 3),
            "running": len(self.scheduler.running),
            "waiting": len(self.scheduler.waiting),
        }
