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
* ``EngineConfig.overlap_steps``: once the batch is a steady greedy decode
  batch, ``step`` queues the next decode step on the device (its token ids
  copied there from this step's argmax) before reading this step's tokens
  back, so the host's scheduling and output handling run while the GPU
  computes.  Every request produces the same tokens and the same block
  tables as without it: a sequence that stops on a stop token at step k had
  step k+1 computed for nothing (its output is dropped), and the blocks step
  k+1 reserved are taken back and reserved again in the reference's order
  (the stopped sequence's blocks freed first).  A step reserves the slot of
  the position after the one it writes (``append_slot`` sees the token list
  that already holds the token being processed), so step k+1 wrote no KV
  into the blocks it reserved and nothing on the device moves;
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
from .scheduler import Request, Scheduler, Status

# output slot of a token still being computed on the device (overlapped steps)
PENDING = -1


@dataclass
class StepOutput:
    req_id: int
    token_id: int
    text_delta: str
    finished: bool
    request: Request = field(repr=False)


@dataclass
class _InFlight:
    """A decode step queued on the device whose tokens are not read yet."""
    reqs: list            # the step's sequences, in batch order
    slots: list           # index of each one's pending token in output_token_ids
    host_ids: torch.Tensor    # pinned int32, filled by an asynchronous copy
    done: torch.cuda.Event    # recorded after that copy
    h2d_bytes: int
    # every running sequence's block-table length before this step was
    # scheduled, in scheduling order (to redo the step's block reservations
    # in the reference's order when an earlier step's sequence stops)
    tables_before: list = field(default_factory=list)


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
        self._inflight: _InFlight | None = None
        self._ids_host: list[torch.Tensor] = []
        self._ids_turn = 0

    # ------------------------------------------------------------- API

    def reset(self) -> None:
        """Forget every request: a fresh block manager and scheduler over
        the same KV pool, model and captured decode graphs (which depend on
        neither), so a new workload starts cold without re-capturing."""
        self.drain()
        self.block_manager = BlockManager(self.cfg.num_blocks, self.cfg.block_size,
                                          self.cfg.enable_prefix_caching)
        self.scheduler = Scheduler(self.cfg, self.block_manager)

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
        for parity tests.  With ``overlap_steps`` the outputs returned may be
        those of a step queued by the previous call (see ``drain``)."""
        if self.cfg.overlap_steps and forced_tokens is None:
            return self._step_overlapped()
        if self._inflight is not None:
            return self.drain()
        return self._step_plain(forced_tokens)

    def _step_plain(self, forced_tokens: list[int] | None) -> list[StepOutput]:
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

    # ------------------------------------------------- overlapped decode

    def drain(self) -> list[StepOutput]:
        """Outputs of the decode step still queued on the device, if any."""
        f, self._inflight = self._inflight, None
        return self._collect(f) if f is not None else []

    def _step_overlapped(self) -> list[StepOutput]:
        if self._inflight is None:
            if not self._overlap_ready(None):
                return self._step_plain(None)
            self._inflight = self._launch(None)
        nxt = self._launch(self._inflight) if self._overlap_ready(self._inflight) else None
        out = self._collect(self._inflight, nxt)
        if nxt is not None and all(r.status is Status.FINISHED for r in nxt.reqs):
            self._collect(nxt)          # every sequence of it has stopped
            nxt = None
        self._inflight = nxt
        return out

    def _overlap_ready(self, inflight: _InFlight | None) -> bool:
        """Whether the next step is a decode of exactly the running sequences
        (after ``inflight``, in its order) that the scheduler serves without
        preempting: no waiting request, greedy sampling, no sequence stopping
        for length at ``inflight``, a free block for every sequence that
        starts one."""
        sch = self.scheduler
        if not self.cuda_graphs or self.cfg.enable_prefix_caching or sch.waiting:
            return False
        run = sch.running
        if not run or any(r.status is not Status.RUNNING or r.temperature > 0.0 for r in run):
            return False
        if inflight is not None:
            if len(inflight.reqs) != len(run) or any(a is not b for a, b in zip(inflight.reqs, run)):
                return False
            # capturing a graph runs a forward, which would overwrite the
            # in-flight step's samples before they are fed
            g = self._graphs.get(len(run))
            if g is None or g.stale():
                return False
            lim = self.cfg.max_model_len
            if any(len(r.output_token_ids) >= r.max_new_tokens or r.context_len() >= lim
                   for r in run):
                return False
        # blocks the step may take: one where the next slot starts a block, one
        # where build_batch extends a table (a prompt ending on a block boundary)
        bs = self.cfg.block_size
        need = sum((r.context_len() % bs == 0) + (len(r.block_table) * bs < r.context_len())
                   for r in run)
        return need <= self.block_manager.num_free()

    def _launch(self, prev: _InFlight | None) -> _InFlight:
        """Schedule and queue one decode step (graph replay) without waiting
        for it.  With ``prev`` (the step queued before it, same sequences in
        the same order) the token ids are ``prev``'s samples, copied on the
        device; the host holds PENDING for them."""
        before = [(r, len(r.block_table)) for r in self.scheduler.running]
        batch = self.scheduler.schedule()
        reqs = batch.decode
        if batch.prefill or not reqs:
            raise RuntimeError("overlapped step: a decode-only batch was expected")
        n = len(reqs)
        if prev is not None and (len(prev.reqs) != n or
                                 any(a is not b for a, b in zip(prev.reqs, reqs))):
            raise RuntimeError("overlapped step: the batch differs from the queued step's")
        ids, pos, slices, tables, ctx = self.build_batch(batch)
        g = self.decode_graph(n, sum(ctx))
        md = StepMeta(ids, pos, slices, tables, ctx, self.cfg.block_size,
                      self.model.cfg.n_heads // self.model.cfg.n_kv_heads, self.device,
                      bt_width=self._bt_width, dest=g.dest, staging=g.staging())
        dm = self.model.dm
        if prev is not None:
            g.md.ids.copy_(dm.next_ids[:n])
        g.run(md)
        if not self._ids_host or self._ids_host[0].numel() < n:
            self._ids_host = [torch.empty(max(n, 64), dtype=torch.int32).pin_memory()
                              for _ in range(2)]
        host = self._ids_host[self._ids_turn]
        self._ids_turn ^= 1
        host[:n].copy_(dm.next_ids[:n], non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        slots = []
        for r in reqs:
            slots.append(len(r.output_token_ids))
            r.output_token_ids.append(PENDING)
        self.last_batch = None
        self.last_logits = None
        return _InFlight(reqs, slots, host, done, md.h2d_bytes, before)

    def _collect(self, f: _InFlight, queued: _InFlight | None = None) -> list[StepOutput]:
        """Wait for a queued step's tokens and apply them (append / finish) as
        ``step`` does; sequences that stopped at an earlier step are skipped.
        ``queued``: the step already queued after ``f``; when a sequence
        stops here, its block reservations are redone in the reference's
        order (``_rereserve``)."""
        f.done.synchronize()
        toks = f.host_ids[: len(f.reqs)].tolist()
        self.last_h2d_bytes = f.h2d_bytes
        self.last_d2h_bytes = 4 * len(f.reqs)
        now = time.perf_counter()
        lim = self.cfg.max_model_len
        rows = []
        for req, idx, tok in zip(f.reqs, f.slots, toks):
            if req.status is Status.FINISHED:
                continue
            finished = (tok in self.eos_ids or idx + 1 >= req.max_new_tokens
                        or len(req.prompt_token_ids) + idx + 1 >= lim)
            rows.append((req, idx, tok, finished))
        redo = queued is not None and any(fin for *_, fin in rows)
        if redo:
            self._take_back(queued)
        outputs: list[StepOutput] = []
        for req, idx, tok, finished in rows:
            req.output_token_ids[idx] = tok
            if req.first_token_time is None:
                req.first_token_time = now
            delta = self.tokenizer.decode([tok], skip_special_tokens=True) if self.tokenizer else ""
            if finished:
                del req.output_token_ids[idx + 1:]     # a later queued step's token
                self.scheduler.finish(req)
            outputs.append(StepOutput(req.req_id, tok, delta, finished, req))
        if redo:
            self._rereserve(queued)
        return outputs

    def _take_back(self, q: _InFlight) -> None:
        """Undo the block reservations of queued step ``q``: its scheduling
        only popped fresh blocks from the top of the free stack (a decode
        step with prefix caching off and no preemption), so pushing each
        table's new tail back, last first, restores the stack exactly."""
        bm = self.block_manager
        for req, n in reversed(q.tables_before):
            while len(req.block_table) > n:
                bid = req.block_table.pop()
                blk = bm.blocks[bid]
                blk.ref_count = 0
                blk.token_ids = []
                bm.free_ids.append(bid)

    def _rereserve(self, q: _InFlight) -> None:
        """Reserve queued step ``q``'s blocks again, as the reference's next
        schedule does after the stopped sequences were freed: ``append_slot``
        per running sequence in order, plus ``build_batch``'s extension.
        ``q`` wrote its KV at the position before the reserved one, inside
        blocks the tables already held, so its device work stays valid."""
        bm, bs = self.block_manager, self.cfg.block_size
        for req, _ in q.tables_before:
            if req.status is not Status.RUNNING:
                continue
            L = req.context_len() - 1          # q's own token is still pending
            bm.append_slot(req.block_table, req.token_view(L))
            if len(req.block_table) * bs < L:
                bm.append_slot(req.block_table, req.token_view(L - 1))

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
