"""Host logic of the overlapped decode steps (no GPU): when the engine may
queue the next step before reading the current one back, and how a queued
step's tokens are applied — placeholders filled, stops on length / stop
token / max_model_len, the token of a step queued after a stop dropped, and
a stopped sequence skipped when the step queued after its stop completes."""
from __future__ import annotations

import torch

from tinybatch_b200.block_manager import BlockManager
from tinybatch_b200.config import EngineConfig
from tinybatch_b200.engine import PENDING, LLMEngine, _InFlight
from tinybatch_b200.scheduler import Request, Scheduler, Status


class _Done:
    def synchronize(self) -> None:
        pass


class _Graph:
    def __init__(self, stale=False):
        self._stale = stale

    def stale(self) -> bool:
        return self._stale


def _engine(num_blocks=64, max_model_len=512, stop=(), prefix=False):
    cfg = EngineConfig(block_size=4, num_blocks=num_blocks, enable_prefix_caching=prefix,
                       max_batch_tokens=512, max_running=16, max_model_len=max_model_len,
                       stop_token_ids=tuple(stop), overlap_steps=True, device="cpu")
    eng = LLMEngine.__new__(LLMEngine)
    eng.cfg = cfg
    eng.cuda_graphs = True
    eng.block_manager = BlockManager(num_blocks, 4, prefix)
    eng.scheduler = Scheduler(cfg, eng.block_manager)
    eng.eos_ids = set(stop)
    eng.tokenizer = None
    eng._inflight = None
    eng._graphs = {}
    eng.last_h2d_bytes = eng.last_d2h_bytes = 0
    return eng


def _running(eng, prompts, max_new):
    reqs = [Request(prompt_token_ids=p, max_new_tokens=m) for p, m in zip(prompts, max_new)]
    for r in reqs:
        eng.scheduler.add(r)
    batch = eng.scheduler.schedule()                 # admits them (prefill)
    assert len(batch.prefill) == len(reqs)
    for r in reqs:
        r.output_token_ids.append(1)                 # the prefill's sample
    return reqs


def _queue(reqs):
    """What _launch records for a step of `reqs`: one PENDING token each."""
    slots = []
    for r in reqs:
        slots.append(len(r.output_token_ids))
        r.output_token_ids.append(PENDING)
    return slots


def _inflight(reqs, slots, toks):
    return _InFlight(list(reqs), slots, torch.tensor(toks, dtype=torch.int32), _Done(), 100)


def test_ready_only_for_a_steady_greedy_decode_batch():
    eng = _engine()
    reqs = _running(eng, [[5] * 6, [6] * 9], [10, 10])
    assert eng._overlap_ready(None)
    f = _inflight(reqs, _queue(reqs), [2, 3])
    assert not eng._overlap_ready(f)                 # no graph captured for 2 sequences yet
    eng._graphs[2] = _Graph(stale=True)
    assert not eng._overlap_ready(f)
    eng._graphs[2] = _Graph()
    assert eng._overlap_ready(f)
    # a waiting request, a sampled one, prefix caching, a different batch
    eng.scheduler.add(Request(prompt_token_ids=[1, 2], max_new_tokens=3))
    assert not eng._overlap_ready(f)
    eng.scheduler.waiting.clear()
    reqs[1].temperature = 0.7
    assert not eng._overlap_ready(f)
    reqs[1].temperature = 0.0
    assert not eng._overlap_ready(_inflight(reqs[:1], [0], [2]))
    eng.cfg.enable_prefix_caching = True
    assert not eng._overlap_ready(f)


def test_not_ready_when_a_sequence_stops_for_length_at_the_queued_step():
    eng = _engine(max_model_len=12)
    reqs = _running(eng, [[5] * 6, [6] * 9], [3, 10])
    eng._graphs[2] = _Graph()
    f = _inflight(reqs, _queue(reqs), [2, 3])        # outputs: [1, PENDING]
    assert eng._overlap_ready(f)
    f2 = _inflight(reqs, _queue(reqs), [4, 5])       # outputs reach 3 = max_new_tokens
    assert not eng._overlap_ready(f2)
    # the second sequence reaches max_model_len 12 (9 prompt + 3 outputs)
    reqs[0].max_new_tokens = 50
    assert not eng._overlap_ready(f2)


def test_not_ready_without_a_free_block_for_every_new_block():
    eng = _engine(num_blocks=4)
    reqs = _running(eng, [[5] * 3, [6] * 7], [10, 10])   # 1 + 2 blocks of 4
    eng._graphs[2] = _Graph()
    # contexts 4 and 8: both next slots start a block; only one block is free
    assert eng.block_manager.num_free() == 1
    f = _inflight(reqs, [0, 0], [0, 0])
    assert not eng._overlap_ready(f)


def test_collect_fills_placeholders_and_stops():
    eng = _engine(stop=[9])
    reqs = _running(eng, [[5] * 6, [6] * 9, [7] * 3], [10, 2, 10])
    f1 = _inflight(reqs, _queue(reqs), [4, 5, 9])
    f2 = _inflight(reqs, _queue(reqs), [6, 7, 8])   # queued before f1 was read
    out = eng._collect(f1)
    assert [(o.token_id, o.finished) for o in out] == [(4, False), (5, True), (9, True)]
    # the stopped sequences lost the token of the step queued after their stop
    assert reqs[0].output_token_ids == [1, 4, PENDING]
    assert reqs[1].output_token_ids == [1, 5] and reqs[1].status is Status.FINISHED
    assert reqs[2].output_token_ids == [1, 9] and reqs[2].status is Status.FINISHED
    assert reqs[1].block_table == [] and reqs[2].block_table == []
    out2 = eng._collect(f2)
    assert [(o.req_id, o.token_id) for o in out2] == [(reqs[0].req_id, 6)]
    assert reqs[0].output_token_ids == [1, 4, 6]
    assert eng.last_d2h_bytes == 4 * 3 and eng.last_h2d_bytes == 100


def test_collect_stops_at_max_model_len():
    eng = _engine(max_model_len=9)
    reqs = _running(eng, [[5] * 7], [50])
    f = _inflight(reqs, _queue(reqs), [3])          # context 9 = max_model_len
    out = eng._collect(f)
    assert out[0].finished and reqs[0].status is Status.FINISHED


def test_drain_returns_the_queued_step_once():
    eng = _engine()
    reqs = _running(eng, [[5] * 6], [10])
    eng._inflight = _inflight(reqs, _queue(reqs), [4])
    assert [o.token_id for o in eng.drain()] == [4]
    assert eng._inflight is None and eng.drain() == []


class _Pools:
    """Stand-in for the KV cache: one CPU pool per layer."""

    def __init__(self, num_blocks, layers=2):
        self.pools = [torch.zeros(num_blocks, 2, 1, 4, 2) for _ in range(layers)]


def _spec_launch(eng):
    """The host part of _launch: schedule the next decode step before the
    previous step's tokens are known, build its batch, queue placeholders;
    each sequence's KV slot of this step is marked in the pools."""
    before = [(r, len(r.block_table)) for r in eng.scheduler.running]
    batch = eng.scheduler.schedule()
    assert not batch.prefill
    eng.build_batch(batch)
    for r in batch.decode:
        pos = r.context_len() - 1
        blk, off = r.block_table[pos // 4], pos % 4
        for pool in eng.kv_cache.pools:
            pool[blk, 0, 0, off, 0] = float(r.req_id)
            pool[blk, 0, 0, off, 1] = float(pos)
    slots = _queue(batch.decode)
    return batch.decode, slots, before


def _plain_run(prompts, max_new, stops, steps, num_blocks):
    """Reference order: every step schedules, then applies its tokens and
    frees what stopped.  Returns the (tables, free stack) after each step's
    tokens are applied and the next step is scheduled."""
    eng = _engine(num_blocks=num_blocks, stop=[9])
    eng.cfg.overlap_steps = False
    reqs = _running(eng, prompts, max_new)
    states = []
    batch = eng.scheduler.schedule()
    eng.build_batch(batch)
    for k in range(steps):
        for i, r in enumerate(list(batch.decode)):
            tok = 9 if (i, k) in stops else 1
            r.output_token_ids.append(tok)
            if tok == 9 or len(r.output_token_ids) >= r.max_new_tokens:
                eng.scheduler.finish(r)
        batch = eng.scheduler.schedule()
        eng.build_batch(batch)
        states.append(([list(r.block_table) for r in reqs], list(eng.block_manager.free_ids)))
    return states


def test_stop_token_keeps_the_reference_block_tables():
    """A sequence stops on a stop token while the next step is already
    queued, at steps where other sequences cross block boundaries: after the
    queued step's reservations are redone, every table and the free stack
    equal the plain engine's, and each continuing sequence's KV slot written
    by the queued step sits in a block its table held before that step (the
    redone reservations never move KV already written)."""
    prompts = [[5] * 7, [6] * 3, [7] * 11, [8] * 2, [4] * 5]
    max_new = [40] * 5
    # (sequence index in the step's batch, step) that emits the stop token
    stops = {(1, 1), (0, 4), (2, 9)}
    steps = 12
    want = _plain_run(prompts, max_new, stops, steps, num_blocks=40)

    eng = _engine(num_blocks=40, stop=[9])
    eng.kv_cache = _Pools(40)
    reqs = _running(eng, prompts, max_new)
    cur = _spec_launch(eng)
    for k in range(steps):
        nxt = _spec_launch(eng)        # queued before step k's tokens are read
        toks = [9 if (i, k) in stops else 1 for i in range(len(cur[0]))]
        f = _inflight(cur[0], cur[1], toks)
        q = _InFlight(nxt[0], nxt[1], torch.zeros(len(nxt[0]), dtype=torch.int32), _Done(), 0,
                      nxt[2])
        eng._collect(f, q)
        # the queued step's own sequences minus those that just stopped
        cur = ([r for r in nxt[0] if r.status is Status.RUNNING],
               [s for r, s in zip(nxt[0], nxt[1]) if r.status is Status.RUNNING])
        tables = [list(r.block_table) for r in reqs]
        assert (tables, list(eng.block_manager.free_ids)) == want[k], k
        before = dict((id(r), n) for r, n in nxt[2])
        for r in cur[0]:
            assert r.output_token_ids[-1] == PENDING
            pos = r.context_len() - 2          # the position the queued step wrote
            assert pos // 4 < before[id(r)]
            blk, off = r.block_table[pos // 4], pos % 4
            for pool in eng.kv_cache.pools:
                assert pool[blk, 0, 0, off, 0].item() == r.req_id
                assert pool[blk, 0, 0, off, 1].item() == pos


def test_reset_starts_cold():
    """reset() forgets every request and the prefix cache, keeping the pool
    and graphs: the next identical workload gets identical tables."""
    eng = _engine(prefix=True)
    eng._graphs[1] = _Graph()
    reqs = _running(eng, [[5] * 9, [5] * 9], [4, 4])
    first = [list(r.block_table) for r in reqs]
    assert eng.block_manager.prefix_hits > 0          # the second prompt hit the first
    eng.reset()
    assert not eng.scheduler.has_work() and eng.block_manager.prefix_hits == 0
    assert eng.block_manager.num_free() == 64 and eng._graphs
    again = [list(r.block_table) for r in _running(eng, [[5] * 9, [5] * 9], [4, 4])]
    assert again == first
