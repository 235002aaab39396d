"""Overlapped decode steps (``EngineConfig.overlap_steps``): the engine queues
step k+1 on the device, fed with step k's samples there, before reading step
k's tokens back.  Every request must produce exactly the tokens of the plain
step-by-step engine, including requests that stop on a stop token (their
speculative step is dropped), requests that reach max_new_tokens at
different steps, and requests admitted while a step is in flight; no block
may leak."""
from __future__ import annotations

import random

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from tinybatch_b200 import _native  # noqa: E402
from tinybatch_b200.config import EngineConfig, named_config  # noqa: E402
from tinybatch_b200.engine import LLMEngine  # noqa: E402
from tinybatch_b200.model import Qwen2Paged  # noqa: E402
from tinybatch_b200.weights import synthetic_weights  # noqa: E402


@pytest.fixture(autouse=True)
def _status_clean():
    _native.status(clear=True)
    yield
    _native.raise_on_status("engine overlap")


@pytest.fixture(scope="module")
def model():
    cfg = named_config("tiny")
    return Qwen2Paged.from_weights(cfg, synthetic_weights(cfg, 0))


def _prompts(n, seed=5):
    rng = random.Random(seed)
    # lengths on and around block boundaries (block 16)
    lens = [16, 31, 32, 33, 5, 47, 64, 1][:n] + [rng.randint(2, 70) for _ in range(max(0, n - 8))]
    return [[rng.randrange(256) for _ in range(k)] for k in lens]


def _engine(model, overlap, stop=()):
    cfg = EngineConfig(block_size=16, num_blocks=160, enable_prefix_caching=False,
                       max_batch_tokens=512, max_running=16, max_model_len=512,
                       stop_token_ids=tuple(stop), overlap_steps=overlap)
    return LLMEngine(cfg, model=model)


def _run(model, overlap, prompts, max_new, stop=(), late=None, late_at=4):
    eng = _engine(model, overlap, stop)
    reqs = [eng.add_request_ids(p, max_new_tokens=m) for p, m in zip(prompts, max_new)]
    steps = 0
    while eng.scheduler.has_work():
        eng.step()
        steps += 1
        if late is not None and steps == late_at:
            reqs += [eng.add_request_ids(p, max_new_tokens=m) for p, m in late]
    eng.drain()
    assert eng.block_manager.num_free() == eng.cfg.num_blocks
    return [list(r.output_token_ids) for r in reqs], eng


def test_overlap_matches_plain_engine(model):
    prompts = _prompts(12)
    max_new = [3, 17, 40, 1, 25, 9, 40, 2, 33, 12, 40, 6]
    plain, _ = _run(model, False, prompts, max_new)
    over, eng = _run(model, True, prompts, max_new)
    assert over == plain
    assert [len(o) for o in over] == max_new
    assert all(t >= 0 for o in over for t in o)


def test_overlap_stop_tokens(model):
    prompts = _prompts(10, seed=9)
    max_new = [30] * 10
    free, _ = _run(model, False, prompts, max_new)
    # stop on a token some request samples mid-stream
    counts = {}
    for o in free:
        for t in o[2:20]:
            counts[t] = counts.get(t, 0) + 1
    stop = max(counts, key=counts.get)
    plain, _ = _run(model, False, prompts, max_new, stop=[stop])
    over, _ = _run(model, True, prompts, max_new, stop=[stop])
    assert over == plain
    assert any(len(o) < 30 for o in over)


def test_overlap_admits_requests_mid_stream(model):
    prompts = _prompts(6, seed=11)
    late = [(p, 8 + i) for i, p in enumerate(_prompts(4, seed=12))]
    plain, _ = _run(model, False, prompts, [20] * 6, late=late)
    over, _ = _run(model, True, prompts, [20] * 6, late=late)
    assert over == plain


def test_overlap_queues_steps_ahead(model):
    """In a steady decode batch every call after the first queues one step
    before reading the previous one."""
    eng = _engine(model, True)
    for p in _prompts(8, seed=13):
        eng.add_request_ids(p, max_new_tokens=12)
    eng.step()                              # prefill
    eng.step()                              # first decode (plain: fills the graph)
    queued = 0
    while eng.scheduler.has_work():
        eng.step()
        queued += eng._inflight is not None
    eng.drain()
    assert queued >= 8
