"""End-to-end parity of the B200 forward with the reference.

Tolerance: logits within max-abs 2e-2 of the
reference's fp32 forward on the same seeded weights (ours run bf16 weights
with fp32 accumulation and an fp32 residual stream), greedy argmax agreement
>= 99% teacher-forced, block tables bit-exact.  Against the CPU oracle fed
the same bf16-rounded weights the bound is tighter (1e-2).
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from oracle import qwen2_ref as R  # noqa: E402
from tinybatch_b200 import _native  # noqa: E402
from tinybatch_b200.config import EngineConfig, named_config  # noqa: E402
from tinybatch_b200.engine import LLMEngine  # noqa: E402
from tinybatch_b200.model import Qwen2Paged  # noqa: E402
from tinybatch_b200.tensor_parallel import tp_forward  # noqa: E402
from tinybatch_b200.weights import reference_test_weights, synthetic_weights  # noqa: E402

ATOL = 2e-2


@pytest.fixture(autouse=True)
def _status_clean():
    _native.status(clear=True)
    yield
    _native.raise_on_status("forward")


def _bf16_round(w):
    return {k: v.to(torch.bfloat16).float() for k, v in w.items()}


@pytest.fixture(scope="module")
def tiny():
    cfg = named_config("tiny")
    w = synthetic_weights(cfg, 0)
    return cfg, w, Qwen2Paged.from_weights(cfg, w)


@pytest.mark.parametrize("name", ["paged_bs16", "paged_small"])
def test_paged_trace_teacher_forced(golden, tiny, name):
    cfg, w, model = tiny
    run = golden[name]
    kv = model.make_kv_cache(run["num_blocks"], run["block_size"])
    wr = _bf16_round(w)
    pools = R.new_pools(cfg.n_layers, run["num_blocks"], run["block_size"], cfg.n_kv_heads,
                        cfg.head_dim)
    worst = 0.0
    for st in run["steps"]:
        out = model.forward(st["token_ids"], st["positions"], st["seq_slices"],
                            st["block_tables"], st["context_lens"], kv).cpu()
        ref = st["logits"]
        err = float((out - ref).abs().max())
        worst = max(worst, err)
        _assert_decisive_argmax(out, ref, err)
        orc = R.paged_forward(cfg, wr, st["token_ids"], st["positions"], st["seq_slices"],
                              st["block_tables"], st["context_lens"], pools, run["block_size"])
        torch.testing.assert_close(out, orc, atol=1e-2, rtol=0)
    assert worst <= ATOL, worst


def _assert_decisive_argmax(out, ref, err):
    """Rows whose reference top-1 leads the runner-up by more than twice the
    observed logit error must pick the same token; closer rows are near-ties
    that a bf16 forward may legitimately flip."""
    top2 = ref.topk(2, dim=-1).values
    decisive = (top2[:, 0] - top2[:, 1]) > 2 * err
    assert bool((out.argmax(-1) == ref.argmax(-1))[decisive].all())


def test_tiny_prefill_and_tp_forward_world1(golden, tiny):
    cfg, w, model = tiny
    case = golden["tiny_tp"]
    ids = torch.tensor(case["ids"])
    kv = model.make_kv_cache(8, 16)
    out = model.forward(ids, torch.arange(16), [(0, 16)], [[5]], [16], kv).cpu()
    torch.testing.assert_close(out, case["paged_last"], atol=ATOL, rtol=0)
    logits = tp_forward(ids, w, cfg, world=1)
    torch.testing.assert_close(logits, case["logits_w1"], atol=ATOL, rtol=0)
    _assert_decisive_argmax(logits, case["logits_w1"], float((logits - case["logits_w1"]).abs().max()))


def test_reference_tp_test_model_world1(golden):
    case = golden["ref_test"]
    cfg = named_config("ref-test")
    w = reference_test_weights(cfg, 0)
    logits = tp_forward(torch.tensor(case["ids"]), w, cfg, world=1)
    torch.testing.assert_close(logits, case["logits_w1"], atol=ATOL, rtol=0)
    _assert_decisive_argmax(logits, case["logits_w1"], float((logits - case["logits_w1"]).abs().max()))


def test_engine_teacher_forced_matches_reference_run(golden, tiny):
    """Our engine (scheduler, block manager, metadata, forward), fed the
    reference run's sampled tokens, rebuilds the reference's flat batches and
    block tables bit for bit and reproduces its logits."""
    cfg, w, model = tiny
    for name in ("paged_bs16", "paged_small"):
        run = golden[name]
        ecfg = EngineConfig(block_size=run["block_size"], num_blocks=run["num_blocks"],
                            max_batch_tokens=run["max_batch_tokens"],
                            max_running=run["max_running"], enable_prefix_caching=run["prefix"])
        eng = LLMEngine(ecfg, model=model)
        for p, n in zip(run["prompts"], run["max_new"]):
            eng.add_request_ids(p, max_new_tokens=n)
        for st in run["steps"]:
            eng.step(forced_tokens=st["next_ids"])
            ids, pos, slices, tables, ctx = eng.last_batch
            assert ids == st["token_ids"] and pos == st["positions"]
            assert slices == [tuple(x) for x in st["seq_slices"]]
            assert [list(t) for t in tables] == st["block_tables"] and ctx == st["context_lens"]
            lg = eng.last_logits[: len(ctx)].cpu()
            err = float((lg - st["logits"]).abs().max())
            assert err <= ATOL, err
            _assert_decisive_argmax(lg, st["logits"], err)
        assert not eng.scheduler.has_work()


def test_engine_prompt_on_block_boundary():
    """A prompt of exactly block_size tokens decodes (the reference engine has
    no block for that first decode token)."""
    cfg = named_config("tiny")
    model = Qwen2Paged.from_weights(cfg, synthetic_weights(cfg, 0))
    eng = LLMEngine(EngineConfig(block_size=16, num_blocks=16, max_batch_tokens=64), model=model)
    out = eng.generate([list(range(16)), list(range(32))], max_new_tokens=5)
    assert [len(o) for o in out] == [5, 5]


@pytest.mark.slow
def test_qwen05b_probe(golden):
    """Config 2 shape (24 layers, bf16 weights) against the reference's fp32
    forward on the same bf16-valued weights.

    Over 24 layers any forward that stores its GEMM inputs, q, the KV cache
    and the attention/SwiGLU outputs in bf16 drifts from the fp32 forward:
    the CPU oracle with exactly those roundings (``emulate_bf16``) lands
    ~0.026-0.031 max-abs / ~0.004 mean-abs away on this case, and two such
    forwards differ from each other by as much (the rounding decisions
    diverge).  So the bound here is relative: our deviation from the fp32
    reference may not exceed the emulated bf16 forward's by more than 30%
    (+5e-3), with absolute caps 4e-2 max / 6e-3 mean; rows whose top-1 lead
    is decisive must pick the same token."""
    case = golden["qwen05b"]
    cfg = named_config(case["cfg"])
    w = synthetic_weights(cfg, case["seed"])
    wb = {k: v.to(torch.bfloat16).float() for k, v in w.items()}
    model = Qwen2Paged.from_weights(cfg, w)
    kv = model.make_kv_cache(16, 16)
    p0, p1 = case["prompts"]
    args = (p0 + p1, list(range(40)) + list(range(17)), [(0, 40), (40, 57)], case["tables"],
            [40, 17])
    dargs = (case["next_ids"], [40, 17], [(0, 1), (1, 2)], case["tables"], [41, 18])
    pre = model.forward(*args, kv).cpu()
    dec = model.forward(*dargs, kv).cpu()
    pools = R.new_pools(cfg.n_layers, 16, 16, cfg.n_kv_heads, cfg.head_dim)
    pre_e = R.paged_forward(cfg, wb, *args, pools, 16, emulate_bf16=True)
    dec_e = R.paged_forward(cfg, wb, *dargs, pools, 16, emulate_bf16=True)
    si = case["sample_idx"]
    for got, emu, ref in ((pre, pre_e, case["prefill"]), (dec, dec_e, case["decode"])):
        ours = (got[:, si] - ref["sample"]).abs()
        emul = (emu[:, si] - ref["sample"]).abs()
        assert float(ours.max()) <= min(4e-2, 1.3 * float(emul.max()) + 5e-3), (ours.max(), emul.max())
        assert float(ours.mean()) <= min(6e-3, 1.3 * float(emul.mean()) + 1e-3), (ours.mean(), emul.mean())
        top = torch.gather(got, 1, ref["top_idx"])
        err = float((top - ref["top_val"]).abs().max())
        assert err <= 4e-2, err
        gap = ref["top_val"][:, 0] - ref["top_val"][:, 1]
        decisive = gap > 2 * err
        assert bool((got.argmax(-1) == ref["argmax"])[decisive].all())
