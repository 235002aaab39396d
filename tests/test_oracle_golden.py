"""Pin the CPU oracle (and the host bookkeeping) to the reference's own outputs.

The golden vectors were produced by running the reference unmodified
(``tests/golden/make_golden.py``).  Weights are regenerated from their seed;
the stored fingerprints prove the draw is the same one the reference saw.
"""
from __future__ import annotations

import pytest
import torch

from oracle import qwen2_ref as R
from tinybatch_b200.block_manager import BlockManager, OutOfBlocks
from tinybatch_b200.config import EngineConfig, named_config
from tinybatch_b200.scheduler import Request, Scheduler
from tinybatch_b200.weights import fingerprint, reference_test_weights, synthetic_weights


def _weights(case):
    cfg = named_config(case["cfg"])
    if case["cfg"] == "ref-test":
        w = reference_test_weights(cfg, case["seed"])
    else:
        w = synthetic_weights(cfg, case["seed"])
    fp = fingerprint(w)
    for k, v in case["fingerprint"].items():
        assert fp[k] == pytest.approx(v, rel=1e-12), k
    return cfg, w


@pytest.mark.parametrize("name", ["tiny_tp", "ref_test"])
def test_tp_forward_matches_reference(golden, name):
    case = golden[name]
    cfg, w = _weights(case)
    ids = torch.tensor(case["ids"])
    torch.testing.assert_close(R.tp_forward(cfg, w, ids, world=1), case["logits_w1"],
                               atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(R.tp_forward(cfg, w, ids, world=2), case["logits_w2"],
                               atol=1e-5, rtol=1e-5)
    # two all-reduces per layer, T x d elements each (the reference ran fp32)
    assert case["stats_w2"]["calls"] == 2 * cfg.n_layers
    assert case["stats_w2"]["bytes"] == 2 * cfg.n_layers * len(case["ids"]) * cfg.d_model * 4


def test_tp_gate_case_matches_reference(golden):
    """The parity-gate model bench.py checks at every tensor-parallel degree:
    the oracle, emulating 1, 2, 4 and 8 ranks, reproduces the reference's
    logits for the bf16-valued draw it recorded."""
    from tinybatch_b200.config import ModelConfig
    case = golden["tp_gate"]
    cfg = ModelConfig(**case["cfg"])
    w = {k: v.float() for k, v in synthetic_weights(cfg, case["seed"], dtype=torch.bfloat16).items()}
    fp = fingerprint(w)
    for k, v in case["fingerprint"].items():
        assert fp[k] == pytest.approx(v, rel=1e-12), k
    ids = torch.tensor(case["ids"])
    for world in (1, 2, 4, 8):
        torch.testing.assert_close(R.tp_forward(cfg, w, ids, world=world), case["logits_w1"],
                                   atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(case["logits_w2"], case["logits_w1"], atol=1e-5, rtol=1e-5)
    assert case["stats_w2"] == {"calls": 2 * cfg.n_layers,
                                "bytes": 2 * cfg.n_layers * len(case["ids"]) * cfg.d_model * 4}


def test_paged_prefill_matches_reference(golden):
    case = golden["tiny_tp"]
    cfg, w = _weights(case)
    pools = R.new_pools(cfg.n_layers, 8, 16, cfg.n_kv_heads, cfg.head_dim)
    out = R.paged_forward(cfg, w, case["ids"], list(range(16)), [(0, 16)], [[5]], [16], pools, 16)
    torch.testing.assert_close(out, case["paged_last"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("name", ["paged_bs16", "paged_small"])
def test_paged_engine_trace_matches_reference(golden, name):
    run = golden[name]
    cfg = named_config("tiny")
    w = synthetic_weights(cfg, 0)
    bs = run["block_size"]
    pools = R.new_pools(cfg.n_layers, run["num_blocks"], bs, cfg.n_kv_heads, cfg.head_dim)
    for st in run["steps"]:
        out = R.paged_forward(cfg, w, st["token_ids"], st["positions"], st["seq_slices"],
                              st["block_tables"], st["context_lens"], pools, bs)
        torch.testing.assert_close(out, st["logits"], atol=1e-5, rtol=1e-5)
        assert out.argmax(-1).tolist() == st["next_ids"]


def test_paged_engine_trace_tables_from_host_scheduler(golden):
    """Our Scheduler + BlockManager, fed the same greedy token stream,
    produce the reference's flat batches and block tables bit for bit."""
    for name in ("paged_bs16", "paged_small"):
        run = golden[name]
        ecfg = EngineConfig(block_size=run["block_size"], num_blocks=run["num_blocks"],
                            enable_prefix_caching=run["prefix"],
                            max_batch_tokens=run["max_batch_tokens"],
                            max_running=run["max_running"])
        bm = BlockManager(run["num_blocks"], run["block_size"], run["prefix"])
        sched = Scheduler(ecfg, bm)
        reqs = [Request(prompt_token_ids=list(p), max_new_tokens=n)
                for p, n in zip(run["prompts"], run["max_new"])]
        idx = {r.req_id: i for i, r in enumerate(reqs)}
        for r in reqs:
            sched.add(r)
        for st in run["steps"]:
            b = sched.schedule()
            ordered = b.prefill + b.decode
            assert [idx[r.req_id] for r in ordered] == st["req"]
            assert [list(r.block_table) for r in ordered] == st["block_tables"]
            assert len(b.prefill) == st["n_prefill"]
            assert bm.num_free() == st["num_free"]
            assert (bm.prefix_hits, bm.prefix_queries) == (st["prefix_hits"], st["prefix_queries"])
            for r, t in zip(ordered, st["next_ids"]):
                r.output_token_ids.append(t)
                if len(r.output_token_ids) >= r.max_new_tokens:
                    sched.finish(r)
        assert [r.preemptions for r in reqs] == run["preemptions"]


def test_block_manager_trace(golden):
    bm = BlockManager(24, 4, True)
    seqs = []
    for rec in golden["bm_trace"]:
        if rec["op"] == "alloc":
            try:
                table, cached = bm.allocate_prompt(list(rec["tokens"]))
                seqs.append((list(rec["tokens"]), table))
                assert (table, cached) == (rec["table"], rec["cached"])
            except OutOfBlocks:
                assert rec.get("error") == "OutOfBlocks"
        elif rec["op"] == "append":
            toks, table = seqs[rec["seq"]]
            try:
                grew = bm.append_slot(table, toks)
                toks.append(rec["token"])
                assert (grew, table) == (rec["grew"], rec["table"])
            except OutOfBlocks:
                assert rec.get("error") == "OutOfBlocks"
        else:
            _, table = seqs.pop(rec["seq"])
            bm.free_table(table)
        assert bm.num_free() == rec["num_free"]
        assert (bm.prefix_hits, bm.prefix_queries) == (rec["hits"], rec["queries"])
        assert bm.free_ids == rec["free_ids"]
        assert list(bm.evictable) == rec["evictable"]
        assert [b.ref_count for b in bm.blocks] == rec["ref_counts"]


def test_scheduler_trace(golden):
    ecfg = EngineConfig(block_size=4, num_blocks=20, enable_prefix_caching=True,
                        max_batch_tokens=40, max_running=5)
    bm = BlockManager(20, 4, True)
    s = Scheduler(ecfg, bm)
    reqs = []
    for rec in golden["sched_trace"]:
        if rec["new"] is not None:
            r = Request(prompt_token_ids=list(rec["new"][0]), max_new_tokens=rec["new"][1])
            reqs.append(r)
            s.add(r)
        idx = {r.req_id: i for i, r in enumerate(reqs)}
        b = s.schedule()
        assert [idx[r.req_id] for r in b.prefill] == rec["prefill"]
        assert [idx[r.req_id] for r in b.decode] == rec["decode"]
        assert [list(r.block_table) for r in b.prefill + b.decode] == rec["tables"]
        assert [r.num_cached_tokens for r in b.prefill] == rec["cached"]
        for r, t in zip(b.prefill + b.decode, rec["appended"]):
            r.output_token_ids.append(t)
            if len(r.output_token_ids) >= r.max_new_tokens:
                s.finish(r)
        assert [idx[r.req_id] for r in s.waiting] == rec["waiting"]
        assert [idx[r.req_id] for r in s.running] == rec["running"]
        assert [r.preemptions for r in reqs] == rec["preemptions"]
        assert bm.num_free() == rec["num_free"]


@pytest.mark.slow
def test_qwen05b_probe_matches_reference(golden):
    case = golden["qwen05b"]
    cfg = named_config(case["cfg"])
    w = synthetic_weights(cfg, case["seed"])
    w = {k: v.to(torch.bfloat16).to(torch.float32) for k, v in w.items()}
    assert float(w["model.embed_tokens.weight"].double().abs().sum()) == pytest.approx(
        case["fingerprint_embed"], rel=1e-12)
    p0, p1 = case["prompts"]
    pools = R.new_pools(cfg.n_layers, 16, 16, cfg.n_kv_heads, cfg.head_dim)
    pre = R.paged_forward(cfg, w, p0 + p1, list(range(40)) + list(range(17)),
                          [(0, 40), (40, 57)], case["tables"], [40, 17], pools, 16)
    dec = R.paged_forward(cfg, w, case["next_ids"], [40, 17], [(0, 1), (1, 2)],
                          case["tables"], [41, 18], pools, 16)
    for got, ref in ((pre, case["prefill"]), (dec, case["decode"])):
        torch.testing.assert_close(got[:, case["sample_idx"]], ref["sample"], atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(torch.gather(got, 1, ref["top_idx"]), ref["top_val"],
                                   atol=1e-4, rtol=1e-4)
        assert got.argmax(-1).tolist() == ref["argmax"].tolist()
