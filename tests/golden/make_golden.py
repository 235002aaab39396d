"""Generate the golden vectors by running the reference implementation.

Usage (from the repository root, in a container where the reference source
tree is available; it never runs on the GPU box)::

    python tests/golden/make_golden.py --reference-src <reference>/src

The reference is imported from ``--reference-src`` and run unmodified on the
CPU in fp32.  Outputs go to ``tests/golden/golden.pt``.  Every case records
its inputs (token ids, block tables, ...) and the reference's outputs; the
weights are regenerated from their seed by ``tinybatch_b200.weights`` and a
per-tensor fingerprint is stored so a changed draw is detected.

Cases:
  tiny_tp      config "tiny" (2 layers, vocab 256, N(0,0.02) seed 0), 16 ids:
               tp_forward(world=1), run_tp_forward(world=2), paged prefill
  ref_test     the reference TP test model (4 layers, vocab 97, randn*0.05
               seed 0) on its 24 ids (seed 1): world 1 and 2, comm stats
  paged_*      engine-style runs (Scheduler + BlockManager + PagedKVCache +
               Qwen2Paged) with greedy decoding, prefix sharing and, in
               paged_small, eviction and preemption; every step's flat batch
               and logits are recorded
  bm_trace     random allocate/append/free sequence against BlockManager
  sched_trace  random admission/decode/finish sequence against Scheduler
  qwen05b      config "qwen2.5-0.5b" (seed 1, bf16-valued weights): two
               prompts, paged prefill and one decode step; top-64 logits
               and a fixed index sample
  tp_gate      a model whose heads, kv heads and d_ff divide 2, 4 and 8 (2
               layers, d 1024, 16 q / 8 kv heads of 64, ff 2048, vocab 512,
               bf16-valued weights seed 7), 40 ids (seed 7): tp_forward at
               world 1 and run_tp_forward at world 2 -- the parity gate
               bench.py runs before timing at every tensor-parallel degree

``--update NAME ...`` recomputes only the named cases and keeps the others.
"""
from __future__ import annotations

import argparse
import random
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from tinybatch_b200.config import named_config  # noqa: E402
from tinybatch_b200.weights import fingerprint, reference_test_weights, synthetic_weights  # noqa: E402


def ref_cfg(ref, cfg):
    return ref.model.ModelConfig(**{k: getattr(cfg, k) for k in (
        "n_layers", "n_heads", "n_kv_heads", "d_model", "head_dim", "d_ff", "vocab_size",
        "rms_eps", "rope_theta", "tie_embeddings", "max_position")})


def ref_model(ref, cfg, w):
    m = ref.model.Qwen2Paged.__new__(ref.model.Qwen2Paged)
    m.cfg, m.w, m.device, m.dtype = ref_cfg(ref, cfg), w, torch.device("cpu"), torch.float32
    return m


def engine_run(ref, cfg, w, prompts, max_new, block_size, num_blocks, max_batch_tokens,
               max_running, prefix=True):
    """Drive the reference Scheduler/BlockManager/model like LLMEngine.step
    (``src/tinybatch/engine.py:94-143``), greedy, recording every step."""
    ecfg = ref.config.EngineConfig(block_size=block_size, num_blocks=num_blocks,
                                   enable_prefix_caching=prefix,
                                   max_batch_tokens=max_batch_tokens, max_running=max_running)
    bm = ref.block_manager.BlockManager(num_blocks, block_size, prefix)
    sched = ref.scheduler.Scheduler(ecfg, bm)
    model = ref_model(ref, cfg, w)
    kv = ref.kv_cache.PagedKVCache(cfg.n_layers, num_blocks, block_size, cfg.n_kv_heads,
                                   cfg.head_dim, torch.device("cpu"), torch.float32)
    reqs = [ref.scheduler.Request(prompt_token_ids=list(p), max_new_tokens=n)
            for p, n in zip(prompts, max_new)]
    index = {r.req_id: i for i, r in enumerate(reqs)}
    for r in reqs:
        sched.add(r)
    steps = []
    while sched.has_work():
        batch = sched.schedule()
        if batch.is_empty():
            break
        ids, pos, slices, tables, ctx = [], [], [], [], []
        for r in batch.prefill:
            s = len(ids)
            ids += r.prompt_token_ids[r.num_cached_tokens:]
            pos += list(range(r.num_cached_tokens, len(r.prompt_token_ids)))
            slices.append((s, len(ids)))
            tables.append(list(r.block_table))
            ctx.append(len(r.prompt_token_ids))
        for r in batch.decode:
            s = len(ids)
            ids.append(r.all_token_ids()[-1])
            pos.append(r.context_len() - 1)
            slices.append((s, len(ids)))
            tables.append(list(r.block_table))
            ctx.append(r.context_len())
        logits = model.forward(torch.tensor(ids), torch.tensor(pos), slices, tables, ctx, kv)
        ordered = batch.prefill + batch.decode
        nxt = [int(logits[i].argmax()) for i in range(len(ordered))]
        steps.append(dict(req=[index[r.req_id] for r in ordered],
                          n_prefill=len(batch.prefill), token_ids=ids, positions=pos,
                          seq_slices=slices, block_tables=tables, context_lens=ctx,
                          logits=logits.clone(), next_ids=nxt,
                          num_free=bm.num_free(), prefix_hits=bm.prefix_hits,
                          prefix_queries=bm.prefix_queries))
        for r, t in zip(ordered, nxt):
            r.output_token_ids.append(t)
            if len(r.output_token_ids) >= r.max_new_tokens:
                sched.finish(r)
    return dict(prompts=[list(p) for p in prompts], max_new=list(max_new),
                block_size=block_size, num_blocks=num_blocks,
                max_batch_tokens=max_batch_tokens, max_running=max_running,
                prefix=prefix, steps=steps,
                outputs=[list(r.output_token_ids) for r in reqs],
                preemptions=[r.preemptions for r in reqs])


def bm_trace(ref, seed=0):
    rng = random.Random(seed)
    bm = ref.block_manager.BlockManager(24, 4, True)
    seqs: list[tuple[list[int], list[int]]] = []
    ops = []
    vocab = [1, 2, 3]                     # tiny vocab -> many shared prefixes
    for _ in range(400):
        kind = rng.random()
        rec: dict = {}
        if kind < 0.35 or not seqs:
            n = rng.randint(1, 14)
            toks = [rng.choice(vocab) for _ in range(n)]
            rec = dict(op="alloc", tokens=list(toks))
            try:
                table, cached = bm.allocate_prompt(toks)
                seqs.append((toks, table))
                rec.update(table=list(table), cached=cached)
            except ref.block_manager.OutOfBlocks:
                rec.update(error="OutOfBlocks")
        elif kind < 0.8:
            i = rng.randrange(len(seqs))
            toks, table = seqs[i]
            rec = dict(op="append", seq=i, token=rng.choice(vocab))
            try:
                grew = bm.append_slot(table, toks)
                toks.append(rec["token"])
                rec.update(grew=grew, table=list(table))
            except ref.block_manager.OutOfBlocks:
                rec.update(error="OutOfBlocks")
        else:
            i = rng.randrange(len(seqs))
            toks, table = seqs.pop(i)
            rec = dict(op="free", seq=i)
            bm.free_table(table)
        rec.update(num_free=bm.num_free(), hits=bm.prefix_hits, queries=bm.prefix_queries,
                   free_ids=list(bm.free_ids), evictable=list(bm.evictable),
                   ref_counts=[b.ref_count for b in bm.blocks])
        ops.append(rec)
    return ops


def sched_trace(ref, seed=0):
    """Random arrivals, decodes and finishes; each step records the new
    request (if any), the batch, the tokens appended and the queues."""
    rng = random.Random(seed)
    ecfg = ref.config.EngineConfig(block_size=4, num_blocks=20, enable_prefix_caching=True,
                                   max_batch_tokens=40, max_running=5)
    bm = ref.block_manager.BlockManager(20, 4, True)
    s = ref.scheduler.Scheduler(ecfg, bm)
    reqs = []
    trace = []
    for _ in range(120):
        new = None
        if rng.random() < 0.4:
            n = rng.randint(2, 22)
            new = ([rng.choice([5, 6]) for _ in range(n)], rng.randint(1, 12))
            r = ref.scheduler.Request(prompt_token_ids=list(new[0]), max_new_tokens=new[1])
            reqs.append(r)
            s.add(r)
        idx = {r.req_id: i for i, r in enumerate(reqs)}
        b = s.schedule()
        rec = dict(new=new, prefill=[idx[r.req_id] for r in b.prefill],
                   decode=[idx[r.req_id] for r in b.decode],
                   tables=[list(r.block_table) for r in b.prefill + b.decode],
                   cached=[r.num_cached_tokens for r in b.prefill], appended=[])
        for r in b.prefill + b.decode:
            t = rng.choice([5, 6, 7])
            rec["appended"].append(t)
            r.output_token_ids.append(t)
            if len(r.output_token_ids) >= r.max_new_tokens:
                s.finish(r)
        rec.update(waiting=[idx[r.req_id] for r in s.waiting],
                   running=[idx[r.req_id] for r in s.running],
                   preemptions=[r.preemptions for r in reqs], num_free=bm.num_free())
        trace.append(rec)
    return trace


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--skip-05b", action="store_true")
    ap.add_argument("--update", nargs="*", default=None,
                    help="recompute only these cases, keep the rest of golden.pt")
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    import tinybatch as _pkg  # noqa: F401
    import tinybatch.block_manager
    import tinybatch.config
    import tinybatch.kv_cache
    import tinybatch.model
    import tinybatch.scheduler
    import tinybatch.tensor_parallel
    ref = sys.modules["tinybatch"]
    torch.set_num_threads(8)
    path = Path(__file__).parent / "golden.pt"
    only = set(args.update) if args.update is not None else None
    out: dict = torch.load(path, weights_only=False) if only is not None else {}

    def want(name: str) -> bool:
        return only is None or name in only

    # ---- tp_gate
    if want("tp_gate"):
        from tinybatch_b200.config import ModelConfig
        cfg = ModelConfig(n_layers=2, d_model=1024, n_heads=16, n_kv_heads=8, head_dim=64,
                          d_ff=2048, vocab_size=512, rope_theta=1e6, rms_eps=1e-6,
                          tie_embeddings=False, max_position=4096)
        w = synthetic_weights(cfg, seed=7, dtype=torch.bfloat16)
        w = {k: v.to(torch.float32) for k, v in w.items()}
        ids = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(7))
        rc = ref_cfg(ref, cfg)
        l1 = ref.tensor_parallel.tp_forward(ids, w, rc, world=1)
        l2, st2 = ref.tensor_parallel.run_tp_forward(2, w, rc, ids, port=29617)
        out["tp_gate"] = dict(cfg={k: getattr(cfg, k) for k in cfg.__dataclass_fields__},
                              seed=7, ids=ids.tolist(), fingerprint=fingerprint(w),
                              logits_w1=l1, logits_w2=l2,
                              stats_w2={k: st2[k] for k in ("calls", "bytes")})
    if only is not None:
        torch.save(out, path)
        print(f"updated {sorted(only)} in {path} ({path.stat().st_size / 1024:.0f} KiB)")
        return

    # ---- tiny_tp
    cfg = named_config("tiny")
    w = synthetic_weights(cfg, seed=0)
    ids = torch.randint(0, cfg.vocab_size, (16,), generator=torch.Generator().manual_seed(0))
    rc = ref_cfg(ref, cfg)
    l1 = ref.tensor_parallel.tp_forward(ids, w, rc, world=1)
    l2, st2 = ref.tensor_parallel.run_tp_forward(2, w, rc, ids, port=29611)
    kv = ref.kv_cache.PagedKVCache(cfg.n_layers, 8, 16, cfg.n_kv_heads, cfg.head_dim,
                                   torch.device("cpu"), torch.float32)
    lp = ref_model(ref, cfg, w).forward(ids, torch.arange(16), [(0, 16)], [[5]], [16], kv)
    out["tiny_tp"] = dict(cfg="tiny", seed=0, ids=ids.tolist(), fingerprint=fingerprint(w),
                          logits_w1=l1, logits_w2=l2,
                          stats_w2={k: st2[k] for k in ("calls", "bytes")}, paged_last=lp)

    # ---- ref_test
    cfg = named_config("ref-test")
    w = reference_test_weights(cfg, seed=0)
    ids = torch.randint(0, cfg.vocab_size, (24,), generator=torch.Generator().manual_seed(1))
    rc = ref_cfg(ref, cfg)
    l1 = ref.tensor_parallel.tp_forward(ids, w, rc, world=1)
    l2, st2 = ref.tensor_parallel.run_tp_forward(2, w, rc, ids, port=29613)
    out["ref_test"] = dict(cfg="ref-test", seed=0, ids=ids.tolist(), fingerprint=fingerprint(w),
                           logits_w1=l1, logits_w2=l2,
                           stats_w2={k: st2[k] for k in ("calls", "bytes")})

    # ---- paged engine runs on the tiny model
    cfg = named_config("tiny")
    w = synthetic_weights(cfg, seed=0)
    rng = random.Random(7)
    shared = [rng.randrange(cfg.vocab_size) for _ in range(32)]
    # prompt lengths avoid multiples of the block size: the reference engine
    # has no block for the first decode token of such a prompt (its
    # append_slot reserves the position after the one being written)
    suffix = [n + (n % 16 == 0) for n in (rng.randint(1, 20) for _ in range(3))]
    prompts = [shared + [rng.randrange(256) for _ in range(n)] for n in suffix]
    prompts += [[rng.randrange(256) for _ in range(n)] for n in (5, 17, 47)]
    max_new = [6, 9, 4, 12, 7, 5]
    out["paged_bs16"] = engine_run(ref, cfg, w, prompts, max_new, block_size=16,
                                   num_blocks=64, max_batch_tokens=96, max_running=4)
    rng = random.Random(11)
    prompts = [[rng.randrange(256) for _ in range(n)] for n in (9, 14, 6, 11)]
    prompts.append(prompts[0][:8] + [3, 4])
    out["paged_small"] = engine_run(ref, cfg, w, prompts, [10, 8, 12, 6, 7], block_size=4,
                                    num_blocks=12, max_batch_tokens=64, max_running=5)

    # ---- host bookkeeping traces
    out["bm_trace"] = bm_trace(ref)
    out["sched_trace"] = sched_trace(ref)

    # ---- 0.5B-shaped probe
    if not args.skip_05b:
        cfg = named_config("qwen2.5-0.5b")
        # config 2 specifies bf16 weights: the reference runs its fp32
        # forward on the bf16-valued draw
        w = synthetic_weights(cfg, seed=1)
        w = {k: v.to(torch.bfloat16).to(torch.float32) for k, v in w.items()}
        rng = random.Random(5)
        p0 = [rng.randrange(cfg.vocab_size) for _ in range(40)]
        p1 = [rng.randrange(cfg.vocab_size) for _ in range(17)]
        bs = 16
        kv = ref.kv_cache.PagedKVCache(cfg.n_layers, 16, bs, cfg.n_kv_heads, cfg.head_dim,
                                       torch.device("cpu"), torch.float32)
        tables = [[3, 7, 1], [9, 2]]
        m = ref_model(ref, cfg, w)
        ids = torch.tensor(p0 + p1)
        pos = torch.tensor(list(range(40)) + list(range(17)))
        pre = m.forward(ids, pos, [(0, 40), (40, 57)], tables, [40, 17], kv)
        nxt = [int(pre[0].argmax()), int(pre[1].argmax())]
        dec = m.forward(torch.tensor(nxt), torch.tensor([40, 17]), [(0, 1), (1, 2)],
                        tables, [41, 18], kv)
        sample = torch.randperm(cfg.vocab_size, generator=torch.Generator().manual_seed(3))[:4096].clone()
        summ = {}
        for name, lg in (("prefill", pre), ("decode", dec)):
            top = lg.topk(64, dim=-1)
            summ[name] = dict(top_idx=top.indices, top_val=top.values,
                              sample=lg[:, sample].clone(), argmax=lg.argmax(-1))
        out["qwen05b"] = dict(cfg="qwen2.5-0.5b", seed=1, prompts=[p0, p1], tables=tables,
                              next_ids=nxt, sample_idx=sample, fingerprint_embed=float(
                                  w["model.embed_tokens.weight"].double().abs().sum()),
                              **summ)

    torch.save(out, path)
    print(f"wrote {path} ({path.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
