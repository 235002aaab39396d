"""Decode throughput of the tensor-parallel paged Qwen2 layer stack on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 14b|0.5b|72b]

Default workload (``--config 14b``, the headline): the Qwen2.5-14B shape (48
layers, d 5120, 40 q / 8 kv heads, hd 128, ff 13824, vocab 152064), bf16
weights N(0, 0.02) drawn on each GPU from seed 3 (random init: no checkpoint
exists offline; each rank draws only its own slices), 128 requests with
prompt lengths uniform in [128, 2048] of random ids (seed 3), 256 output
tokens each, greedy, block_size 16.  TP = N (one process per GPU,
``torchrun``).

A step is one decode step of all 128 running sequences (128 new tokens).
Prefill of the prompts runs first, untimed.  Then:
  value  K back-to-back decode steps on the device with every step's
         metadata already in HBM; the sampled ids feed the next step on the
         device (device-to-device copy); CUDA events, max over ranks
  e2e    K more steps through ``LLMEngine.step`` (host scheduler, pinned
         host->device metadata copy, forward, argmax, device->host ids) with
         ``overlap_steps``: each call queues the next decode step before it
         reads the current one's ids, so the host work of a step runs while
         the device computes; the step still queued after the K-th call is
         collected (``drain``) inside the timed region and counted
The weights (29 GB) and the KV cache stream from HBM every step, far larger
than the 126 MB L2, so no flush is needed between steps.

``--config 0.5b`` (Qwen2.5-0.5B shape, 32 requests, prompts U[32, 512],
outputs U[16, 256], seed 1, TP 1 or 2) and ``--config 72b`` (Qwen2.5-72B
shape, 256 requests sharing one 1024-token prefix plus suffixes U[32, 256],
outputs U[16, 256], prefix caching on, seed 4, TP 8) run the whole workload
through ``LLMEngine`` with continuous batching, as the reference's own
benchmark does: value = generated tokens / wall time of the run.

Parity gate (every run, before timing; a breach prints the line and exits 1):
  forward  a model whose heads and d_ff divide 1..8 ranks (the golden case
           ``tp_gate``), sharded over the N ranks through ``tp_forward``,
           against the logits the reference itself produced for it
           (tests/golden/golden.pt): max-abs <= 2e-2, argmax agreement, the
           logits identical on every rank
  fused    (N > 1) one fused row-parallel GEMM + all-reduce call at M = 128,
           5120 x 5120, one-shot and two-shot, against an fp32 sum of the same
           bf16 inputs (torch on the GPU): the error beyond one bf16 rounding
           of the reduced values <= 2e-2, and h bit-identical on every rank

CPU legs (the reference's algorithm restated in ``oracle/``, fp32, timed on
the box's host cores): one full-width decoder layer of the decode step over
the same contexts the GPU arm decodes, extrapolated to all layers, plus the
LM head (timed on an eighth of the vocabulary, x8).  At N > 1 every rank
runs its shard of the layer with a gloo all-reduce, as the reference's
``tensor_parallel.py`` does, on cores / N threads each.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BLOCK = 16

# name -> workload of one --config
WORKLOADS = {
    "14b": dict(model="qwen2.5-14b", seed=3, n_req=128, prompt=(128, 2048), out=256,
                mode="steady", prefix=False),
    "0.5b": dict(model="qwen2.5-0.5b", seed=1, n_req=32, prompt=(32, 512), out=(16, 256),
                 mode="run", prefix=False),
    "72b": dict(model="qwen2.5-72b", seed=4, n_req=256, prompt=(32, 256), out=(16, 256),
                mode="run", prefix=True, shared_prefix=1024),
}


def make_prompts(vocab: int, wl: dict) -> tuple[list[list[int]], list[int]]:
    """Prompts and output lengths of a workload (``random.Random(seed)``)."""
    rng = random.Random(wl["seed"])
    n = wl["n_req"]
    if wl.get("shared_prefix"):
        prefix = [rng.randrange(vocab) for _ in range(wl["shared_prefix"])]
        lens = [rng.randint(*wl["prompt"]) for _ in range(n)]
        prompts = [prefix + [rng.randrange(vocab) for _ in range(L)] for L in lens]
    else:
        lens = [rng.randint(*wl["prompt"]) for _ in range(n)]
        prompts = [[rng.randrange(vocab) for _ in range(L)] for L in lens]
    out = wl["out"]
    outs = [out] * n if isinstance(out, int) else [rng.randint(*out) for _ in range(n)]
    return prompts, outs


def decode_contexts(prompts: list[list[int]], warmup: int, steps: int) -> list[int]:
    """Context lengths of the steady decode steps in the middle of the timed
    region (after the prefill's first token, W warm-up steps and K/2 timed
    steps); the CPU legs time the same contexts."""
    return [len(p) + 2 + warmup + steps // 2 for p in prompts]


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def peaks() -> tuple[dict, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi samples (every 100 ms) of this GPU while the timed regions run."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)       # first sample before the timed region starts
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- CPU legs

def cpu_decode_sample(cfg, ctx_lens: list[int], rank: int = 0, world: int = 1, group=None,
                      reps: int = 2) -> dict:
    """Time the reference's algorithm (the oracle's fp32 restatement, host
    cores) on this rank's shard of one full-width decoder layer of a decode
    step for every sequence, and on an eighth of the LM head, and extrapolate
    to the whole model.  The layer is the reference's tensor-parallel layer
    (``src/tinybatch/tensor_parallel.py:86-116``) with the paged per-sequence
    attention of ``src/tinybatch/model.py:131-147``; the row-parallel partial
    sums go through ``dist.all_reduce`` on the gloo ``group`` when world > 1.
    The head is replicated on every rank, as the reference computes it.
    Returns the per-rank times and tokens/s (max over ranks)."""
    import torch.distributed as dist

    from oracle import qwen2_ref as R
    gen = torch.Generator().manual_seed(0)
    d, hd = cfg.d_model, cfg.head_dim
    nh, nkv, ff = cfg.n_heads // world, cfg.n_kv_heads // world, cfg.d_ff // world

    def rnd(*shape):
        return torch.randn(*shape, generator=gen) * 0.02

    # the rank's slices (random values: only the time is measured)
    wq, bq = rnd(nh * hd, d), rnd(nh * hd)
    wk, bk = rnd(nkv * hd, d), rnd(nkv * hd)
    wv, bv = rnd(nkv * hd, d), rnd(nkv * hd)
    wo, wg, wu, wd = rnd(d, nh * hd), rnd(ff, d), rnd(ff, d), rnd(d, ff)
    ones = torch.ones(d)
    n = len(ctx_lens)
    tables, nb = [], 0
    for c in ctx_lens:
        k = -(-c // BLOCK)
        tables.append(list(range(nb, nb + k)))
        nb += k
    pool = torch.randn(nb, 2, nkv, BLOCK, hd, generator=gen) * 0.5
    h = torch.randn(n, d, generator=gen)
    positions = torch.tensor([c - 1 for c in ctx_lens])
    slices = [(i, i + 1) for i in range(n)]
    v8 = -(-cfg.vocab_size // 8)
    head = torch.full((v8, d), 0.01)

    def allreduce(x):
        if world > 1:
            dist.all_reduce(x, op=dist.ReduceOp.SUM, group=group)
        return x

    def layer(h):
        x = R.rms_norm(h, ones, cfg.rms_eps)
        q = R.rope(R.linear(x, wq, bq).view(n, nh, hd), positions, cfg.rope_theta)
        k = R.rope(R.linear(x, wk, bk).view(n, nkv, hd), positions, cfg.rope_theta)
        v = R.linear(x, wv, bv).view(n, nkv, hd)
        R.kv_write(pool, k, v, positions, slices, tables, BLOCK)
        attn = torch.empty(n, nh * hd)
        for i, (table, ctx) in enumerate(zip(tables, ctx_lens)):
            keys, vals = R.kv_gather(pool, table, ctx)
            attn[i] = R.attention(q[i:i + 1], keys, vals, first_pos=ctx - 1).reshape(-1)
        h = h + allreduce(R.linear(attn, wo))
        x = R.rms_norm(h, ones, cfg.rms_eps)
        a = torch.nn.functional.silu(R.linear(x, wg)) * R.linear(x, wu)
        return h + allreduce(R.linear(a, wd))

    t_layer, t_head = [], []
    for _ in range(reps):
        t0 = time.perf_counter()
        layer(h)
        t1 = time.perf_counter()
        R.linear(R.rms_norm(h, ones, cfg.rms_eps), head)
        t2 = time.perf_counter()
        t_layer.append(t1 - t0)
        t_head.append((t2 - t1) * cfg.vocab_size / v8)
    times = torch.tensor([min(t_layer), min(t_head)], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX, group=group)
    layer_s, head_s = float(times[0]), float(times[1])
    step_s = cfg.n_layers * layer_s + head_s
    return {"layer_s": layer_s, "lm_head_s": head_s, "step_s": step_s,
            "tokens_per_s": n / step_s, "sample_s": sum(t_layer) / reps + sum(t_head) / reps / 8}


def cpu_baseline_line(cfg, ctx, rank, world, group, threads) -> dict:
    torch.set_num_threads(threads)
    info = cpu_decode_sample(cfg, ctx, rank, world, group)
    tp = f"TP={world} over gloo, " if world > 1 else ""
    return {"value": info["tokens_per_s"], "unit": "tokens/s", "cores": threads * world,
            "threads_per_rank": threads, "kind": "port",
            "extrapolated_from": f"1 full-width layer x{cfg.n_layers} + LM head "
                                 "(timed on 1/8 of the vocabulary, x8)",
            "layer_s": round(info["layer_s"], 4), "lm_head_s": round(info["lm_head_s"], 4),
            "sample": f"{tp}one fp32 decoder layer for all {len(ctx)} sequences (paged KV "
                      "gather + SDPA as the reference), contexts of the timed steps"}


def run_reference(args) -> None:
    """The reference's algorithm for this path on the host cores (its fp32
    restatement in oracle/; the reference itself is Python and is not on the
    GPU box).  Each step times one full-width layer of the decode step and an
    eighth of the LM head (the faster of two samples, as the GPU arm's CPU
    leg does); ``value`` extrapolates to the whole model."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from tinybatch_b200.config import named_config
    wl = WORKLOADS[args.config]
    cfg = named_config(wl["model"])
    threads = host_cores()
    torch.set_num_threads(threads)
    prompts, _ = make_prompts(cfg.vocab_size, wl)
    ctx = decode_contexts(prompts, args.warmup, args.steps)
    for _ in range(args.warmup):
        cpu_decode_sample(cfg, ctx, reps=1)
    infos, walls = [], []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        infos.append(cpu_decode_sample(cfg, ctx))     # min of two samples, as the CPU leg
        walls.append(time.perf_counter() - t0)
    value = statistics.median(i["tokens_per_s"] for i in infos)
    layer_s = statistics.median(i["layer_s"] for i in infos)
    head_s = statistics.median(i["lm_head_s"] for i in infos)
    line = {
        "impl": "reference", "metric": "decode_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # a step is one bounded sample (one layer + 1/8 of the head); value
        # extrapolates it to the whole decode step
        "ms_per_step": 1e3 * statistics.mean(walls),
        "extrapolated_ms_per_decode_step": 1e3 * (cfg.n_layers * layer_s + head_s),
        "extrapolated_from": f"1 full-width layer x{cfg.n_layers} + LM head (timed on 1/8 of "
                             "the vocabulary, x8)",
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"{wl['model']} decode, {len(prompts)} requests, TP=1 on host "
                               "cores, contexts of the GPU arm's timed steps"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "layer_s": round(layer_s, 4), "lm_head_s": round(head_s, 4),
                         "sample": "per step: one full-width fp32 decoder layer for all "
                                   f"{len(prompts)} sequences (paged KV gather + SDPA as the "
                                   "reference) + 1/8 of the LM head, faster of two samples"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU arm

def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_over_ranks(x: float, world: int, op: str = "max") -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.MIN)
    return float(t.item())


def same_on_all_ranks(t: torch.Tensor, world: int) -> bool:
    """Whether tensor t (on this rank's GPU) is bit-identical on every rank."""
    if world == 1:
        return True
    import torch.distributed as dist
    words = t.contiguous().view(-1).view(torch.int32).to(torch.int64)
    idx = torch.arange(words.numel(), device=words.device, dtype=torch.int64)
    sig = torch.stack([words.sum(), (words * (idx % 65521 + 1)).sum()])
    allsig = [torch.empty_like(sig) for _ in range(world)]
    dist.all_gather(allsig, sig)
    return all(torch.equal(s, allsig[0]) for s in allsig)


def parity_gate(rank: int, world: int, dev) -> dict:
    """The checks described in the module docstring; every rank takes part."""
    from tinybatch_b200.config import ModelConfig
    from tinybatch_b200.tensor_parallel import release, shard_weights, tp_forward
    from tinybatch_b200.weights import synthetic_weights
    gold = torch.load(os.path.join(ROOT, "tests", "golden", "golden.pt"),
                      weights_only=False)["tp_gate"]
    cfg = ModelConfig(**gold["cfg"])
    w = synthetic_weights(cfg, gold["seed"], dtype=torch.bfloat16)
    shard = shard_weights(w, cfg, rank, world)
    stats = {"calls": 0, "bytes": 0, "seconds": 0.0}
    logits = tp_forward(torch.tensor(gold["ids"], device=dev), shard, cfg, world,
                        stats if world > 1 else None)
    torch.cuda.synchronize()
    ident = same_on_all_ranks(logits, world)
    release()
    ref = gold["logits_w1"].to(dev)
    err = float((logits - ref).abs().max())
    agree = float((logits.argmax(-1) == ref.argmax(-1)).float().mean()) * 100
    top2 = ref.topk(2, dim=-1).values
    decisive = (top2[:, 0] - top2[:, 1]) > 2 * err
    dec_ok = bool((logits.argmax(-1) == ref.argmax(-1))[decisive].all())
    out = {"forward": {"model": "tp_gate (2 layers, d 1024, 16/8 heads, ff 2048, vocab 512)",
                       "reference": "tests/golden/golden.pt, logits of the reference's own run",
                       "tokens": len(gold["ids"]),
                       "max_abs": reduce_over_ranks(err, world),
                       "argmax_agree_pct": reduce_over_ranks(agree, world, "min"),
                       "decisive_argmax_ok": bool(reduce_over_ranks(float(dec_ok), world, "min")),
                       "logits_identical_across_ranks": ident,
                       "allreduce_calls": stats["calls"] if world > 1 else 0,
                       "allreduce_seconds": stats["seconds"] if world > 1 else 0.0}}
    ok = out["forward"]["max_abs"] <= 2e-2 and out["forward"]["decisive_argmax_ok"] and ident
    if world > 1:
        from tinybatch_b200 import _native, ops
        from tinybatch_b200.comm import TPComm
        from tinybatch_b200.runtime import plan_gemm
        M, N, K = 128, 5120, 5120
        kt = K // world
        g = torch.Generator(device=dev).manual_seed(2)
        xs = [torch.randn(M, kt, generator=g, device=dev).to(torch.bfloat16) for _ in range(world)]
        ws = [(torch.randn(N, kt, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
              for _ in range(world)]
        h0 = torch.randn(M, N, generator=g, device=dev)
        gn = torch.ones(N, dtype=torch.bfloat16, device=dev)
        ref = h0.clone()
        for r in range(world):                      # the all-reduce SUM in rank order
            ref += xs[r].float() @ ws[r].float().t()
        comm = TPComm.from_process_group(dev, n_cols=N, max_rows=M)
        bn, splits = plan_gemm(M, N, kt)
        fused = {}
        try:
            for two_shot in (False, True):
                h = h0.clone()
                hg = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
                sq = torch.empty(ops.row_parts(N, bn, splits), M, device=dev)
                comm.row_linear_residual(xs[rank], ws[rank], h, gn, hg, sq, bn=bn, splits=splits,
                                         two_shot=two_shot)
                torch.cuda.synchronize()
                code = _native.status(clear=True)
                excess = float(((h - ref).abs() - 2.0 ** -8 * (ref - h0).abs()).max())
                sq_err = float(((sq.sum(0) - ref.square().sum(1)).abs()
                                / ref.square().sum(1)).max())
                key = "two_shot" if two_shot else "one_shot"
                fused[key] = {"excess_over_bf16_rounding": reduce_over_ranks(excess, world),
                              "sumsq_rel_err": reduce_over_ranks(sq_err, world),
                              "status": int(reduce_over_ranks(float(code), world)),
                              "h_bitident_across_ranks": same_on_all_ranks(h, world)}
                f = fused[key]
                ok = ok and f["excess_over_bf16_rounding"] <= 2e-2 and f["sumsq_rel_err"] <= 1e-3 \
                    and f["status"] == 0 and f["h_bitident_across_ranks"]
        finally:
            comm.close()
        out["fused_row_gemm_allreduce"] = {"M": M, "N": N, "K": K, "bn": bn, "splits": splits,
                                           **fused}
    out["ok"] = bool(ok)
    torch.cuda.empty_cache()
    return out


def build_model(wl, cfg, rank, world, dev, max_tokens, comm):
    from tinybatch_b200.model import Qwen2Paged
    from tinybatch_b200.weights import synthetic_rank_weights
    w = synthetic_rank_weights(cfg, wl["seed"], rank, world, device=dev)
    model = Qwen2Paged.from_weights(cfg, w, device=dev, rank=rank, world=world, comm=comm,
                                    max_tokens=max_tokens, max_seqs=wl["n_req"], sharded=True)
    del w
    torch.cuda.empty_cache()
    return model


def kernel_breakdown(prof: list, pk: dict) -> dict:
    kinds: dict[str, dict] = {}
    for kind, s, e, nbytes, flops in prof:
        k = kinds.setdefault(kind, {"launches": 0, "ms": 0.0, "bytes": 0.0, "flops": 0.0})
        k["launches"] += 1
        k["ms"] += s.elapsed_time(e)
        k["bytes"] += nbytes
        k["flops"] += flops
    total_ms = sum(k["ms"] for k in kinds.values()) or 1.0
    for k in kinds.values():
        k["share"] = k["ms"] / total_ms
        k["GBps"] = k["bytes"] / (k["ms"] / 1e3) / 1e9 if k["ms"] else None
        k["TFLOPs"] = k["flops"] / (k["ms"] / 1e3) / 1e12 if k["ms"] else None
        k["hbm_frac"] = k["GBps"] / pk["hbm_gbs"] if k["GBps"] else None
    return kinds


def run_ours(args) -> None:
    from tinybatch_b200.config import EngineConfig, named_config
    from tinybatch_b200.engine import LLMEngine

    rank, world, local = setup_dist()
    dev = torch.device("cuda", local)
    wl = WORKLOADS[args.config]
    cfg = named_config(wl["model"])

    gate = parity_gate(rank, world, dev)
    if not gate["ok"]:
        if rank == 0:
            print(json.dumps({"metric": "decode_tokens_per_s", "value": None, "n_gpus": world,
                              "error": "parity gate failed", "parity": gate}), flush=True)
        sys.exit(1)

    comm = None
    if world > 1:
        from tinybatch_b200.comm import TPComm
        comm = TPComm.from_process_group(dev, n_cols=cfg.d_model, max_rows=args.max_batch_tokens)
    model = build_model(wl, cfg, rank, world, dev, args.max_batch_tokens, comm)
    prompts, outs = make_prompts(cfg.vocab_size, wl)
    if wl["mode"] == "run":
        run_workload(args, wl, cfg, rank, world, local, dev, model, prompts, outs, gate)
    else:
        run_steady(args, wl, cfg, rank, world, local, dev, model, prompts, gate)
    if world > 1:
        import torch.distributed as dist
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def _cpu_leg(args, cfg, ctx, rank, world):
    """The CPU baseline: rank 0 alone at N=1, every rank (gloo) at N>1."""
    if args.skip_cpu:
        return None
    cores = host_cores()
    if world == 1:
        return cpu_baseline_line(cfg, ctx, 0, 1, None, cores)
    import torch.distributed as dist
    group = dist.new_group(backend="gloo")
    line = cpu_baseline_line(cfg, ctx, rank, world, group, max(1, cores // world))
    dist.destroy_process_group(group)
    return line


def prefill_flops(cfg, prompt_lens: list[int]) -> float:
    """Algorithmic flop of prefilling the prompts with no cached prefix: the
    projections (2 x tokens x weights per layer), causal attention
    (4 x head_dim x q heads x visible query-key pairs per layer) and the LM
    head on each prompt's last token."""
    hd, d = cfg.head_dim, cfg.d_model
    per_tok = 2 * (d * (cfg.n_heads + 2 * cfg.n_kv_heads) * hd + cfg.n_heads * hd * d
                   + 3 * d * cfg.d_ff)
    tokens = sum(prompt_lens)
    pairs = sum(p * (p + 1) // 2 for p in prompt_lens)
    return float(cfg.n_layers * (per_tok * tokens + 4 * hd * cfg.n_heads * pairs)
                 + 2 * cfg.vocab_size * d * len(prompt_lens))


def run_steady(args, wl, cfg, rank, world, local, dev, model, prompts, gate) -> None:
    from tinybatch_b200.config import EngineConfig
    from tinybatch_b200.engine import LLMEngine
    from tinybatch_b200.runtime import StepMeta

    n_req, out_tokens = wl["n_req"], wl["out"]
    num_blocks = sum(-(-(len(p) + out_tokens + 1) // BLOCK) for p in prompts) + 64
    ecfg = EngineConfig(block_size=BLOCK, num_blocks=num_blocks, enable_prefix_caching=False,
                        max_batch_tokens=args.max_batch_tokens, max_running=n_req,
                        max_model_len=4096, max_new_tokens=out_tokens, device=str(dev),
                        overlap_steps=True)
    eng = LLMEngine(ecfg, model=model)
    reqs = [eng.add_request_ids(p, max_new_tokens=out_tokens) for p in prompts]

    # prefill (untimed): until every request runs and the batch is decode-only
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    prefill_steps = 0
    while eng.scheduler.waiting or any(len(r.output_token_ids) == 0 for r in reqs):
        eng.step()
        prefill_steps += 1
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    prompt_tokens = sum(len(p) for p in prompts)

    for _ in range(args.warmup):
        eng.step()
    eng.drain()        # no step queued across the boundary of a timed region
    assert all(len(r.output_token_ids) + args.steps * 2 + 2 < out_tokens for r in reqs)

    # ---- value: K device-resident decode steps, each one CUDA-graph replay
    graph = eng.decode_graph(n_req)
    group = cfg.n_heads // cfg.n_kv_heads
    metas, placeholders = [], []
    for _ in range(args.steps):
        batch = eng.scheduler.schedule()
        assert not batch.prefill and len(batch.decode) == n_req
        ids, pos, slices, tables, ctx = eng.build_batch(batch)
        md = StepMeta(ids, pos, slices, tables, ctx, BLOCK, group, dev, bt_width=eng._bt_width)
        assert graph.matches(md)
        metas.append(md)
        for r in batch.decode:
            r.output_token_ids.append(-1)           # replaced by the device's sample below
        placeholders.append(list(batch.decode))
    torch.cuda.synchronize()
    hist = torch.empty(args.steps, n_req, dtype=torch.int32, device=dev)
    nxt = model.dm.next_ids
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")     # profilers select the timed steps by this range
        start.record()
        for k, md in enumerate(metas):
            graph.dest.copy_(md.buf)
            graph.md.ids.copy_(nxt[:n_req])
            graph.graph.replay()
            hist[k].copy_(nxt[:n_req])
        end.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        barrier(world)
        h = hist.cpu().tolist()
        for k, batch in enumerate(placeholders):
            for j, r in enumerate(batch):
                idx = len(r.output_token_ids) - args.steps + k
                r.output_token_ids[idx] = h[k][j]

        # ---- e2e: K steps through the public engine API (host buffers, copies inside)
        torch.cuda.synchronize()
        barrier(world)
        t_e2e0 = time.perf_counter()
        e0.record()
        # overlapped engine steps: each call queues the next decode step before
        # reading this one's tokens; the step still queued after the last call
        # is collected inside the timed region and its tokens counted
        h2d = d2h = 0
        e2e_tokens = e2e_steps = 0
        for k in range(args.steps + 1):
            outs = eng.step() if k < args.steps else eng.drain()
            if outs:
                e2e_tokens += len(outs)
                e2e_steps += 1
                h2d += eng.last_h2d_bytes
                d2h += eng.last_d2h_bytes
        e1.record()
        torch.cuda.synchronize()
        wall_e2e = time.perf_counter() - t_e2e0
    dt = reduce_over_ranks(start.elapsed_time(end) / 1e3, world)
    dt_e2e = reduce_over_ranks(max(e0.elapsed_time(e1) / 1e3, 0.0), world)
    value = n_req * args.steps / dt
    e2e = e2e_tokens / dt_e2e
    graph_launches = args.steps * (5 * cfg.n_layers + 3)

    # ---- per-kernel device times: one eager decode step queued behind a
    # sleep kernel, so every launch is enqueued before the GPU reaches it and
    # the events around each launch time the kernel, not the host
    md_prof = StepMeta([r.all_token_ids()[-1] for r in reqs], [r.context_len() - 1 for r in reqs],
                       [(i, i + 1) for i in range(n_req)], [r.block_table for r in reqs],
                       [r.context_len() for r in reqs], BLOCK, group, dev)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda._sleep(60_000_000)
    model.dm.prof = []
    model.forward_meta(md_prof, eng.kv_cache, sample=True)
    torch.cuda.synchronize()
    prof = model.dm.prof
    model.dm.prof = None
    eng.drain()

    pk, src = peaks()
    kinds = kernel_breakdown(prof, pk)
    top = max(kinds, key=lambda n: kinds[n]["ms"])
    tk = kinds[top]
    per_launch_bytes = tk["bytes"] / tk["launches"]
    per_launch_s = tk["ms"] / tk["launches"] / 1e3
    achieved = per_launch_bytes / per_launch_s / 1e9
    # DRAM bytes per launch of the top kernel: the ratio of ncu-measured
    # traffic to algorithmic bytes in a captured small case of the same
    # kernel (profiles/traffic.json), scaled to this launch's algorithmic bytes
    traffic = None
    tr_path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tr_path):
        with open(tr_path) as f:
            rec = json.load(f).get(f"{top}@tp{world}")
        if rec:
            traffic = per_launch_bytes * rec["dram_bytes_per_launch"] / rec["algorithmic_bytes_per_launch"]

    ctx = decode_contexts(prompts, args.warmup, args.steps)
    cpu = _cpu_leg(args, cfg, ctx, rank, world)
    if rank == 0:
        pf_flops = prefill_flops(cfg, [len(p) for p in prompts])
        pf_peak = pk["bf16_tflops_sustained"] * world
        line = {
            "metric": "decode_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompt ids)",
            "config": {"workload": f"{wl['model']} decode, {n_req} requests, prompts "
                                   f"U[{wl['prompt'][0]},{wl['prompt'][1]}], {out_tokens} output "
                                   f"tokens, block 16, TP={world}",
                       "tp": world, "global_batch": n_req,
                       "l2": "no flush: 29 GB of weights and the KV cache stream every step",
                       "prefill_s": round(prefill_s, 2), "prefill_steps": prefill_steps,
                       "prefill_tokens_per_s": round(prompt_tokens / prefill_s, 1)},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d // e2e_steps,
                    "d2h_bytes_per_step": d2h // e2e_steps, "wall_s": round(wall_e2e, 3),
                    "steps": e2e_steps, "overlap_steps": True},
            "gpu_launches": graph_launches,
            "roofline": {"kernel": top, "bound": "hbm", "achieved": achieved,
                         "peak": pk["hbm_gbs"], "peak_source": src, "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "traffic": traffic},
            "kernels": {n: {kk: (round(vv, 4) if isinstance(vv, float) else vv)
                            for kk, vv in k.items()} for n, k in kinds.items()},
            "clocks": clocks.summary(),
            "parity": gate,
            "prefill": {"prompts": n_req, "prompt_tokens": prompt_tokens,
                        "steps": prefill_steps, "wall_s": round(prefill_s, 3),
                        "tokens_per_s": round(prompt_tokens / prefill_s, 1),
                        "flop": pf_flops, "tflops": round(pf_flops / prefill_s / 1e12, 1),
                        "peak_tflops": pf_peak, "peak": f"bf16 sustained x {world} ({src})",
                        "frac": round(pf_flops / prefill_s / 1e12 / pf_peak, 3),
                        "timing": "host wall clock over the engine's prefill steps "
                                  "(scheduling and metadata included)"},
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)


def run_workload(args, wl, cfg, rank, world, local, dev, model, prompts, outs, gate) -> None:
    """The whole workload through LLMEngine with continuous batching (every
    request submitted at once): generated tokens / wall time, as the
    reference's benchmark reports it (``benchmarks/bench.py:88-99``)."""
    from tinybatch_b200.config import EngineConfig
    from tinybatch_b200.engine import LLMEngine

    n_req = wl["n_req"]
    num_blocks = sum(-(-(len(p) + o + 1) // BLOCK) for p, o in zip(prompts, outs)) + 64
    ecfg = EngineConfig(block_size=BLOCK, num_blocks=num_blocks,
                        enable_prefix_caching=wl["prefix"], max_batch_tokens=args.max_batch_tokens,
                        max_running=n_req, max_model_len=4096, max_new_tokens=max(outs),
                        device=str(dev), overlap_steps=not wl["prefix"])

    eng = LLMEngine(ecfg, model=model)

    def one_run():
        eng.reset()          # cold block manager and scheduler; pool and graphs kept
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        reqs = [eng.add_request_ids(p, max_new_tokens=o) for p, o in zip(prompts, outs)]
        steps = 0
        while eng.scheduler.has_work():
            eng.step()
            steps += 1
        eng.drain()                 # an overlapped step still queued
        torch.cuda.synchronize()
        wall = reduce_over_ranks(time.perf_counter() - t0, world)
        return eng, reqs, wall, steps

    one_run()            # warm-up run: captures the decode graph of every batch size
    with ClockSampler(local) as clocks:
        eng, reqs, wall, steps = one_run()
    gen = sum(len(r.output_token_ids) for r in reqs)
    value = gen / wall
    bm = eng.block_manager
    if rank == 0:
        line = {
            "metric": "generated_tokens_per_s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": 1, "ms_per_step": 1e3 * wall / steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompt ids)",
            "config": {"workload": f"{wl['model']}, {n_req} requests at once, continuous batching, "
                                   f"prefix caching {'on' if wl['prefix'] else 'off'}, TP={world}",
                       "tp": world, "prompt_tokens": sum(len(p) for p in prompts),
                       "generated_tokens": gen, "engine_steps": steps,
                       "prefix_hit_rate": round(bm.hit_rate(), 4),
                       "prefix_hits": bm.prefix_hits, "prefix_queries": bm.prefix_queries},
            "e2e": {"value": value, "unit": "tokens/s", "note": "the run is end to end: host "
                    "scheduler, metadata copies and sampled ids inside the wall time"},
            "clocks": clocks.summary(),
            "parity": gate,
        }
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default="14b")
    ap.add_argument("--max-batch-tokens", type=int, default=16384)
    ap.add_argument("--skip-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
