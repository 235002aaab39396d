"""Per-kernel device times of one decode step at the benchmark's shapes, and
the small case the ncu captures run on.

    python -m tinybatch_b200.kernelbench [--tp T] [--layers L] [--reps R]
    python -m tinybatch_b200.kernelbench --prefill N [--prompt-len P] [--cached C]
    python -m tinybatch_b200.kernelbench --plan qkv=256x5,o=128x2 ...   (override the planner)

Workload: the Qwen2.5-14B layer shapes (d 5120, 40 q / 8 kv heads, hd 128,
ff 13824, vocab 152064) cut to ``L`` decoder layers (default 1) and sharded
as rank 0 of a ``T``-way tensor-parallel group (no exchange: the row-parallel
launches run their single-rank form), random bf16 weights (seed 3); 128
sequences decoding one token each with the benchmark's context lengths
(prompt lengths uniform in [128, 2048], seed 3, plus 8 generated tokens),
block size 16, each sequence's blocks contiguous in the pool.  About 4 GB on
the device at L = 1, so a profiler can replay any launch.

Every repetition queues one eager forward behind a sleep kernel (so the
events around each launch time the kernel, not the host) and records, per
launch kind, the device time, the algorithmic HBM bytes and the flops the
runtime attributes to it.  Printed per kind (JSON, one line each): launches
per step, microseconds per launch (median over repetitions), achieved GB/s
and TFLOP/s, and the fraction of the roofline

    T_roof = max(bytes / HBM copy bandwidth, flops / bf16 GEMM rate)

with the burst figures of MEASURED_PEAKS.json (a copy and a cuBLAS GEMM
measured on this pool's B200s).

``--prefill N``: one prefill forward of N prompts instead (lengths drawn from
the 14B benchmark's U[128, 2048] with its seed, or all ``--prompt-len`` P);
with ``--cached C`` every prompt continues a C-token prefix already in the
pool (the 72B workload's shared 1024-token prefix), so attention reads C + P
keys for the P new tokens.  Prompt tokens/s of the forward and, for
attention, causal (query, key) pairs x 4 flops per head dim against the bf16
tensor rate.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import statistics

import torch

from . import _native
from .config import named_config
from .model import Qwen2Paged
from .weights import synthetic_weights

N_SEQ = 128
BLOCK = 16
SEED = 3


def peaks() -> tuple[dict, str]:
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    path = os.path.join(root, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def context_lengths(n: int = N_SEQ, generated: int = 8) -> list[int]:
    """The benchmark's prompt lengths (same generator, same draws) plus the
    tokens generated so far."""
    rng = random.Random(SEED)
    return [rng.randint(128, 2048) + generated for _ in range(n)]


def build(tp: int, layers: int, device: torch.device):
    cfg = named_config("qwen2.5-14b", n_layers=layers)
    w = synthetic_weights(cfg, SEED, dtype=torch.bfloat16, device=device)
    model = Qwen2Paged.from_weights(cfg, w, device=device, rank=0, world=tp, comm=None,
                                    max_tokens=N_SEQ, max_seqs=N_SEQ)
    del w
    torch.cuda.empty_cache()
    ctx = context_lengths()
    tables, nb = [], 0
    for c in ctx:
        k = -(-c // BLOCK)
        tables.append(list(range(nb, nb + k)))
        nb += k
    cache = model.make_kv_cache(nb, BLOCK)
    g = torch.Generator(device=device).manual_seed(SEED)
    for pool in cache.pools:
        pool.copy_(torch.randn(pool.shape, generator=g, device=device).mul_(0.5))
    ids = torch.randint(0, cfg.vocab_size, (N_SEQ,), generator=torch.Generator().manual_seed(SEED))
    md = model.metadata(ids.tolist(), [c - 1 for c in ctx], [(i, i + 1) for i in range(N_SEQ)],
                        tables, ctx, BLOCK)
    return cfg, model, cache, md


def parse_plan(text: str | None) -> dict:
    """'qkv=256x5,o=128x2' -> {'qkv': (256, 5), 'o': (128, 2)} (tile width x
    split-K factor per projection: qkv, o, gu, down, lm)."""
    out = {}
    for item in (text or "").split(","):
        if item:
            k, v = item.split("=")
            bn, sp = v.split("x")
            out[k] = (int(bn), int(sp))
    return out


def run(tp: int = 1, layers: int = 1, reps: int = 5,
        split_tokens: int | None = None, plan: dict | None = None) -> list[dict]:
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg, model, cache, md = build(tp, layers, dev)
    model.dm.split_tokens = split_tokens
    if plan:
        planner = model.dm.plans

        def plans(T, n):
            p = planner(T, n)
            p.update(plan)
            return p
        model.dm.plans = plans
    for _ in range(2):
        model.forward_meta(md, cache, sample=True)
    torch.cuda.synchronize()
    _native.raise_on_status("kernelbench warm-up")
    times: dict[str, list[float]] = {}
    meta: dict[str, tuple[int, float, float]] = {}
    for _ in range(reps):
        torch.cuda._sleep(50_000_000)
        model.dm.prof = []
        model.forward_meta(md, cache, sample=True)
        torch.cuda.synchronize()
        per: dict[str, list] = {}
        for kind, s, e, nbytes, flops in model.dm.prof:
            per.setdefault(kind, []).append((s.elapsed_time(e) * 1e3, nbytes, flops))
        for kind, lst in per.items():
            times.setdefault(kind, []).append(sum(t for t, _, _ in lst) / len(lst))
            meta[kind] = (len(lst), sum(b for _, b, _ in lst) / len(lst),
                          sum(f for _, _, f in lst) / len(lst))
        model.dm.prof = None
    # the whole forward, launches back to back (no events between them)
    fwd = []
    for _ in range(reps):
        torch.cuda._sleep(50_000_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        model.forward_meta(md, cache, sample=True)
        e1.record()
        torch.cuda.synchronize()
        fwd.append(e0.elapsed_time(e1) * 1e3)
    _native.raise_on_status("kernelbench")
    pk, src = peaks()
    rows = [{"kernel": "forward", "tp": tp, "layers": layers,
             "plans": {k: list(v) for k, v in model.dm.plans(N_SEQ, N_SEQ).items()},
             "split_tokens": split_tokens or "auto", "launches_per_step": 1,
             "us_per_launch": round(statistics.median(fwd), 2)}]
    for kind, ts in times.items():
        n, nbytes, flops = meta[kind]
        us = statistics.median(ts)
        t_hbm = nbytes / (pk["hbm_gbs"] * 1e9)
        t_tc = flops / (pk["bf16_tflops"] * 1e12)
        bound = "hbm" if t_hbm >= t_tc else "tensor"
        rows.append({"kernel": kind, "tp": tp, "launches_per_step": n, "us_per_launch": round(us, 2),
                     "bytes_per_launch": int(nbytes), "GBps": round(nbytes / us / 1e3, 1),
                     "TFLOPs": round(flops / us / 1e6, 1), "bound": bound,
                     "us_roofline": round(max(t_hbm, t_tc) * 1e6, 2),
                     "frac": round(max(t_hbm, t_tc) * 1e6 / us, 3), "peaks": src})
    rows.sort(key=lambda r: -r["us_per_launch"] * r["launches_per_step"])
    return rows


def run_prefill(n: int, prompt_len: int | None, cached: int, tp: int = 1, layers: int = 1,
                reps: int = 3) -> list[dict]:
    dev = torch.device("cuda", torch.cuda.current_device())
    rng = random.Random(SEED)
    lens = [prompt_len or rng.randint(128, 2048) for _ in range(n)]
    T = sum(lens)
    cfg = named_config("qwen2.5-14b", n_layers=layers)
    w = synthetic_weights(cfg, SEED, dtype=torch.bfloat16, device=dev)
    model = Qwen2Paged.from_weights(cfg, w, device=dev, rank=0, world=tp, comm=None,
                                    max_tokens=T, max_seqs=n)
    del w
    torch.cuda.empty_cache()
    tables, nb = [], 0
    for L in lens:
        k = -(-(cached + L) // BLOCK)
        tables.append(list(range(nb, nb + k)))
        nb += k
    cache = model.make_kv_cache(nb, BLOCK)
    g = torch.Generator(device=dev).manual_seed(SEED)
    for pool in cache.pools:
        pool.copy_(torch.randn(pool.shape, generator=g, device=dev).mul_(0.5))
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(SEED))
    pos, slices, s0 = [], [], 0
    for L in lens:
        pos += list(range(cached, cached + L))
        slices.append((s0, s0 + L))
        s0 += L
    md = model.metadata(ids.tolist(), pos, slices, tables, [cached + L for L in lens], BLOCK)
    model.forward_meta(md, cache)
    torch.cuda.synchronize()
    _native.raise_on_status("kernelbench prefill warm-up")
    times: dict[str, list[float]] = {}
    meta: dict[str, tuple[int, float, float]] = {}
    fwd = []
    for _ in range(reps):
        torch.cuda._sleep(50_000_000)
        model.dm.prof = []
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        model.forward_meta(md, cache)
        e1.record()
        torch.cuda.synchronize()
        fwd.append(e0.elapsed_time(e1) * 1e3)
        per: dict[str, list] = {}
        for kind, s, e, nbytes, flops in model.dm.prof:
            per.setdefault(kind, []).append((s.elapsed_time(e) * 1e3, nbytes, flops))
        for kind, lst in per.items():
            times.setdefault(kind, []).append(sum(t for t, _, _ in lst) / len(lst))
            meta[kind] = (len(lst), sum(b for _, b, _ in lst) / len(lst),
                          sum(f for _, _, f in lst) / len(lst))
        model.dm.prof = None
    _native.raise_on_status("kernelbench prefill")
    pk, src = peaks()
    us_fwd = statistics.median(fwd)
    rows = [{"kernel": "prefill_forward", "tp": tp, "layers": layers, "prompts": n,
             "prompt_tokens": T, "cached_prefix": cached, "us": round(us_fwd, 1),
             "prompt_tokens_per_s": round(T / us_fwd * 1e6, 1)}]
    for kind, ts in times.items():
        n_l, nbytes, flops = meta[kind]
        us = statistics.median(ts)
        t_hbm = nbytes / (pk["hbm_gbs"] * 1e9)
        t_tc = flops / (pk["bf16_tflops"] * 1e12)
        rows.append({"kernel": kind, "tp": tp, "launches_per_step": n_l,
                     "us_per_launch": round(us, 2), "TFLOPs": round(flops / us / 1e6, 1),
                     "GBps": round(nbytes / us / 1e3, 1),
                     "bound": "hbm" if t_hbm >= t_tc else "tensor",
                     "frac": round(max(t_hbm, t_tc) * 1e6 / us, 3), "peaks": src})
    rows.sort(key=lambda r: -r.get("us_per_launch", 0) * r.get("launches_per_step", 0))
    return rows


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1, help="shard as rank 0 of this many ranks")
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--split-tokens", default=None,
                    help="decode split-KV size (default: the runtime's policy); comma list")
    ap.add_argument("--plan", default=None,
                    help="override GEMM plans, e.g. qkv=256x5,o=128x2 (tile width x splits)")
    ap.add_argument("--prefill", type=int, default=0, help="prefill N prompts instead")
    ap.add_argument("--prompt-len", type=int, default=None)
    ap.add_argument("--cached", type=int, default=0)
    args = ap.parse_args()
    if args.prefill:
        for r in run_prefill(args.prefill, args.prompt_len, args.cached, args.tp, args.layers,
                             args.reps):
            print(json.dumps(r), flush=True)
        return
    splits = [None] if args.split_tokens is None else [int(v) or None for v in
                                                       args.split_tokens.split(",")]
    for st in splits:
        for r in run(args.tp, args.layers, args.reps, st, parse_plan(args.plan)):
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
