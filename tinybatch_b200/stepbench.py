"""Tensor-parallel decode-step timing on a few full-width layers.

    torchrun --nproc-per-node T -m tinybatch_b200.stepbench [--layers L] [--reps R]

The Qwen2.5-14B layer shapes cut to L decoder layers (default 8: ~2.5 GB of
weights per rank at T = 2, far beyond the L2, so every step streams them from
HBM as the full model does), bf16 weights N(0, 0.02) seed 3, sharded over the
T ranks with the fused row-parallel exchange; 128 sequences decoding one
token each with the 14B benchmark's context lengths (prompt lengths uniform in
[128, 2048], seed 3, plus 8 generated tokens), block size 16, KV pool filled
with random values.  One decode step (embedding, L layers, vocabulary-parallel
head, argmax) is captured as a CUDA graph and replayed R times back to back;
printed: the device time per step and per layer (CUDA events, max over
ranks) and the device status word.  A cheap stand-in for ``bench.py`` when
comparing builds of the per-layer kernels and the exchange.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import random

import torch
import torch.distributed as dist

from . import _native
from .comm import TPComm
from .config import named_config
from .model import Qwen2Paged
from .runtime import DecodeGraph, StepMeta
from .weights import synthetic_rank_weights

N_SEQ = 128
BLOCK = 16
SEED = 3


def run(layers: int, reps: int) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    cfg = named_config("qwen2.5-14b", n_layers=layers)
    comm = TPComm.from_process_group(dev, n_cols=cfg.d_model, max_rows=2 * N_SEQ) \
        if world > 1 else None
    w = synthetic_rank_weights(cfg, SEED, rank, world, device=dev)
    model = Qwen2Paged.from_weights(cfg, w, device=dev, rank=rank, world=world, comm=comm,
                                    max_tokens=2 * N_SEQ, max_seqs=N_SEQ, sharded=True)
    del w
    torch.cuda.empty_cache()
    rng = random.Random(SEED)
    ctx = [rng.randint(128, 2048) + 8 for _ in range(N_SEQ)]
    tables, nb = [], 0
    for c in ctx:
        k = -(-c // BLOCK)
        tables.append(list(range(nb, nb + k)))
        nb += k
    cache = model.make_kv_cache(nb, BLOCK)
    g = torch.Generator(device=dev).manual_seed(SEED)
    for pool in cache.pools:
        pool.copy_(torch.randn(pool.shape, generator=g, device=dev).mul_(0.5))
    bt_width = 4096 // BLOCK + 1
    graph = DecodeGraph(model.dm, cache.pools, N_SEQ, bt_width, 4096, BLOCK, ctx_total=sum(ctx))
    ids = [rng.randrange(cfg.vocab_size) for _ in ctx]
    md = StepMeta(ids, [c - 1 for c in ctx], [(i, i + 1) for i in range(N_SEQ)], tables, ctx,
                  BLOCK, cfg.n_heads // cfg.n_kv_heads, dev, bt_width=bt_width)
    graph.run(md)
    for _ in range(5):
        graph.graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.graph.replay()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    status = _native.status(clear=True)
    del graph
    if comm is not None:
        comm.close()
    ms = float(t.item())
    if rank != 0:
        return None
    return {"tp": world, "layers": layers, "sequences": N_SEQ, "reps": reps,
            "ms_per_step": round(ms, 4), "us_per_layer": round(ms * 1e3 / layers, 2),
            "status": status}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--reps", type=int, default=40)
    ap.add_argument("--tag", default="")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    r = run(args.layers, args.reps)
    if r is not None:
        r["tag"] = args.tag
        print(json.dumps(r), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
