"""Decode throughput of the tensor-parallel paged Qwen2 layer stack on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (Qwen2.5-14B shape): 48 layers, d 5120, 40 q / 8
kv heads, hd 128, ff 13824, vocab 152064, bf16 weights N(0, 0.02) drawn on
the device from seed 3 (random init: no checkpoint exists offline); 128
requests with prompt lengths uniform in [128, 2048] of random ids (seed 3),
256 output tokens each, greedy, block_size 16.  TP = N (one process per GPU,
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

CONFIG = "qwen2.5-14b"
N_REQ = 128
OUT_TOKENS = 256
PROMPT_RANGE = (128, 2048)
SEED = 3
BLOCK = 16


def make_prompts(vocab: int, n: int = N_REQ, seed: int = SEED) -> list[list[int]]:
    rng = random.Random(seed)
    lens = [rng.randint(*PROMPT_RANGE) for _ in range(n)]
    return [[rng.randrange(vocab) for _ in range(L)] for L in lens]


def peaks() -> tuple[dict, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi samples (200 ms) of this GPU during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
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
        for line in getattr(self, "lines", []):
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

def cpu_decode_sample(cfg, ctx_lens: list[int], reps: int = 1) -> tuple[float, dict]:
    """Time the oracle (the reference's algorithm, fp32, host cores) on one
    full-width decoder layer of a decode step for every sequence, plus the
    LM head, and extrapolate to the whole model: tokens/s."""
    from oracle import qwen2_ref as R
    torch.manual_seed(0)
    d, hd = cfg.d_model, cfg.head_dim
    qd, kvd = cfg.n_heads * hd, cfg.n_kv_heads * hd
    p = "model.layers.0."
    w = {p + "input_layernorm.weight": torch.ones(d), p + "post_attention_layernorm.weight": torch.ones(d),
         p + "self_attn.q_proj.weight": torch.randn(qd, d) * 0.02, p + "self_attn.q_proj.bias": torch.randn(qd) * 0.02,
         p + "self_attn.k_proj.weight": torch.randn(kvd, d) * 0.02, p + "self_attn.k_proj.bias": torch.randn(kvd) * 0.02,
         p + "self_attn.v_proj.weight": torch.randn(kvd, d) * 0.02, p + "self_attn.v_proj.bias": torch.randn(kvd) * 0.02,
         p + "self_attn.o_proj.weight": torch.randn(d, qd) * 0.02,
         p + "mlp.gate_proj.weight": torch.randn(cfg.d_ff, d) * 0.02,
         p + "mlp.up_proj.weight": torch.randn(cfg.d_ff, d) * 0.02,
         p + "mlp.down_proj.weight": torch.randn(d, cfg.d_ff) * 0.02}
    n = len(ctx_lens)
    tables, nb = [], 0
    for c in ctx_lens:
        k = -(-c // BLOCK)
        tables.append(list(range(nb, nb + k)))
        nb += k
    pool = torch.randn(nb, 2, cfg.n_kv_heads, BLOCK, hd) * 0.5
    h = torch.randn(n, d)
    positions = torch.tensor([c - 1 for c in ctx_lens])
    slices = [(i, i + 1) for i in range(n)]
    head = torch.full((cfg.vocab_size, d), 0.01)
    t_layer, t_head = [], []
    for _ in range(reps):
        t0 = time.perf_counter()
        R.paged_layer(cfg, w, 0, h, positions, slices, tables, ctx_lens, pool, BLOCK)
        t1 = time.perf_counter()
        R.linear(R.rms_norm(h, torch.ones(d), cfg.rms_eps), head)
        t2 = time.perf_counter()
        t_layer.append(t1 - t0)
        t_head.append(t2 - t1)
    step_s = cfg.n_layers * min(t_layer) + min(t_head)
    info = {"layer_s": min(t_layer), "lm_head_s": min(t_head), "step_s": step_s}
    return n / step_s, info


def run_reference(args) -> None:
    """The reference's own algorithm for this path on the host cores (the
    oracle restatement; the reference itself is Python and is not present on
    the GPU box)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from tinybatch_b200.config import named_config
    cfg = named_config(CONFIG)
    torch.set_num_threads(os.cpu_count() or 1)
    prompts = make_prompts(cfg.vocab_size)
    ctx = [len(p) + 1 for p in prompts]
    for _ in range(args.warmup):
        cpu_decode_sample(cfg, ctx)
    vals = []
    for _ in range(args.steps):
        v, info = cpu_decode_sample(cfg, ctx)
        vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": "decode_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * N_REQ / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{CONFIG} decode, {N_REQ} requests, prompts U[128,2048], TP=1 on host cores"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": "per step: one full-width fp32 decoder layer for all 128 sequences "
                                   "(paged KV gather + SDPA as the reference) + LM head, x48 layers"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args) -> None:
    from tinybatch_b200.config import EngineConfig, named_config
    from tinybatch_b200.engine import LLMEngine
    from tinybatch_b200.model import Qwen2Paged
    from tinybatch_b200.weights import synthetic_weights

    rank, world, local = setup_dist()
    dev = torch.device("cuda", local)
    cfg = named_config(CONFIG)
    comm = None
    if world > 1:
        from tinybatch_b200.comm import TPComm
        comm = TPComm.from_process_group(dev, n_cols=cfg.d_model, max_rows=args.max_batch_tokens)

    w = synthetic_weights(cfg, SEED, dtype=torch.bfloat16, device=dev)
    model = Qwen2Paged.from_weights(cfg, w, device=dev, rank=rank, world=world, comm=comm,
                                    max_tokens=args.max_batch_tokens, max_seqs=N_REQ)
    del w
    torch.cuda.empty_cache()

    prompts = make_prompts(cfg.vocab_size)
    num_blocks = sum(-(-(len(p) + OUT_TOKENS + 1) // BLOCK) for p in prompts) + 64
    ecfg = EngineConfig(block_size=BLOCK, num_blocks=num_blocks, enable_prefix_caching=False,
                        max_batch_tokens=args.max_batch_tokens, max_running=N_REQ,
                        max_model_len=4096, max_new_tokens=OUT_TOKENS, device=str(dev),
                        overlap_steps=True)
    eng = LLMEngine(ecfg, model=model)
    reqs = [eng.add_request_ids(p, max_new_tokens=OUT_TOKENS) for p in prompts]

    # prefill (untimed): until every request runs and the batch is decode-only
    t0 = time.perf_counter()
    prefill_steps = 0
    while eng.scheduler.waiting or any(len(r.output_token_ids) == 0 for r in reqs):
        eng.step()
        prefill_steps += 1
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0

    for _ in range(args.warmup):
        eng.step()
    eng.drain()        # no step queued across the boundary of a timed region
    assert all(len(r.output_token_ids) + args.steps * 2 + 2 < OUT_TOKENS for r in reqs)

    # ---- value: K device-resident decode steps, each one CUDA-graph replay
    from tinybatch_b200.runtime import StepMeta
    graph = eng.decode_graph(N_REQ)
    group = cfg.n_heads // cfg.n_kv_heads
    metas, placeholders = [], []
    for _ in range(args.steps):
        batch = eng.scheduler.schedule()
        assert not batch.prefill and len(batch.decode) == N_REQ
        ids, pos, slices, tables, ctx = eng.build_batch(batch)
        md = StepMeta(ids, pos, slices, tables, ctx, BLOCK, group, dev, bt_width=eng._bt_width)
        assert graph.matches(md)
        metas.append(md)
        for r in batch.decode:
            r.output_token_ids.append(-1)           # replaced by the device's sample below
        placeholders.append(list(batch.decode))
    torch.cuda.synchronize()
    hist = torch.empty(args.steps, N_REQ, dtype=torch.int32, device=dev)
    nxt = model.dm.next_ids
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.nvtx.range_push("timed")     # profilers select the timed steps by this range
        start.record()
        for k, md in enumerate(metas):
            graph.dest.copy_(md.buf)
            graph.md.ids.copy_(nxt[:N_REQ])
            graph.graph.replay()
            hist[k].copy_(nxt[:N_REQ])
        end.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier(world)
    dt = max_over_ranks(start.elapsed_time(end) / 1e3, world)
    h = hist.cpu().tolist()
    for k, batch in enumerate(placeholders):
        for j, r in enumerate(batch):
            idx = len(r.output_token_ids) - args.steps + k
            r.output_token_ids[idx] = h[k][j]
    value = N_REQ * args.steps / dt
    graph_launches = args.steps * (5 * cfg.n_layers + 3)

    # ---- per-kernel device times: one eager decode step queued behind a
    # sleep kernel, so every launch is enqueued before the GPU reaches it and
    # the events around each launch time the kernel, not the host
    md_prof = StepMeta([r.all_token_ids()[-1] for r in reqs], [r.context_len() - 1 for r in reqs],
                       [(i, i + 1) for i in range(N_REQ)], [r.block_table for r in reqs],
                       [r.context_len() for r in reqs], BLOCK, group, dev)
    torch.cuda.synchronize()
    torch.cuda._sleep(60_000_000)
    model.dm.prof = []
    model.forward_meta(md_prof, eng.kv_cache, sample=True)
    torch.cuda.synchronize()
    prof = model.dm.prof
    model.dm.prof = None

    # ---- e2e: K steps through the public engine API (host buffers, copies inside)
    torch.cuda.synchronize()
    barrier(world)
    t_e2e0 = time.perf_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    # overlapped engine steps: each call queues the next decode step before
    # reading this one's tokens; the step still queued after the last call is
    # collected inside the timed region and its tokens counted
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
    dt_e2e = max_over_ranks(max(e0.elapsed_time(e1) / 1e3, 0.0), world)
    wall_e2e = time.perf_counter() - t_e2e0
    e2e = e2e_tokens / dt_e2e

    # ---- per-kernel breakdown
    pk, src = peaks()
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

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.skip_cpu:
            torch.set_num_threads(os.cpu_count() or 1)
            ctx = [len(r.prompt_token_ids) + len(r.output_token_ids) for r in reqs]
            v, info = cpu_decode_sample(cfg, ctx)
            cpu = {"value": v, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                   "sample": "one full-width fp32 decoder layer of a 128-sequence decode step "
                             f"({info['layer_s']:.2f} s) + LM head ({info['lm_head_s']:.2f} s), "
                             "extrapolated x48 layers"}
        line = {
            "metric": "decode_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompt ids)",
            "config": {"workload": f"{CONFIG} decode, {N_REQ} requests, prompts U[128,2048], "
                                   f"{OUT_TOKENS} output tokens, block 16, TP={world}",
                       "tp": world, "global_batch": N_REQ,
                       "l2": "no flush: 29 GB of weights and the KV cache stream every step",
                       "prefill_s": round(prefill_s, 2), "prefill_steps": prefill_steps},
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
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
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
