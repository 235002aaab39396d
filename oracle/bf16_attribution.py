"""Attribute the bf16-storage deviation of the Qwen2 forward to single
tensors (test infrastructure: CPU only, never on the product path).

    python -m oracle.bf16_attribution --config qwen2.5-14b --layers 4 --seed 3 \
        --prompts 200,500,900,1400

Runs the oracle's fp32 paged forward (prefill of the prompts, then one
decode step fed the fp32 forward's greedy tokens) and, on the same batches,
the ``emulate_bf16`` forward with every stored tensor rounded, with each
``BF16_TENSORS`` name rounded alone, and with all but one rounded.  Prints
the max-abs / mean-abs logit deviation from fp32 and the argmax agreement of
each variant.  Weights: ``synthetic_weights(cfg, seed)`` cast to bf16 (the
values the GPU path holds), then fp32.
"""
from __future__ import annotations

import argparse
import json
import random
import time

import torch

from oracle import qwen2_ref as R


def run(cfg, w, prompts, bs, emulate, forced=None):
    plens = [len(p) for p in prompts]
    tables, nb = [], 0
    for n in plens:
        k = -(-(n + 4) // bs)
        tables.append(list(range(nb, nb + k)))
        nb += k
    ids = sum(prompts, [])
    pos = sum([list(range(n)) for n in plens], [])
    sl, o = [], 0
    for n in plens:
        sl.append((o, o + n))
        o += n
    pools = R.new_pools(cfg.n_layers, nb, bs, cfg.n_kv_heads, cfg.head_dim)
    pre = R.paged_forward(cfg, w, ids, pos, sl, tables, plens, pools, bs, emulate_bf16=emulate)
    nxt = pre.argmax(-1).tolist() if forced is None else forced
    dec = R.paged_forward(cfg, w, nxt, plens, [(i, i + 1) for i in range(len(plens))], tables,
                          [n + 1 for n in plens], pools, bs, emulate_bf16=emulate)
    return [pre, dec], nxt


def main() -> None:
    from tinybatch_b200.config import named_config
    from tinybatch_b200.weights import synthetic_weights
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="qwen2.5-14b")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--prompts", default="200,500,900,1400")
    ap.add_argument("--threads", type=int, default=8)
    args = ap.parse_args()
    torch.set_num_threads(args.threads)
    cfg = named_config(args.config, n_layers=args.layers)
    w = {k: v.float() for k, v in synthetic_weights(cfg, args.seed, dtype=torch.bfloat16).items()}
    rng = random.Random(args.seed)
    prompts = [[rng.randrange(cfg.vocab_size) for _ in range(int(n))]
               for n in args.prompts.split(",")]
    ref, nxt = run(cfg, w, prompts, 16, False)
    print(f"fp32 logit std {float(ref[0].std()):.3f}", flush=True)
    variants = [("all_stored", True), ("all+p", R.BF16_TENSORS)]
    variants += [("only_" + n, {n}) for n in sorted(R.BF16_TENSORS)]
    variants += [("all_but_" + n, R.BF16_TENSORS - {n}) for n in sorted(R.BF16_TENSORS)]
    res = {}
    for name, emu in variants:
        t0 = time.time()
        out, _ = run(cfg, w, prompts, 16, emu, forced=nxt)
        mx = max(float((a - b).abs().max()) for a, b in zip(out, ref))
        mean = sum(float((a - b).abs().mean()) for a, b in zip(out, ref)) / len(out)
        agree = sum(int((a.argmax(-1) == b.argmax(-1)).sum()) for a, b in zip(out, ref))
        res[name] = {"max_abs": mx, "mean_abs": mean, "argmax_agree": agree,
                     "rows": 2 * len(prompts)}
        print(f"{name:18s} max {mx:.4f} mean {mean:.5f} argmax {agree}/{2 * len(prompts)} "
              f"({time.time() - t0:.0f} s)", flush=True)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
