"""How far the reference's own forward run in bf16 lands from its fp32
forward (it runs every tensor, the residual stream included, in the model
dtype).  Needs the reference source tree, like make_golden.py; prints one
line, writes nothing.

    python tests/golden/reference_bf16.py --reference-src <reference>/src \
        --config qwen2.5-14b --layers 4 --seed 3 --prompts 200,500,900,1400

Same weights and prompts as ``python -m oracle.bf16_attribution`` with the
same arguments: prefill of the prompts, then one decode step fed the fp32
run's greedy tokens (teacher-forced) on both dtypes.
"""
from __future__ import annotations

import argparse
import random
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from tests.golden.make_golden import ref_cfg  # noqa: E402
from tinybatch_b200.config import named_config  # noqa: E402
from tinybatch_b200.weights import synthetic_weights  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--config", default="qwen2.5-14b")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--prompts", default="200,500,900,1400")
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    import tinybatch.kv_cache
    import tinybatch.model
    ref = sys.modules["tinybatch"]
    torch.set_num_threads(8)
    cfg = named_config(args.config, n_layers=args.layers)
    w = synthetic_weights(cfg, args.seed, dtype=torch.bfloat16)
    rng = random.Random(args.seed)
    plens = [int(n) for n in args.prompts.split(",")]
    prompts = [[rng.randrange(cfg.vocab_size) for _ in range(n)] for n in plens]
    bs = 16
    tables, nb = [], 0
    for n in plens:
        k = -(-(n + 4) // bs)
        tables.append(list(range(nb, nb + k)))
        nb += k
    ids = torch.tensor(sum(prompts, []))
    pos = torch.tensor(sum([list(range(n)) for n in plens], []))
    sl, o = [], 0
    for n in plens:
        sl.append((o, o + n))
        o += n

    def run(dtype, nxt=None):
        m = ref.model.Qwen2Paged.__new__(ref.model.Qwen2Paged)
        m.cfg, m.device, m.dtype = ref_cfg(ref, cfg), torch.device("cpu"), dtype
        m.w = {k: v.to(dtype) for k, v in w.items()}
        kv = ref.kv_cache.PagedKVCache(cfg.n_layers, nb, bs, cfg.n_kv_heads, cfg.head_dim,
                                       torch.device("cpu"), dtype)
        pre = m.forward(ids, pos, sl, tables, plens, kv)
        nxt = pre.argmax(-1) if nxt is None else nxt
        dec = m.forward(nxt, torch.tensor(plens), [(i, i + 1) for i in range(len(plens))],
                        tables, [n + 1 for n in plens], kv)
        return [pre, dec], nxt

    f, nxt = run(torch.float32)
    b, _ = run(torch.bfloat16, nxt)
    mx = max(float((x - y).abs().max()) for x, y in zip(f, b))
    mean = sum(float((x - y).abs().mean()) for x, y in zip(f, b)) / 2
    agree = sum(int((x.argmax(-1) == y.argmax(-1)).sum()) for x, y in zip(f, b))
    print(f"reference bf16 vs fp32: max-abs {mx:.4f} mean-abs {mean:.5f} "
          f"argmax {agree}/{2 * len(plens)}")


if __name__ == "__main__":
    main()
