"""Host-side launch planning of the runtime (no GPU): GEMM tile / split
choice and its shared-memory fit, deferred-norm part counts, the decode
split-KV policy and the metadata packing that orders decode sequences."""
from __future__ import annotations

import numpy as np
import torch

from tinybatch_b200 import ops
from tinybatch_b200.runtime import (StepMeta, cluster_fits, decode_split_tokens, plan_gemm)


def test_cluster_fit_rule():
    # one member receives splits x ceil(pairs/splits) x chunks/pair 8 KiB chunks
    assert cluster_fits(256, 6) and cluster_fits(256, 8) and cluster_fits(256, 7)
    assert cluster_fits(256, 6, paired=True) and not cluster_fits(256, 7, paired=True)
    for bn in (64, 128, 192):
        assert all(cluster_fits(bn, s, p) for s in range(2, 9) for p in (False, True))


def test_plans_respect_fit_and_k():
    for (M, N, K, paired) in [(128, 7168, 5120, True), (128, 5120, 5120, False),
                              (1, 896, 896, False), (4096, 27648, 5120, True),
                              (16, 152064, 5120, False)]:
        bn, s = plan_gemm(M, N, K, paired=paired)
        assert bn in (64, 128, 192, 256) and 1 <= s <= 8
        assert s == 1 or cluster_fits(bn, s, paired)
        assert s <= -(-K // 64)


def test_row_parts():
    assert ops.row_parts(5120, 256, 6) == 120
    assert ops.row_parts(5120, 256, 6, "global") == 20
    assert ops.row_parts(896, 128, 1) == 7


def test_decode_split_policy():
    # 128 sequences x 8 kv heads fill the GPU twice over: one CTA each
    assert decode_split_tokens(128, 8, 128 * 1100, 2304) == 2304
    # few sequences: keys cut so that about 2 x 444 CTAs run
    s = decode_split_tokens(2, 8, 2 * 32768, 32768)
    assert s % 16 == 0 and 256 <= s <= 8192
    assert 600 <= 2 * 8 * -(-32768 // s) <= 1300
    assert decode_split_tokens(1, 2, 20, 20) == 256


def test_step_meta_orders_decode_longest_first():
    ctx = [5, 40, 17, 40, 3]
    tables = [list(range(i * 3, i * 3 + 3)) for i in range(len(ctx))]
    md = StepMeta([1] * 5, [c - 1 for c in ctx], [(i, i + 1) for i in range(5)], tables, ctx,
                  16, 4, "cpu", pinned=False)
    order = md.dec_order.numpy()
    assert sorted(order.tolist()) == list(range(5))
    assert np.all(np.diff(np.asarray(ctx)[order]) <= 0)
    assert order.tolist() == [1, 3, 2, 0, 4]      # stable among equal lengths
    assert md.dec_ctx.numpy().tolist() == ctx
