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


def test_plans_follow_measured_rankings():
    """Decode shapes (M = 128) whose (bn, splits) were timed on a B200 in
    graph replay: the planner must pick the faster of each measured pair.
    o_proj TP=1: (128, 3) 16.1 us vs (256, 6) 18.1; down TP=1: (128, 3) 32.0
    vs (256, 6) 33.4; o_proj TP=4: (128, 3) 9.9 vs (64, 1) 13.0; down TP=4:
    (128, 3) 13.5 vs (64, 1) 22.8; down at M = 4096: (192, 1) 515 vs (256, 2)
    598."""
    assert plan_gemm(128, 5120, 5120) == (128, 3)
    assert plan_gemm(128, 5120, 13824) == (128, 3)
    assert plan_gemm(128, 5120, 1280) == (128, 3)
    assert plan_gemm(128, 5120, 3456) == (128, 3)
    assert plan_gemm(4096, 5120, 13824) == (192, 1)


def test_vocab_shards_cover_the_vocabulary_in_rank_order():
    from tinybatch_b200.runtime import vocab_shard
    for V, t in [(152064, 8), (509, 2), (509, 8), (7, 8), (256, 4)]:
        cols = []
        for r in range(t):
            c0, n = vocab_shard(V, r, t)
            assert n >= 0 and c0 == min(r * -(-V // t), V)
            cols += list(range(c0, c0 + n))
        assert cols == list(range(V))
    assert vocab_shard(152064, 3, 8) == (3 * 19008, 19008)


def test_row_parts():
    assert ops.row_parts(5120, 256, 6) == 120
    assert ops.row_parts(5120, 256, 6, "global") == 20
    assert ops.row_parts(896, 128, 1) == 7


def test_decode_split_policy():
    # 128 sequences x 8 kv heads fill the GPU twice over: one CTA each
    assert decode_split_tokens(128, 8, 128 * 1100, 2304) == 2304
    # few sequences: keys cut so that about 0.6 x 444 CTAs run
    s = decode_split_tokens(2, 8, 2 * 32768, 32768)
    assert s % 16 == 0 and 256 <= s <= 8192
    assert 200 <= 2 * 8 * -(-32768 // s) <= 330
    # TP=8 shard of the 14B decode (one kv head per rank): ~512-token pieces
    assert 480 <= decode_split_tokens(128, 1, 141000, 2304) <= 560
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


def _loop_pack(token_ids, positions, slices, tables, ctx, bs, group, bt_width):
    """Plain-loop restatement of the StepMeta layout (the checker)."""
    ids = np.asarray(token_ids, dtype=np.int32)
    pos = np.asarray(positions, dtype=np.int32)
    T, n = len(ids), len(slices)
    starts = np.array([s for s, _ in slices], dtype=np.int32)
    ends = np.array([e for _, e in slices], dtype=np.int32)
    qlen = ends - starts
    ctx = np.asarray(ctx, dtype=np.int32)
    slots = np.full(T, -1, dtype=np.int32)
    for i, (s, e) in enumerate(slices):
        for t in range(s, e):
            slots[t] = tables[i][pos[t] // bs] * bs + pos[t] % bs
    row_dst = np.full(T, -1, dtype=np.int32)
    for i, (s, e) in enumerate(slices):
        if e > s:
            row_dst[e - 1] = i
    is_dec = qlen * group <= 16

    def subset(mask):
        idx = [i for i in range(n) if mask[i]]
        ld = max([len(tables[i]) for i in idx] + [bt_width, 1])
        bt = np.full((len(idx), ld), -1, dtype=np.int32)
        for r, i in enumerate(idx):
            bt[r, :len(tables[i])] = tables[i]
        return starts[idx], qlen[idx], ctx[idx], bt, np.asarray(idx)

    d = subset(is_dec)
    p = subset(~is_dec)
    order = np.argsort(-d[2], kind="stable").astype(np.int32)
    # (prefill sequence, 256-row tile), most keys read first (stable)
    tiles = []
    for r, (ql, c) in enumerate(zip(p[1].tolist(), p[2].tolist())):
        for t in range(-(-ql * group // 256)):
            last = min(t * 256 + 255, ql * group - 1)
            tiles.append((-min(c, c - ql + last // group + 1), len(tiles), r, t))
    work = np.asarray([(r, t) for *_, r, t in sorted(tiles)], dtype=np.int32).reshape(-1, 2)
    return np.concatenate([ids, pos, slots, row_dst, d[0], d[1], d[2], d[3].ravel(), order,
                           p[0], p[1], p[2], p[3].ravel(), work.ravel()]).astype(np.int32)


def test_step_meta_packing_matches_loop_restatement():
    rng = np.random.default_rng(11)
    for trial in range(30):
        n = int(rng.integers(1, 40))
        qlens = [int(rng.choice([1, 1, 1, int(rng.integers(2, 90))])) for _ in range(n)]
        ctxs = [q + int(rng.integers(0, 300)) for q in qlens]
        tables, nb = [], 0
        for c in ctxs:
            k = -(-c // 16) + int(rng.integers(0, 2))
            tables.append(list(rng.permutation(5000)[:k]))
        ids, pos, slices = [], [], []
        for q, c in zip(qlens, ctxs):
            s = len(ids)
            ids += list(rng.integers(0, 1000, q))
            pos += list(range(c - q, c))
            slices.append((s, s + q))
        bt_width = int(rng.choice([0, 40]))
        md = StepMeta(ids, pos, slices, tables, ctxs, 16, 5, "cpu", pinned=False, bt_width=bt_width)
        want = _loop_pack(ids, pos, slices, tables, ctxs, 16, 5, bt_width)
        got = md.buf.numpy()
        assert got.shape == want.shape and np.array_equal(got, want), trial


def test_step_meta_rejects_position_beyond_table():
    import pytest
    with pytest.raises(IndexError):
        StepMeta([1], [40], [(0, 1)], [[3, 4]], [41], 16, 4, "cpu", pinned=False)


def test_token_view_matches_list():
    from tinybatch_b200.scheduler import TokenView
    p, o = list(range(100, 137)), list(range(900, 911))
    full = p + o
    for limit in (None, 0, 5, 37, 40, 48, 60):
        v = TokenView(p, o, limit)
        ref = full if limit is None else full[:limit]
        assert len(v) == len(ref) and list(v) == ref
        for a in range(-3, len(ref) + 3, 4):
            for b in range(-3, len(ref) + 3, 5):
                assert v[a:b] == ref[a:b], (limit, a, b)
        for k in range(-len(ref), len(ref)):
            assert v[k] == ref[k]


def test_prefill_work_list():
    """(sequence, 256-row tile) pairs covering every query row once, ordered
    by the keys a tile reads (its last row's causal limit), most first."""
    from tinybatch_b200.runtime import PREFILL_ROWS, prefill_work
    q_len, ctx, G = [300, 5, 64, 1], [300, 900, 64, 40], 5
    w = prefill_work(q_len, ctx, G)
    want = sorted((r, t) for r, ql in enumerate(q_len) for t in range(-(-ql * G // PREFILL_ROWS)))
    assert sorted(map(tuple, w.tolist())) == want

    def keys(r, t):
        last = min(t * PREFILL_ROWS + PREFILL_ROWS - 1, q_len[r] * G - 1)
        return min(ctx[r], ctx[r] - q_len[r] + last // G + 1)

    cost = [keys(r, t) for r, t in w.tolist()]
    assert cost == sorted(cost, reverse=True)
    assert cost[0] == 900                  # the one-row tile over a 895-token cached prefix
    assert prefill_work([], [], G).shape == (0, 2)
