"""Kernel-level parity on the B200: each fused kernel against an fp32
PyTorch/oracle restatement of the same op, through the C ABI.

Tolerances: the GEMMs read bf16 operands and accumulate in fp32, so against
an fp32 product of the same bf16 values only the summation order differs
(rtol 2e-3 / atol 2e-3 relative to the output scale).  Epilogues that round
to bf16 are compared at bf16 resolution (atol/rtol 1.6e-2).
"""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU-only hosts, never run there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from oracle import qwen2_ref as R  # noqa: E402
from tinybatch_b200 import _native, ops  # noqa: E402
from tinybatch_b200.runtime import prefill_work  # noqa: E402

DEV = "cuda"


@pytest.fixture(autouse=True)
def _status_clean():
    _native.status(clear=True)
    yield
    _native.raise_on_status("kernel")


def _rand(*shape, scale=1.0, seed=0, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).to(DEV)


GEMM_CASES = [
    # M, N, K, bn, splits
    (128, 256, 512, 128, 1),
    (1, 64, 64, 64, 1),
    (200, 384, 1024, 128, 1),
    (77, 97, 64, 64, 1),
    (128, 64, 32, 64, 1),
    (300, 512, 1024, 256, 1),
    (128, 576, 1024, 192, 1),
    (128, 512, 1024, 128, 2),
    (64, 640, 1344, 128, 3),
    (130, 256, 4096, 256, 5),
    (128, 960, 2048, 192, 4),
    (100, 384, 4096, 64, 8),
    (128, 1280, 2048, 256, 6),
    # more tiles than SMs: persistent CTAs walk several tiles each
    (1024, 4608, 512, 128, 1),
    (777, 5120, 320, 256, 1),
]


@pytest.mark.parametrize("split_mode", ["cluster", "global"])
@pytest.mark.parametrize("M,N,K,bn,splits", GEMM_CASES)
def test_linear_f32(M, N, K, bn, splits, split_mode):
    if splits == 1 and split_mode == "global":
        pytest.skip("no split")
    x = _rand(M, K, seed=1)
    w = _rand(N, K, scale=1 / math.sqrt(K), seed=2)
    ld = (N + 3) // 4 * 4
    out = torch.full((M, ld), float("nan"), device=DEV)
    ops.linear(x, w, out, bn=bn, splits=splits, split_mode=split_mode)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    torch.testing.assert_close(out[:, :N], ref, atol=2e-3, rtol=2e-3)


def test_linear_rowscale_bf16():
    M, N, K = 96, 256, 512
    x = _rand(M, K, seed=3)
    w = _rand(N, K, scale=1 / math.sqrt(K), seed=4)
    sq = torch.rand(3, 128, device=DEV) * 100 + 1
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.linear(x, w, out, sq=sq, inv_d=1 / 512, eps=1e-6, bn=128)
    torch.cuda.synchronize()
    scale = torch.rsqrt(sq[:, :M].sum(0) / 512 + 1e-6)
    ref = (x.float() @ w.float().t()) * scale[:, None]
    torch.testing.assert_close(out.float(), ref, atol=1.6e-2, rtol=1.6e-2)


@pytest.mark.parametrize("M,N,K,bn,splits,mode", [
    (128, 512, 640, 128, 1, "cluster"), (37, 256, 1024, 64, 4, "global"),
    (37, 256, 1024, 64, 4, "cluster"), (260, 896, 896, 128, 1, "cluster"),
    (128, 5120, 5120, 256, 7, "cluster"), (96, 896, 896, 192, 3, "cluster"),
    (128, 2048, 2048, 256, 8, "cluster"), (20, 640, 1280, 128, 5, "cluster"),
    (1100, 5120, 256, 128, 1, "cluster"), (1024, 2048, 192, 64, 1, "cluster")])
def test_row_linear_residual(M, N, K, bn, splits, mode):
    x = _rand(M, K, seed=5)
    w = _rand(N, K, scale=1 / math.sqrt(K), seed=6)
    h0 = torch.randn(M, N, device=DEV)
    g = _rand(N, seed=7) + 1.0
    h = h0.clone()
    hg = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    parts = ops.row_parts(N, bn, splits, mode)
    sq = torch.empty(parts, M, device=DEV)
    row_dst = torch.full((M,), -1, dtype=torch.int32, device=DEV)
    row_dst[M - 1] = 0
    row_dst[M // 2] = 1
    hg2 = torch.zeros(2, N, dtype=torch.bfloat16, device=DEV)
    sq2 = torch.zeros(parts, 2, device=DEV)
    ops.row_linear_residual(x, w, h, g, hg, sq, row_dst=row_dst, hg2=hg2, sq2=sq2, bn=bn,
                            splits=splits, split_mode=mode)
    torch.cuda.synchronize()
    href = h0 + x.float() @ w.float().t()
    torch.testing.assert_close(h, href, atol=2e-3, rtol=2e-3)
    torch.testing.assert_close(hg.float(), href * g.float(), atol=1.6e-2, rtol=1.6e-2)
    torch.testing.assert_close(sq.sum(0), href.square().sum(1), rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(hg2[0], hg[M - 1])
    torch.testing.assert_close(hg2[1], hg[M // 2])
    torch.testing.assert_close(sq2[:, 0], sq[:, M - 1])


@pytest.mark.parametrize("M,F,K,bn,splits,mode", [
    (128, 256, 512, 128, 1, "cluster"), (50, 192, 896, 128, 2, "global"),
    (50, 192, 896, 128, 2, "cluster"), (200, 128, 256, 256, 1, "cluster"),
    (128, 1728, 640, 192, 2, "cluster"), (128, 864, 1024, 192, 1, "cluster"),
    (128, 992, 1024, 256, 3, "cluster"), (64, 720, 1280, 192, 5, "cluster"),
    (700, 3456, 256, 192, 1, "cluster")])
def test_gate_up_swiglu(M, F, K, bn, splits, mode):
    x = _rand(M, K, seed=8)
    wg = _rand(F, K, scale=1 / math.sqrt(K), seed=9)
    wu = _rand(F, K, scale=1 / math.sqrt(K), seed=10)
    half = bn // 2
    n_tiles = (F + half - 1) // half
    wgu = torch.zeros(n_tiles * bn, K, dtype=torch.bfloat16, device=DEV)
    for t in range(n_tiles):
        f0, f1 = t * half, min(F, (t + 1) * half)
        wgu[t * bn: t * bn + f1 - f0] = wg[f0:f1]
        wgu[t * bn + half: t * bn + half + f1 - f0] = wu[f0:f1]
    sq = torch.rand(1, M, device=DEV) * K + 1
    act = torch.empty(M, F, dtype=torch.bfloat16, device=DEV)
    ops.gate_up_swiglu(x, wgu, act, n_feat=F, sq=sq, inv_d=1 / K, eps=1e-6, bn=bn, splits=splits,
                       split_mode=mode)
    torch.cuda.synchronize()
    s = torch.rsqrt(sq[0] / K + 1e-6)[:, None]
    gate = (x.float() @ wg.float().t()) * s
    up = (x.float() @ wu.float().t()) * s
    ref = torch.nn.functional.silu(gate) * up
    torch.testing.assert_close(act.float(), ref, atol=1.6e-2, rtol=1.6e-2)


@pytest.mark.parametrize("hq,hkv,hd,bn,bs,splits", [
    (4, 2, 16, 64, 16, 1), (14, 2, 64, 128, 16, 1), (40, 8, 128, 128, 16, 1),
    (5, 1, 128, 256, 4, 1), (40, 8, 128, 256, 16, 4), (14, 2, 64, 192, 16, 2),
    (5, 1, 128, 128, 16, 3), (4, 2, 16, 64, 16, 2), (14, 2, 64, 256, 16, 3),
    (40, 8, 128, 256, 16, 5), (40, 8, 128, 128, 16, 1), (14, 2, 64, 64, 16, 1)])
def test_qkv_rope_kv(hq, hkv, hd, bn, bs, splits):
    # 1000 rows with one split: more tiles than SMs (persistent CTAs)
    M, K = (1000 if splits == 1 and bn <= 128 else 70), max(256, 128 * splits)
    N = (hq + 2 * hkv) * hd
    x = _rand(M, K, seed=11)
    w = _rand(N, K, scale=1 / math.sqrt(K), seed=12)
    bias = _rand(N, scale=0.1, seed=13)
    theta = 1e6
    max_pos = 4096
    cos, sin = R.rope_tables(torch.arange(max_pos), hd, theta)
    cos, sin = cos.to(DEV), sin.to(DEV)
    pos = torch.randint(0, max_pos, (M,), generator=torch.Generator().manual_seed(1))
    num_blocks = 64
    perm = torch.randperm(num_blocks * bs, generator=torch.Generator().manual_seed(2))[:M]
    slots = perm.to(torch.int32)
    q = torch.empty(M, hq * hd, dtype=torch.bfloat16, device=DEV)
    pool = torch.zeros(num_blocks, 2, hkv, bs, hd, dtype=torch.bfloat16, device=DEV)
    sq = torch.rand(2, M, device=DEV) * K + 1
    ops.qkv_rope_kv(x, w, bias, n_q_heads=hq, n_kv_heads=hkv, head_dim=hd, sq=sq, inv_d=1 / K,
                    eps=1e-6, rope_cos=cos, rope_sin=sin, positions=pos.to(torch.int32).to(DEV),
                    slots=slots.to(DEV), q_out=q, kv_pool=pool, block_size=bs, bn=bn,
                    splits=splits)
    torch.cuda.synchronize()
    s = torch.rsqrt(sq.sum(0) / K + 1e-6)[:, None].cpu()
    y = (x.float().cpu() @ w.float().cpu().t()) * s + bias.float().cpu()
    qr = R.rope(y[:, : hq * hd].view(M, hq, hd), pos, theta).reshape(M, -1)
    kr = R.rope(y[:, hq * hd:(hq + hkv) * hd].view(M, hkv, hd), pos, theta)
    vr = y[:, (hq + hkv) * hd:].view(M, hkv, hd)
    torch.testing.assert_close(q.float().cpu(), qr, atol=1.6e-2, rtol=1.6e-2)
    pc = pool.float().cpu()
    for m in range(M):
        b, o = int(slots[m]) // bs, int(slots[m]) % bs
        torch.testing.assert_close(pc[b, 0, :, o], kr[m], atol=1.6e-2, rtol=1.6e-2)
        torch.testing.assert_close(pc[b, 1, :, o], vr[m], atol=1.6e-2, rtol=1.6e-2)


def test_cluster_split_that_does_not_fit_is_rejected():
    """bn 256 with 7 cluster members: the RoPE-paired chunks one member
    receives exceed its pipeline buffers; the launcher refuses the call."""
    hq, hkv, hd, M, K = 40, 8, 128, 16, 1024
    N = (hq + 2 * hkv) * hd
    cos, sin = R.rope_tables(torch.arange(64), hd, 1e6)
    with pytest.raises(_native.NativeError, match="do not fit"):
        ops.qkv_rope_kv(_rand(M, K), _rand(N, K), _rand(N), n_q_heads=hq, n_kv_heads=hkv,
                        head_dim=hd, sq=None, inv_d=0.0, eps=0.0, rope_cos=cos.to(DEV),
                        rope_sin=sin.to(DEV), positions=torch.zeros(M, dtype=torch.int32, device=DEV),
                        slots=torch.zeros(M, dtype=torch.int32, device=DEV),
                        q_out=torch.empty(M, hq * hd, dtype=torch.bfloat16, device=DEV),
                        kv_pool=torch.zeros(4, 2, hkv, 16, hd, dtype=torch.bfloat16, device=DEV),
                        block_size=16, bn=256, splits=7)


def _paged_case(hq, hkv, hd, bs, q_lens, ctx_lens, seed=0):
    """Random pool + tables; returns device tensors and an fp32 reference."""
    g = torch.Generator().manual_seed(seed)
    n = len(q_lens)
    nb_per = [(c + bs - 1) // bs for c in ctx_lens]
    num_blocks = sum(nb_per) + 3
    perm = torch.randperm(num_blocks, generator=g).tolist()
    tables, k = [], 0
    for nb in nb_per:
        tables.append(perm[k:k + nb])
        k += nb
    bt_ld = max(nb_per)
    bt = torch.full((n, bt_ld), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    pool = (torch.randn(num_blocks, 2, hkv, bs, hd, generator=g)).to(torch.bfloat16)
    T = sum(q_lens)
    q = torch.randn(T, hq * hd, generator=g).to(torch.bfloat16)
    q_start = torch.tensor([sum(q_lens[:i]) for i in range(n)], dtype=torch.int32)
    ref = torch.empty(T, hq * hd)
    pf = pool.float()
    for i in range(n):
        keys, vals = R.kv_gather(pf, tables[i], ctx_lens[i])
        s0 = int(q_start[i])
        out = R.attention(q[s0:s0 + q_lens[i]].float().view(q_lens[i], hq, hd), keys, vals,
                          first_pos=ctx_lens[i] - q_lens[i])
        ref[s0:s0 + q_lens[i]] = out.reshape(q_lens[i], -1)
    dev = dict(q=q.to(DEV), pool=pool.to(DEV), bt=bt.to(DEV), q_start=q_start.to(DEV),
               q_len=torch.tensor(q_lens, dtype=torch.int32, device=DEV),
               ctx=torch.tensor(ctx_lens, dtype=torch.int32, device=DEV))
    return dev, ref


@pytest.mark.parametrize("hq,hkv,hd,bs", [(40, 8, 128, 16), (14, 2, 64, 16), (4, 2, 16, 4),
                                          (64, 8, 128, 16)])
@pytest.mark.parametrize("split_tokens,ordered", [(512, False), (64, False), (4096, True),
                                                  (256, True)])
def test_paged_attention_decode(hq, hkv, hd, bs, split_tokens, ordered):
    """Split-KV (merged in the launch by the last split of each sequence and
    kv head) and one-CTA-per-sequence decode, in index order or dispatched
    longest first."""
    ctx = [1, 15, 16, 17, 100, 700, 1300, 33, 3000]
    d, ref = _paged_case(hq, hkv, hd, bs, [1] * len(ctx), ctx, seed=3)
    out = torch.zeros(len(ctx), hq * hd, dtype=torch.bfloat16, device=DEV)
    order = None
    if ordered:
        order = torch.tensor(sorted(range(len(ctx)), key=lambda i: -ctx[i]), dtype=torch.int32,
                             device=DEV)
    arena = ops.Scratch(DEV, 1 << 16)
    for _ in range(2):   # the second call reuses the arena: arrival counters were reset
        out.zero_()
        ops.paged_attention_decode(d["q"], out, d["pool"], n_q_heads=hq, n_kv_heads=hkv,
                                   head_dim=hd, block_size=bs, block_tables=d["bt"],
                                   q_start=d["q_start"], q_len=d["q_len"], ctx_len=d["ctx"],
                                   max_ctx=max(ctx), split_tokens=split_tokens, seq_order=order,
                                   scratch=arena)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("hq,hkv,hd,bs", [(40, 8, 128, 16), (14, 2, 64, 16), (4, 2, 16, 4)])
def test_paged_attention_prefill(hq, hkv, hd, bs):
    q_lens = [37, 5, 64, 130, 2]
    ctx = [37, 21, 64, 200, 2]          # seq 1 and 3 have a cached prefix
    d, ref = _paged_case(hq, hkv, hd, bs, q_lens, ctx, seed=4)
    G = hq // hkv
    work = torch.tensor(prefill_work(q_lens, ctx, G), dtype=torch.int32, device=DEV)
    out = torch.zeros(sum(q_lens), hq * hd, dtype=torch.bfloat16, device=DEV)
    ops.paged_attention_prefill(d["q"], out, d["pool"], n_q_heads=hq, n_kv_heads=hkv,
                                head_dim=hd, block_size=bs, block_tables=d["bt"],
                                q_start=d["q_start"], q_len=d["q_len"], ctx_len=d["ctx"],
                                work=work)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("hq,hkv,hd,bs", [(40, 8, 128, 16), (64, 8, 128, 32), (14, 2, 64, 16)])
def test_paged_attention_prefill_long(hq, hkv, hd, bs):
    """Prefill over many 128-key tiles (the two-stage ring and both S buffers
    reused several times), cached prefixes of several tiles, rows of the
    last tile only partly valid, a one-token prompt."""
    q_lens = [700, 129, 260, 1, 40]
    ctx = [700, 900, 260, 513, 777]
    d, ref = _paged_case(hq, hkv, hd, bs, q_lens, ctx, seed=9)
    G = hq // hkv
    work = torch.tensor(prefill_work(q_lens, ctx, G), dtype=torch.int32, device=DEV)
    out = torch.zeros(sum(q_lens), hq * hd, dtype=torch.bfloat16, device=DEV)
    for _ in range(2):
        ops.paged_attention_prefill(d["q"], out, d["pool"], n_q_heads=hq, n_kv_heads=hkv,
                                    head_dim=hd, block_size=bs, block_tables=d["bt"],
                                    q_start=d["q_start"], q_len=d["q_len"], ctx_len=d["ctx"],
                                    work=work)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("hq,hkv,hd,bs", [(40, 8, 128, 16), (4, 2, 16, 4)])
def test_paged_attention_prefill_rejects_bad_work(hq, hkv, hd, bs):
    """Work entries naming no sequence of the call, a row tile past the prompt
    or a negative tile are refused in the kernel (status BAD_INDEX, nothing
    read through them, valid entries of the same call still computed)."""
    q_lens, ctx = [40, 7], [40, 30]
    d, ref = _paged_case(hq, hkv, hd, bs, q_lens, ctx, seed=5)
    G = hq // hkv
    good = prefill_work(q_lens, ctx, G).tolist()
    bad = [[2, 0], [0, 5], [1, -1]]
    work = torch.tensor(good + bad, dtype=torch.int32, device=DEV)
    out = torch.zeros(sum(q_lens), hq * hd, dtype=torch.bfloat16, device=DEV)
    ops.paged_attention_prefill(d["q"], out, d["pool"], n_q_heads=hq, n_kv_heads=hkv,
                                head_dim=hd, block_size=bs, block_tables=d["bt"],
                                q_start=d["q_start"], q_len=d["q_len"], ctx_len=d["ctx"],
                                work=work)
    torch.cuda.synchronize()
    assert _native.status(clear=True) == 103      # TB_STATUS_BAD_INDEX
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-2, rtol=2e-2)


def test_embed_and_argmax():
    V, d, M = 1000, 256, 9
    emb = _rand(V, d, scale=0.5, seed=14)
    g = _rand(d, seed=15)
    ids = torch.randint(0, V, (M,), generator=torch.Generator().manual_seed(3)).to(torch.int32)
    h = torch.empty(M, d, device=DEV)
    hg = torch.empty(M, d, dtype=torch.bfloat16, device=DEV)
    sq = torch.empty(1, M, device=DEV)
    ops.embed(ids.to(DEV), emb, g, h, hg, sq)
    logits = torch.randn(M, 152064, device=DEV)
    logits[3, 17] = 100.0
    logits[3, 900] = 100.0            # tie -> first index
    am = torch.empty(M, dtype=torch.int32, device=DEV)
    ops.argmax(logits, am)
    torch.cuda.synchronize()
    ref_h = emb.float()[ids.long().to(DEV)]
    torch.testing.assert_close(h, ref_h)
    torch.testing.assert_close(hg.float(), ref_h * g.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(sq[0], ref_h.square().sum(1), rtol=1e-4, atol=1e-4)
    assert am.tolist() == logits.argmax(1).tolist()
    assert int(am[3]) == 17


def test_split_k_calls_share_one_arena():
    """Split-K GEMMs with different tile counts reuse one scratch arena: the
    arrival counters must not alias an earlier call's partial tiles."""
    arena = ops.Scratch(DEV, 1 << 20)
    shapes = [(40, 256, 2048, 64, 8), (57, 4096, 896, 256, 3), (1, 152064 // 8, 896, 256, 3),
              (40, 256, 2048, 64, 8)]
    for i, (M, N, K, bn, splits) in enumerate(shapes):
        x = _rand(M, K, seed=20 + i)
        w = _rand(N, K, scale=1 / math.sqrt(K), seed=30 + i)
        out = torch.empty(M, N, device=DEV)
        ops.linear(x, w, out, bn=bn, splits=splits, scratch=arena, split_mode="global")
        torch.cuda.synchronize()
        torch.testing.assert_close(out, x.float() @ w.float().t(), atol=2e-3, rtol=2e-3)


def test_cluster_occupancy_query():
    for bn in (64, 128, 192, 256):
        for c in (1, 2, 4, 8):
            assert ops.max_active_clusters(bn, c) >= 1
