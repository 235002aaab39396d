"""Tensor parallelism on 2+ GPUs: the fused GEMM + all-reduce epilogue over
NVLink peer memory, checked against the reference's own TP=2 run (golden
logits) and against the CPU oracle of the row-parallel block.

Tolerances: logits as the single-GPU forward (max-abs 2e-2).  The op-level
block exchanges bf16 partials (one-shot) or bf16 partials and bf16 sums
(two-shot, like the reference's bf16 all-reduce); against an fp32 reference
of the same bf16 inputs the error may exceed 2e-2 by at most one bf16
rounding of the reduced value (2^-8 relative).
"""
from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 CUDA devices", allow_module_level=True)

from tinybatch_b200.config import named_config  # noqa: E402
from tinybatch_b200.tensor_parallel import _spawn, run_tp_forward  # noqa: E402
from tinybatch_b200.weights import reference_test_weights, synthetic_weights  # noqa: E402

PORT = 29611 + (os.getpid() % 1000)


def test_run_tp_forward_world2_matches_reference(golden):
    case = golden["ref_test"]
    cfg = named_config("ref-test")
    w = reference_test_weights(cfg, 0)
    logits, stats = run_tp_forward(2, w, cfg, torch.tensor(case["ids"]), port=PORT, timeout_s=240)
    ref = case["logits_w2"]
    err = float((logits - ref).abs().max())
    assert err <= 2e-2, err
    top2 = ref.topk(2, dim=-1).values
    decisive = (top2[:, 0] - top2[:, 1]) > 2 * err
    assert bool((logits.argmax(-1) == ref.argmax(-1))[decisive].all())
    # exactly two fused all-reduces per layer, T x d bf16 each
    assert stats["calls"] == 2 * cfg.n_layers
    assert stats["bytes"] == 2 * cfg.n_layers * len(case["ids"]) * cfg.d_model * 2


def _op_worker(rank, world, port, cases, queue):
    """Row-parallel block alone: h += sum_r x_r W_r^T, then the norm prologue."""
    import datetime

    import torch.distributed as dist

    from oracle import qwen2_ref as R
    from tinybatch_b200 import _native, ops
    from tinybatch_b200.comm import TPComm

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    comm = None
    try:
        dev = torch.device("cuda", rank)
        N_max = max(c[1] for c in cases)
        errs = []
        for ci, (M, N, K, bn, splits, two_shot) in enumerate(cases):
            if comm is None or comm.n_cols != N:
                if comm is not None:
                    comm.close()
                comm = TPComm(rank, world, dev, N, max_rows=4096)
            g = torch.Generator().manual_seed(100 + ci)
            xs = [torch.randn(M, K // world, generator=g).to(torch.bfloat16) for _ in range(world)]
            ws = [(torch.randn(N, K // world, generator=g) / K ** 0.5).to(torch.bfloat16)
                  for _ in range(world)]
            h0 = torch.randn(M, N, generator=g)
            gn = torch.ones(N, dtype=torch.bfloat16)
            h = h0.to(dev).clone()
            hg = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            parts = ops.row_parts(N, bn, splits)
            sq = torch.empty(parts, M, device=dev)
            comm.row_linear_residual(xs[rank].to(dev), ws[rank].to(dev), h, gn.to(dev), hg, sq,
                                     bn=bn, splits=splits, two_shot=two_shot)
            torch.cuda.synchronize()
            code = _native.status(clear=True)
            href, _ = R.row_gemm_allreduce_norm(xs, [w.t() for w in ws], h0, gn, 1e-6)
            # error beyond bf16 resolution of the exchanged values (|h| is O(1..8))
            excess = (h.cpu() - href).abs() - 2.0 ** -8 * (href - h0).abs()
            errs.append((float(excess.max()),
                         float((sq.sum(0).cpu() - href.square().sum(1)).abs().max()
                               / href.square().sum(1).abs().max()), code,
                         h.cpu().double().sum().item()))
        queue.put((rank, errs))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("two_shot", [False, True])
def test_fused_row_gemm_allreduce_world2(two_shot):
    cases = [(1, 5120, 5120, 256, 4, two_shot), (64, 5120, 1024, 128, 2, two_shot),
             (300, 896, 896, 128, 1, two_shot), (128, 5120, 13824, 192, 4, two_shot),
             (2048, 5120, 512, 128, 1, two_shot)]   # 640 tiles: several per persistent CTA
    _check_fused(2, cases, PORT + 7)


def _check_fused(world, cases, port):
    res = _spawn(world, _op_worker, (cases,), port=port, timeout_s=300, collect_all=True)
    for per_case in zip(*res):
        for err, sq_err, code, _ in per_case:
            assert code == 0
            assert err <= 2e-2, err
            assert sq_err <= 1e-3, sq_err
        # the replicated residual is bit-identical on every rank
        assert len({hsum for *_, hsum in per_case}) == 1


@pytest.mark.parametrize("world", [4, 8])
def test_fused_row_gemm_allreduce_world4_8(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} CUDA devices")
    cases = [(1, 5120, 5120, 128, 3, False), (64, 5120, 5120, 64, 1, True),
             (128, 5120, 13824, 128, 3, None), (1024, 5120, 1024, 128, 1, True)]
    _check_fused(world, cases, PORT + 20 + world)


def _small_tp_config():
    """2 layers, 16 q / 8 kv heads of 64, ff 2048, vocab 512: divisible at TP 2/4/8."""
    from tinybatch_b200.config import ModelConfig
    return ModelConfig(n_layers=2, d_model=1024, n_heads=16, n_kv_heads=8, head_dim=64,
                       d_ff=2048, vocab_size=512, rope_theta=1e6, rms_eps=1e-6,
                       tie_embeddings=False, max_position=4096)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_run_tp_forward_matches_oracle(world):
    """Sharded forward over `world` GPUs vs the single-process fp32 oracle on
    the same (bf16-valued) weights: logits within 2e-2."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} CUDA devices")
    from oracle import qwen2_ref as R
    cfg = _small_tp_config()
    w = synthetic_weights(cfg, 7, dtype=torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(7))
    logits, stats = run_tp_forward(world, w, cfg, ids, port=PORT + 40 + world, timeout_s=300)
    ref = R.tp_forward(cfg, {k: v.float() for k, v in w.items()}, ids, world=1)
    err = float((logits - ref).abs().max())
    assert err <= 2e-2, err
    assert stats["calls"] == 2 * cfg.n_layers


def _sample_worker(rank, world, port, cfg, w, queue):
    """One decode step of 24 sequences sampled on the device with the
    vocabulary-parallel head, and the same step's full logits from the
    replicated head; reports both."""
    import datetime
    import random

    import torch.distributed as dist

    from tinybatch_b200 import _native
    from tinybatch_b200.comm import TPComm
    from tinybatch_b200.model import Qwen2Paged

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    comm = TPComm(rank, world, dev, cfg.d_model, max_rows=256)
    try:
        model = Qwen2Paged.from_weights(cfg, w, device=dev, rank=rank, world=world, comm=comm,
                                        max_tokens=64, max_seqs=64)
        rng = random.Random(3)
        ctx = [rng.randint(1, 200) for _ in range(24)]
        tables, nb = [], 0
        for c in ctx:
            k = -(-c // 16)
            tables.append(list(range(nb, nb + k)))
            nb += k
        cache = model.make_kv_cache(nb, 16)
        g = torch.Generator(device=dev).manual_seed(5)
        for pool in cache.pools:
            pool.copy_(torch.randn(pool.shape, generator=g, device=dev).mul_(0.5))
        ids = [rng.randrange(cfg.vocab_size) for _ in ctx]
        md = model.metadata(ids, [c - 1 for c in ctx], [(i, i + 1) for i in range(24)], tables,
                            ctx, 16)
        full = model.dm.forward(md, cache.pools, sample=False).clone()
        model.dm.forward(md, cache.pools, sample=True)
        got = model.dm.next_ids[:24].clone()
        torch.cuda.synchronize()
        _native.raise_on_status(f"rank {rank}")
        queue.put((rank, (full.cpu(), got.cpu())))
    finally:
        comm.close()
        dist.destroy_process_group()


def _vocab_parallel_case(world, tie):
    from tinybatch_b200.config import ModelConfig
    # vocabulary not divisible by the degree: ragged shards
    cfg = ModelConfig(n_layers=2, d_model=1024, n_heads=16, n_kv_heads=8, head_dim=64,
                      d_ff=2048, vocab_size=509, rope_theta=1e6, rms_eps=1e-6,
                      tie_embeddings=False, max_position=4096)
    w = synthetic_weights(cfg, 11, dtype=torch.bfloat16)
    if tie:
        # every logit 0 except two equal ones in the first and the last shard:
        # the answer is the smaller of the two when positive, else index 0
        head = torch.zeros_like(w["lm_head.weight"])
        v = torch.randn(cfg.d_model, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
        head[5] = v
        head[cfg.vocab_size - 2] = v
        w["lm_head.weight"] = head
    return cfg, w


@pytest.mark.parametrize("world,tie", [(2, False), (2, True), (4, False), (8, True)])
def test_vocab_parallel_sampling(world, tie):
    """Greedy ids from the vocabulary-parallel head + cross-rank argmax equal
    torch.argmax of the replicated head's logits on every rank (exactly for
    the constructed ties; wherever the top-2 gap is decisive otherwise)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} CUDA devices")
    cfg, w = _vocab_parallel_case(world, tie)
    res = _spawn(world, _sample_worker, (cfg, w), port=PORT + 60 + world + 10 * tie,
                 timeout_s=300, collect_all=True)
    full, ids0 = res[0]
    for r in range(1, world):
        assert torch.equal(res[r][1], ids0), f"rank {r} sampled different ids"
    ref = full.argmax(-1).to(torch.int32)
    if tie:
        assert torch.equal(ids0, ref)
        assert set(ids0.tolist()) <= {0, 5}
    else:
        top2 = full.topk(2, dim=-1).values
        decisive = (top2[:, 0] - top2[:, 1]) > 1e-3
        assert int(decisive.sum()) >= 20
        assert torch.equal(ids0[decisive], ref[decisive])


def _mixed_worker(rank, world, port, cfg, w, queue):
    """Back-to-back forwards on one communicator, some sampling on the device
    (row-parallel exchanges plus an argmax exchange) and some returning full
    logits (row-parallel exchanges only), in an order that reuses every
    buffer half many times; then tp_forward's exchange timing."""
    import datetime
    import random

    import torch.distributed as dist

    from tinybatch_b200 import _native
    from tinybatch_b200.comm import TPComm
    from tinybatch_b200.model import Qwen2Paged
    from tinybatch_b200.tensor_parallel import shard_weights, tp_forward

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    comm = TPComm(rank, world, dev, cfg.d_model, max_rows=256)
    try:
        model = Qwen2Paged.from_weights(cfg, w, device=dev, rank=rank, world=world, comm=comm,
                                        max_tokens=64, max_seqs=64)
        rng = random.Random(4)
        ctx = [rng.randint(1, 100) for _ in range(16)]
        tables, nb = [], 0
        for c in ctx:
            k = -(-c // 16)
            tables.append(list(range(nb, nb + k)))
            nb += k
        cache = model.make_kv_cache(nb, 16)
        g = torch.Generator(device=dev).manual_seed(6)
        for pool in cache.pools:
            pool.copy_(torch.randn(pool.shape, generator=g, device=dev).mul_(0.5))
        ids = [rng.randrange(cfg.vocab_size) for _ in ctx]
        md = model.metadata(ids, [c - 1 for c in ctx], [(i, i + 1) for i in range(16)], tables,
                            ctx, 16)
        logits, sampled = [], []
        for sample in (False, False, True, False, True, True, False, True, False, False):
            out = model.dm.forward(md, cache.pools, sample=sample)
            if sample:
                sampled.append(model.dm.next_ids[:16].clone())
            else:
                logits.append(out.clone())
        torch.cuda.synchronize()
        _native.raise_on_status(f"rank {rank}")
        same_logits = all(torch.equal(x, logits[0]) for x in logits)
        same_ids = all(torch.equal(x, sampled[0]) for x in sampled)
        stats = {"calls": 0, "bytes": 0, "seconds": 0.0}
        shard = shard_weights(w, cfg, rank, world)
        ids_t = torch.randint(0, cfg.vocab_size, (24,), generator=torch.Generator().manual_seed(1))
        tp_forward(ids_t, shard, cfg, world, stats)
        torch.cuda.synchronize()
        _native.raise_on_status(f"rank {rank} tp_forward")
        queue.put((rank, (same_logits, same_ids, logits[0].argmax(-1).cpu(), sampled[0].cpu(),
                          stats)))
    finally:
        from tinybatch_b200.comm import close_all
        close_all()
        dist.destroy_process_group()


def test_mixed_sampled_and_full_forwards_world2():
    """Forwards with and without device sampling, back to back, on one
    communicator: every repeat of the same step gives the same logits and the
    same ids on every rank, no wait runs out, and tp_forward reports the
    exchanges' device time in comm_stats["seconds"]."""
    cfg = _small_tp_config()
    w = synthetic_weights(cfg, 9, dtype=torch.bfloat16)
    res = _spawn(2, _mixed_worker, (cfg, w), port=PORT + 90, timeout_s=300, collect_all=True)
    for same_logits, same_ids, full_arg, ids, stats in res:
        assert same_logits and same_ids
        assert stats["calls"] == 2 * cfg.n_layers
        assert 0.0 < stats["seconds"] < 1.0, stats
    assert torch.equal(res[0][3], res[1][3])
    assert torch.equal(res[0][2], res[1][2])
