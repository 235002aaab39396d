"""Host-side tensor-parallel plumbing on CPU ranks (gloo, world size 2):
sharding rules, the IPC-handle exchange the communicator performs at start,
and failure handling of the multi-process runner (a rank that raises, a rank
that never reports) -- all without a GPU."""
from __future__ import annotations

import datetime
import os
import time

import pytest
import torch
import torch.distributed as dist

from tinybatch_b200.comm import exchange_handles
from tinybatch_b200.config import named_config
from tinybatch_b200.tensor_parallel import _spawn, shard_weights
from tinybatch_b200.weights import reference_test_weights

PORT = 30111 + (os.getpid() % 1000)


def _init(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=30))


def _exchange_worker(rank, world, port, queue):
    _init(rank, world, port)
    try:
        mine = bytes([rank * 16 + i for i in range(64)])
        queue.put((rank, exchange_handles(mine)))
    finally:
        dist.destroy_process_group()


def _raising_worker(rank, world, port, queue):
    if rank == 1:
        raise ValueError("planted failure on rank 1")
    time.sleep(30)            # rank 0 would wait for its partner forever
    queue.put((rank, "late"))


def _silent_worker(rank, world, port, queue):
    time.sleep(60)            # never reports


def _partial_sum_worker(rank, world, port, w, cfg, x, queue):
    """The row-parallel reduction of the reference (shard, local F.linear,
    all_reduce SUM over gloo): what the fused kernel replaces."""
    _init(rank, world, port)
    try:
        p = "model.layers.0."
        sw = shard_weights(w, cfg, rank, world)
        part = x.chunk(world, dim=1)[rank] @ sw[p + "self_attn.o_proj.weight"].t()
        dist.all_reduce(part)
        queue.put((rank, part))
    finally:
        dist.destroy_process_group()


def test_shard_shapes_and_divisibility():
    cfg = named_config("ref-test")
    w = reference_test_weights(cfg)
    s = shard_weights(w, cfg, rank=0, world=2)
    assert s["model.layers.0.self_attn.q_proj.weight"].shape[0] == cfg.n_heads * cfg.head_dim // 2
    assert s["model.layers.0.self_attn.q_proj.bias"].shape[0] == cfg.n_heads * cfg.head_dim // 2
    assert s["model.layers.0.self_attn.o_proj.weight"].shape[1] == cfg.n_heads * cfg.head_dim // 2
    assert s["model.layers.0.mlp.down_proj.weight"].shape[1] == cfg.d_ff // 2
    assert s["model.embed_tokens.weight"].shape == w["model.embed_tokens.weight"].shape
    with pytest.raises(AssertionError):
        shard_weights(w, cfg, rank=0, world=3)


def test_handle_exchange_world2():
    res = _spawn(2, _exchange_worker, (), port=PORT, timeout_s=60, collect_all=True)
    want = [bytes([r * 16 + i for i in range(64)]) for r in range(2)]
    assert res[0] == want and res[1] == want


def test_row_parallel_sum_equals_single_process():
    cfg = named_config("ref-test")
    w = reference_test_weights(cfg)
    x = torch.randn(24, cfg.n_heads * cfg.head_dim, generator=torch.Generator().manual_seed(5))
    res = _spawn(2, _partial_sum_worker, (w, cfg, x), port=PORT + 1, timeout_s=60,
                 collect_all=True)
    full = x @ w["model.layers.0.self_attn.o_proj.weight"].t()
    for r in res:
        torch.testing.assert_close(r, full, atol=1e-5, rtol=1e-5)


def test_failed_rank_raises_promptly():
    t0 = time.time()
    with pytest.raises(RuntimeError, match="rank 1"):
        _spawn(2, _raising_worker, (), port=PORT + 2, timeout_s=60)
    assert time.time() - t0 < 25


def test_silent_rank_times_out():
    t0 = time.time()
    with pytest.raises(RuntimeError, match="no result"):
        _spawn(2, _silent_worker, (), port=PORT + 3, timeout_s=3)
    assert time.time() - t0 < 20


def test_exchange_sequence_parity_rules():
    """Consecutive exchanges of one kind must alternate buffer halves: an
    explicit seq with the previous call's parity is refused, an implicit one
    takes the other half."""
    from tinybatch_b200.comm import TPComm
    assert TPComm._next(None, 1, "x") == 0
    assert TPComm._next(None, 0, "x") == 1
    assert TPComm._next(0, 1, "x") == 0
    assert TPComm._next(7, 0, "x") == 7
    with pytest.raises(ValueError):
        TPComm._next(2, 0, "x")
    with pytest.raises(ValueError):
        TPComm._next(-1, 0, "x")
    # a forward's row-parallel sites 0 .. 2L-1 start at parity 0 and end at 1,
    # so back-to-back forwards (sampled or not) keep alternating
    last = 1
    for _ in range(3):
        for site in range(2 * 4):
            last = TPComm._next(site, last, "forward") & 1


def _cpu_leg_worker(rank, world, port, queue):
    """bench.py's CPU baseline at TP=2: each rank times its shard of a decoder
    layer with gloo all-reduces; the reported times are the max over ranks."""
    import bench
    _init(rank, world, port)
    try:
        cfg = named_config("tiny")
        info = bench.cpu_decode_sample(cfg, [5, 17, 33, 64], rank, world, dist.group.WORLD)
        queue.put((rank, info))
    finally:
        dist.destroy_process_group()


def test_bench_cpu_leg_tp2():
    res = _spawn(2, _cpu_leg_worker, (), port=PORT + 40, timeout_s=120, collect_all=True)
    a, b = res
    assert a["layer_s"] == b["layer_s"] and a["lm_head_s"] == b["lm_head_s"]
    cfg = named_config("tiny")
    assert a["step_s"] == pytest.approx(cfg.n_layers * a["layer_s"] + a["lm_head_s"])
    assert a["tokens_per_s"] == pytest.approx(4 / a["step_s"])
