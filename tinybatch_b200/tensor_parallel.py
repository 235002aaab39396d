"""Megatron-style tensor parallelism on B200s — the reference's API
(``src/tinybatch/tensor_parallel.py``) over the fused kernels.

* ``shard_weights(w, cfg, rank, world)``: same split as the reference
  (``:35-61``): q/k/v weight+bias and gate/up by output rows, o/down by input
  columns, the rest replicated; ``AssertionError`` when heads, kv heads or
  d_ff do not divide the degree.
* ``tp_forward(token_ids, w, cfg, world, comm_stats)``: cache-free causal
  prefill of one sequence on this rank's shard, returning full fp32 logits
  ``[T, vocab]`` (``:64-117``).  It must be called in every rank's process
  (one process per GPU, ``torch.distributed`` initialised for world > 1).
  The two all-reduces per layer run inside the o_proj / down_proj GEMM
  epilogues over NVLink peer memory; ``comm_stats`` counts them exactly like
  the reference's wrapper (``calls`` += 1 and ``bytes`` += numel * element
  size of the reduced ``[T, d]`` bf16 tensor per all-reduce).
* ``run_tp_forward(world, w, cfg, token_ids, port)``: spawns one process per
  GPU, returns rank 0's ``(logits, stats)`` (``:138-151``), with timeouts so
  a dead rank ends the call with an error instead of a hang.
"""
from __future__ import annotations

import os
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from .config import ModelConfig
from .runtime import StepMeta

COL_SUFFIXES = ("q_proj.weight", "k_proj.weight", "v_proj.weight", "q_proj.bias",
                "k_proj.bias", "v_proj.bias", "gate_proj.weight", "up_proj.weight")
ROW_SUFFIXES = ("o_proj.weight", "down_proj.weight")


def shard_weights(w: dict, cfg: ModelConfig, rank: int, world: int) -> dict:
    """This rank's slice of a full Qwen2 weight dict (F.linear layout)."""
    assert cfg.n_heads % world == 0, "q heads must divide tp degree"
    assert cfg.n_kv_heads % world == 0, "kv heads must divide tp degree"
    assert cfg.d_ff % world == 0, "d_ff must divide tp degree"
    out = {}
    for k, v in w.items():
        if k.endswith(COL_SUFFIXES):
            out[k] = v.chunk(world, dim=0)[rank].contiguous()
        elif k.endswith(ROW_SUFFIXES):
            out[k] = v.chunk(world, dim=1)[rank].contiguous()
        else:
            out[k] = v
    return out


_MODELS: dict = {}


def _rank_model(w: dict, cfg: ModelConfig, world: int):
    """Build (once per weight dict) this rank's device model."""
    from .model import Qwen2Paged
    key = (id(w), world)
    if key not in _MODELS:
        rank = dist.get_rank() if world > 1 else 0
        comm = None
        if world > 1:
            from .comm import TPComm
            comm = TPComm.from_process_group(torch.device("cuda", torch.cuda.current_device()))
        dev = torch.device("cuda", torch.cuda.current_device())
        model = Qwen2Paged.from_weights(cfg, w, device=dev, rank=rank, world=world, comm=comm,
                                        sharded=True)
        _MODELS[key] = (model, w)       # keeps w alive so its id stays unique
    return _MODELS[key][0]


@torch.inference_mode()
def tp_forward(token_ids: torch.Tensor, w: dict, cfg: ModelConfig, world: int,
               comm_stats: dict | None = None) -> torch.Tensor:
    """Prefill forward over this rank's shard ``w``; logits ``[T, vocab]`` fp32
    (identical on every rank)."""
    m = _rank_model(w, cfg, world)
    ids = token_ids.detach().cpu().tolist()
    T = len(ids)
    bs = 16
    nb = -(-T // bs)
    kv = m.make_kv_cache(nb, bs)
    md_all = StepMeta(ids, list(range(T)), [(0, T)], [list(range(nb))], [T], bs,
                      cfg.n_heads // cfg.n_kv_heads, m.device, all_logits=True)
    logits = m.dm.forward(md_all, kv.pools)
    if comm_stats is not None and world > 1:
        comm_stats["calls"] += 2 * cfg.n_layers
        comm_stats["bytes"] += 2 * cfg.n_layers * T * cfg.d_model * 2
        comm_stats.setdefault("seconds", 0.0)
    out = logits.clone()
    return out.cpu() if token_ids.device.type == "cpu" else out


def _worker(rank: int, world: int, w: dict, cfg: ModelConfig, token_ids: torch.Tensor,
            port: int, queue, timeout_s: float) -> None:
    import datetime
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s),
                            device_id=torch.device("cuda", rank))
    try:
        shard = shard_weights(w, cfg, rank, world)
        stats = {"calls": 0, "bytes": 0, "seconds": 0.0}
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        logits = tp_forward(token_ids, shard, cfg, world, stats)
        torch.cuda.synchronize()
        stats["wall_seconds"] = time.perf_counter() - t0
        if rank == 0:
            queue.put((logits.cpu(), stats))
    except BaseException as e:  # report instead of leaving rank 0's caller waiting
        if rank == 0:
            queue.put(e)
        raise
    finally:
        from .comm import close_all
        close_all()
        dist.destroy_process_group()


def run_tp_forward(world: int, w: dict, cfg: ModelConfig, token_ids: torch.Tensor,
                   port: int = 29517, timeout_s: float = 300.0) -> tuple[torch.Tensor, dict]:
    """Spawn ``world`` GPU processes, run the sharded forward, return rank 0's
    ``(logits, stats)``.  Raises ``RuntimeError`` if a rank dies or the call
    exceeds ``timeout_s``."""
    if torch.cuda.device_count() < world:
        raise RuntimeError(f"run_tp_forward needs {world} GPUs, found {torch.cuda.device_count()}")
    ctx = mp.get_context("spawn")
    queue = ctx.SimpleQueue()
    procs = [ctx.Process(target=_worker, args=(r, world, w, cfg, token_ids, port, queue, timeout_s))
             for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.time() + timeout_s
    result = None
    while result is None:
        if not queue.empty():
            result = queue.get()
            break
        dead = [p for p in procs if p.exitcode not in (None, 0)]
        if dead:
            break
        if time.time() > deadline:
            break
        time.sleep(0.05)
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
        if p.is_alive():
            p.kill()
            p.join()
    if result is None:
        codes = [p.exitcode for p in procs]
        raise RuntimeError(f"tensor-parallel forward failed or timed out (exit codes {codes})")
    if isinstance(result, BaseException):
        raise RuntimeError(f"rank 0 failed: {result!r}")
    return result
