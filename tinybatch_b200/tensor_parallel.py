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
  size of the reduced ``[T, d]`` bf16 tensor per all-reduce) and adds to
  ``seconds`` the exchange's device-measured share of each fused call (the
  longest span any CTA spent from its first push to holding every sum).
* ``run_tp_forward(world, w, cfg, token_ids, port)``: spawns one process per
  GPU, returns rank 0's ``(logits, stats)`` (``:138-151``), with timeouts so
  a dead rank ends the call with an error instead of a hang.
"""
from __future__ import annotations

import os
import pickle
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


# The device model of the last weight dict tp_forward saw in this process
# (key (id(w), world)); a new dict replaces it, so repeated calls with fresh
# dicts do not accumulate device memory.  The entry keeps w alive, so its id
# cannot be reused by another dict while it is cached.
_MODEL: dict = {}


def _rank_model(w: dict, cfg: ModelConfig, world: int):
    """This rank's device model for weight dict ``w`` (built once per dict)."""
    from .model import Qwen2Paged
    key = (id(w), world)
    if _MODEL.get("key") != key:
        release()
        rank = dist.get_rank() if world > 1 else 0
        comm = None
        if world > 1:
            from .comm import TPComm
            comm = TPComm.from_process_group(torch.device("cuda", torch.cuda.current_device()),
                                             n_cols=cfg.d_model, max_rows=4096)
        dev = torch.device("cuda", torch.cuda.current_device())
        model = Qwen2Paged.from_weights(cfg, w, device=dev, rank=rank, world=world, comm=comm,
                                        sharded=True)
        _MODEL.update(key=key, model=model, w=w)
    return _MODEL["model"]


def release() -> None:
    """Drop the cached device model of ``tp_forward`` (closing its
    communicator: every rank must call this together)."""
    old = _MODEL.pop("model", None)
    _MODEL.clear()
    if old is not None and old.dm.comm is not None:
        old.dm.comm.close()
    del old
    torch.cuda.empty_cache()


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
    timed = comm_stats is not None and world > 1
    if timed:
        m.dm.exchange_spans = torch.zeros(m.dm.n_sites, dtype=torch.int64, device=m.device)
    try:
        logits = m.dm.forward(md_all, kv.pools)
    finally:
        spans, m.dm.exchange_spans = m.dm.exchange_spans, None
    if timed:
        comm_stats["calls"] += 2 * cfg.n_layers
        comm_stats["bytes"] += 2 * cfg.n_layers * T * cfg.d_model * 2
        comm_stats["seconds"] = comm_stats.get("seconds", 0.0) + float(spans.sum().item()) * 1e-9
    out = logits.clone()
    return out.cpu() if token_ids.device.type == "cpu" else out


def _worker(rank: int, world: int, port: int, w: dict, cfg: ModelConfig,
            token_ids: torch.Tensor, timeout_s: float, queue) -> None:
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
            queue.put((0, (logits.cpu(), stats)))
    finally:
        from .comm import close_all
        close_all()
        dist.destroy_process_group()


class _Reporter:
    """Queue front that sends every report by value (plain pickle), so a
    tensor in it stays readable after the sending rank has exited."""

    def __init__(self, queue):
        self._q = queue

    def put(self, item) -> None:
        self._q.put(pickle.dumps(item))


def _entry(target, rank, world, port, args, queue):
    """Process body: run ``target``; report an exception to the parent."""
    rep = _Reporter(queue)
    try:
        target(rank, world, port, *args, rep)
    except BaseException as e:  # the parent turns this into a RuntimeError
        rep.put((rank, RuntimeError(f"rank {rank}: {e!r}")))
        raise


def _spawn(world: int, target, args: tuple, port: int, timeout_s: float,
           collect_all: bool = False) -> list:
    """Run ``target(rank, world, port, *args, queue)`` in ``world`` spawned
    processes; each rank reports ``queue.put((rank, payload))`` (rank 0 only
    unless ``collect_all``).  Returns the payloads indexed by rank.  Raises
    ``RuntimeError`` when a rank reports an exception, exits with an error,
    or the results do not arrive within ``timeout_s``; surviving processes
    are then killed, so a dead rank never leaves the caller waiting."""
    ctx = mp.get_context("spawn")
    queue = ctx.SimpleQueue()
    procs = [ctx.Process(target=_entry, args=(target, r, world, port, args, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    need = world if collect_all else 1
    got: dict[int, object] = {}
    error = None
    deadline = time.time() + timeout_s
    while len(got) < need and error is None:
        while not queue.empty():
            rank, payload = pickle.loads(queue.get())
            if isinstance(payload, BaseException):
                error = payload
                break
            got[rank] = payload
        if error is None and len(got) < need:
            dead = [(i, p.exitcode) for i, p in enumerate(procs) if p.exitcode not in (None, 0)]
            if dead:
                error = RuntimeError(f"rank(s) exited with errors: {dead}")
            elif time.time() > deadline:
                error = RuntimeError(f"no result within {timeout_s:.0f} s")
            else:
                time.sleep(0.02)
    for p in procs:
        p.join(timeout=5.0 if error is None else 0.5)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    if error is not None:
        raise RuntimeError(f"tensor-parallel run failed: {error}")
    if not collect_all:
        return [got[0]]
    return [got[r] for r in range(world)]


def run_tp_forward(world: int, w: dict, cfg: ModelConfig, token_ids: torch.Tensor,
                   port: int = 29517, timeout_s: float = 300.0) -> tuple[torch.Tensor, dict]:
    """Spawn ``world`` GPU processes, run the sharded forward, return rank 0's
    ``(logits, stats)``.  Raises ``RuntimeError`` if a rank dies or the call
    exceeds ``timeout_s``."""
    if torch.cuda.device_count() < world:
        raise RuntimeError(f"run_tp_forward needs {world} GPUs, found {torch.cuda.device_count()}")
    return _spawn(world, _worker, (w, cfg, token_ids, timeout_s), port, timeout_s)[0]
