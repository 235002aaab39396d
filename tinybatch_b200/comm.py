"""Tensor-parallel communicator: the all-reduce that the reference runs as
``dist.all_reduce`` (``src/tinybatch/tensor_parallel.py:76-84``) lives in the
row-parallel GEMM epilogue here; this module sets up the peer memory it uses.

One process per GPU.  ``torch.distributed`` (any backend) is used once, at
construction, to exchange the 64-byte CUDA IPC handles of every rank's
exchange allocation; from then on ranks talk only through NVLink peer memory
inside the kernels.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as N
from . import ops

_OPEN: list["TPComm"] = []


def exchange_handles(mine: bytes, group=None) -> list[bytes]:
    """All ranks' handles in rank order (all_gather over ``group``)."""
    world = dist.get_world_size(group)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor(list(mine), dtype=torch.uint8, device=dev)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t, group=group)
    return [bytes(o.cpu().tolist()) for o in out]


class TPComm:
    """Peer-memory communicator of one rank (see include/tinybatch_b200.h).

    Every exchange names a sequence number whose parity selects one of two
    buffer halves; consecutive row-parallel exchanges must alternate parity
    (and so must consecutive argmax exchanges unless a row-parallel one lies
    between them).  Calls without ``seq`` take the next parity; calls with
    one (the forward passes ``2 * layer + j``) are checked against the
    previous call and raise ``ValueError`` when they would reuse a half."""

    # one-shot (every rank sends its partial to every rank) while a rank's
    # pushed bytes stay at or below this; two-shot (owner reduce, then
    # broadcast) above.  Measured crossover: one-shot faster at t = 2 with
    # 1.3 MB pushed (M = 128, N = 5120), two-shot faster at t = 4 with 3.9 MB
    # and at t = 2 with 5.2 MB
    TWO_SHOT_BYTES = 2 << 20

    def __init__(self, rank: int, world: int, device, n_cols: int, max_rows: int = 16384,
                 group=None, handles_fn=None):
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.n_cols, self.max_rows = n_cols, max_rows
        self.group = group
        lib = N.load()
        handle = ctypes.create_string_buffer(64)
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            N.check(lib.tb_comm_create(rank, world, max_rows, n_cols, ctypes.byref(ptr), handle),
                    "tb_comm_create")
        self._ptr = ptr
        handles = (handles_fn or exchange_handles)(handle.raw, group)
        if len(handles) != world or any(len(h) != 64 for h in handles):
            raise RuntimeError("communicator handle exchange returned malformed handles")
        blob = ctypes.create_string_buffer(b"".join(handles), 64 * world)
        with torch.cuda.device(self.device):
            N.check(lib.tb_comm_open(self._ptr, blob), "tb_comm_open")
        self.closed = False
        # parity of the last row-parallel / argmax exchange (the first call uses 0)
        self._row_par = 1
        self._am_par = 1
        # every rank has mapped every peer before any kernel may write into it
        if world > 1 and dist.is_initialized():
            dist.barrier(group)
        _OPEN.append(self)

    @classmethod
    def from_process_group(cls, device, n_cols: int | None = None, **kw) -> "TPComm":
        rank, world = dist.get_rank(), dist.get_world_size()
        if n_cols is None:
            raise ValueError("n_cols (the model's d_model) is required")
        return cls(rank, world, device, n_cols, **kw)

    @staticmethod
    def _next(seq: int | None, last: int, what: str) -> int:
        if seq is None:
            return 1 - last
        if seq < 0 or (seq & 1) == last:
            raise ValueError(f"{what}: seq {seq} has the parity of the previous exchange")
        return seq

    def use_two_shot(self, M: int, n_cols: int) -> bool:
        return (self.world - 1) * M * n_cols * 2 > self.TWO_SHOT_BYTES

    def row_linear_residual(self, x, w, h, g_next, hg, sq_out, *, seq: int | None = None,
                            row_dst=None, hg2=None, sq2=None, bn=128, splits=1,
                            two_shot: bool | None = None, span=None, **_):
        """Row-parallel projection + fused all-reduce + residual + norm
        prologue.  ``span``: optional device int64 element that the call
        raises to its exchange span in ns (``tb_row_linear_allreduce_residual``)."""
        M, K = x.shape
        Nn = w.shape[0]
        if two_shot is None:
            two_shot = self.use_two_shot(M, Nn)
        seq = self._next(seq, self._row_par, "row-parallel exchange")
        ptr = N.ptr
        N.check(N.load().tb_row_linear_allreduce_residual(
            ptr(x), x.stride(0), ptr(w), w.stride(0), M, Nn, K, ptr(h), h.stride(0), ptr(g_next),
            ptr(hg), hg.stride(0), ptr(sq_out), sq_out.stride(0), ptr(row_dst), ptr(hg2), ptr(sq2),
            sq2.stride(0) if sq2 is not None else 0, self._ptr, seq, int(bool(two_shot)),
            ptr(span), bn, splits, N.stream_ptr()),
            "tb_row_linear_allreduce_residual")
        self._row_par = seq & 1

    def argmax(self, logits, n_local: int, col0: int, out, *, seq: int | None = None) -> None:
        """out[m] = torch.argmax over the whole vocabulary of row m, from this
        rank's shard logits[:, :n_local] (global columns col0 ...)."""
        seq = self._next(seq, self._am_par, "argmax exchange")
        N.check(N.load().tb_argmax_vocab_parallel(
            self._ptr, N.ptr(logits), logits.stride(0), logits.shape[0], n_local, col0,
            N.ptr(out), seq, N.stream_ptr()), "tb_argmax_vocab_parallel")
        self._am_par = seq & 1

    def close(self, barrier: bool = True) -> None:
        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        if barrier and self.world > 1 and dist.is_initialized():
            dist.barrier(self.group)      # no peer may still be writing into our buffers
        with torch.cuda.device(self.device):
            N.check(N.load().tb_comm_destroy(self._ptr), "tb_comm_destroy")
        self.closed = True
        if self in _OPEN:
            _OPEN.remove(self)


def close_all() -> None:
    for c in list(_OPEN):
        c.close(barrier=False)
