"""Thin torch-tensor wrappers over the C ABI (one function per fused kernel).

Every function checks shapes on the host, calls the library on the current
CUDA stream and raises ``NativeError`` on a nonzero return code.  Scratch
buffers come from a ``Scratch`` arena owned by the caller (nothing here
allocates per call except when no arena is given).
"""
from __future__ import annotations

import torch

from . import _native as N
from ._native import ptr


class Scratch:
    """A zero-initialised device arena reused by every call that needs
    split-K or split-KV scratch.  Grows (re-zeroed) when a call needs more."""

    def __init__(self, device, nbytes: int = 0):
        self.device = torch.device(device)
        self.buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=self.device)
        self.version = 0        # bumped on every growth (captured graphs must check it)
        self._retired: list[torch.Tensor] = []

    def get(self, nbytes: int) -> tuple[int | None, int]:
        if nbytes == 0:
            return None, 0
        if nbytes > self.buf.numel():
            # the old buffer stays alive: a graph captured on it never reads freed memory
            self._retired.append(self.buf)
            self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self.version += 1
        return self.buf.data_ptr(), self.buf.numel()


def _gemm_scratch(scratch: Scratch | None, device, M, n_cols, bn, splits, split_mode):
    """Scratch for a GEMM call: none for cluster split-K (the default),
    caller scratch for ``split_mode="global"``."""
    if splits <= 1 or split_mode == "cluster":
        return None, 0, None
    if split_mode != "global":
        raise ValueError(f"split_mode must be 'cluster' or 'global', not {split_mode!r}")
    return _scratch(scratch, device, N.load().tb_gemm_scratch_bytes(M, n_cols, bn, splits))


def _scratch(scratch: Scratch | None, device, nbytes: int):
    if nbytes == 0:
        return None, 0, None
    if scratch is None:
        scratch = Scratch(device, nbytes)
    p, n = scratch.get(nbytes)
    return p, n, scratch


def _sq(sq):
    """(ptr, parts, ld) of a deferred-norm partial-sum buffer [parts, ld] or None."""
    if sq is None:
        return None, 0, 0
    return ptr(sq), sq.shape[0], sq.stride(0)


def linear(x, w, out, *, sq=None, inv_d=0.0, eps=0.0, bn=128, splits=1, scratch=None,
           split_mode="cluster"):
    lib = N.load()
    M, K = x.shape
    Nn = w.shape[0]
    ws, wsn, _ = _gemm_scratch(scratch, x.device, M, Nn, bn, splits, split_mode)
    sp, parts, sld = _sq(sq)
    N.check(lib.tb_linear(ptr(x), x.stride(0), ptr(w), w.stride(0), M, Nn, K, sp, parts, sld,
                          inv_d, eps, ptr(out), out.stride(0), int(out.dtype == torch.float32),
                          bn, splits, ws, wsn, N.stream_ptr()), "tb_linear")
    return out


def qkv_rope_kv(x, w_qkv, bias, *, n_q_heads, n_kv_heads, head_dim, sq, inv_d, eps,
                rope_cos, rope_sin, positions, slots, q_out, kv_pool, block_size,
                bn=128, splits=1, scratch=None, split_mode="cluster"):
    lib = N.load()
    M, K = x.shape
    Nn = w_qkv.shape[0]
    ws, wsn, _ = _gemm_scratch(scratch, x.device, M, Nn, bn, splits, split_mode)
    sp, parts, sld = _sq(sq)
    N.check(lib.tb_qkv_rope_kv(ptr(x), x.stride(0), ptr(w_qkv), w_qkv.stride(0), ptr(bias), M,
                               K, n_q_heads, n_kv_heads, head_dim, sp, parts, sld, inv_d, eps,
                               ptr(rope_cos), ptr(rope_sin), rope_cos.shape[0], ptr(positions),
                               ptr(slots), ptr(q_out), q_out.stride(0), ptr(kv_pool),
                               block_size, bn, splits, ws, wsn, N.stream_ptr()),
            "tb_qkv_rope_kv")


def gate_up_swiglu(x, w_gu, act, *, n_feat, sq, inv_d, eps, bn=128, splits=1, scratch=None,
                   split_mode="cluster"):
    lib = N.load()
    M, K = x.shape
    Nn = w_gu.shape[0]
    ws, wsn, _ = _gemm_scratch(scratch, x.device, M, Nn, bn, splits, split_mode)
    sp, parts, sld = _sq(sq)
    N.check(lib.tb_gate_up_swiglu(ptr(x), x.stride(0), ptr(w_gu), w_gu.stride(0), M, K, n_feat,
                                  sp, parts, sld, inv_d, eps, ptr(act), act.stride(0), bn,
                                  splits, ws, wsn, N.stream_ptr()),
            "tb_gate_up_swiglu")
    return act


def row_parts(n_cols: int, bn: int, splits: int, split_mode: str = "cluster") -> int:
    """Rows of deferred-norm partial sums a row-parallel call writes: one per
    column tile, or per (column tile, cluster member) with cluster split-K."""
    tiles = -(-n_cols // bn)
    return tiles * splits if (splits > 1 and split_mode == "cluster") else tiles


def row_linear_residual(x, w, h, g_next, hg, sq_out, *, row_dst=None, hg2=None, sq2=None,
                        bn=128, splits=1, scratch=None, split_mode="cluster"):
    lib = N.load()
    M, K = x.shape
    Nn = w.shape[0]
    ws, wsn, _ = _gemm_scratch(scratch, x.device, M, Nn, bn, splits, split_mode)
    N.check(lib.tb_row_linear_residual(
        ptr(x), x.stride(0), ptr(w), w.stride(0), M, Nn, K, ptr(h), h.stride(0), ptr(g_next),
        ptr(hg), hg.stride(0), ptr(sq_out), sq_out.stride(0), ptr(row_dst), ptr(hg2),
        ptr(sq2), sq2.stride(0) if sq2 is not None else 0, bn, splits, ws, wsn,
        N.stream_ptr()), "tb_row_linear_residual")


def paged_attention_decode(q, out, kv_pool, *, n_q_heads, n_kv_heads, head_dim, block_size,
                           block_tables, q_start, q_len, ctx_len, max_ctx, split_tokens=512,
                           seq_order=None, scratch=None):
    """``seq_order`` (optional int32 [n]): the order in which sequences are
    dispatched (e.g. longest first)."""
    lib = N.load()
    n = ctx_len.shape[0]
    ws, wsn, _ = _scratch(scratch, q.device, lib.tb_attention_scratch_bytes(
        n, n_kv_heads, head_dim, max_ctx, split_tokens))
    N.check(lib.tb_paged_attention_decode(
        ptr(q), q.stride(0), ptr(out), out.stride(0), ptr(kv_pool), kv_pool.shape[0],
        n_q_heads, n_kv_heads, head_dim, block_size, ptr(block_tables), block_tables.stride(0),
        ptr(q_start), ptr(q_len), ptr(ctx_len), ptr(seq_order), n, max_ctx, split_tokens, ws,
        wsn, N.stream_ptr()), "tb_paged_attention_decode")


def paged_attention_prefill(q, out, kv_pool, *, n_q_heads, n_kv_heads, head_dim, block_size,
                            block_tables, q_start, q_len, ctx_len, work):
    if work.dim() != 2 or work.shape[1] != 2 or work.dtype != torch.int32:
        raise ValueError("work must be an int32 [n_work, 2] tensor of (sequence, row tile)")
    lib = N.load()
    n = ctx_len.shape[0]
    N.check(lib.tb_paged_attention_prefill(
        ptr(q), q.stride(0), ptr(out), out.stride(0), ptr(kv_pool), kv_pool.shape[0],
        n_q_heads, n_kv_heads, head_dim, block_size, ptr(block_tables), block_tables.stride(0),
        ptr(q_start), ptr(q_len), ptr(ctx_len), n, ptr(work), work.shape[0], N.stream_ptr()),
        "tb_paged_attention_prefill")


def embed(ids, emb, g, h, hg, sq):
    lib = N.load()
    M = ids.shape[0]
    N.check(lib.tb_embed(ptr(ids), M, ptr(emb), emb.stride(0), emb.shape[1], emb.shape[0],
                         ptr(g), ptr(h), h.stride(0), ptr(hg), hg.stride(0), ptr(sq),
                         N.stream_ptr()), "tb_embed")


def argmax(logits, out):
    lib = N.load()
    M, V = logits.shape
    N.check(lib.tb_argmax(ptr(logits), logits.stride(0), M, V, ptr(out), N.stream_ptr()),
            "tb_argmax")
    return out


def max_active_clusters(bn: int, cluster: int) -> int:
    import ctypes
    out = ctypes.c_int(0)
    N.check(N.load().tb_gemm_max_active_clusters(bn, cluster, ctypes.byref(out)),
            "tb_gemm_max_active_clusters")
    return out.value
