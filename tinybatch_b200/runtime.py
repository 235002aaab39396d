"""Device-side forward of the (tensor-parallel) paged Qwen2 model on one rank.

Per decoder layer the forward is five kernel launches, all from the C ABI:

  1. tb_qkv_rope_kv          column-parallel q|k|v GEMM; epilogue applies the
                             deferred input RMSNorm, bias and RoPE, writes q
                             and scatters k, v into the paged pool
  2. tb_paged_attention_*    GQA attention over the pool through block tables
  3. tb_row_linear_residual  row-parallel o_proj; epilogue: (all-reduce,)
                             residual add, next-norm prologue (h*g, sum h^2)
  4. tb_gate_up_swiglu       column-parallel gate|up GEMM with SwiGLU epilogue
  5. tb_row_linear_residual  row-parallel down_proj, same epilogue as 3

The residual stream ``h`` stays fp32 on the device.  RMSNorm is never a
separate pass: the row-parallel epilogue stores ``hg = bf16(h * g)`` and
per-tile partial sums of ``h^2``; the next GEMM multiplies its rows by
``rsqrt(mean(h^2) + eps)``, which equals ``rms_norm(h, g) @ W^T``
(``src/tinybatch/model.py:65-69``).
"""
from __future__ import annotations

import itertools
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from . import ops
from .config import ModelConfig

SMS = 148


# ------------------------------------------------------------------ planning

_CLUSTERS: list[int] | None = None
# clusters of 1..8 GEMM CTAs resident at once on a B200 (one CTA per SM);
# replaced by the device's own answer on first use
_CLUSTERS_B200 = [148, 74, 45, 33, 26, 22, 15, 15]


def _cluster_capacity() -> list[int]:
    global _CLUSTERS
    if _CLUSTERS is None:
        try:
            _CLUSTERS = [ops.max_active_clusters(128, c) for c in range(1, 9)]
        except Exception:
            _CLUSTERS = list(_CLUSTERS_B200)
    return _CLUSTERS


# Shared-memory ring of each tile width (stages x (A + B) bytes); cluster
# split-K receives the members' partial chunks in it.
_RING_BYTES = {64: 8 * (16384 + 8192), 128: 6 * (16384 + 16384), 192: 5 * (16384 + 24576),
               256: 4 * (16384 + 32768)}


def cluster_fits(bn: int, splits: int, paired: bool = False) -> bool:
    """Whether a cluster member's share of the partial chunks fits its ring:
    splits x ceil(pairs / splits) x chunks-per-pair x (128 x 16 fp32)."""
    np_, cp = (bn // 32, 2) if paired else (bn // 16, 1)
    return splits * -(-np_ // splits) * cp * 8192 <= _RING_BYTES[bn]


def plan_gemm(M: int, N: int, K: int, bns=(64, 128, 192, 256), max_splits: int = 8,
              paired: bool = False) -> tuple[int, int]:
    """Tile width and cluster split-K factor for C[M,N] = A[M,K] B[N,K]^T.

    Time model, fitted to device timelines of the decode shapes on B200:
    a CTA streams its B slice from HBM at min(50 GB/s, 6 TB/s / active
    CTAs), takes its A and B boxes into shared memory at ~95 GB/s (A comes
    from L2 but still passes through the SM's copy engine: narrow tiles pay
    for it), or is bound by its share of the tensor pipe (~10.8 TFLOP/s per
    SM), whichever is slowest; its epilogue then costs ~1.5 us of
    launch and prologue, ~0.9 us per 16-column chunk it finishes and, with
    split-K, one cluster barrier (~1.3 us) plus the partial chunks it stores
    into the other members' shared memory at ~25 GB/s.  A launch with more
    CTAs than fit at once runs ceil(CTAs / resident CTAs) waves.
    ``paired``: the epilogue finishes chunk pairs (SwiGLU, RoPE); only
    (bn, splits) whose cluster chunks fit shared memory are considered."""
    cap = _cluster_capacity()
    tm = -(-M // 128)
    num_k = -(-K // 64)
    best = None
    for bn in bns:
        tiles = tm * -(-N // bn)
        for s in range(1, max_splits + 1):
            if s > num_k or (s > 1 and num_k / s < 2):
                break
            if s > 1 and not cluster_fits(bn, s, paired):
                continue
            ctas = tiles * s
            k_it = -(-num_k // s)
            b_bytes = k_it * 64 * 2 * bn
            ab_bytes = b_bytes + k_it * 64 * 2 * 128
            cta_flops = 2.0 * 128 * bn * 64 * k_it
            epi = 1.5e-6 + 0.9e-6 * (bn / 16) / s
            if s > 1:
                epi += 1.3e-6 + (bn * 128 * 4 * (s - 1) / s) / 25e9
            if tiles <= cap[s - 1]:
                bw = min(50e9, 6.0e12 / ctas)
                t = max(b_bytes / bw, ab_bytes / 95e9, cta_flops / 10.8e12) + epi
            else:     # several waves of fully busy SMs (39 GB/s each); a tail
                # wave costs a whole wave (and, in a fused all-reduce, another
                # exchange round trip)
                waves = -(-ctas // (cap[s - 1] * s))
                t = waves * (max(b_bytes / 39e9, ab_bytes / 95e9, cta_flops / 10.8e12) + epi)
            if best is None or t < best[0]:
                best = (t, bn, s)
    return best[1], best[2]


def vocab_shard(vocab: int, rank: int, world: int) -> tuple[int, int]:
    """(first column, columns) of a rank's slice of a vocabulary-parallel LM
    head: ceil(vocab / world) columns per rank in rank order, the last slice
    shorter (possibly empty)."""
    per = -(-vocab // world)
    col0 = min(rank * per, vocab)
    return col0, max(0, min(per, vocab - col0))


# Resident CTAs of the decode attention kernel on a B200 (148 SMs x 3).
ATTN_SLOTS = 148 * 3
ATTN_MAX_SPLIT = 8192


def decode_split_tokens(n_seqs: int, n_kv: int, ctx_total: int, max_ctx: int,
                        slots: int = ATTN_SLOTS) -> int:
    """Keys per split-KV piece of a decode attention launch.  Measured on the
    14B decode shards (TP 1-8): fastest when the launch has about 0.6 CTAs
    per resident slot.  So when the (sequence, kv head) pairs alone reach
    that, every pair runs as one CTA (dispatched longest first, no merge);
    otherwise the keys are cut to about that many CTAs.  A multiple of 16 in
    [256, 8192]."""
    target = 0.6 * slots
    if n_seqs * n_kv >= target:
        split = max_ctx
    else:
        split = -(-ctx_total * n_kv // int(target))
    return min(ATTN_MAX_SPLIT, max(256, -(-split // 16) * 16))


# ------------------------------------------------------------------ weights

@dataclass
class LayerWeights:
    wqkv: torch.Tensor   # [(Hq+2Hkv)/t*hd, d]
    bqkv: torch.Tensor   # [(Hq+2Hkv)/t*hd]
    wo: torch.Tensor     # [d, Hq/t*hd]
    wgu: torch.Tensor    # [tiles*gu_bn, d] interleaved gate/up
    wd: torch.Tensor     # [d, ff/t]
    ln_in: torch.Tensor  # [d]
    ln_post: torch.Tensor


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, bn: int) -> torch.Tensor:
    """Rows of tile t: gate rows of features [t*bn/2, (t+1)*bn/2), then the
    matching up rows; the last tile is padded with zero rows."""
    F, K = gate.shape
    half = bn // 2
    tiles = -(-F // half)
    out = torch.zeros(tiles, 2, half, K, dtype=gate.dtype, device=gate.device)
    pad = tiles * half - F
    g = torch.nn.functional.pad(gate, (0, 0, 0, pad)).view(tiles, half, K)
    u = torch.nn.functional.pad(up, (0, 0, 0, pad)).view(tiles, half, K)
    out[:, 0] = g
    out[:, 1] = u
    return out.view(tiles * bn, K)


class RankWeights:
    """One tensor-parallel rank's weights, packed for the fused kernels, bf16
    on the rank's device.  ``w`` is the full (unsharded) HF-named dict; the
    split is the Megatron one of ``src/tinybatch/tensor_parallel.py:35-61``."""

    # gate/up tile: 96 features of gate + 96 of up; 13824/t features give
    # 144 tiles at t = 1, 72 at t = 2 ... so decode fills ~144 SMs at any degree
    GU_BN = 192

    def __init__(self, cfg: ModelConfig, w: dict, rank: int = 0, world: int = 1,
                 device="cuda", sharded: bool = False):
        assert cfg.n_heads % world == 0, "q heads must divide tp degree"
        assert cfg.n_kv_heads % world == 0, "kv heads must divide tp degree"
        assert cfg.d_ff % world == 0, "d_ff must divide tp degree"
        self.cfg, self.rank, self.world = cfg, rank, world
        self.device = torch.device(device)
        bf = torch.bfloat16

        def dev(t):
            return t.detach().to(device=self.device, dtype=bf).contiguous()

        def col(t):
            return dev(t if sharded else t.chunk(world, dim=0)[rank])

        def row(t):
            return dev(t if sharded else t.chunk(world, dim=1)[rank])

        self.n_q = cfg.n_heads // world
        self.n_kv = cfg.n_kv_heads // world
        self.ff = cfg.d_ff // world
        self.layers: list[LayerWeights] = []
        for i in range(cfg.n_layers):
            p = f"model.layers.{i}."
            q, k, v = (col(w[p + f"self_attn.{n}_proj.weight"]) for n in "qkv")
            biases = []
            for n, rows in (("q", q.shape[0]), ("k", k.shape[0]), ("v", v.shape[0])):
                b = w.get(p + f"self_attn.{n}_proj.bias")
                biases.append(col(b) if b is not None else torch.zeros(rows, dtype=bf, device=self.device))
            self.layers.append(LayerWeights(
                wqkv=torch.cat([q, k, v], 0).contiguous(),
                bqkv=torch.cat(biases, 0).contiguous(),
                wo=row(w[p + "self_attn.o_proj.weight"]),
                wgu=interleave_gate_up(col(w[p + "mlp.gate_proj.weight"]),
                                       col(w[p + "mlp.up_proj.weight"]), self.GU_BN).contiguous(),
                wd=row(w[p + "mlp.down_proj.weight"]),
                ln_in=dev(w[p + "input_layernorm.weight"]),
                ln_post=dev(w[p + "post_attention_layernorm.weight"]),
            ))
        self.emb = dev(w["model.embed_tokens.weight"])
        head = w.get("lm_head.weight")
        tied = head is None or head is w["model.embed_tokens.weight"]
        self.lm_head = self.emb if tied else dev(head)
        self.final_norm = dev(w["model.norm.weight"])
        self.rope_cos, self.rope_sin = rope_tables(cfg, self.device)


def rope_tables(cfg: ModelConfig, device) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin [max_position, hd/2] with the reference's arithmetic
    (``src/tinybatch/model.py:75-77``: inv_freq = 1/theta^(arange(0,hd,2)/hd),
    angle = float(pos) * inv_freq), computed once on the CPU."""
    hd = cfg.head_dim
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
    ang = torch.arange(cfg.max_position, dtype=torch.float32)[:, None] * inv_freq[None, :]
    return ang.cos().to(device).contiguous(), ang.sin().to(device).contiguous()


# ------------------------------------------------------------------ metadata

PREFILL_ROWS = 256      # query rows per prefill attention work item (two 128-row tiles)


def prefill_work(q_len, ctx, group: int) -> np.ndarray:
    """Prefill attention work list: (sequence, tile of 256 query rows) pairs,
    row = token * group + head, ordered by the keys each tile reads (its last
    row's causal limit), most first, so long tiles start early."""
    items, cost = [], []
    for r, (ql, c) in enumerate(zip(np.asarray(q_len).tolist(), np.asarray(ctx).tolist())):
        rows = ql * group
        first = c - ql
        for t in range(-(-rows // PREFILL_ROWS)):
            last = min(t * PREFILL_ROWS + PREFILL_ROWS - 1, rows - 1)
            items.append((r, t))
            cost.append(min(c, first + last // group + 1))
    order = sorted(range(len(items)), key=lambda i: -cost[i])
    return np.asarray([items[i] for i in order], dtype=np.int32).reshape(-1, 2)


class StepMeta:
    """Device int32 metadata of one flat mixed batch, built on the host with
    numpy and shipped in one host->device copy.  Block tables may be lists
    or int numpy arrays.

    Fields: ids, positions, slots [T]; row_dst [T] (sequence index of each
    sequence's last token, else -1); for the decode subset (q_len*G <= 16)
    and the prefill subset: q_start, q_len, ctx_len [n], block tables
    [n, bt_ld] (-1 padded); the decode subset's order by descending context
    length; the prefill (sequence, 256-row tile) work list (``prefill_work``)."""

    def __init__(self, token_ids, positions, seq_slices, block_tables, context_lens,
                 block_size: int, group: int, device, pinned: bool = True,
                 all_logits: bool = False, bt_width: int = 0,
                 dest: torch.Tensor | None = None, staging: torch.Tensor | None = None):
        """``bt_width`` pads the block tables to at least that many columns
        (a fixed layout for CUDA-graph replay); ``dest``, a device int32
        buffer of exactly the packed size, receives the metadata instead of
        a fresh allocation; ``staging``, a pinned int32 host buffer at least
        that large, is reused for the copy instead of pinning a new one (the
        caller keeps it untouched until the copy has completed)."""
        if isinstance(token_ids, torch.Tensor):
            token_ids = token_ids.detach().cpu().numpy()
        if isinstance(positions, torch.Tensor):
            positions = positions.detach().cpu().numpy()
        ids = np.asarray(token_ids, dtype=np.int64).astype(np.int32)
        pos = np.asarray(positions, dtype=np.int64).astype(np.int32)
        T = ids.shape[0]
        n = len(seq_slices)
        starts = np.fromiter((s for s, _ in seq_slices), dtype=np.int32, count=n)
        ends = np.fromiter((e for _, e in seq_slices), dtype=np.int32, count=n)
        qlen = ends - starts
        ctx = np.asarray(context_lens, dtype=np.int32)
        # block tables as one flat array with row offsets (one pass over the lists)
        lens = np.fromiter(map(len, block_tables), dtype=np.int64, count=n)
        offs = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(lens, out=offs[1:])
        if n and all(isinstance(t, np.ndarray) for t in block_tables):
            flat_bt = np.concatenate(block_tables).astype(np.int64, copy=False)
        else:
            flat_bt = np.fromiter(itertools.chain.from_iterable(block_tables), dtype=np.int64,
                                  count=int(offs[-1]))
        # slot of every token: table[p // bs] * bs + p % bs
        slots = np.full(T, -1, dtype=np.int32)
        n_tok = int(qlen.sum())
        if n_tok:
            tok_seq = np.repeat(np.arange(n), qlen)
            first_of_seq = np.repeat(np.cumsum(qlen) - qlen, qlen)
            tok = np.arange(n_tok) - first_of_seq + np.repeat(starts, qlen)
            p = pos[tok].astype(np.int64)
            blk = p // block_size
            if np.any(blk >= lens[tok_seq]) or np.any(p < 0):
                raise IndexError("a token position lies beyond its sequence's block table")
            slots[tok] = (flat_bt[offs[tok_seq] + blk] * block_size + p % block_size).astype(np.int32)
        if all_logits:          # every token row gets logits (tp_forward)
            row_dst = np.arange(T, dtype=np.int32)
        else:
            row_dst = np.full(T, -1, dtype=np.int32)
            row_dst[ends[qlen > 0] - 1] = np.nonzero(qlen > 0)[0].astype(np.int32)
        self.n_out = T if all_logits else n
        is_dec = qlen * group <= 16
        self.T, self.n = T, n
        self.group = group

        def subset(mask):
            idx = np.nonzero(mask)[0]
            rl = lens[idx]
            bt_ld = max(int(rl.max()) if len(idx) else 0, bt_width, 1)
            bt = np.full((len(idx), bt_ld), -1, dtype=np.int32)
            if len(idx):
                cols = np.arange(bt_ld)
                valid = cols[None, :] < rl[:, None]
                bt[valid] = flat_bt[(offs[idx][:, None] + cols[None, :])[valid]]
            return idx, starts[idx], qlen[idx], ctx[idx], bt

        d_idx, d_qs, d_ql, d_ctx, d_bt = subset(is_dec)
        p_idx, p_qs, p_ql, p_ctx, p_bt = subset(~is_dec)
        work = prefill_work(p_ql, p_ctx, group)
        # decode sequences longest first: the attention grid dispatches in this order
        d_order = np.argsort(-d_ctx, kind="stable").astype(np.int32)
        parts = [ids, pos, slots, row_dst, d_qs, d_ql, d_ctx, d_bt.ravel(), d_order, p_qs, p_ql,
                 p_ctx, p_bt.ravel(), work.ravel()]
        flat = np.concatenate(parts).astype(np.int32)
        if staging is not None and staging.numel() >= flat.size:
            host = staging[: flat.size]
            host.numpy()[:] = flat
        else:
            host = torch.from_numpy(flat)
            if pinned and torch.device(device).type == "cuda":
                host = host.pin_memory()
        if dest is not None:
            if dest.numel() != flat.size:
                raise ValueError("metadata layout differs from the destination buffer")
            dest.copy_(host, non_blocking=True)
            buf = dest
        else:
            buf = host.to(device, non_blocking=True)
        self.buf = buf
        self.layout = (T, n, int(is_dec.sum()), d_bt.shape[1], p_bt.shape[1], work.shape[0],
                       all_logits)
        self.h2d_bytes = flat.nbytes
        views, o = [], 0
        for a in parts:
            views.append(buf[o:o + a.size])
            o += a.size
        (self.ids, self.positions, self.slots, self.row_dst, self.dec_q_start, self.dec_q_len,
         self.dec_ctx, dbt, self.dec_order, self.pre_q_start, self.pre_q_len, self.pre_ctx, pbt,
         wk) = views
        self.dec_bt = dbt.view(len(d_idx), d_bt.shape[1])
        self.pre_bt = pbt.view(len(p_idx), p_bt.shape[1])
        self.work = wk.view(-1, 2)
        self.n_dec, self.n_pre = len(d_idx), len(p_idx)
        self.dec_ctx_sum = int(d_ctx.astype(np.int64).sum())
        self.pre_ctx_sum = int(p_ctx.astype(np.int64).sum())
        self.dec_tokens = int(d_ql.astype(np.int64).sum())
        # causal (query, key) pairs of the prefill subset, for the flop count
        first = (p_ctx - p_ql).astype(np.int64)
        ql = p_ql.astype(np.int64)
        self.pre_pairs = int((ql * first + ql * (ql + 1) // 2).sum())
        self.dec_max_ctx = int(d_ctx.max()) if len(d_idx) else 1
        self._keep = (host, buf)


# ------------------------------------------------------------------ forward

class DeviceModel:
    """Buffers and the launch sequence of the forward on one rank."""

    def __init__(self, weights: RankWeights, max_tokens: int = 2048, max_seqs: int = 256,
                 comm=None, split_tokens: int | None = None):
        self.w = weights
        self.cfg = weights.cfg
        self.device = weights.device
        self.comm = comm
        # decode split-KV size (None: decode_split_tokens per call)
        self.split_tokens = split_tokens
        # with a communicator, sampled steps score only this rank's slice of
        # the vocabulary and exchange argmax candidates (tb_argmax_vocab_parallel);
        # full logits (sample=False) still come from the whole, replicated head
        self.vocab_parallel = comm is not None
        # row-parallel exchange sites of one forward: o_proj (2l) and down_proj
        # (2l + 1) of every layer, passed as the exchange's sequence number, so
        # every forward starts at parity 0 and ends at parity 1
        self.n_sites = 2 * self.cfg.n_layers
        # when a device int64 tensor [n_sites], every row-parallel exchange
        # raises its element to the exchange's span in ns (tp_forward's
        # comm_stats["seconds"])
        self.exchange_spans: torch.Tensor | None = None
        # split-K scratch (arrival counters must stay zero between calls) and
        # split-KV attention scratch live in separate arenas
        self.scratch = ops.Scratch(self.device, 1 << 20)
        self.attn_scratch = ops.Scratch(self.device, 1 << 20)
        # when a list, every launch appends (kind, start event, end event,
        # algorithmic bytes, flops) -- used by the benchmark's roofline
        self.prof: list | None = None
        self._alloc(max_tokens, max_seqs)

    def _run(self, kind: str, nbytes: float, flops: float, fn, *a, **kw):
        if self.prof is None:
            return fn(*a, **kw)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        r = fn(*a, **kw)
        e.record()
        self.prof.append((kind, s, e, nbytes, flops))
        return r

    def generation(self) -> tuple:
        """Changes whenever a buffer a captured graph may point to is replaced."""
        return (self._alloc_gen, self.scratch.version, self.attn_scratch.version)

    def _alloc(self, T: int, S: int) -> None:
        cfg, w, dev = self.cfg, self.w, self.device
        self._alloc_gen = getattr(self, "_alloc_gen", -1) + 1
        # previous buffers stay referenced so a stale graph cannot touch freed memory
        self._retired = getattr(self, "_retired", [])
        if hasattr(self, "h"):
            self._retired.append((self.h, self.hg, self.sq, self.q, self.attn, self.act,
                                  self.hg_last, self.sq_last, self.logits, self.next_ids))
        d = cfg.d_model
        self.T_max, self.S_max = T, S
        # deferred-norm partial sums: one row per (column tile, cluster member)
        self.parts_max = max(-(-d // 64), 1) * 8
        self.h = torch.zeros(T, d, device=dev)
        self.hg = torch.zeros(T, d, device=dev, dtype=torch.bfloat16)
        self.sq = torch.zeros(self.parts_max, T, device=dev)
        self.q = torch.zeros(T, w.n_q * cfg.head_dim, device=dev, dtype=torch.bfloat16)
        self.attn = torch.zeros(T, w.n_q * cfg.head_dim, device=dev, dtype=torch.bfloat16)
        ff_pad = -(-w.ff // 64) * 64
        self.act = torch.zeros(T, ff_pad, device=dev, dtype=torch.bfloat16)
        self.hg_last = torch.zeros(S, d, device=dev, dtype=torch.bfloat16)
        self.sq_last = torch.zeros(self.parts_max, S, device=dev)
        v_pad = -(-cfg.vocab_size // 4) * 4      # fp32 rows stay 16-byte aligned
        self.logits = torch.zeros(S, v_pad, device=dev)[:, :cfg.vocab_size]
        self.next_ids = torch.zeros(S, dtype=torch.int32, device=dev)

    def ensure(self, T: int, S: int) -> None:
        if T > self.T_max or S > self.S_max:
            self._alloc(max(T, self.T_max), max(S, self.S_max))

    # one row-parallel projection: residual (+ all-reduce) + norm prologue
    def _row(self, x, wmat, g_next, T, last: bool, md: StepMeta, site: int, plan):
        bn, splits = plan
        kw = dict(bn=bn, splits=splits, scratch=self.scratch)
        if last:
            kw.update(row_dst=md.row_dst, hg2=self.hg_last, sq2=self.sq_last)
        Nn, K = wmat.shape
        nbytes = 2 * Nn * K + 2 * T * K + T * Nn * (4 + 4 + 2)
        proj = "o_proj" if site % 2 == 0 else "down_proj"
        if self.comm is None:
            self._run(f"{proj}_residual", nbytes, 2.0 * T * Nn * K, ops.row_linear_residual, x,
                      wmat, self.h[:T], g_next, self.hg[:T], self.sq, **kw)
        else:
            span = self.exchange_spans[site] if self.exchange_spans is not None else None
            self._run(f"{proj}_allreduce_residual", nbytes, 2.0 * T * Nn * K,
                      self.comm.row_linear_residual, x, wmat, self.h[:T], g_next, self.hg[:T],
                      self.sq, seq=site, span=span, **kw)
        return ops.row_parts(Nn, bn, splits)

    def plans(self, T: int, n: int) -> dict:
        """(bn, splits) of every projection of a forward over T tokens with n
        sampled rows (all layers share their shapes)."""
        cfg, W = self.cfg, self.w
        L = W.layers[0]
        hd = cfg.head_dim
        return {
            "qkv": plan_gemm(T, L.wqkv.shape[0], cfg.d_model,
                             bns=tuple(b for b in (64, 128, 192, 256) if b % hd == 0),
                             paired=hd >= 32),
            "o": plan_gemm(T, L.wo.shape[0], L.wo.shape[1]),
            "gu": (RankWeights.GU_BN,
                   plan_gemm(T, L.wgu.shape[0], cfg.d_model, bns=(RankWeights.GU_BN,),
                             paired=True)[1]),
            "down": plan_gemm(T, L.wd.shape[0], L.wd.shape[1]),
            "lm": plan_gemm(n, cfg.vocab_size, cfg.d_model),
            "lm_shard": plan_gemm(n, max(1, vocab_shard(cfg.vocab_size, 0, self._world())[1]),
                                  cfg.d_model),
        }

    def _world(self) -> int:
        return self.comm.world if self.comm is not None else 1

    def forward(self, md: StepMeta, kv_pools: list[torch.Tensor], compute_logits: bool = True,
                sample: bool = False, attn_max_ctx: int | None = None,
                attn_split: int | None = None):
        """Launch the forward.  ``attn_max_ctx`` sizes the decode attention
        grid (default: this batch's longest context); a CUDA graph passes its
        bound so one capture serves every context length up to it, and
        ``attn_split`` its split-KV size."""
        cfg, W = self.cfg, self.w
        T, n = md.T, md.n_out
        self.ensure(T, n)
        d, hd = cfg.d_model, cfg.head_dim
        inv_d, eps = 1.0 / d, cfg.rms_eps
        bs = kv_pools[0].shape[3]
        pl = self.plans(T, n)
        self._run("embed", T * d * (2 + 4 + 2), 0.0, ops.embed, md.ids, W.emb, W.layers[0].ln_in,
                  self.h[:T], self.hg[:T], self.sq[0])
        kv_row = 2 * W.n_kv * hd * 2          # K+V bytes of one token in one layer
        dec_ctx = md.dec_ctx_sum
        pre_ctx = md.pre_ctx_sum
        parts = 1
        for li, L in enumerate(W.layers):
            pool = kv_pools[li]
            bn, splits = pl["qkv"]
            Nq = L.wqkv.shape[0]
            self._run("qkv_rope_kv", 2 * Nq * d + 2 * T * d + 2 * T * Nq, 2.0 * T * Nq * d,
                      ops.qkv_rope_kv, self.hg[:T], L.wqkv, L.bqkv, n_q_heads=W.n_q, n_kv_heads=W.n_kv,
                            head_dim=hd, sq=self.sq[:parts], inv_d=inv_d, eps=eps,
                            rope_cos=W.rope_cos, rope_sin=W.rope_sin, positions=md.positions,
                            slots=md.slots, q_out=self.q[:T], kv_pool=pool, block_size=bs,
                            bn=bn, splits=splits, scratch=self.scratch)
            akw = dict(n_q_heads=W.n_q, n_kv_heads=W.n_kv, head_dim=hd, block_size=bs)
            qrow = W.n_q * hd * 2
            if md.n_dec:
                mc = attn_max_ctx or md.dec_max_ctx
                split = attn_split or self.split_tokens or decode_split_tokens(
                    md.n_dec, W.n_kv, md.n_dec * mc if attn_max_ctx else md.dec_ctx_sum, mc)
                self._run(
                    "attention_decode", dec_ctx * kv_row + 2 * md.dec_tokens * qrow,
                    4.0 * md.dec_ctx_sum * W.n_q * hd, ops.paged_attention_decode,
                    self.q, self.attn, pool, block_tables=md.dec_bt, q_start=md.dec_q_start,
                    q_len=md.dec_q_len, ctx_len=md.dec_ctx, seq_order=md.dec_order,
                    max_ctx=mc, split_tokens=split, scratch=self.attn_scratch, **akw)
            if md.n_pre:
                self._run(
                    "attention_prefill", pre_ctx * kv_row + 2 * (T - md.dec_tokens) * qrow,
                    4.0 * md.pre_pairs * W.n_q * hd, ops.paged_attention_prefill,
                    self.q, self.attn, pool, block_tables=md.pre_bt, q_start=md.pre_q_start,
                    q_len=md.pre_q_len, ctx_len=md.pre_ctx, work=md.work, **akw)
            parts = self._row(self.attn[:T], L.wo, L.ln_post, T, False, md, 2 * li, pl["o"])
            bn, splits = pl["gu"]
            Ngu = L.wgu.shape[0]
            self._run("gate_up_swiglu", 2 * Ngu * d + 2 * T * d + 2 * T * W.ff, 2.0 * T * Ngu * d,
                      ops.gate_up_swiglu, self.hg[:T], L.wgu, self.act[:T], n_feat=W.ff,
                      sq=self.sq[:parts], inv_d=inv_d, eps=eps, bn=bn, splits=splits,
                      scratch=self.scratch)
            last = li == len(W.layers) - 1
            g_next = W.final_norm if last else W.layers[li + 1].ln_in
            parts = self._row(self.act[:T, :W.ff], L.wd, g_next, T, last, md, 2 * li + 1,
                              pl["down"])
        if not compute_logits:
            return None
        V = cfg.vocab_size
        if sample and self.comm is not None and self.vocab_parallel:
            # each rank scores its vocabulary slice; the argmax exchanges one
            # (value, index) candidate per row and rank
            col0, nv = vocab_shard(V, self.comm.rank, self.comm.world)
            out = self.logits[:n, :nv]
            if nv:
                bn, splits = pl["lm_shard"]
                self._run("lm_head", 2 * nv * d + 2 * n * d + 4 * n * nv, 2.0 * n * nv * d,
                          ops.linear, self.hg_last[:n], W.lm_head[col0:col0 + nv], out,
                          sq=self.sq_last[:parts], inv_d=inv_d, eps=eps, bn=bn, splits=splits,
                          scratch=self.scratch)
            self._run("argmax", 4 * n * nv, 0.0, self.comm.argmax, self.logits[:n], nv, col0,
                      self.next_ids[:n])
            return out
        bn, splits = pl["lm"]
        out = self.logits[:n]
        self._run("lm_head", 2 * V * d + 2 * n * d + 4 * n * V, 2.0 * n * V * d, ops.linear,
                  self.hg_last[:n], W.lm_head, out, sq=self.sq_last[:parts], inv_d=inv_d,
                  eps=eps, bn=bn, splits=splits, scratch=self.scratch)
        if sample:
            self._run("argmax", 4 * n * V, 0.0, ops.argmax, out, self.next_ids[:n])
        return out


class DecodeGraph:
    """One decode step of ``n`` sequences captured as a CUDA graph.

    The graph reads its metadata from a static device buffer laid out for
    ``n`` decode sequences with block tables ``bt_width`` wide; attention is
    sized for contexts up to ``max_ctx``.  ``run(md)`` expects ``md`` built
    into ``self.dest`` (``StepMeta(..., bt_width=, dest=graph.dest)``), or
    copies it there, then replays: every kernel of the step, no host work."""

    def __init__(self, dm: DeviceModel, kv_pools, n: int, bt_width: int, max_ctx: int,
                 block_size: int, ctx_total: int | None = None):
        """``ctx_total``: the summed context length of a typical batch (the
        one being captured for): the split-KV size is chosen for it."""
        self.dm, self.pools = dm, kv_pools
        self.n, self.bt_width, self.max_ctx = n, bt_width, max_ctx
        group = dm.cfg.n_heads // dm.cfg.n_kv_heads
        self.split = dm.split_tokens or decode_split_tokens(
            n, dm.w.n_kv, ctx_total if ctx_total else n * max_ctx, max_ctx)
        # a valid dummy batch: every sequence has one token at position 0 in block 0
        self.md = StepMeta([0] * n, [0] * n, [(i, i + 1) for i in range(n)],
                           [[0]] * n, [1] * n, block_size, group, dm.device,
                           bt_width=bt_width)
        self.dest = self.md.buf
        # two pinned host buffers, alternated by staging(): a step's metadata
        # copy is issued from one while the previous step's may still be reading
        # the other
        self._staging = [torch.empty(self.dest.numel(), dtype=torch.int32).pin_memory()
                         for _ in range(2)]
        self._turn = 0
        # one eager run (sizes the scratch arenas and sets kernel attributes
        # outside the capture) on a throw-away one-block pool per layer, so the
        # dummy batch never writes into the live cache; the capture itself
        # executes nothing and records the real pools
        p0 = kv_pools[0]
        dummy = [torch.zeros((1,) + tuple(p0.shape[1:]), dtype=p0.dtype, device=p0.device)
                 for _ in kv_pools]
        dm.forward(self.md, dummy, sample=True, attn_max_ctx=max_ctx, attn_split=self.split)
        torch.cuda.synchronize(dm.device)
        del dummy
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            dm.forward(self.md, kv_pools, sample=True, attn_max_ctx=max_ctx,
                       attn_split=self.split)
        torch.cuda.synchronize(dm.device)
        self.gen = dm.generation()

    def staging(self) -> torch.Tensor:
        """The next pinned host buffer for a ``StepMeta(..., dest=self.dest)``."""
        self._turn ^= 1
        return self._staging[self._turn]

    def stale(self) -> bool:
        return self.gen != self.dm.generation()

    def matches(self, md: StepMeta) -> bool:
        return md.layout == self.md.layout and md.dec_max_ctx <= self.max_ctx

    def run(self, md: StepMeta) -> None:
        if self.stale():
            raise RuntimeError("decode graph is stale: a buffer it uses was reallocated")
        if md.buf.data_ptr() != self.dest.data_ptr():
            if not self.matches(md):
                raise ValueError("batch does not fit the captured decode graph")
            self.dest.copy_(md.buf)
        self.graph.replay()
