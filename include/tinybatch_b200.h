/*
 * tinybatch_b200 — C ABI of the B200 (sm_100a) kernels for the tensor-parallel
 * paged Qwen2 layer.
 *
 * Conventions
 *   - Every pointer argument is a device pointer unless its name ends in _h.
 *   - bf16 means IEEE bfloat16 (__nv_bfloat16), row-major, leading dimension
 *     (ld*) in elements; weights are in F.linear layout [out, in].
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).
 *   - Every call returns TB_OK (0) or a TB_ERR_* code; tb_last_error() gives
 *     the message of the last failure on the calling thread.  No call
 *     allocates device memory: scratch space ("ws") is owned by the caller.
 *   - Split-K scratch must be zero-filled when first handed to the library;
 *     every call leaves its arrival counters at zero again.
 *   - Device-side problems (a bounded wait that ran out, an out-of-range
 *     block id or position) are recorded in a device status word and read
 *     with tb_status(); the kernel that saw them finishes without faulting.
 *
 * Reference interfaces (coindef/tinybatch, paths relative to its root):
 *   src/tinybatch/model.py         Qwen2Paged.forward  :100-158
 *   src/tinybatch/kv_cache.py      PagedKVCache.write/gather :25-45
 *   src/tinybatch/tensor_parallel.py  tp_forward :64-117, allreduce :76-84
 *   src/tinybatch/engine.py        LLMEngine._sample greedy argmax :149-151
 */
#ifndef TINYBATCH_B200_H
#define TINYBATCH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_OK 0
#define TB_ERR_ARG 1     /* invalid shape, alignment or pointer */
#define TB_ERR_CUDA 2    /* a CUDA call failed */
#define TB_ERR_TIMEOUT 3 /* a bounded wait (device or peer) ran out */
#define TB_ERR_STATE 4   /* communicator not initialised / already closed */

/* Device status codes (tb_status). */
#define TB_STATUS_MBAR_TIMEOUT 101 /* a pipeline barrier wait ran out */
#define TB_STATUS_PEER_TIMEOUT 102 /* a wait for a peer GPU's data ran out */
#define TB_STATUS_BAD_INDEX 103    /* block id / position / slot out of range */

int tb_version(void);
const char* tb_last_error(void);

/* Debug timeline: while buf is not NULL, every GEMM launched afterwards by
 * this process writes, per CTA c, %globaltimer stamps (ns) to buf[16*c + k]
 * for k = 0 start, 1 loads issued, 2 accumulator ready, 3 partials pushed
 * to the peer ranks, 4 owned sums sent (two-shot), 5 every value of the
 * all-reduce received, 6 end, 7 split-K
 * chunks stored to their cluster owners, 8 every cluster member's chunks
 * arrived (unreached points are left as they were).  The tcgen05 prefill
 * attention (CTA c = work item + n_work * kv head) writes 32 entries per CTA
 * at buf[32*c + k]: %globaltimer at k = 0 (start) and 31 (end), and clock64
 * stamps (SM cycles; 30 / 29 = start / end) of its pipeline: 1 Q stored, 26 Q seen
 * by the MMA thread, 27 output read, and for key tiles j < 3 at 2 + 8j: K
 * loads start / issued, V loads start / issued, S issued, S read, P stored,
 * PV issued.  buf must hold 16
 * entries per CTA of the largest GEMM launch and 32 per CTA of the largest
 * prefill.  Not thread-safe; NULL turns it off. */
int tb_debug_trace(unsigned long long* buf);

/* Read (and optionally clear) the device status word of the current device.
 * Synchronises the device. */
int tb_status(unsigned int* code_h, int clear);

/* ------------------------------------------------------------------ GEMMs
 * Common arguments of the GEMM entry points:
 *   x [M, K] bf16 (ldx), w [N, K] bf16 (ldw): out = x . w^T, fp32 accumulate
 *   sq, sq_parts, sq_ld, inv_d, eps: deferred RMSNorm of x.  When sq is not
 *     NULL, row m of the product is scaled by
 *     rsqrt(inv_d * sum_{p<sq_parts} sq[p*sq_ld + m] + eps), i.e. x holds
 *     h * norm_weight and sq holds partial sums of h^2 — exactly
 *     rms_norm(h) . w^T of src/tinybatch/model.py:65-69.
 *   bn: output tile width (64, 128, 192 or 256); splits: split-K factor.
 *   ws/ws_bytes: how split-K partials are combined.
 *     ws == NULL, splits in 2..8: the splits of an output tile run as one
 *       thread-block cluster; each CTA stores every 16-column chunk of its
 *       fp32 partial into the shared memory of the member that owns the
 *       chunk (distributed shared memory), and each owner sums its chunks in
 *       split order (deterministic, no scratch) and finishes them.  The
 *       chunks a member receives must fit its pipeline buffers: calls whose
 *       (bn, splits) do not fit fail with TB_ERR_ARG (bn 256 with 7 splits
 *       for the gate/up and the head_dim >= 32 QKV projections).
 *     ws != NULL: partials go through caller scratch of at least
 *       tb_gemm_scratch_bytes(M, N, bn, splits) bytes: a fixed 64 KiB region
 *       of per-tile arrival counters (zero when first handed over, left zero
 *       by every call, so one arena can serve every GEMM), then fp32 partial
 *       tiles; the last CTA of a tile to arrive reduces them.
 *     Unused when splits == 1.
 */
size_t tb_gemm_scratch_bytes(int M, int N, int bn, int splits);

/* How many clusters of `cluster` GEMM CTAs (tile width bn) fit on the current
 * device at once (cudaOccupancyMaxActiveClusters); for choosing splits. */
int tb_gemm_max_active_clusters(int bn, int cluster, int* out_h);

/* Plain projection: out = rowscale * x . w^T, fp32 (out_f32=1) or bf16.
 * Replaces F.linear of the LM head (src/tinybatch/model.py:158,
 * tensor_parallel.py:117). */
int tb_linear(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
              const float* sq, int sq_parts, int sq_ld, float inv_d, float eps,
              void* out, int ld_out, int out_f32, int bn, int splits,
              void* ws, size_t ws_bytes, void* stream);

/* Bytes of split-K scratch built into the library for
 * tb_linear_static_scratch: 4 KiB of arrival counters (at most 1024 output
 * tiles) followed by fp32 partial tiles. */
#define TB_STATIC_SCRATCH_BYTES (8u << 20)

/* tb_linear for callers that cannot allocate device memory (no counterpart
 * in the reference).  Some callers may not call cudaMalloc at all -- code
 * running inside a custom allocator, or next to a framework that has already
 * reserved all device memory for its own pool -- yet still want the split-K
 * projection, which needs scratch for its partial tiles.  This variant takes
 * that scratch from a fixed array inside the library
 * (TB_STATIC_SCRATCH_BYTES per device, held by every GPU that loads the
 * library until the process exits) and allocates nothing.  Arguments and
 * result are those of tb_linear without ws/ws_bytes.
 *   - A call whose split-K scratch would exceed the array (or 1024 tiles)
 *     fails with TB_ERR_ARG and a message naming the size it needed.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current); make that first call
 *     before any stream capture.  After a device reset (a new primary
 *     context) the next call looks it up again.
 *   - All calls on a device share the array and it keeps the last call's
 *     contents; each call clears the counters it needs.  Calls that may run
 *     at the same time on one device (unordered streams) race on it. */
int tb_linear_static_scratch(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
                             const float* sq, int sq_parts, int sq_ld, float inv_d, float eps,
                             void* out, int ld_out, int out_f32, int bn, int splits,
                             void* stream);

/* Column-parallel fused QKV projection.  w_qkv = [Wq; Wk; Wv] of this rank's
 * heads ([(Hq+2Hkv)*hd, K]), bias likewise.  Epilogue: rowscale, + bias,
 * NeoX RoPE of q and k with the fp32 tables rope_cos/rope_sin
 * [max_pos, hd/2], q -> q_out [M, Hq*hd]; k, v -> kv_pool
 * [num_blocks, 2, Hkv, block_size, hd] at flat slot slots[m]
 * (= block*block_size + offset).
 * Replaces q/k/v F.linear + _rope + PagedKVCache.write
 * (src/tinybatch/model.py:119-128, kv_cache.py:25-38,
 *  tensor_parallel.py:92-97).  bn must be a multiple of hd; rope_cos and
 * rope_sin 16-byte aligned. */
int tb_qkv_rope_kv(const void* x, int ldx, const void* w_qkv, int ldw, const void* bias,
                   int M, int K, int n_q_heads, int n_kv_heads, int head_dim,
                   const float* sq, int sq_parts, int sq_ld, float inv_d, float eps,
                   const float* rope_cos, const float* rope_sin, int max_pos,
                   const int* positions, const int* slots,
                   void* q_out, int ld_q, void* kv_pool, int block_size,
                   int bn, int splits, void* ws, size_t ws_bytes, void* stream);

/* Column-parallel gate/up projection with SwiGLU epilogue.  w_gu holds, for
 * each output tile t of width bn, the bn/2 gate rows of features
 * [t*bn/2, (t+1)*bn/2) followed by the matching bn/2 up rows (zero rows pad
 * the last tile).  act [M, n_feat] = silu(g) * u.
 * Replaces gate/up F.linear + F.silu(gate)*up (src/tinybatch/model.py:152-154,
 * tensor_parallel.py:111-114). */
int tb_gate_up_swiglu(const void* x, int ldx, const void* w_gu, int ldw, int M, int K,
                      int n_feat, const float* sq, int sq_parts, int sq_ld, float inv_d,
                      float eps, void* act, int ld_act, int bn, int splits,
                      void* ws, size_t ws_bytes, void* stream);

/* Row-parallel projection + residual + next-norm prologue, single rank:
 *   h[m, :] += x . w^T  (fp32 residual stream, in place)
 *   hg = bf16(h * g_next), sq_out[part, m] = partial sums of h^2 over the row
 * so the next GEMM applies rms_norm(h) * g_next through its rowscale.
 * Optional gather: when row_dst is not NULL and row_dst[m] >= 0, row m of hg
 * and of sq_out is also written to row row_dst[m] of hg2 / sq2.
 * Replaces h + F.linear(attn, Wo) / h + F.linear(act, Wd) and the following
 * _rms_norm (src/tinybatch/model.py:149-151,154,156; tensor_parallel.py:108-110,114,116).
 * The number of sq parts written is ceil(N / bn), times splits with cluster
 * split-K (ws == NULL, splits > 1: one part per cluster member). */
int tb_row_linear_residual(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
                           float* h, int ld_h, const void* g_next, void* hg, int ld_hg,
                           float* sq_out, int sq_out_ld, const int* row_dst, void* hg2,
                           float* sq2, int sq2_ld, int bn, int splits, void* ws,
                           size_t ws_bytes, void* stream);

/* ------------------------------------------------- tensor-parallel comm
 * One communicator per rank (one process per GPU).  It owns one device
 * allocation per rank (exchange buffers for max_rows x n_cols bf16 partials
 * and sums, argmax candidate slots for max_rows rows), made at creation and
 * shared with the other ranks through CUDA IPC:
 *   1. tb_comm_create on every rank -> a 64-byte cudaIpcMemHandle;
 *   2. exchange the handles (e.g. torch.distributed all_gather);
 *   3. tb_comm_open with all world handles in rank order;
 *   4. the exchange calls below, the same calls in the same order on every
 *      rank;
 *   5. after a barrier, tb_comm_destroy.
 * The exchanges carry no flags: every buffer word holds an all-ones sentinel
 * until a peer's data lands, the receiver polls the data itself and puts the
 * sentinel back.  Each call names a sequence number `seq`; its parity picks
 * one of two buffer halves.  Rules (the caller keeps them; a violation can
 * mix two calls' data):
 *   - consecutive tb_row_linear_allreduce_residual calls on a communicator
 *     have seq of alternating parity (e.g. 2l and 2l+1 for layer l);
 *   - consecutive tb_argmax_vocab_parallel calls alternate parity too, or
 *     have at least one row-parallel call between them.
 * A wait that runs out (5 s) sets TB_STATUS_PEER_TIMEOUT and leaves data in
 * the buffers: destroy and recreate the communicator after one.
 * Replaces torch.distributed all_reduce(SUM) in the reference's
 * tensor_parallel.py:76-84 (called at :108 and :114). */
int tb_comm_create(int rank, int world, int max_rows, int n_cols, void** comm_out,
                   void* ipc_handle_out);
int tb_comm_open(void* comm, const void* ipc_handles);
int tb_comm_destroy(void* comm);

/* Row-parallel projection with the all-reduce fused into its epilogue:
 *   h += sum over ranks of (x_r . w_r^T)   (x_r, w_r: this rank's K shard)
 * then hg / sq_out as tb_row_linear_residual.  Each CTA pushes its bf16
 * partial of every 16-column unit of its tile over NVLink: two_shot = 0 to
 * every rank, which sums the world partials in rank order; two_shot = 1 to
 * the unit's owner rank ((tile * bn/16 + unit) % world), which sums them in
 * rank order and sends the bf16 sum to every rank.  Every rank adds the same
 * values, so h stays identical on all ranks.  Every rank must make the same
 * calls (same M, N, K, bn, splits, seq, two_shot) in the same order.
 * span_ns (optional device pointer): the call raises *span_ns to the longest
 * time, in ns, that any of its CTAs spent between starting to push and
 * holding every sum it needs (the exchange's share of the call).
 * Replaces allreduce(F.linear(attn, Wo)) / allreduce(F.linear(act, Wd)) + the
 * residual add and next _rms_norm (tensor_parallel.py:76-84, :108-110, :114-116). */
int tb_row_linear_allreduce_residual(const void* x, int ldx, const void* w, int ldw, int M, int N,
                                     int K, float* h, int ld_h, const void* g_next, void* hg,
                                     int ld_hg, float* sq_out, int sq_out_ld, const int* row_dst,
                                     void* hg2, float* sq2, int sq2_ld, void* comm, int seq,
                                     int two_shot, unsigned long long* span_ns, int bn,
                                     int splits, void* stream);

/* Greedy sampling over a vocabulary-parallel LM head: row m of logits
 * (fp32, row pitch ld) holds this rank's n_local vocabulary columns, global
 * columns col0 .. col0+n_local-1 (shards ordered by rank).  Every rank
 * writes out[m] = the first index of the row's maximum over the whole
 * vocabulary (torch.argmax of the full row; 0 when no value exceeds -inf).
 * One (value, index) candidate per row and rank travels through the
 * communicator (seq: see the rules above).  M <= max_rows.  Replaces the
 * replicated F.linear(h, lm_head) + argmax of the reference
 * (tensor_parallel.py:117, engine.py:149-151) for the sampled rows. */
int tb_argmax_vocab_parallel(void* comm, const float* logits, int ld, int M, int n_local,
                             int col0, int* out, int seq, void* stream);

/* ------------------------------------------------------------- attention
 * Paged GQA attention reading K/V through block tables (no gather copy).
 *   q [*, Hq*hd] bf16 (ld_q), out [*, Hq*hd] bf16 (ld_out)
 *   block_tables [n_seqs, bt_ld] int32, q_start/q_len/ctx_len [n_seqs] int32
 * Sequence s has query rows q_start[s] .. +q_len[s]; its query token i sits at
 * position ctx_len[s]-q_len[s]+i and attends to keys 0..that position.
 * Replaces PagedKVCache.gather + repeat_interleave + SDPA
 * (src/tinybatch/model.py:131-147, kv_cache.py:40-45, tensor_parallel.py:99-105).
 *
 * _decode: every sequence must have q_len*Hq/Hkv <= 16 (decode steps).
 *   Keys are split into pieces of split_tokens (a multiple of 16); grid is
 *   sized for max_ctx.  Scratch: tb_attention_scratch_bytes, zero-filled
 *   before its first use; its first 64 KiB hold per-(seq, kv head) arrival
 *   counters that every completed call leaves at zero (the last split CTA
 *   of a pair merges the splits in split order, in the same launch).
 *   At most 16384 (sequence, kv head) pairs per call with more than one split.
 *   split_tokens <= 8192.  seq_order (optional, [n_seqs] int32, a
 *   permutation): sequences are dispatched in this order (longest first
 *   keeps the tail of the launch short); NULL = index order.
 * _prefill: any q_len; work_pairs [n_work, 2] int32 = (seq, tile) with
 *   tiles of 256 query rows (row = token * Hq/Hkv + head in the group), best
 *   ordered longest first; entries naming no sequence of the call, a tile
 *   past its prompt, or a context longer than bt_ld blocks set
 *   TB_STATUS_BAD_INDEX.  head_dim 64 / 128 with block_size a multiple of 16
 *   run on the tensor cores (tcgen05: two 128-row tiles per CTA share each
 *   K/V tile; S, P and O in TMEM). */
size_t tb_attention_scratch_bytes(int n_seqs, int n_kv_heads, int head_dim, int max_ctx,
                                  int split_tokens);
int tb_paged_attention_decode(const void* q, int ld_q, void* out, int ld_out,
                              const void* kv_pool, int num_blocks, int n_q_heads,
                              int n_kv_heads, int head_dim, int block_size,
                              const int* block_tables, int bt_ld, const int* q_start,
                              const int* q_len, const int* ctx_len, const int* seq_order,
                              int n_seqs, int max_ctx, int split_tokens, void* ws,
                              size_t ws_bytes, void* stream);
int tb_paged_attention_prefill(const void* q, int ld_q, void* out, int ld_out,
                               const void* kv_pool, int num_blocks, int n_q_heads,
                               int n_kv_heads, int head_dim, int block_size,
                               const int* block_tables, int bt_ld, const int* q_start,
                               const int* q_len, const int* ctx_len, int n_seqs,
                               const int* work_pairs, int n_work, void* stream);

/* ------------------------------------------------------ embedding, sampling */

/* h[m] = float(emb[ids[m]]); hg = bf16(h * g); sq[m] = sum h^2 (one part).
 * Replaces F.embedding + the first _rms_norm (src/tinybatch/model.py:112,116). */
int tb_embed(const int* ids, int M, const void* emb, int ld_emb, int d, int vocab,
             const void* g, float* h, int ld_h, void* hg, int ld_hg, float* sq, void* stream);

/* out[m] = argmax_n logits[m, n] (first maximal index), logits fp32.
 * Replaces the greedy branch of LLMEngine._sample (src/tinybatch/engine.py:149-151). */
int tb_argmax(const float* logits, int ld, int M, int N, int* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TINYBATCH_B200_H */
