// tcgen05 GEMM with fused epilogues for the Qwen2 layer.
//
//   C[M, N] = A[M, K] . B[N, K]^T        A, B bf16, K-major (row-major, K inner)
//
// A is the activation (tokens x features), B a weight in F.linear layout
// [out_features, in_features].  One CTA computes one 128 x BN output tile
// over a K range (split-K across blockIdx.y):
//   warp 0      TMA producer: 128x64 A and BNx64 B boxes, 128-byte swizzle,
//               STAGES-deep ring of shared-memory slots guarded by mbarriers
//   warp 1      allocates BN TMEM columns; one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) x4 per slot and frees the
//               slot with tcgen05.commit
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator (warp w reads
//               TMEM lanes 32*(w%4)..+31, one output row per thread), then
//               the fused op of the GemmArgs kind below
// Split-K runs in one of two forms.  Cluster (default): the splits of a tile
// form a thread-block cluster; each member stores every 16-column chunk of
// its fp32 partial into the shared memory of the member that owns the chunk,
// and each owner sums its chunks in member order (deterministic) and runs the
// epilogue on them.  Global (caller scratch): each CTA writes its partial to
// the workspace; the last CTA of a tile to arrive (per-tile arrival counter)
// sums the partials in split order and runs the epilogue.
#pragma once

#include "../../include/tinybatch_b200.h"
#include "common.cuh"

namespace tb {

enum EpiKind : int {
  EPI_F32 = 0,     // out fp32 = acc * rowscale                 (lm_head logits)
  EPI_BF16 = 1,    // out bf16 = acc * rowscale
  EPI_QKV = 2,     // bias + RoPE; q -> q_out, k/v -> paged KV pool
  EPI_SWIGLU = 3,  // interleaved gate/up tiles -> silu(g) * u
  EPI_RESID = 4,   // h += acc; hg = bf16(h * g_next); per-tile sum(h^2)
};

constexpr int TB_MAX_RANKS = 8;

// Device view of a tensor-parallel communicator (comm.cu).  Every rank owns
// one allocation with the same layout; rs/ag/am[p] point into rank p's
// allocation (peer-mapped for p != rank).
//   rs[p]  [2 parity][world src][plane] bf16: partials pushed by each source
//          rank (one-shot: every column of every row; two-shot: the rows
//          rank p owns); a plane holds a whole output tile by tile, each tile
//          as [16-column unit][half][128 rows][8 columns]
//   ag[p]  [2 parity][plane] bf16: reduced sums (two-shot)
//   am[p]  [2 parity][world src][max_rows] u64: argmax candidates
// No flags: every buffer holds the all-ones sentinel word (TB_SENTINEL) until
// a peer stores data into it with 8-byte-atomic stores, the receiver polls
// the data words themselves and puts the sentinel back once it has read
// them.  A call's parity (seq & 1) picks the buffer half; consecutive calls
// of one kind alternate parity, so a rank can only write a half again after
// every rank has finished reading it (each call needs every rank's data,
// and a rank pushes call seq+1's data only after its call seq completed).
struct CommDev {
  int rank, world;  // world <= 1: no all-reduce
  int two_shot;
  int par;          // parity of this call (seq & 1)
  int max_rows, n_cols;
  unsigned long long* span_ns;  // optional: max over CTAs of the exchange span
  __nv_bfloat16* rs[TB_MAX_RANKS];
  __nv_bfloat16* ag[TB_MAX_RANKS];
  unsigned long long* am[TB_MAX_RANKS];
};

struct GemmArgs {
  int M, N, K;
  int tiles_m, tiles_n, splits, group_m;
  // Deferred RMSNorm of the A operand: row m is scaled by
  // rsqrt(sum_p sq[p * sq_ld + m] * inv_d + eps) (sq == nullptr: scale 1).
  const float* sq;
  int sq_parts, sq_ld;
  float inv_d, eps;
  // split-K scratch: ws [tiles][splits][BN][128] fp32, counters [tiles] int32 (zeroed)
  float* ws;
  int* counters;
  // EPI_F32 / EPI_BF16 / EPI_SWIGLU / EPI_QKV(q) output
  void* out;
  int ld_out;
  // EPI_QKV
  const __nv_bfloat16* bias;
  const float* rope_cos;  // [max_pos, head_dim/2]
  const float* rope_sin;
  const int* positions;   // [M]
  const int* slots;       // [M] block * block_size + offset in block
  __nv_bfloat16* kv_pool; // [num_blocks, 2, n_kv_heads, block_size, head_dim]
  int n_q_heads, n_kv_heads, head_dim, block_size, max_pos;
  // EPI_RESID
  float* h;
  int ld_h;
  const __nv_bfloat16* gnext;
  __nv_bfloat16* hg;
  int ld_hg;
  float* sq_out;           // [parts, sq_out_ld]: tiles_n parts, tiles_n * splits in cluster split-K
  int sq_out_ld;
  const int* row_dst;      // optional: row m also written to row row_dst[m] of hg2/sq2
  __nv_bfloat16* hg2;
  float* sq2;
  int sq2_ld;
  // EPI_SWIGLU
  int n_feat;
  // EPI_RESID across tensor-parallel ranks (comm.world > 1)
  CommDev comm;
  // debug timeline (tb_debug_trace): per CTA 16 globaltimer stamps, or null
  unsigned long long* trace;
};

// Timeline points recorded when GemmArgs::trace is set.
enum TracePoint : int {
  TR_START = 0,       // CTA set up (barriers, TMEM)
  TR_LOADS_ISSUED,    // producer issued its last TMA load
  TR_ACC_READY,       // epilogue saw the accumulator complete
  TR_PUSHED,          // partials pushed (all-reduce)
  TR_PARTNERS,        // every source's partials received (all-reduce)
  TR_SUMS,            // reduced sums received (two-shot)
  TR_END,             // epilogue done
  TR_PARKED,          // cluster split: partial chunks stored to their owners
  TR_CLUSTER_SYNC,    // cluster split: every member's chunks arrived
  TR_BODY,            // residual finisher: every chunk updated (warp 2)
  TR_COMBINED,        // residual finisher: first chunk updated (warp 2)
  TR_POINTS = 16,
};

}  // namespace tb
