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
// one allocation with the same layout; rs/ag/flags[p] point into rank p's
// allocation (peer-mapped for p != rank).
//   rs[p]    [2 parity][world src][plane] bf16: partial sums pushed by each
//            source rank (one-shot: every column; two-shot: the columns rank
//            p owns); a plane holds a whole output tile by tile, each tile as
//            [16-column unit][half][128 rows][8 columns]
//   ag[p]    [2 parity][plane] bf16: reduced sums (two-shot)
//   flags[p] [2 kind][2 parity][world src][max_ctas] u32: "source src's CTA
//            c has delivered call `epoch`" (kind 0: partials, 1: sums)
//   state    this rank's step counter; a call's epoch is
//            state[0] * n_sites + site + 1, its parity epoch & 1
struct CommDev {
  int rank, world;  // world <= 1: no all-reduce
  int two_shot;
  int site, n_sites;
  int max_rows, n_cols, max_ctas;
  uint32_t* state;
  __nv_bfloat16* rs[TB_MAX_RANKS];
  __nv_bfloat16* ag[TB_MAX_RANKS];
  uint32_t* flags[TB_MAX_RANKS];
};

// An L2 warm-up request for the weight the next kernel streams: a bf16
// matrix [rows, k] with row pitch ld elements, read by `splits` K segments
// (split-K boundaries of 64-column blocks); the first `bytes` of every
// (row, segment) are prefetched, in 256 x 256 tensor boxes (the kernel's
// third tensor map).  base == nullptr: none.
struct L2Prefetch {
  const char* base;
  long long ld;
  int rows, k, splits, bytes;
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
  // issued by warp 0 once this CTA's main loop is done
  L2Prefetch pf;
};

// Timeline points recorded when GemmArgs::trace is set.
enum TracePoint : int {
  TR_START = 0,       // CTA set up (barriers, TMEM)
  TR_LOADS_ISSUED,    // producer issued its last TMA load
  TR_ACC_READY,       // epilogue saw the accumulator complete
  TR_PUSHED,          // partials pushed and fenced (all-reduce)
  TR_PARTNERS,        // partner flags observed (all-reduce)
  TR_SUMS,            // reduced sums delivered (two-shot)
  TR_END,             // epilogue done
  TR_PARKED,          // cluster split: partial chunks stored to their owners
  TR_CLUSTER_SYNC,    // cluster split: every member's chunks arrived
  TR_BODY,            // residual finisher: every chunk updated (warp 2)
  TR_COMBINED,        // residual finisher: first chunk updated (warp 2)
  TR_POINTS = 16,
};

// Host side (gemm.cu): validate and copy an L2 warm-up request into g.
int gemm_set_prefetch(GemmArgs& g, const tb_l2_prefetch* p);

}  // namespace tb
