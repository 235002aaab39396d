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
// With split-K each CTA writes its fp32 partial to the caller's workspace;
// the last CTA of a tile to arrive (per-tile arrival counter) sums the
// partials in split order (deterministic) and runs the epilogue.
#pragma once

#include "common.cuh"

namespace tb {

enum EpiKind : int {
  EPI_F32 = 0,     // out fp32 = acc * rowscale                 (lm_head logits)
  EPI_BF16 = 1,    // out bf16 = acc * rowscale
  EPI_QKV = 2,     // bias + RoPE; q -> q_out, k/v -> paged KV pool
  EPI_SWIGLU = 3,  // interleaved gate/up tiles -> silu(g) * u
  EPI_RESID = 4,   // h += acc; hg = bf16(h * g_next); per-tile sum(h^2)
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
  float* sq_out;           // [tiles_n, sq_out_ld]
  int sq_out_ld;
  const int* row_dst;      // optional: row m also written to row row_dst[m] of hg2/sq2
  __nv_bfloat16* hg2;
  float* sq2;
  int sq2_ld;
  // EPI_SWIGLU
  int n_feat;
};

}  // namespace tb
