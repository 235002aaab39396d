// Paged GQA attention that reads K/V straight from the block pool.
//
// Pool layout (unchanged from the reference): [num_blocks, 2, n_kv, bs, hd]
// bf16, K at index 0 and V at 1; token at position p of a sequence lives in
// block table[p / bs], slot p % bs.
//
// Rows.  For one (sequence, kv head) the query rows are the pairs
// (query token i, head g in the kv head's group of G = Hq/Hkv heads), row
// r = i*G + g.  Query token i sits at absolute position ctx - q_len + i and
// sees keys 0 .. ctx - q_len + i (causal with a cached prefix).
//
// Math.  S = Q K^T and O = P V run on mma.sync m16n8k16 (bf16 in, fp32
// accumulate) over 16-token key chunks staged in shared memory with
// cp.async (16-byte pieces, XOR-swizzled so ldmatrix is conflict-free);
// softmax is the online (running max / running sum) form in base 2.
//
//   decode kernels  q_len*G <= 16 rows; one CTA per (split, kv head, seq);
//                   4 warps take interleaved key chunks of the split and
//                   merge their (max, sum, O) in shared memory; with more
//                   than one split the CTA writes (O/l, log2 l + max) to the
//                   workspace and the last split CTA of the (seq, kv head)
//                   to finish merges all splits in split order (an arrival
//                   counter per pair, reset by the merging CTA).  Chunks arrive by
//                   TMA (a producer warp, 8-slot mbarrier ring) when the
//                   block size is a multiple of 16 and hd is 64 or 128,
//                   else by per-lane cp.async.
//   prefill         256 query rows per CTA (a work item (sequence, 256-row
//                   tile) per kv head): for head_dim 64 / 128 and block sizes
//                   that are multiples of 16 on tcgen05 (attn_prefill_tc_kernel:
//                   cp.async gathers, S and O in TMEM); otherwise 8 warps of
//                   16 rows on mma.sync with key chunks shared by the warps.
#include "attention.cuh"
#include "common.cuh"
#include "host.h"

namespace tb {

extern unsigned long long* g_debug_trace;   // tb_debug_trace (null: no timeline)


__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// One arrival on `bar` once every cp.async this thread issued so far has
// landed (the barrier's count includes the arrival).
__device__ __forceinline__ void cp_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 16-token chunk of K (or V) for one kv head: [16][HD] bf16, 16-byte pieces
// XOR-swizzled within each row.
template <int HD>
struct ChunkLayout {
  static constexpr int CPR = HD / 8;                   // 16-byte pieces per row
  static constexpr int XM = (CPR < 8 ? CPR : 8) - 1;  // swizzle mask
  static constexpr int BYTES = 16 * HD * 2;
  __device__ static __forceinline__ int off(int t, int c) { return t * HD * 2 + ((c ^ (t & XM)) << 4); }
};

// Issue the cp.async pieces of key chunk `chunk` (K and V) handled by this
// thread (thread `tid` of `nthr`).
template <int HD>
__device__ __forceinline__ void load_chunk(const AttnArgs& a, const int* table, int kvh, int ctx,
                                           int chunk, uint32_t sk, uint32_t sv, int tid, int nthr) {
  using C = ChunkLayout<HD>;
  const size_t head_stride = (size_t)a.block_size * HD;
  for (int i = tid; i < 16 * C::CPR; i += nthr) {
    const int t = i / C::CPR, c = i % C::CPR;
    const int p = chunk * 16 + t;
    bool ok = p < ctx;
    const __nv_bfloat16* src = a.pool;
    if (ok) {
      const int blk = table[p / a.block_size];
      if (blk < 0 || blk >= a.num_blocks) {
        set_status(ERR_BAD_INDEX);
        ok = false;
      } else {
        src = a.pool + ((size_t)blk * 2 * a.n_kv_heads + kvh) * head_stride +
              (size_t)(p % a.block_size) * HD + c * 8;
      }
    }
    cp_async16(sk + C::off(t, c), src, ok);
    cp_async16(sv + C::off(t, c), ok ? src + (size_t)a.n_kv_heads * head_stride : src, ok);
  }
}

// 16-token chunk written by TMA with 128-byte swizzling: the head dimension
// is cut in 64-element halves, each a [16 rows][128 B] box whose 16-byte units
// are XOR-permuted by (row % 8); halves are 2 KiB apart.
template <int HD>
struct TmaChunkLayout {
  static constexpr int BYTES = 16 * HD * 2;
  __device__ static __forceinline__ int off(int t, int c) {
    return (c >> 3) * 2048 + t * 128 + (((c & 7) ^ (t & 7)) << 4);
  }
};

// Per-warp flash state for 16 rows: thread holds rows lane/4 and lane/4+8.
// C gives the shared-memory layout of a K or V chunk.
template <int HD, class C = ChunkLayout<HD>>
struct Flash {
  float o[HD / 8][4];
  float m[2], l[2];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
  }

  // One 16-key chunk.  qa: A fragments of Q; `limit[h]` = last key position
  // row-half h may see (inclusive); keys >= ctx are masked too.
  __device__ __forceinline__ void step(const uint32_t (*qa)[4], uint32_t sk, uint32_t sv,
                                       int chunk, int ctx, const int* limit, float scale_log2,
                                       int lane) {
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t b[4];
      const int tok = (mi >> 1) * 8 + rr;
      ldsm_x4(sk + C::off(tok, ks * 2 + (mi & 1)), b);
      mma16816(s[0], qa[ks], b[0], b[1]);
      mma16816(s[1], qa[ks], b[2], b[3]);
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int p = chunk * 16 + nt * 8 + 2 * (lane & 3) + (e & 1);
        float v = s[nt][e] * scale_log2;
        if (p >= ctx || p > limit[h]) v = -INFINITY;
        s[nt][e] = v;
        mx[h] = fmaxf(mx[h], v);
      }
    float alpha[2], mu[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float mn = fmaxf(m[h], mx[h]);
      mu[h] = mn == -INFINITY ? 0.f : mn;
      alpha[h] = exp2f(m[h] - mu[h]);
      m[h] = mn;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[nt][e] - mu[e >> 1]);
        s[nt][e] = p;
        rs[e >> 1] += p;
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) l[h] = l[h] * alpha[h] + rs[h];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(s[0][0], s[0][1]);
    pa[1] = pack_bf16x2(s[0][2], s[0][3]);
    pa[2] = pack_bf16x2(s[1][0], s[1][1]);
    pa[3] = pack_bf16x2(s[1][2], s[1][3]);
#pragma unroll
    for (int dt = 0; dt < HD / 16; ++dt) {
      uint32_t b[4];
      const int tok = (mi & 1) * 8 + rr;
      ldsm_x4_t(sv + C::off(tok, dt * 2 + (mi >> 1)), b);
      mma16816(o[2 * dt], pa, b[0], b[1]);
      mma16816(o[2 * dt + 1], pa, b[2], b[3]);
    }
  }

  __device__ __forceinline__ void finish_sum() {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
    }
  }
};

// A fragments of 16 query rows (rows >= nrows are zero).
template <int HD>
__device__ __forceinline__ void load_q(const AttnArgs& a, int q0, int G, int kvh, int row0,
                                       int nrows, int lane, uint32_t (*qa)[4]) {
  const int g4 = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = row0 + g4 + half * 8;
    const bool ok = (r - row0) < nrows;
    const __nv_bfloat16* src =
        ok ? a.q + (size_t)(q0 + r / G) * a.ld_q + (size_t)(kvh * G + r % G) * HD : a.q;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t lo = 0, hi = 0;
      if (ok) {
        lo = *reinterpret_cast<const uint32_t*>(src + ks * 16 + 2 * t4);
        hi = *reinterpret_cast<const uint32_t*>(src + ks * 16 + 8 + 2 * t4);
      }
      qa[ks][half] = lo;
      qa[ks][2 + half] = hi;
    }
  }
}

// Merge the n_splits partial results of (seq, kv head) in split order:
// out = sum_s 2^(lse_s - M) O_s / sum_s 2^(lse_s - M), M = max_s lse_s.
// The partials were written by other CTAs of this launch: read through L2.
template <int HD>
__device__ __forceinline__ void merge_splits(const AttnArgs& a, int seq, int kvh, int n_splits,
                                             int q0, int G, int nrows) {
  const size_t base0 = ((size_t)seq * a.n_kv_heads + kvh) * a.max_splits;
  for (int i = threadIdx.x; i < nrows * HD; i += blockDim.x) {
    const int r = i / HD, c = i % HD;
    float M = -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, __ldcg(a.ws_lse + (base0 + s) * 16 + r));
    const float mu = M == -INFINITY ? 0.f : M;
    float W = 0.f, acc = 0.f;
#pragma unroll 4
    for (int s = 0; s < n_splits; ++s) {
      const float w = exp2f(__ldcg(a.ws_lse + (base0 + s) * 16 + r) - mu);
      W += w;
      acc += w * __ldcg(a.ws_o + ((base0 + s) * 16 + r) * HD + c);
    }
    a.out[(size_t)(q0 + r / G) * a.ld_out + (size_t)(kvh * G + r % G) * HD + c] =
        __float2bfloat16_rn(W > 0.f ? acc / W : 0.f);
  }
}

// Merge the per-warp flash states of nw warps (smem: O[nw][16][HD] fp32,
// m[nw][16], l[nw][16], then one int) and write the normalised rows:
// straight to `out` when the sequence has one split, else (O/l, max +
// log2 l) to the split workspace, after which the last split CTA of this
// (seq, kv head) to arrive merges every split.  Called by every thread of the
// CTA after the key loop.
template <int HD, class F>
__device__ __forceinline__ void merge_warps(const AttnArgs& a, F& f, uint8_t* smem, int nw,
                                            int warp, int lane, int seq, int kvh, int split,
                                            int n_splits, int q0, int G, int nrows,
                                            bool participates) {
  constexpr int LD = HD + 4;  // padded rows: no bank conflicts on the fragment stores
  float* so = reinterpret_cast<float*>(smem);
  float* sm = so + nw * 16 * LD;
  float* sl = sm + nw * 16;
  if (participates) {
    const int g4 = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = g4 + (e >> 1) * 8, c = nt * 8 + 2 * t4 + (e & 1);
        so[(warp * 16 + r) * LD + c] = f.o[nt][e];
      }
    if (t4 == 0) {
      sm[warp * 16 + g4] = f.m[0];
      sm[warp * 16 + g4 + 8] = f.m[1];
      sl[warp * 16 + g4] = f.l[0];
      sl[warp * 16 + g4 + 8] = f.l[1];
    }
  }
  __syncthreads();
  const bool direct = n_splits == 1;
  for (int i = threadIdx.x; i < nrows * HD; i += blockDim.x) {
    const int r = i / HD, c = i % HD;
    float M = -INFINITY;
    for (int w = 0; w < nw; ++w) M = fmaxf(M, sm[w * 16 + r]);
    const float mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, acc = 0.f;
    for (int w = 0; w < nw; ++w) {
      const float sc = exp2f(sm[w * 16 + r] - mu);
      L += sl[w * 16 + r] * sc;
      acc += so[(w * 16 + r) * LD + c] * sc;
    }
    const float val = L > 0.f ? acc / L : 0.f;
    if (direct) {
      a.out[(size_t)(q0 + r / G) * a.ld_out + (size_t)(kvh * G + r % G) * HD + c] =
          __float2bfloat16_rn(val);
    } else {
      const size_t base = (((size_t)seq * a.n_kv_heads + kvh) * a.max_splits + split) * 16 + r;
      a.ws_o[base * HD + c] = val;
      if (c == 0) a.ws_lse[base] = L > 0.f ? mu + log2f(L) : -INFINITY;
    }
  }
  if (direct) return;
  // publish this split, then count arrivals; the last CTA merges
  int* last = reinterpret_cast<int*>(sl + nw * 16);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* cnt = a.ws_count + (size_t)seq * a.n_kv_heads + kvh;
    const int prev = atomicAdd(cnt, 1);
    const int is_last = prev == n_splits - 1;
    if (is_last) *cnt = 0;   // ready for the next call
    *last = is_last;
  }
  __syncthreads();
  if (!*last) return;
  __threadfence();
  merge_splits<HD>(a, seq, kvh, n_splits, q0, G, nrows);
}

constexpr int DEC_STAGES = 3;

template <int HD>
__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnArgs a) {
  using C = ChunkLayout<HD>;
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int seq = a.seq_order != nullptr ? a.seq_order[blockIdx.z] : (int)blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (seq < 0 || seq >= a.n_seqs) {
    if (threadIdx.x == 0) set_status(ERR_BAD_INDEX);
    return;
  }
  const int ctx = a.ctx_len[seq], qlen = a.q_len[seq], q0 = a.q_start[seq];
  const int G = a.n_q_heads / a.n_kv_heads;
  const int nrows = qlen * G;
  const int n_chunks = (ctx + 15) / 16;
  const int n_splits = (n_chunks + a.split_chunks - 1) / a.split_chunks;
  if (split >= n_splits || nrows <= 0) return;
  if (nrows > 16) {
    set_status(ERR_BAD_INDEX);
    return;
  }
  const int c_begin = split * a.split_chunks;
  const int c_end = min(c_begin + a.split_chunks, n_chunks);
  const int* table = a.block_tables + (size_t)seq * a.bt_ld;

  uint32_t qa[HD / 16][4];
  load_q<HD>(a, q0, G, kvh, 0, nrows, lane, qa);
  int limit[2];
  {
    const int first = ctx - qlen;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = min((lane >> 2) + 8 * h, nrows - 1);
      limit[h] = first + r / G;
    }
  }

  const uint32_t ring = smem_u32(smem) + warp * DEC_STAGES * 2 * C::BYTES;
  Flash<HD> f;
  f.init();
  // this warp's chunks: c_begin + warp + 4*j
  const int my_n = c_end - c_begin - warp > 0 ? (c_end - c_begin - warp + 3) / 4 : 0;
#pragma unroll
  for (int j = 0; j < DEC_STAGES - 1; ++j) {
    if (j < my_n) {
      const uint32_t st = ring + j * 2 * C::BYTES;
      load_chunk<HD>(a, table, kvh, ctx, c_begin + warp + 4 * j, st, st + C::BYTES, lane, 32);
    }
    cp_commit();
  }
  for (int j = 0; j < my_n; ++j) {
    cp_wait<DEC_STAGES - 2>();
    __syncwarp();
    const uint32_t st = ring + (j % DEC_STAGES) * 2 * C::BYTES;
    f.step(qa, st, st + C::BYTES, c_begin + warp + 4 * j, ctx, limit, a.scale_log2, lane);
    __syncwarp();
    const int jn = j + DEC_STAGES - 1;
    if (jn < my_n) {
      const uint32_t sn = ring + (jn % DEC_STAGES) * 2 * C::BYTES;
      load_chunk<HD>(a, table, kvh, ctx, c_begin + warp + 4 * jn, sn, sn + C::BYTES, lane, 32);
    }
    cp_commit();
  }
  cp_wait<0>();
  f.finish_sum();
  __syncthreads();
  merge_warps<HD>(a, f, smem, 4, warp, lane, seq, kvh, split, n_splits, q0, G, nrows, true);
}

// Decode attention with TMA key/value loads (head_dim 64 or 128, block size a
// multiple of 16).  Warp 4 issues, for every 16-token chunk of the split, one
// 2-D TMA box per 64-column half of K and of V straight from the pool (the
// pool viewed as [num_blocks*2*n_kv*bs rows, hd]), into an 8-slot ring guarded
// by mbarriers; warps 0-3 consume chunks round-robin and merge at the end.
constexpr int TMA_STAGES = 8;
constexpr int TMA_THREADS = 160;
constexpr int TMA_MAX_SPLIT_CHUNKS = 512;   // split_tokens <= 8192
// Chunk i goes to slot i % TMA_STAGES and to consumer warp i % 4.  With the
// stage count a multiple of 4 every slot has a single consumer warp, which
// waits on its slot's phases strictly in order; otherwise a warp could wait
// for a phase two ahead of the slot's current one, and mbarrier parity waits
// cannot tell those apart.
static_assert(TMA_STAGES % 4 == 0, "each ring slot must belong to one consumer warp");

template <int HD>
__global__ void __launch_bounds__(TMA_THREADS, 3)
    attn_decode_tma_kernel(const __grid_constant__ CUtensorMap pool_map, const AttnArgs a) {
  using C = TmaChunkLayout<HD>;
  constexpr int SLOT = 2 * C::BYTES;  // K then V
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TMA_STAGES * SLOT);
  uint64_t* empty = full + TMA_STAGES;
  int* chunk_row = reinterpret_cast<int*>(empty + TMA_STAGES);  // [split_chunks] pool row of K

  const int split = blockIdx.x, kvh = blockIdx.y;
  // step metadata and block tables come from host copies, not from the
  // previous kernel: read them before waiting
  const int seq = a.seq_order != nullptr ? a.seq_order[blockIdx.z] : (int)blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (seq < 0 || seq >= a.n_seqs) {
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) set_status(ERR_BAD_INDEX);
    return;
  }
  const int ctx = a.ctx_len[seq], qlen = a.q_len[seq], q0 = a.q_start[seq];
  const int G = a.n_q_heads / a.n_kv_heads;
  const int nrows = qlen * G;
  const int n_chunks = (ctx + 15) / 16;
  const int n_splits = (n_chunks + a.split_chunks - 1) / a.split_chunks;
  if (threadIdx.x == 0) pdl_trigger();
  if (split >= n_splits || nrows <= 0) {
    pdl_wait();
    return;
  }
  if (nrows > 16) {
    pdl_wait();
    if (threadIdx.x == 0) set_status(ERR_BAD_INDEX);
    return;
  }
  const int c_begin = split * a.split_chunks;
  const int n_mine = min(c_begin + a.split_chunks, n_chunks) - c_begin;
  const int* table = a.block_tables + (size_t)seq * a.bt_ld;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TMA_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  Flash<HD, C> f;
  f.init();
  if (warp == 4) {
    // ---- producer: the split's pool rows first (one coalesced pass over the
    // block table), then one TMA box per K/V half per chunk
    for (int i = lane; i < n_mine; i += 32) {
      const int p0 = (c_begin + i) * 16;
      int blk = table[p0 / a.block_size];
      if (blk < 0 || blk >= a.num_blocks) {
        set_status(ERR_BAD_INDEX);
        blk = 0;  // load something valid; the result is flagged
      }
      chunk_row[i] = ((blk * 2) * a.n_kv_heads + kvh) * a.block_size + p0 % a.block_size;
    }
    __syncwarp();
    pdl_wait();   // K/V of this step are written by the preceding QKV kernel
    if (lane == 0) {
      prefetch_tmap(&pool_map);
      const int rows_per_kv = a.n_kv_heads * a.block_size;
      for (int i = 0; i < n_mine; ++i) {
        const int s = i % TMA_STAGES;
        if (i >= TMA_STAGES && !mbar_wait(&empty[s], ((i / TMA_STAGES) - 1) & 1)) break;
        const int row_k = chunk_row[i];
        uint8_t* dst = smem + s * SLOT;
        mbar_arrive_expect_tx(&full[s], SLOT);
#pragma unroll
        for (int hf = 0; hf < HD / 64; ++hf) {
          tma_load_2d(dst + hf * 2048, &pool_map, &full[s], hf * 64, row_k);
          tma_load_2d(dst + C::BYTES + hf * 2048, &pool_map, &full[s], hf * 64, row_k + rows_per_kv);
        }
      }
    }
  } else {
    // ---- consumers: warp w takes chunks w, w+4, ...
    pdl_wait();
    uint32_t qa[HD / 16][4];
    load_q<HD>(a, q0, G, kvh, 0, nrows, lane, qa);
    int limit[2];
    const int first = ctx - qlen;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = min((lane >> 2) + 8 * h, nrows - 1);
      limit[h] = first + r / G;
    }
    const uint32_t base = smem_u32(smem);
    for (int i = warp; i < n_mine; i += 4) {
      const int s = i % TMA_STAGES;
      if (!mbar_wait(&full[s], (i / TMA_STAGES) & 1)) break;
      const uint32_t sk = base + s * SLOT;
      f.step(qa, sk, sk + C::BYTES, c_begin + i, ctx, limit, a.scale_log2, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    f.finish_sum();
  }
  __syncthreads();   // ring drained: every issued load was consumed
  merge_warps<HD>(a, f, smem, 4, warp, lane, seq, kvh, split, n_splits, q0, G, nrows, warp < 4);
}

constexpr int PF_STAGES = 2;

constexpr int PF_ROWS = 256;   // query rows per prefill work item

// A prefill work item (sequence, 256-row tile) that names a sequence of the
// call, a row tile inside its prompt, a prompt no longer than its context and
// a context its block-table row can hold.
__device__ __forceinline__ bool prefill_item_ok(const AttnArgs& a, int seq, int rt) {
  if (seq < 0 || seq >= a.n_seqs || rt < 0) return false;
  const int ctx = a.ctx_len[seq], qlen = a.q_len[seq];
  const int G = a.n_q_heads / a.n_kv_heads;
  return qlen >= 1 && qlen <= ctx && rt * PF_ROWS < qlen * G &&
         (ctx + a.block_size - 1) / a.block_size <= a.bt_ld;
}

template <int HD>
__global__ void __launch_bounds__(256) attn_prefill_kernel(const AttnArgs a) {
  using C = ChunkLayout<HD>;
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const int seq = a.work[2 * blockIdx.x], rt = a.work[2 * blockIdx.x + 1];
  const int kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (!prefill_item_ok(a, seq, rt)) {
    if (threadIdx.x == 0) set_status(ERR_BAD_INDEX);
    return;
  }
  const int ctx = a.ctx_len[seq], qlen = a.q_len[seq], q0 = a.q_start[seq];
  const int G = a.n_q_heads / a.n_kv_heads;
  const int nrows_total = qlen * G;
  // the work item's rows in two passes of 128 (8 warps x 16 rows)
  for (int sub = 0; sub < PF_ROWS / 128; ++sub) {
  const int r128 = rt * (PF_ROWS / 128) + sub;
  if (r128 * 128 >= nrows_total) break;
  const int row0 = r128 * 128 + warp * 16;
  const int nrows = max(0, min(16, nrows_total - row0));
  const int first = ctx - qlen;
  const int* table = a.block_tables + (size_t)seq * a.bt_ld;
  // keys needed by the whole CTA: up to the last row's causal limit
  const int last_row = min(r128 * 128 + 127, nrows_total - 1);
  const int cta_keys = min(ctx, first + last_row / G + 1);
  const int n_chunks = (cta_keys + 15) / 16;

  uint32_t qa[HD / 16][4];
  load_q<HD>(a, q0, G, kvh, row0, nrows, lane, qa);
  int limit[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = row0 + min((lane >> 2) + 8 * h, max(nrows - 1, 0));
    limit[h] = first + r / G;
  }
  const int warp_keys = nrows > 0 ? min(ctx, first + (row0 + nrows - 1) / G + 1) : 0;

  const uint32_t ring = smem_u32(smem);
  Flash<HD> f;
  f.init();
  if (n_chunks > 0) load_chunk<HD>(a, table, kvh, ctx, 0, ring, ring + C::BYTES, threadIdx.x, 256);
  cp_commit();
  for (int ci = 0; ci < n_chunks; ++ci) {
    if (ci + 1 < n_chunks) {
      const uint32_t sn = ring + ((ci + 1) % PF_STAGES) * 2 * C::BYTES;
      load_chunk<HD>(a, table, kvh, ctx, ci + 1, sn, sn + C::BYTES, threadIdx.x, 256);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t st = ring + (ci % PF_STAGES) * 2 * C::BYTES;
    if (ci * 16 < warp_keys) f.step(qa, st, st + C::BYTES, ci, ctx, limit, a.scale_log2, lane);
    __syncthreads();
  }
  cp_wait<0>();
  f.finish_sum();
  const int g4 = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g4 + 8 * h;
    if (r >= nrows) continue;
    const int R = row0 + r;
    const float inv = f.l[h] > 0.f ? 1.f / f.l[h] : 0.f;
    __nv_bfloat16* dst = a.out + (size_t)(q0 + R / G) * a.ld_out + (size_t)(kvh * G + R % G) * HD;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      const int c = nt * 8 + 2 * t4;
      *reinterpret_cast<uint32_t*>(dst + c) =
          pack_bf16x2(f.o[nt][2 * h] * inv, f.o[nt][2 * h + 1] * inv);
    }
  }
  __syncthreads();   // the next pass refills the chunk ring
  }
}

// ------------------------------------------------------ prefill, tcgen05
//
// One CTA per (work item = (sequence, 256-row tile), kv head): two query
// tiles A and B of 128 rows share every K/V tile.  Row r of tile x is query
// row R = 256 * tile + 128 * x + r: token R / G, head R % G of the kv head's
// group.  Keys go in tiles of 128 (8 chunks of 16 tokens, each chunk one
// block-table lookup), up to the last row's causal limit.
//   warps 0/2  loaders of K / V: every key tile gathered from the pool
//              through the block table with 16-byte cp.async pieces (a warp
//              instruction moves two whole 256-byte key rows), written in the
//              128-byte-swizzled layout the MMA descriptors describe, into
//              two-stage rings (a K stage is refilled once both S MMAs of
//              its tile are done, a V stage once both PV MMAs are done).  A
//              stage's barrier completes when its pieces have landed
//              (cp.async arrivals) and the MMA thread fences them over to
//              the async proxy.  (TMA boxes of one 16-token block half --
//              2 KiB, all the pool keeps contiguous at block size 16 --
//              issued at ~40 ns each from one thread, left the tensor pipe
//              waiting.)
//   warp 1     TMEM owner and MMA issuer.  Per query tile x: S_x = Q_x K_j^T
//              (M 128, N 128 keys, K = HD) into S_x in TMEM; once the
//              softmax has written P_x (bf16, over the first 64 columns of
//              S_x), O_x += P_x V_j with P read from TMEM and V in place as
//              an MN-major operand; S_x for the next key tile follows once
//              that PV is complete (it overwrites P_x).  The two tiles'
//              chains interleave, so one tile's MMAs run while the other's
//              softmax works.
//   warp 3     spare: completes the first warpgroup, whose registers go to
//              the softmax warpgroups (setmaxnreg)
//   warps 4-7  softmax of tile A, warps 8-11 of tile B: one query row per
//              thread (TMEM lane = row): Q into shared memory, then per key
//              tile the row's 128 scores into registers, the row max, P =
//              exp2(S - ref) into TMEM, and the running sum
// O_x stays in TMEM across the key tiles.  A row's exponent reference `ref`
// moves only when its running max exceeds it by more than PT_RESCALE (log2
// units): then the row's O is rescaled in TMEM (after the PV MMAs issued so
// far complete) and its sum by the same factor.  Otherwise P and O carry a
// factor of at most 2^PT_RESCALE, which the final division by the sum
// removes; bf16 rounding of P is relative, so the factor costs no precision.
// Shared-memory tiles use the 128-byte swizzle (rows of 64 bf16, 16-byte
// pieces XOR-permuted by row % 8, 8-row atoms 1024 B apart).
constexpr int PT_ROWS = 128;     // query rows per tile (two tiles per CTA)
constexpr int PT_KEYS = 128;     // keys per tile
constexpr int PT_THREADS = 384;  // K loader, MMA, V loader, spare; 2 x 4 softmax warps
// Registers per thread: the launch gives every thread PT_REGS_LAUNCH; the
// first warpgroup (loaders, MMA) drops to PT_REGS_LOW and the two softmax
// warpgroups rise to PT_REGS_HIGH, so a row's 128 scores stay in registers
// without spilling.
constexpr int PT_REGS_LAUNCH = 168, PT_REGS_LOW = 56, PT_REGS_HIGH = 224;
static_assert(128 * PT_REGS_LOW + 256 * PT_REGS_HIGH <= PT_THREADS * PT_REGS_LAUNCH,
              "register split above the launch total");
constexpr float PT_RESCALE = 8.f;

// Debug timeline of a prefill CTA (tb_debug_trace), PT_TR_POINTS slots:
// 0 / 31 %globaltimer at the first softmax thread's start / end, 30 its
// clock64 at start (29: at end); the other slots are clock64 stamps (SM
// cycles): 1 Q stored, 26 the MMA thread sees Q, 27 the output is read from
// TMEM, and for key tiles k < 3 at 2 + 8k: +0 / +1 K_k loads start / issued,
// +2 / +3 V_k loads start / issued (loaders; start = its stage is free),
// +4 S_A,k issued (MMA), +5 S_A,k in registers, +6 P_A,k stored (first
// softmax thread), +7 PV_A,k issued (MMA).
enum : int { PT_TR_Q = 1, PT_TR_TILES = 3, PT_TR_QSEEN = 26, PT_TR_OREAD = 27, PT_TR_CLK1 = 29,
             PT_TR_CLK0 = 30, PT_TR_END = 31, PT_TR_POINTS = 32 };

__device__ __forceinline__ void pt_put(const AttnArgs& a, int point, unsigned long long v) {
  if (a.trace != nullptr)
    a.trace[(size_t)(blockIdx.x + blockIdx.y * gridDim.x) * PT_TR_POINTS + point] = v;
}
__device__ __forceinline__ void pt_clk(const AttnArgs& a, int point) {
  if (a.trace != nullptr) pt_put(a, point, (unsigned long long)clock64());
}
__device__ __forceinline__ void pt_tile(const AttnArgs& a, int k, int what) {
  if (a.trace != nullptr && k < PT_TR_TILES) pt_clk(a, 2 + 8 * k + what);
}

template <int HD>
struct PrefillTcLayout {
  static constexpr int HALVES = HD / 64;                  // 64-column halves
  static constexpr int HALF = PT_ROWS * 128;              // one [128][64] bf16 half: 16 KiB
  static constexpr int Q_TILE = HALVES * HALF;
  static constexpr int KV_HALF = PT_KEYS * 128;           // [128 keys][64] bf16
  static constexpr int KV_PART = HALVES * KV_HALF;        // K (or V) of one key tile
  static constexpr int STAGE = 2 * KV_PART;               // K then V
  static constexpr int OFF_Q = 0;                         // Q_A then Q_B
  static constexpr int OFF_KV = 2 * Q_TILE;
  static constexpr int OFF_BAR = OFF_KV + 2 * STAGE;
  static constexpr int N_BARS = 17;
  static constexpr int SMEM = OFF_BAR + 24 * 8 + 1024;     // barriers + TMEM slot + alignment slack
  static constexpr uint32_t TMEM_COLS = 512;
  // S_A, S_B (P_x over the first 64 columns of S_x), O_A, O_B
  __device__ static constexpr uint32_t col_s(int x) { return (uint32_t)(x * PT_KEYS); }
  __device__ static constexpr uint32_t col_o(int x) { return (uint32_t)(2 * PT_KEYS + x * HD); }
  static_assert(2 * PT_KEYS + 2 * HD <= TMEM_COLS, "TMEM: two S and two O");
  static_assert(N_BARS * 8 + 4 <= 24 * 8, "barrier area");
  static_assert(SMEM <= 232448, "prefill shared memory above 227 KiB");
};

// Byte offset of 16-byte piece c (0..7) of row r in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

template <int HD>
__global__ void __launch_bounds__(PT_THREADS, 1)
    attn_prefill_tc_kernel(const AttnArgs a) {
  using L = PrefillTcLayout<HD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* k_full = bars;         // [2] by stage
  uint64_t* k_empty = bars + 2;    // [2]
  uint64_t* v_full = bars + 4;     // [2]
  uint64_t* v_empty = bars + 6;    // [2]
  uint64_t* s_full = bars + 8;     // [2] by query tile
  uint64_t* p_full = bars + 10;    // [2] by query tile: P written, S read
  uint64_t* pv_done = bars + 12;   // [2] by query tile
  uint64_t* q_full = bars + 14;
  uint64_t* mma_idle = bars + 15;  // every MMA of the CTA complete (before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::N_BARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // step metadata comes from host copies, not from the previous kernel
  const int seq = a.work[2 * blockIdx.x], rt = a.work[2 * blockIdx.x + 1];
  const int kvh = blockIdx.y;
  if (!prefill_item_ok(a, seq, rt)) {   // uniform over the CTA: nothing set up yet
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) set_status(ERR_BAD_INDEX);
    return;
  }
  const int ctx = a.ctx_len[seq], qlen = a.q_len[seq], q0 = a.q_start[seq];
  const int G = a.n_q_heads / a.n_kv_heads;
  const int nrows_total = qlen * G;
  const int first = ctx - qlen;
  const int last_row = min(rt * PF_ROWS + PF_ROWS - 1, nrows_total - 1);
  const int keys = max(1, min(ctx, first + last_row / G + 1));   // keys this CTA needs
  const int n_tiles = (keys + PT_KEYS - 1) / PT_KEYS;
  const bool has_b = rt * PF_ROWS + PT_ROWS < nrows_total;      // tile B holds a row
  const int* table = a.block_tables + (size_t)seq * a.bt_ld;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 32);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 32);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], PT_ROWS);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(q_full, 2 * PT_ROWS);
    mbar_init(mma_idle, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) pdl_trigger();
  const uint32_t sbase = smem_u32(smem);

  if (warp < 4) {
  setmaxnreg_dec<PT_REGS_LOW>();
  if (warp == 0 || warp == 2) {
    // ---------------- loaders: K (warp 0) and V (warp 2)
    const int is_v = warp != 0;
    uint64_t* full = is_v ? v_full : k_full;
    uint64_t* empty = is_v ? v_empty : k_empty;
    const int last_chunk = (keys - 1) / 16;
    constexpr int PPK = HD / 8;                      // 16-byte pieces per key row
    constexpr int KEYS_PER_INSN = 32 / PPK;          // key rows one warp instruction moves
    // lane c < 8: the block-table entry of chunk c of the tile (chunks past
    // the CTA's last one repeat it: their keys are masked), one tile ahead
    auto entry = [&](int j) {
      return lane < PT_KEYS / 16 ? table[min(j * (PT_KEYS / 16) + lane, last_chunk) * 16 /
                                         a.block_size]
                                 : 0;
    };
    int blk = entry(0);
    pdl_wait();   // the pool is written by the previous kernel
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      const int blk_next = j + 1 < n_tiles ? entry(j + 1) : 0;
      if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(&empty[st], ((j >> 1) - 1) & 1))) break;
      if (lane == 0) pt_tile(a, j, 2 * is_v);
      // lane c: first pool row of chunk c
      int b = blk;
      if (lane < PT_KEYS / 16 && (b < 0 || b >= a.num_blocks)) {
        set_status(ERR_BAD_INDEX);
        b = 0;
      }
      const int key0 = min(j * (PT_KEYS / 16) + lane, last_chunk) * 16;
      const int rk = (int)(((size_t)b * 2 * a.n_kv_heads + (size_t)is_v * a.n_kv_heads + kvh) *
                               a.block_size + key0 % a.block_size);
      const uint32_t stage = sbase + L::OFF_KV + st * L::STAGE + is_v * L::KV_PART;
#pragma unroll 1
      for (int c = 0; c < PT_KEYS / 16; ++c) {
        const int row0 = __shfl_sync(0xffffffffu, rk, c);
#pragma unroll
        for (int i = 0; i < 16 / KEYS_PER_INSN; ++i) {
          const int kk = i * KEYS_PER_INSN + lane / PPK;   // key within the chunk
          const int pc = lane % PPK, h = pc >> 3, pw = pc & 7;
          const int key = c * 16 + kk;                      // key within the tile
          const __nv_bfloat16* src = a.pool + (size_t)(row0 + kk) * HD + pc * 8;
          cp_async16(stage + h * L::KV_HALF + key * 128 + ((pw ^ (key & 7)) << 4), src, true);
        }
      }
      // the stage's barrier completes once every lane's pieces have landed;
      // the MMA thread makes them visible to the tensor core (proxy fence)
      cp_arrive_noinc(&full[st]);
      if (lane == 0) pt_tile(a, j, 2 * is_v + 1);
      blk = blk_next;
    }
    cp_wait<0>();   // nothing in flight at exit
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_m128(PT_KEYS);
      constexpr uint32_t idesc_o = idesc_bf16_m128(HD) | (1u << 16);   // B (V) MN-major
      bool ok = mbar_wait(q_full, 0);
      tc_fence_after();
      pt_clk(a, PT_TR_QSEEN);
      const int nx = has_b ? 2 : 1;
      auto issue_s = [&](int x, int j) {
        const uint32_t qbase = sbase + L::OFF_Q + x * L::Q_TILE;
        const uint32_t kbase = sbase + L::OFF_KV + (j & 1) * L::STAGE;
#pragma unroll
        for (int h = 0; h < L::HALVES; ++h)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_bf16(tmem + L::col_s(x), sw128_desc(qbase + h * L::HALF + kk * 32),
                        sw128_desc(kbase + h * L::KV_HALF + kk * 32), idesc_s,
                        (h | kk) ? 1u : 0u);
        tc_commit(&s_full[x]);
        if (x == 0) pt_tile(a, j, 4);
      };
      auto issue_pv = [&](int x, int j) -> bool {
        if (!mbar_wait(&p_full[x], j & 1)) return false;
        tc_fence_after();
        const uint32_t vbase = sbase + L::OFF_KV + (j & 1) * L::STAGE + L::KV_PART;
#pragma unroll
        for (int ks = 0; ks < PT_KEYS / 16; ++ks)
          tc_mma_bf16_ts(tmem + L::col_o(x), tmem + L::col_s(x) + ks * 8,
                         sw128_mn_desc(vbase + ks * 2048, L::KV_HALF, 1024), idesc_o,
                         (j > 0 || ks > 0) ? 1u : 0u);
        tc_commit(&pv_done[x]);
        if (x == 0) pt_tile(a, j, 7);
        return true;
      };
      if (ok) ok = mbar_wait(&k_full[0], 0);
      if (ok) {
        tc_fence_after();
        fence_proxy_async_smem();   // K arrived through cp.async (generic proxy)
        for (int x = 0; x < nx; ++x) issue_s(x, 0);
        tc_commit(&k_empty[0]);
      }
      for (int j = 0; j < n_tiles && ok; ++j) {
        const bool next = j + 1 < n_tiles;
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1)) break;
        fence_proxy_async_smem();   // V arrived through cp.async (generic proxy)
        bool k_ready = false;
        for (int x = 0; x < nx && ok; ++x) {
          ok = issue_pv(x, j);
          if (!ok || !next) continue;
          if (!k_ready) {
            ok = mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1);
            fence_proxy_async_smem();
            k_ready = true;
          }
          // S_x of the next key tile overwrites P_x: issue it once PV_x is done
          if (ok) ok = mbar_wait(&pv_done[x], j & 1);
          if (ok) {
            tc_fence_after();
            issue_s(x, j + 1);
          }
        }
        if (!ok) break;
        tc_commit(&v_empty[j & 1]);
        if (next) tc_commit(&k_empty[(j + 1) & 1]);
      }
      tc_commit(mma_idle);
      mbar_wait(mma_idle, 0);
    }
  }   // warp 3: nothing to do
  } else {
    setmaxnreg_inc<PT_REGS_HIGH>();
    // ---------------- softmax: one query row per thread, tile x
    const int x = (warp - 4) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;                 // TMEM lane of this thread
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int R = rt * PF_ROWS + x * PT_ROWS + r;
    const bool valid = R < nrows_total;
    const int limit = valid ? first + R / G : -1;   // last key this row sees
    const bool tracer = threadIdx.x == 128;
    if (tracer && a.trace != nullptr) {
      pt_put(a, 0, globaltimer_ns());
      pt_clk(a, PT_TR_CLK0);
    }
    pdl_wait();   // q is written by the previous kernel
    {
      uint8_t* qs = smem + L::OFF_Q + x * L::Q_TILE;
      const __nv_bfloat16* src =
          a.q + (size_t)(q0 + (valid ? R / G : 0)) * a.ld_q + (size_t)(kvh * G + R % G) * HD;
      uint4 v[HD / 8];
#pragma unroll
      for (int c = 0; c < HD / 8; ++c)
        v[c] = valid ? *reinterpret_cast<const uint4*>(src + c * 8) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int c = 0; c < HD / 8; ++c)
        *reinterpret_cast<uint4*>(qs + (c >> 3) * L::HALF + sw128_off(r, c & 7)) = v[c];
      fence_proxy_async_smem();
      mbar_arrive(q_full);
      if (tracer) pt_clk(a, PT_TR_Q);
    }
    if (x == 1 && !has_b) {
      // no row of tile B: nothing to compute
    } else {
      const uint32_t ts = tmem + L::col_s(x) + lane_off;   // S_x, and P_x over its first 64 columns
      const uint32_t to = tmem + L::col_o(x) + lane_off;
      float ref = -INFINITY, l = 0.f;   // exponent reference (log2 units) and running sum
      const float sc = a.scale_log2;
      int done = 0;
      for (int j = 0; j < n_tiles; ++j) {
        // waits are made warp-uniform: the TMEM accesses below are warp-collective
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x], j & 1))) break;
        tc_fence_after();
        float s[PT_KEYS];
        tmem_ld64(ts, s);
        tmem_ld64(ts + 64, s + 64);
        if (tracer) pt_tile(a, j, 5);
        const int k0 = j * PT_KEYS;
        if (k0 + PT_KEYS - 1 > limit) {   // the causal edge (or an empty row)
#pragma unroll
          for (int e = 0; e < PT_KEYS; ++e)
            if (k0 + e > limit) s[e] = -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int e = 0; e < PT_KEYS; e += 2) mx = fmax3(mx, s[e], s[e + 1]);
        mx *= sc;
        const bool move = mx > ref + PT_RESCALE;   // any finite max when ref is -inf
        const bool rescale = move && ref != -INFINITY;
        const float alpha = rescale ? ex2_approx(ref - mx) : 1.f;
        if (__any_sync(0xffffffffu, rescale)) {
          // O holds PV_0 .. PV_{j-1}: once the last of them is complete,
          // scale the warp's rows in place (alpha = 1 for rows that keep
          // their ref)
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[x], (j - 1) & 1))) break;
          tc_fence_after();
#pragma unroll
          for (int c0 = 0; c0 < HD; c0 += 32) {
            float v[32];
            tmem_ld32(to + c0, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= alpha;
            tmem_st32(to + c0, v);
          }
        }
        if (move) ref = mx;
        l *= alpha;
        const float mu = ref == -INFINITY ? 0.f : ref;
        const float2 sc2 = make_float2(sc, sc), nmu2 = make_float2(-mu, -mu);
        float2 sum2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c0 = 0; c0 < PT_KEYS; c0 += 32) {
          uint32_t w[16];   // 32 keys, two bf16 per 32-bit column
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 xv = fma2(make_float2(s[c0 + e], s[c0 + e + 1]), sc2, nmu2);
            const float2 pv = make_float2(ex2_approx(xv.x), ex2_approx(xv.y));
            sum2 = add2(sum2, pv);
            w[e >> 1] = pack_bf16x2(pv.x, pv.y);
          }
          tmem_st16(ts + (c0 >> 1), w);
        }
        tmem_wait_st();
        l += sum2.x + sum2.y;
        tc_fence_before();               // P (and a rescaled O) precede PV
        mbar_arrive(&p_full[x]);         // P_x is in TMEM, S_x has been read
        if (tracer) pt_tile(a, j, 6);
        done = j + 1;
      }
      if (done == n_tiles &&
          __all_sync(0xffffffffu, mbar_wait(&pv_done[x], (n_tiles - 1) & 1))) {
        tc_fence_after();
        if (tracer) pt_clk(a, PT_TR_OREAD);
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* dst = a.out + (size_t)(q0 + (valid ? R / G : 0)) * a.ld_out +
                             (size_t)(kvh * G + R % G) * HD;
#pragma unroll
        for (int c0 = 0; c0 < HD; c0 += 32) {
          float v[32];
          tmem_ld32(to + c0, v);   // warp-collective: every lane loads
          if (valid) {
#pragma unroll
            for (int c = 0; c < 32; c += 8) {
              uint4 u;
              u.x = pack_bf16x2(v[c] * inv, v[c + 1] * inv);
              u.y = pack_bf16x2(v[c + 2] * inv, v[c + 3] * inv);
              u.z = pack_bf16x2(v[c + 4] * inv, v[c + 5] * inv);
              u.w = pack_bf16x2(v[c + 6] * inv, v[c + 7] * inv);
              *reinterpret_cast<uint4*>(dst + c0 + c) = u;
            }
          }
        }
      }
    }
    if (tracer && a.trace != nullptr) {
      pt_clk(a, PT_TR_CLK1);
      pt_put(a, PT_TR_END, globaltimer_ns());
    }
  }
  if (warp == 1) pdl_wait();   // every CTA waits before it exits (PDL chain)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

template <int HD>
static int decode_tma_launch(const AttnArgs& a, cudaStream_t st) {
  constexpr int SLOT = 2 * TmaChunkLayout<HD>::BYTES;
  const int merge = (4 * 16 * (HD + 4) + 2 * 4 * 16) * 4 + 16;
  const int ring = TMA_STAGES * SLOT + 2 * TMA_STAGES * 8 + TMA_MAX_SPLIT_CHUNKS * 4;
  const int smem = (ring > merge ? ring : merge) + 1024;
  if (a.split_chunks > TMA_MAX_SPLIT_CHUNKS) return arg_err("split_tokens above 8192");
  static std::atomic<unsigned long long> attr_devs{0};
  if (int rc = smem_attr_once(attn_decode_tma_kernel<HD>, smem, attr_devs,
                              "attention smem attribute", true))
    return rc;
  CUtensorMap map;
  const uint64_t rows = (uint64_t)a.num_blocks * 2 * a.n_kv_heads * a.block_size;
  int rc = make_tmap_2d(&map, a.pool, HD, rows, (uint64_t)HD * 2, 64, 16);
  if (rc) return rc;
  return launch_pdl(attn_decode_tma_kernel<HD>, dim3(a.max_splits, a.n_kv_heads, a.n_seqs),
                    dim3(TMA_THREADS), smem, st, 1, "attention decode launch", map, a);
}

template <int HD>
static int decode_launch(const AttnArgs& a, cudaStream_t st) {
  const int smem_ring = 4 * DEC_STAGES * 2 * ChunkLayout<HD>::BYTES;
  const int smem_merge = (4 * 16 * (HD + 4) + 2 * 4 * 16) * 4 + 16;
  const int smem = smem_ring > smem_merge ? smem_ring : smem_merge;
  static std::atomic<unsigned long long> attr_devs{0};
  if (int rc = smem_attr_once(attn_decode_kernel<HD>, smem, attr_devs, "attention smem attribute"))
    return rc;
  return launch_pdl(attn_decode_kernel<HD>, dim3(a.max_splits, a.n_kv_heads, a.n_seqs),
                    dim3(128), smem, st, 1, "attention decode launch", a);
}

template <int HD>
static int prefill_launch(const AttnArgs& a, int n_work, cudaStream_t st) {
  const int smem = PF_STAGES * 2 * ChunkLayout<HD>::BYTES;
  return launch_pdl(attn_prefill_kernel<HD>, dim3(n_work, a.n_kv_heads), dim3(256), smem, st, 1,
                    "attention prefill launch", a);
}

template <int HD>
static int prefill_tc_launch(const AttnArgs& a, int n_work, cudaStream_t st) {
  using L = PrefillTcLayout<HD>;
  static std::atomic<unsigned long long> attr_devs{0};
  if (int rc = smem_attr_once(attn_prefill_tc_kernel<HD>, L::SMEM, attr_devs,
                              "prefill smem attribute"))
    return rc;
  // the softmax warpgroups' setmaxnreg.inc waits for registers the first
  // warpgroup releases: refuse a build whose launch total cannot cover it
  static std::atomic<int> regs_ok{0};
  if (!regs_ok.load(std::memory_order_acquire)) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, attn_prefill_tc_kernel<HD>);
    if (e != cudaSuccess) return host_err(e, "prefill attributes");
    if (fa.numRegs * PT_THREADS < 128 * PT_REGS_LOW + 256 * PT_REGS_HIGH)
      return arg_err("prefill kernel built with too few registers for its register split");
    regs_ok.store(1, std::memory_order_release);
  }
  const uint64_t rows = (uint64_t)a.num_blocks * 2 * a.n_kv_heads * a.block_size;
  if (rows >= (1ull << 31)) return arg_err("KV pool rows beyond 2^31");
  AttnArgs at = a;
  at.trace = g_debug_trace;
  return launch_pdl(attn_prefill_tc_kernel<HD>, dim3(n_work, a.n_kv_heads), dim3(PT_THREADS),
                    L::SMEM, st, 1, "attention prefill launch", at);
}

static int check_common(const AttnArgs& a, int head_dim) {
  if (a.n_kv_heads <= 0 || a.n_q_heads % a.n_kv_heads) return arg_err("heads: Hq % Hkv != 0");
  if (a.block_size <= 0 || a.num_blocks <= 0) return arg_err("block_size / num_blocks");
  if ((a.ld_q % 8) || (a.ld_out % 8)) return arg_err("ld_q / ld_out must be multiples of 8");
  if (head_dim != 16 && head_dim != 64 && head_dim != 128) return arg_err("head_dim must be 16, 64 or 128");
  return TB_OK;
}

int attn_decode(AttnArgs a, int head_dim, cudaStream_t st) {
  int rc = check_common(a, head_dim);
  if (rc) return rc;
  if (a.n_q_heads / a.n_kv_heads > 16) return arg_err("GQA group larger than 16");
  if (a.split_chunks <= 0 || a.max_splits <= 0) return arg_err("split sizes");
  if (a.max_splits > 1 && (a.ws_o == nullptr || a.ws_lse == nullptr || a.ws_count == nullptr))
    return arg_err("split workspace");
  if (a.n_seqs == 0) return TB_OK;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  // TMA boxes need 16-token chunks inside one block and a 16-byte aligned pool
  const bool tma = a.block_size % 16 == 0 && reinterpret_cast<uintptr_t>(a.pool) % 16 == 0;
  switch (head_dim) {
    case 16: return decode_launch<16>(a, st);
    case 64: return tma ? decode_tma_launch<64>(a, st) : decode_launch<64>(a, st);
    default: return tma ? decode_tma_launch<128>(a, st) : decode_launch<128>(a, st);
  }
}

int attn_prefill(AttnArgs a, int head_dim, int n_work, cudaStream_t st) {
  int rc = check_common(a, head_dim);
  if (rc) return rc;
  if (n_work == 0) return TB_OK;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  // TMA boxes need 16-token chunks inside one block and a 16-byte aligned pool
  const bool tc = a.block_size % 16 == 0 && reinterpret_cast<uintptr_t>(a.pool) % 16 == 0;
  switch (head_dim) {
    case 16: return prefill_launch<16>(a, n_work, st);
    case 64: return tc ? prefill_tc_launch<64>(a, n_work, st) : prefill_launch<64>(a, n_work, st);
    default: return tc ? prefill_tc_launch<128>(a, n_work, st) : prefill_launch<128>(a, n_work, st);
  }
}

}  // namespace tb
