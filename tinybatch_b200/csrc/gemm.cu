// tcgen05 GEMM kernel and its host launcher (see gemm.cuh for the design).
#include <stdio.h>
#include <string.h>

#include "gemm.cuh"
#include "host.h"

namespace tb {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int A_BYTES = BM * BK * 2;
constexpr int GEMM_THREADS = 192;

// How a split-K launch combines its partial accumulators.
enum SplitMode : int {
  SPLIT_NONE = 0,     // one CTA per tile
  SPLIT_GLOBAL = 1,   // partials in caller scratch; last CTA to arrive reduces
  SPLIT_CLUSTER = 2,  // the splits of a tile form a thread-block cluster; each
                      // CTA stores every 16-column chunk of its partial into
                      // the shared memory of the chunk's owner CTA (DSMEM)
                      // and reduces the chunks it owns locally
};

__device__ __forceinline__ void trace_at(const GemmArgs& g, int point) {
  if (g.trace != nullptr)
    g.trace[(size_t)(blockIdx.x + blockIdx.y * gridDim.x) * TR_POINTS + point] = globaltimer_ns();
}

constexpr int tmem_cols(int bn) { return bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256; }

template <int BN, int STAGES>
struct GemmLayout {
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = STAGES * A_BYTES;
  static constexpr int OFF_BAR = OFF_B + STAGES * B_BYTES;
  static constexpr int BAR_BYTES = (2 * STAGES + 1) * 8 + 16 + 4 * BM * 4;  // + RowStage arrays
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;                // + alignment slack
  // cluster mode receives the members' partial chunks over the stage ring
  static constexpr int RING = OFF_BAR;
};

// Bytes of shared memory a cluster member receives: `splits` sources, each
// sending the ceil(np / splits) pairs of cp 16-column chunks this member owns,
// 128 rows x 16 fp32 per chunk.
__host__ __device__ constexpr int cluster_region_bytes(int np, int cp, int splits) {
  return splits * ((np + splits - 1) / splits) * cp * BM * 16 * 4;
}

// Deferred RMSNorm scale of row m: rsqrt(mean of h^2 + eps) from the
// per-part partial sums the producing kernel wrote.
__device__ __forceinline__ float row_scale(const GemmArgs& g, int m) {
  if (g.sq == nullptr || m >= g.M) return 1.f;
  float s = 0.f;
  int p = 0;
  for (; p + 8 <= g.sq_parts; p += 8) {
    float t[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) t[i] = g.sq[(size_t)(p + i) * g.sq_ld + m];
#pragma unroll
    for (int i = 0; i < 8; ++i) s += t[i];
  }
  for (; p < g.sq_parts; ++p) s += g.sq[(size_t)p * g.sq_ld + m];
  return rsqrtf(s * g.inv_d + g.eps);
}

// How a tile's columns are grouped for the epilogue and, in cluster split-K,
// which member owns them.  The unit of work is a "pair" of cp 16-column
// chunks that one thread finishes together: a single chunk (plain outputs,
// residual; 16-wide heads), the gate and up chunks of the same features
// (SwiGLU: gate columns [0, BN/2), up columns [BN/2, BN)), or the two chunks a
// RoPE rotation mixes (QKV, head_dim >= 32: columns j and j + head_dim/2 of a
// head).  Pair p belongs to cluster member p % splits, at slot
// (p / splits) * cp + which of that member's receive region.
struct TileUnits {
  int np;    // pairs in the tile
  int cp;    // chunks per pair: 1 or 2
  int hc;    // paired kinds: chunks per half (SwiGLU: per tile half; QKV: per head half)
  int kind;  // 0 single chunks, 1 SwiGLU halves, 2 RoPE halves of each head
  __device__ __forceinline__ int chunk(int p, int which) const {
    if (kind == 0) return p;
    if (kind == 1) return p + which * hc;
    return (p / hc) * 2 * hc + which * hc + p % hc;
  }
  __device__ __forceinline__ void pair_of(int k, int& p, int& which) const {
    if (kind == 0) {
      p = k;
      which = 0;
    } else if (kind == 1) {
      which = k / hc;
      p = k % hc;
    } else {
      const int r = k % (2 * hc);
      which = r / hc;
      p = (k / (2 * hc)) * hc + r % hc;
    }
  }
};

template <int BN, int EPI>
__device__ __forceinline__ TileUnits tile_units(const GemmArgs& g) {
  if constexpr (EPI == EPI_SWIGLU) return {BN / 32, 2, BN / 32, 1};
  if constexpr (EPI == EPI_QKV) {
    if (g.head_dim >= 32) return {BN / 32, 2, g.head_dim / 32, 2};
  }
  return {BN / 16, 1, 0, 0};
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

// 16 bytes into the shared memory of a cluster member (a mapa address).
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// ------------------------------------------------------------- staging
// A 16-column chunk of a 128-row tile in shared memory: [4 float4][BM rows],
// chunks numbered [source][slot] (cluster split-K keeps one source per
// member).  A warp reading TMEM (one row per thread) stores 512 contiguous
// bytes per instruction, which also keeps its DSMEM stores dense; the
// finisher's lanes read 8 consecutive rows per 8-lane phase (no bank
// conflicts).
__device__ __forceinline__ uint32_t stage_off(int src, int slot, int nslot, int row, int i) {
  return (uint32_t)((((src * nslot + slot) * 4 + i) * BM + row) * 16);
}

// Staged float4 at byte offset `off` of the CTA's shared memory (plain C++
// accesses: independent loads pipeline; the barriers around them are
// memory-clobbering asm, which orders them).
__device__ __forceinline__ const float4& staged(const uint8_t* smem, uint32_t off) {
  return *reinterpret_cast<const float4*>(smem + off);
}

// Sum over the sources of float4 i of chunk `slot`, row `row`, in source
// order (at most 8 sources, all loads issued before the first add).
__device__ __forceinline__ float4 stage_sum(const uint8_t* smem, int nsrc, int nslot, int slot,
                                            int row, int i) {
  float4 v[8];
#pragma unroll
  for (int s = 0; s < 8; ++s)
    if (s < nsrc) v[s] = staged(smem, stage_off(s, slot, nslot, row, i));
  float4 a = v[0];
#pragma unroll
  for (int s = 1; s < 8; ++s) {
    if (s < nsrc) {
      a.x += v[s].x;
      a.y += v[s].y;
      a.z += v[s].z;
      a.w += v[s].w;
    }
  }
  return a;
}

// Accumulator access for the epilogue: columns [16k, 16k+16) of this
// thread's row.  In SPLIT_NONE / SPLIT_GLOBAL mode it reads TMEM (collective
// over the warp: every lane calls it); in SPLIT_CLUSTER mode it sums, in
// member order, the partials the cluster members stored at `slot` of this
// CTA's receive region.
template <int BN>
struct AccReader {
  uint32_t taddr;   // TMEM address of this warp's lane quarter, column 0
  int mode, splits, z, row;
  const float* ws;  // SPLIT_GLOBAL: this tile's workspace, [splits][BN][128]
  const uint8_t* smem;  // SPLIT_CLUSTER: the receive region (this CTA's shared memory)
  int nslot;        // SPLIT_CLUSTER: chunk slots per source member
  __device__ __forceinline__ void load16(int k, int slot, float* v) const {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.f;
    if (mode == SPLIT_CLUSTER) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = stage_sum(smem, splits, nslot, slot, row, i);
        v[4 * i] = a.x;
        v[4 * i + 1] = a.y;
        v[4 * i + 2] = a.z;
        v[4 * i + 3] = a.w;
      }
      return;
    }
    float own[16];
    tmem_ld16(taddr + 16 * k, own);
    if (mode == SPLIT_NONE) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = own[j];
      return;
    }
    for (int s = 0; s < splits; ++s) {
      if (s == z) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += own[j];
      } else {
        const float* p = ws + ((size_t)s * BN + 16 * k) * BM + row;
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += __ldcg(p + (size_t)j * BM);
      }
    }
  }
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Residual inputs of the first PF 16-column units this thread updates (its row
// of h and the next norm's weight), loaded by the epilogue warps before they
// wait for the accumulator: they do not depend on it, so their latency hides
// under the main loop.
constexpr int PF = 3;
struct ResidPre {
  float h[PF][16];
  uint32_t g[PF][8];  // bf16 pairs
};

__device__ __forceinline__ void load_resid_inputs(const GemmArgs& g, int m, int n, float* h16,
                                                  uint32_t* g8) {
  const float4* hp = reinterpret_cast<const float4*>(g.h + (size_t)m * g.ld_h + n);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 x = hp[i];
    h16[4 * i] = x.x;
    h16[4 * i + 1] = x.y;
    h16[4 * i + 2] = x.z;
    h16[4 * i + 3] = x.w;
  }
  const uint4 a = *reinterpret_cast<const uint4*>(g.gnext + n);
  const uint4 b = *reinterpret_cast<const uint4*>(g.gnext + n + 8);
  g8[0] = a.x; g8[1] = a.y; g8[2] = a.z; g8[3] = a.w;
  g8[4] = b.x; g8[5] = b.y; g8[6] = b.z; g8[7] = b.w;
}

template <int BN>
__device__ __forceinline__ void resid_prefetch(const GemmArgs& g, int tm, int tn, int row,
                                               int own, int n_own, ResidPre& p) {
  const int m = tm * BM + row;
  if (m >= g.M) return;
#pragma unroll
  for (int k = 0; k < PF; ++k) {
    const int u = own + k * n_own;
    const int n = tn * BN + u * 16;
    if (u < BN / 16 && n < g.N) load_resid_inputs(g, m, n, p.h[k], p.g[k]);
  }
}

// h = h_old + v (h_old, g given), hg = bf16(h * g) (and its copy in hg2 row
// dst if dst >= 0); returns the sum of the new h^2 over the 16 columns.
__device__ __forceinline__ float resid_update(const GemmArgs& g, int m, int n, int dst,
                                              const float* v, const float* h_old,
                                              const uint32_t* g8) {
  float hn[16], o[16], ss = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) hn[j] = h_old[j] + v[j];
  float4* hp = reinterpret_cast<float4*>(g.h + (size_t)m * g.ld_h + n);
#pragma unroll
  for (int i = 0; i < 4; ++i) hp[i] = make_float4(hn[4 * i], hn[4 * i + 1], hn[4 * i + 2], hn[4 * i + 3]);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    __nv_bfloat162 w2 = *reinterpret_cast<const __nv_bfloat162*>(&g8[i]);
    const float2 wf = __bfloat1622float2(w2);
    o[2 * i] = hn[2 * i] * wf.x;
    o[2 * i + 1] = hn[2 * i + 1] * wf.y;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) ss += hn[j] * hn[j];
  __nv_bfloat16* hgp = g.hg + (size_t)m * g.ld_hg + n;
  store_bf16x8(hgp, o);
  store_bf16x8(hgp + 8, o + 8);
  if (dst >= 0) {
    __nv_bfloat16* p2 = g.hg2 + (size_t)dst * g.ld_hg + n;
    store_bf16x8(p2, o);
    store_bf16x8(p2 + 8, o + 8);
  }
  return ss;
}

// Runs `body(k, u, n, h_old, g8)` for every 16-column unit this thread
// updates: units own, own + n_own, ... of the tile below N; the first PF take
// their residual inputs from the prefetch, later ones load them on the spot.
// `body` may contain warp-collective accumulator reads: the unit loop is
// uniform across the warp.
template <int BN, class Body>
__device__ __forceinline__ void for_resid_units(const GemmArgs& g, int m, int tn, int own,
                                                int n_own, const ResidPre& pre, Body body) {
  constexpr int U = BN / 16;
  const bool valid = m < g.M;
#pragma unroll
  for (int k = 0; k < PF; ++k) {
    const int u = own + k * n_own;
    const int n = tn * BN + u * 16;
    if (u < U && n < g.N) body(u, n, pre.h[k], pre.g[k]);
  }
  for (int u = own + PF * n_own; u < U; u += n_own) {
    const int n = tn * BN + u * 16;
    if (n >= g.N) break;
    float h16[16];
    uint32_t g8[8];
    if (valid) load_resid_inputs(g, m, n, h16, g8);
    body(u, n, h16, g8);
  }
}

// 16 fp32 values as two 16-byte packets of bf16 (words w[0..3]; never the
// sentinel).
__device__ __forceinline__ void pack_pkts(const float* v, unsigned long long* w) {
  uint32_t b[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) b[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = not_sentinel((unsigned long long)b[2 * i] | ((unsigned long long)b[2 * i + 1] << 32));
}

// v[0..15] += the 16 bf16 values of packets w[0..3].
__device__ __forceinline__ void add_pkts(const unsigned long long* w, float* v) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = (uint32_t)w[i], hi = (uint32_t)(w[i] >> 32);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lo));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hi));
    v[4 * i] += a.x;
    v[4 * i + 1] += a.y;
    v[4 * i + 2] += b.x;
    v[4 * i + 3] += b.y;
  }
}

// Row-parallel epilogue with the all-reduce across tensor-parallel ranks
// fused in (the 128 epilogue threads, one output row each).
//
//   one-shot  every rank pushes its bf16 partial of each 16-column unit of
//             the CTA's columns to every rank; each rank sums the world
//             partials in rank order
//   two-shot  unit u of tile t is owned by rank (t * BN/16 + u) % world:
//             every rank pushes its partial of the unit to the owner only;
//             the owner sums them in rank order and pushes the bf16 sum to
//             every rank
// Every rank then adds the same bf16 values to its replicated fp32 residual,
// so h stays bit-identical on all ranks.  A CTA's partners are the CTAs with
// the same tile and split on the other ranks.
//
// No flags: the exchange buffers hold the sentinel until the data lands
// (8-byte-atomic packet stores over NVLink); each receiving thread polls its
// own packets, sums them, and writes the sentinel back.  One NVLink
// traversal per phase, no round trip for a release or a flag.
//
// Exchange layout: [tile][16-column unit][half][128 rows][8 columns] bf16, the
// epilogue's own thread order (thread = row), so one warp store or load
// instruction moves 512 contiguous bytes.
template <int BN>
__device__ __forceinline__ float run_resid_tp(const GemmArgs& g, const AccReader<BN>& acc, int tm,
                                              int tn, int row, int own, int n_own,
                                              const ResidPre& pre, uint64_t* acc_free) {
  const CommDev& c = g.comm;
  const int m = tm * BM + row;
  const bool valid = m < g.M;
  const int N = g.N, W = c.world;
  // plane: every tile of a max_rows x n_cols output, padded to whole tiles
  const size_t plane = (size_t)((c.max_rows + BM - 1) / BM) * BM * (size_t)(c.n_cols + 256);
  const bool leader = threadIdx.x == 64;
  constexpr int U = BN / 16;
  const size_t tile_base = ((size_t)tm * g.tiles_n + tn) * U;
  const uint64_t t_start = (c.span_ns != nullptr && leader) ? globaltimer_ns() : 0;
  uint64_t t0 = 0;   // start of this thread's current peer wait
  auto xoff = [&](int u, int half) {
    return (((tile_base + u) * 2 + half) * BM + row) * 8;
  };
  auto rs_at = [&](int p, int src) { return c.rs[p] + ((size_t)c.par * W + src) * plane; };
  auto ag_at = [&](int p) { return c.ag[p] + (size_t)c.par * plane; };
  auto owner = [&](int u) { return (int)((tile_base + u) % (size_t)W); };
  auto push = [&](__nv_bfloat16* base, int u, const unsigned long long* w) {
    st_pkt(base + xoff(u, 0), w[0], w[1]);
    st_pkt(base + xoff(u, 1), w[2], w[3]);
  };
  // v = sum over sources s (rank order) of unit u in buffer src(s); every
  // packet is polled until it has landed, then reset to the sentinel.  The
  // loads of up to 4 sources are in flight at once.
  auto recv_sum = [&](auto src, int nsrc, int u, float* v) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.f;
#pragma unroll
    for (int s0 = 0; s0 < TB_MAX_RANKS; s0 += 4) {
      if (s0 < nsrc) {
        unsigned long long d[4][4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (s0 + k < nsrc) {
            ld_pkt(src(s0 + k) + xoff(u, 0), d[k][0], d[k][1]);
            ld_pkt(src(s0 + k) + xoff(u, 1), d[k][2], d[k][3]);
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (s0 + k < nsrc) {
            poll_pkt(src(s0 + k) + xoff(u, 0), d[k][0], d[k][1], t0);
            poll_pkt(src(s0 + k) + xoff(u, 1), d[k][2], d[k][3], t0);
            add_pkts(d[k], v);
            st_pkt(src(s0 + k) + xoff(u, 0), TB_SENTINEL, TB_SENTINEL);
            st_pkt(src(s0 + k) + xoff(u, 1), TB_SENTINEL, TB_SENTINEL);
          }
        }
      }
    }
  };

  // 1. push this rank's partials
  for (int u = own; u < U; u += n_own) {
    const int n = tn * BN + u * 16;
    if (n >= N) break;
    float v[16];
    acc.load16(u, u / n_own, v);   // warp-collective: every lane of the warp
    if (!valid) continue;
    unsigned long long w[4];
    pack_pkts(v, w);
    if (c.two_shot) {
      push(rs_at(owner(u), c.rank), u, w);
    } else {
      for (int p = 0; p < W; ++p) push(rs_at(p, c.rank), u, w);
    }
  }
  if (acc_free != nullptr) {
    // the accumulator has been read: a persistent CTA's MMA warp may reuse it
    tc_fence_before();
    epi_bar();
    if (leader) mbar_arrive(acc_free);
  }
  if (leader) trace_at(g, TR_PUSHED);

  const int dst = (valid && g.row_dst != nullptr) ? g.row_dst[m] : -1;
  float ss = 0.f;
  if (!c.two_shot) {
    // 2. sum the world partials in rank order and apply
    for_resid_units<BN>(g, m, tn, own, n_own, pre,
                        [&](int u, int n, const float* h_old, const uint32_t* g8) {
                          if (!valid) return;
                          float v[16];
                          recv_sum([&](int s) { return rs_at(c.rank, s); }, W, u, v);
                          ss += resid_update(g, m, n, dst, v, h_old, g8);
                        });
  } else {
    // 2'. owners reduce their units and send the bf16 sums to every rank
    for (int u = own; u < U; u += n_own) {
      const int n = tn * BN + u * 16;
      if (n >= N) break;
      if (!valid || owner(u) != c.rank) continue;
      float v[16];
      recv_sum([&](int s) { return rs_at(c.rank, s); }, W, u, v);
      unsigned long long w[4];
      pack_pkts(v, w);
      for (int p = 0; p < W; ++p) push(ag_at(p), u, w);
    }
    if (leader) trace_at(g, TR_PARTNERS);
    // 3. every rank applies the same reduced sums
    for_resid_units<BN>(g, m, tn, own, n_own, pre,
                        [&](int u, int n, const float* h_old, const uint32_t* g8) {
                          if (!valid) return;
                          float v[16];
                          recv_sum([&](int) { return ag_at(c.rank); }, 1, u, v);
                          ss += resid_update(g, m, n, dst, v, h_old, g8);
                        });
  }
  if (c.span_ns != nullptr) {
    epi_bar();   // every row of the tile has its values
    if (leader) atomicMax(c.span_ns, (unsigned long long)(globaltimer_ns() - t_start));
  }
  if (leader) trace_at(g, TR_SUMS);
  return ss;
}

// This CTA's partial row sum of h^2 -> row `part` of sq_out (and of sq2 for
// gathered rows).
__device__ __forceinline__ void store_row_sumsq(const GemmArgs& g, int tm, int part, int row,
                                                float ss) {
  const int m = tm * BM + row;
  if (m >= g.M) return;
  g.sq_out[(size_t)part * g.sq_out_ld + m] = ss;
  if (g.row_dst != nullptr) {
    const int dst = g.row_dst[m];
    if (dst >= 0) g.sq2[(size_t)part * g.sq2_ld + dst] = ss;
  }
}

// ------------------------------------------------------------ finisher
// Per-row values of the tile, written by the epilogue warps (one row per
// thread) before the accumulator is ready and read by the finisher.
struct RowStage {
  float* rs;  // deferred-norm scale
  int* pos;   // QKV: rotary position
  int* slot;  // QKV: KV-cache slot (-1: none)
  int* dst;   // RESID: gathered row of hg2 / sq2 (-1: none)
};

template <int EPI>
__device__ __forceinline__ void stage_rows(const GemmArgs& g, const RowStage& rw, int tm,
                                           int row) {
  const int m = tm * BM + row;
  rw.rs[row] = row_scale(g, m);
  if constexpr (EPI == EPI_QKV) {
    int pos = 0, slot = -1;
    if (m < g.M) {
      pos = g.positions[m];
      slot = g.slots[m];
      if (pos < 0 || pos >= g.max_pos || slot < 0) {
        set_status(ERR_BAD_INDEX);
        pos = 0;
        slot = -1;
      }
    }
    rw.pos[row] = pos;
    rw.slot[row] = slot;
  }
  if constexpr (EPI == EPI_RESID)
    rw.dst[row] = (m < g.M && g.row_dst != nullptr) ? g.row_dst[m] : -1;
}

// Copy this CTA's accumulator (TMEM, one row per thread) into the staging
// chunks: in cluster split-K straight into the shared memory of the member
// that owns each chunk (source z), else into this CTA's own staging area
// (source 0).  64 columns per TMEM load.
template <int BN>
__device__ __forceinline__ void stage_acc(const AccReader<BN>& acc, const TileUnits& tu, int S,
                                          int z, uint8_t* smem, int nslot, int row,
                                          bool cluster) {
  const uint32_t region = smem_u32(smem);
#pragma unroll 1
  for (int k0 = 0; k0 < BN / 16; k0 += 4) {
    float v[64];
    tmem_ld64(acc.taddr + 16 * k0, v);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      int p, which;
      tu.pair_of(k0 + kk, p, which);
      const int slot = (p / S) * tu.cp + which;
      if (cluster) {
        const uint32_t dst = cluster_map(region, (uint32_t)(p % S));
#pragma unroll
        for (int i = 0; i < 4; ++i)
          st_cluster_v4(dst + stage_off(z, slot, nslot, row, i), v[16 * kk + 4 * i],
                        v[16 * kk + 4 * i + 1], v[16 * kk + 4 * i + 2], v[16 * kk + 4 * i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          *reinterpret_cast<float4*>(smem + stage_off(0, slot, nslot, row, i)) =
              make_float4(v[16 * kk + 4 * i], v[16 * kk + 4 * i + 1], v[16 * kk + 4 * i + 2],
                          v[16 * kk + 4 * i + 3]);
      }
    }
  }
}

// Global split-K, last CTA of a tile: own accumulator + the other splits'
// workspace partials, summed in split order, into the staging area.
template <int BN>
__device__ __forceinline__ void stage_global(const AccReader<BN>& acc, const TileUnits& tu,
                                             uint8_t* smem, int nslot, int row) {
  for (int k = 0; k < BN / 16; ++k) {
    float v[16];
    acc.load16(k, 0, v);
    int p, which;
    tu.pair_of(k, p, which);
    const int slot = p * tu.cp + which;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<float4*>(smem + stage_off(0, slot, nslot, row, i)) =
          make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}

__device__ __forceinline__ uint2 pack_bf16x4(float a, float b, float c, float d) {
  return make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
}

// Finisher thread layout: thread t (0..127), lane l = t % 32 of epilogue
// warp w = t / 32, handles float4 i = l / 8 (columns 4i..4i+3 of a chunk) of
// rows fin_row(t) + 32 j, j < 4, where fin_row(t) = l % 8 + 8 w: one warp
// instruction covers 8 rows x 64 contiguous bytes of a row-major output, and
// the 4 threads of a row are lanes l, l^8, l^16, l^24.
__device__ __forceinline__ int fin_piece(int t) { return (t & 31) >> 3; }
__device__ __forceinline__ int fin_row(int t) { return (t & 7) + 8 * (t >> 5); }
//
// Residual inputs of one chunk for a finisher thread: its 4 rows of h (4
// float4) and 4 bf16 of g_next.
struct FinIn {
  float4 h[4];
  uint2 g;
};

// The inputs of the first n (<= FIN_PRE) chunks a finisher thread handles,
// loaded while the main loop runs.  A cluster member owns at most
// ceil(pairs / splits) chunks (3 for bn 128 x 3 and bn 256 x 6), so they all
// arrive in one round trip instead of one per chunk; chunks beyond these
// are loaded one chunk ahead.
constexpr int FIN_PRE = 4;
struct FinPre {
  FinIn c[FIN_PRE];
  int n;
  // c[k] for a k < FIN_PRE known only at run time (selects: the array stays
  // in registers)
  __device__ __forceinline__ FinIn at(int k) const {
    FinIn r = c[0];
#pragma unroll
    for (int j = 1; j < FIN_PRE; ++j)
      if (k == j) r = c[j];
    return r;
  }
};

__device__ __forceinline__ void load_fin_inputs(const GemmArgs& g, int tm, int r0, int n,
                                                FinIn& p) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int m = tm * BM + r0 + 32 * j;
    p.h[j] = m < g.M ? *reinterpret_cast<const float4*>(g.h + (size_t)m * g.ld_h + n)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  p.g = *reinterpret_cast<const uint2*>(g.gnext + n);
}

template <int BN>
__device__ __forceinline__ void fin_prefetch(const GemmArgs& g, int tm, int tn, int own, int step,
                                             int t, FinPre& p) {
  p.n = 0;
#pragma unroll
  for (int k = 0; k < FIN_PRE; ++k) {
    const int u = own + k * step;
    if (u < BN / 16 && tn * BN + u * 16 < g.N) {
      load_fin_inputs(g, tm, fin_row(t), tn * BN + u * 16 + 4 * fin_piece(t), p.c[k]);
      p.n = k + 1;
    }
  }
}

// h += acc; hg = bf16(h * g_next) (and its copy in row dst of hg2), for the
// chunks p0, p0 + step, ... below p_end (staging slots 0, 1, ...); the row
// sums of the new h^2 are added to ss (this thread's 4 rows).  One rolled
// loop over the chunks (the epilogue code runs from a cold instruction cache:
// compact code matters); the inputs of the first pre->n chunks come from
// `pre` when given, every later chunk's are loaded one chunk ahead.
template <int BN>
__device__ __forceinline__ void finish_resid(const GemmArgs& g, const RowStage& rw,
                                             const uint8_t* smem, int nsrc, int nslot, int tm,
                                             int tn, int p0, int p_end, int step, int t,
                                             const FinPre* pre, float* ss) {
  const int U = min(BN / 16, p_end);
  const int i = fin_piece(t), r0 = fin_row(t);
  const int npre = pre != nullptr ? pre->n : 0;
  FinIn cur;
  if (npre > 0) cur = pre->c[0];
  else if (p0 < U && tn * BN + p0 * 16 < g.N)
    load_fin_inputs(g, tm, r0, tn * BN + p0 * 16 + 4 * i, cur);
  int lp = 0;
#pragma unroll 1
  for (int u = p0; u < U && tn * BN + u * 16 < g.N; u += step, ++lp) {
    const int un = u + step;
    FinIn nxt;
    if (lp + 1 < npre) nxt = pre->at(lp + 1);
    else if (un < U && tn * BN + un * 16 < g.N)
      load_fin_inputs(g, tm, r0, tn * BN + un * 16 + 4 * i, nxt);
    const int n = tn * BN + u * 16 + 4 * i;
    const float2 ga = bf16x2_to_float2(cur.g.x), gb = bf16x2_to_float2(cur.g.y);
    // all four rows' sums first: their shared-memory loads overlap
    float4 acc4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc4[j] = stage_sum(smem, nsrc, nslot, lp, r0 + 32 * j, i);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = r0 + 32 * j, m = tm * BM + row;
      if (m >= g.M) continue;
      const float4 a = acc4[j];
      const float4 hn = make_float4(cur.h[j].x + a.x, cur.h[j].y + a.y, cur.h[j].z + a.z,
                                    cur.h[j].w + a.w);
      *reinterpret_cast<float4*>(g.h + (size_t)m * g.ld_h + n) = hn;
      ss[j] += hn.x * hn.x + hn.y * hn.y + hn.z * hn.z + hn.w * hn.w;
      const uint2 o = pack_bf16x4(hn.x * ga.x, hn.y * ga.y, hn.z * gb.x, hn.w * gb.y);
      *reinterpret_cast<uint2*>(g.hg + (size_t)m * g.ld_hg + n) = o;
      const int dst = rw.dst[row];
      if (dst >= 0) *reinterpret_cast<uint2*>(g.hg2 + (size_t)dst * g.ld_hg + n) = o;
    }
    cur = nxt;
  }
}

// The row sums of h^2 a finisher thread accumulated (4 rows, its 4 columns
// of each chunk), reduced over the 4 threads of each row -> row `part` of
// sq_out / sq2.
__device__ __forceinline__ void store_ss(const GemmArgs& g, int tm, int part, int t, float* ss) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], 8);
    ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], 16);
  }
  if (fin_piece(t) == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) store_row_sumsq(g, tm, part, fin_row(t) + 32 * j, ss[j]);
  }
}

// out = rowscale * acc, fp32 or bf16.
template <int BN, int EPI>
__device__ __forceinline__ void finish_linear(const GemmArgs& g, const RowStage& rw,
                                              const uint8_t* smem, int nsrc, int nslot, int tm,
                                              int tn, int own, int p_end, int n_own, int t) {
  const int i = fin_piece(t), r0 = fin_row(t);
  const int U = min(BN / 16, p_end);
  for (int u = own, lp = 0; u < U; u += n_own, ++lp) {
    const int n = tn * BN + u * 16 + 4 * i;
    if (tn * BN + u * 16 >= g.N) break;
    float4 acc4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc4[j] = stage_sum(smem, nsrc, nslot, lp, r0 + 32 * j, i);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = r0 + 32 * j, m = tm * BM + row;
      if (m >= g.M) continue;
      const float4 a = acc4[j];
      const float rs = rw.rs[row];
      const float v[4] = {a.x * rs, a.y * rs, a.z * rs, a.w * rs};
      if constexpr (EPI == EPI_F32) {
        float* o = reinterpret_cast<float*>(g.out) + (size_t)m * g.ld_out + n;
        if (n + 4 <= g.N) *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
        else
          for (int e = 0; e < 4 && n + e < g.N; ++e) o[e] = v[e];
      } else {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)m * g.ld_out + n;
        if (n + 4 <= g.N) *reinterpret_cast<uint2*>(o) = pack_bf16x4(v[0], v[1], v[2], v[3]);
        else
          for (int e = 0; e < 4 && n + e < g.N; ++e) o[e] = __float2bfloat16_rn(v[e]);
      }
    }
  }
}

// act = silu(gate) * up: the tile's first BN/2 columns are the gate rows of
// features [tn*BN/2, (tn+1)*BN/2), the last BN/2 the matching up rows.
template <int BN>
__device__ __forceinline__ void finish_swiglu(const GemmArgs& g, const RowStage& rw,
                                              const uint8_t* smem, int nsrc, int nslot, int tm,
                                              int tn, int own, int p_end, int n_own, int t) {
  const int i = fin_piece(t), r0 = fin_row(t);
  const int NP = min(BN / 32, p_end);
  for (int p = own, lp = 0; p < NP; p += n_own, ++lp) {
    const int f0 = tn * (BN / 2) + p * 16;
    if (f0 >= g.n_feat) break;
    float4 ga4[4], ua4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ga4[j] = stage_sum(smem, nsrc, nslot, 2 * lp, r0 + 32 * j, i);
      ua4[j] = stage_sum(smem, nsrc, nslot, 2 * lp + 1, r0 + 32 * j, i);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = r0 + 32 * j, m = tm * BM + row;
      if (m >= g.M) continue;
      const float4 a = ga4[j], b = ua4[j];
      const float rs = rw.rs[row];
      const float gv[4] = {a.x * rs, a.y * rs, a.z * rs, a.w * rs};
      const float uv[4] = {b.x * rs, b.y * rs, b.z * rs, b.w * rs};
      float y[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = gv[e] / (1.f + __expf(-gv[e])) * uv[e];
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)m * g.ld_out +
                                f0 + 4 * i) = pack_bf16x4(y[0], y[1], y[2], y[3]);
    }
  }
}

// Bias + RoPE of the q and k heads (bias only for v), q to q_out, k and v to
// the paged KV pool at each row's slot.  head_dim >= 32: a pair holds 16
// columns of a head's first half and their rotary partners half a head
// later; head_dim 16: a pair is one head, whose halves sit with threads i
// and i ^ 2.
template <int BN>
__device__ __forceinline__ void finish_qkv(const GemmArgs& g, const RowStage& rw, const uint8_t* smem,
                                           int nsrc, int nslot, int tm, int tn, int own,
                                           int p_end, int n_own, int t) {
  const int i = fin_piece(t), r0 = fin_row(t);
  const int hd = g.head_dim, half = hd >> 1;
  const int heads_in_tile = BN / hd;
  const int total_heads = g.n_q_heads + 2 * g.n_kv_heads;
  const TileUnits tu = tile_units<BN, EPI_QKV>(g);
  const int per_head = tu.kind == 2 ? tu.hc : 1;
  const int NP = min(tu.np, p_end);
  for (int p = own, lp = 0; p < NP; p += n_own, ++lp) {
    const int hh = p / per_head, jj = p % per_head;
    const int head = tn * heads_in_tile + hh;
    if (hh >= heads_in_tile || head >= total_heads) break;
    const int n0 = head * hd;
    const bool is_q = head < g.n_q_heads;
    const int is_v = head >= g.n_q_heads + g.n_kv_heads;
    const int kvh = is_q ? 0 : head - g.n_q_heads - (is_v ? g.n_kv_heads : 0);
    const bool rotate = !is_v;
    auto dst_of = [&](int m, int kslot) -> __nv_bfloat16* {
      if (is_q) return reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)m * g.ld_out + n0;
      const int blk = kslot / g.block_size, off = kslot % g.block_size;
      return g.kv_pool + ((((size_t)blk * 2 + is_v) * g.n_kv_heads + kvh) * g.block_size + off) * hd;
    };
    if (tu.kind == 2) {
      const int c_lo = jj * 16 + 4 * i, c_hi = half + c_lo;
      const uint2 bl2 = *reinterpret_cast<const uint2*>(g.bias + n0 + c_lo);
      const uint2 bh2 = *reinterpret_cast<const uint2*>(g.bias + n0 + c_hi);
      const float2 bl0 = bf16x2_to_float2(bl2.x), bl1 = bf16x2_to_float2(bl2.y);
      const float2 bh0 = bf16x2_to_float2(bh2.x), bh1 = bf16x2_to_float2(bh2.y);
      const float bl[4] = {bl0.x, bl0.y, bl1.x, bl1.y}, bh[4] = {bh0.x, bh0.y, bh1.x, bh1.y};
      // every input of the four rows first (shared sums, rotary cos/sin as
      // one 16-byte load each), so their latencies overlap
      float4 lo4[4], hi4[4], cs4[4], sn4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        lo4[j] = stage_sum(smem, nsrc, nslot, 2 * lp, r0 + 32 * j, i);
        hi4[j] = stage_sum(smem, nsrc, nslot, 2 * lp + 1, r0 + 32 * j, i);
        if (rotate) {
          const size_t f = (size_t)rw.pos[r0 + 32 * j] * half + c_lo;
          cs4[j] = *reinterpret_cast<const float4*>(g.rope_cos + f);
          sn4[j] = *reinterpret_cast<const float4*>(g.rope_sin + f);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int row = r0 + 32 * j, m = tm * BM + row;
        if (m >= g.M) continue;
        const int kslot = rw.slot[row];
        if (!is_q && kslot < 0) continue;
        const float4 a = lo4[j], b = hi4[j];
        const float rs = rw.rs[row];
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
        const float cv[4] = {cs4[j].x, cs4[j].y, cs4[j].z, cs4[j].w};
        const float sv[4] = {sn4[j].x, sn4[j].y, sn4[j].z, sn4[j].w};
        float o1[4], o2[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x1 = av[e] * rs + bl[e], x2 = bv[e] * rs + bh[e];
          if (rotate) {
            o1[e] = x1 * cv[e] - x2 * sv[e];
            o2[e] = x2 * cv[e] + x1 * sv[e];
          } else {
            o1[e] = x1;
            o2[e] = x2;
          }
        }
        __nv_bfloat16* d = dst_of(m, kslot);
        *reinterpret_cast<uint2*>(d + c_lo) = pack_bf16x4(o1[0], o1[1], o1[2], o1[3]);
        *reinterpret_cast<uint2*>(d + c_hi) = pack_bf16x4(o2[0], o2[1], o2[2], o2[3]);
      }
    } else {
      const int c = 4 * i;
      const uint2 b2 = *reinterpret_cast<const uint2*>(g.bias + n0 + c);
      const float2 b0 = bf16x2_to_float2(b2.x), b1 = bf16x2_to_float2(b2.y);
      const float bias4[4] = {b0.x, b0.y, b1.x, b1.y};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int row = r0 + 32 * j, m = tm * BM + row;
        const float4 a = stage_sum(smem, nsrc, nslot, lp, row, i);
        const float rs = rw.rs[row];
        const float av[4] = {a.x, a.y, a.z, a.w};
        float x[4], o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = av[e] * rs + bias4[e];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);   // thread of piece i ^ 2
          if (rotate) {
            const size_t f = (size_t)rw.pos[row] * half + (i & 1) * 4 + e;
            const float cs = g.rope_cos[f], sn = g.rope_sin[f];
            o[e] = i < 2 ? x[e] * cs - partner * sn : x[e] * cs + partner * sn;
          } else {
            o[e] = x[e];
          }
        }
        const int kslot = rw.slot[row];
        if (m < g.M && (is_q || kslot >= 0))
          *reinterpret_cast<uint2*>(dst_of(m, kslot) + c) = pack_bf16x4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// Finish the pairs p0, p0 + step, ... below p_end of tile (tm, tn) from the
// staging area (nsrc sources of nslot chunks; the k-th pair at slots
// k * cp + which).  EPI_RESID adds its row sums of h^2 to ss.
template <int BN, int EPI>
__device__ __forceinline__ void finish(const GemmArgs& g, const RowStage& rw, const uint8_t* smem,
                                       int nsrc, int nslot, int tm, int tn, int p0, int p_end,
                                       int step, int t, const FinPre* pre, float* ss) {
  if constexpr (EPI == EPI_RESID)
    finish_resid<BN>(g, rw, smem, nsrc, nslot, tm, tn, p0, p_end, step, t, pre, ss);
  else if constexpr (EPI == EPI_SWIGLU)
    finish_swiglu<BN>(g, rw, smem, nsrc, nslot, tm, tn, p0, p_end, step, t);
  else if constexpr (EPI == EPI_QKV)
    finish_qkv<BN>(g, rw, smem, nsrc, nslot, tm, tn, p0, p_end, step, t);
  else
    finish_linear<BN, EPI>(g, rw, smem, nsrc, nslot, tm, tn, p0, p_end, step, t);
}

// Split-K GEMM: one CTA per (tile, k-slice).  With scratch the slices park
// fp32 partials in global memory and the last to arrive finishes the tile;
// without it a tile's slices form one cluster and push their partials into
// the owners' shared memory.
template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a,
                   const __grid_constant__ CUtensorMap tma_b, const GemmArgs g) {
  using L = GemmLayout<BN, STAGES>;
  constexpr uint32_t TCOLS = tmem_cols(BN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* sA = smem + L::OFF_A;
  uint8_t* sB = smem + L::OFF_B;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* row_rs = reinterpret_cast<float*>(tmem_slot + 4);  // [BM] per-row values (RowStage)
  int* row_pos = reinterpret_cast<int*>(row_rs + BM);
  int* row_slot = row_pos + BM;
  int* row_dst = row_slot + BM;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // split-K only: launches without it run gemm_persistent_kernel
  const int mode = g.ws != nullptr ? SPLIT_GLOBAL : SPLIT_CLUSTER;

  // grouped raster: m fastest inside a group of group_m row tiles
  const int tile = mode == SPLIT_CLUSTER ? (int)blockIdx.x / g.splits : (int)blockIdx.x;
  const int z = mode == SPLIT_CLUSTER ? (int)blockIdx.x % g.splits : (int)blockIdx.y;
  const int per_group = g.group_m * g.tiles_n;
  const int first_m = (tile / per_group) * g.group_m;
  const int gsize = min(g.tiles_m - first_m, g.group_m);
  const int tm = first_m + (tile % per_group) % gsize;
  const int tn = (tile % per_group) / gsize;
  const int num_k = (g.K + BK - 1) / BK;
  const int kb = (int)((long long)z * num_k / g.splits);
  const int ke = (int)((long long)(z + 1) * num_k / g.splits);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TCOLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) {
    pdl_trigger();
    trace_at(g, TR_START);
  }

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    // The weight tiles of the first stages do not depend on earlier kernels:
    // fetch them before waiting for the previous kernel, then the activations.
    const int pre = min(STAGES, ke - kb);
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], A_BYTES + L::B_BYTES);
      tma_load_2d(sB + i * L::B_BYTES, &tma_b, &full[i], (kb + i) * BK, tn * BN);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(sA + i * A_BYTES, &tma_a, &full[i], (kb + i) * BK, tm * BM);
    for (int it = kb + pre; it < ke; ++it) {
      const int i = it - kb, s = i % STAGES;
      if (!mbar_wait(&empty[s], ((i / STAGES) - 1) & 1)) break;
      mbar_arrive_expect_tx(&full[s], A_BYTES + L::B_BYTES);
      tma_load_2d(sA + s * A_BYTES, &tma_a, &full[s], it * BK, tm * BM);
      tma_load_2d(sB + s * L::B_BYTES, &tma_b, &full[s], it * BK, tn * BN);
    }
    trace_at(g, TR_LOADS_ISSUED);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = idesc_bf16_m128(BN);
    bool ok = true;
    for (int it = kb; it < ke; ++it) {
      const int i = it - kb, s = i % STAGES;
      if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * L::B_BYTES);
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk)
        tc_mma_bf16(tmem_base, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc,
                    (i > 0 || kk > 0) ? 1u : 0u);
      tc_commit(&empty[s]);
    }
    if (ok) tc_commit(done);
    else mbar_arrive(done);
  }
  __syncwarp();

  const int q = warp & 3;
  const int row = q * 32 + lane;   // TMEM lane of this thread (epilogue warps)
  const int t = threadIdx.x - 64;  // finisher thread index (epilogue warps)
  const TileUnits tu = tile_units<BN, EPI>(g);
  const int S = mode == SPLIT_CLUSTER ? g.splits : 1;
  const int nslot = ((tu.np + S - 1) / S) * tu.cp;
  // the row-parallel projection across tensor-parallel ranks keeps one row
  // per thread end to end (its exchange layout is row-major per thread)
  const bool tp = EPI == EPI_RESID && g.comm.world > 1;
  AccReader<BN> acc;
  acc.taddr = tmem_base + ((uint32_t)(q * 32) << 16);
  acc.mode = mode;
  acc.splits = g.splits;
  acc.z = z;
  acc.row = row;
  acc.ws = nullptr;
  acc.smem = smem;
  acc.nslot = nslot;
  const RowStage rw{row_rs, row_pos, row_slot, row_dst};

  ResidPre pre;     // tensor-parallel residual: one row per thread
  FinPre fpre;      // finisher: inputs of its first chunks
  if (warp >= 2) {
    pdl_wait();   // the epilogue reads and writes buffers earlier kernels use
    // inputs that do not depend on the accumulator load under the main loop
    stage_rows<EPI>(g, rw, tm, row);
    if constexpr (EPI == EPI_RESID) {
      if (tp) resid_prefetch<BN>(g, tm, tn, row, mode == SPLIT_CLUSTER ? z : 0, S, pre);
      else fin_prefetch<BN>(g, tm, tn, mode == SPLIT_CLUSTER ? z : 0, S, t, fpre);
    }
  }
  if (mode == SPLIT_CLUSTER) {
    if (warp >= 2) {
      mbar_wait(done, 0);
      tc_fence_after();
      if (threadIdx.x == 64) trace_at(g, TR_ACC_READY);
    }
    // 1. every member's MMAs are complete, so every stage ring is free
    cluster_sync_all();
    // 2. store each 16-column chunk of this partial into its owner's ring
    if (warp >= 2) {
      stage_acc<BN>(acc, tu, S, z, smem, nslot, row, true);
      if (threadIdx.x == 64) trace_at(g, TR_PARKED);
    }
    // 3. every chunk has arrived; from here on each CTA reads only its own
    //    shared memory, so members may exit independently
    cluster_sync_all();
    if (threadIdx.x == 64) trace_at(g, TR_CLUSTER_SYNC);
    if (warp >= 2) {
      if (tp) {
        const float ss = run_resid_tp<BN>(g, acc, tm, tn, row, z, S, pre, nullptr);
        store_row_sumsq(g, tm, tn * S + z, row, ss);
      } else {
        float ss[4] = {0.f, 0.f, 0.f, 0.f};
        finish<BN, EPI>(g, rw, smem, S, nslot, tm, tn, z, 1 << 30, S, t, &fpre, ss);
        if constexpr (EPI == EPI_RESID) store_ss(g, tm, tn * S + z, t, ss);
      }
      if (threadIdx.x == 64) trace_at(g, TR_END);
    }
  } else if (warp >= 2) {
    mbar_wait(done, 0);
    tc_fence_after();
    if (threadIdx.x == 64) trace_at(g, TR_ACC_READY);
    bool run;
    {
      const size_t tile_lin = (size_t)tm * g.tiles_n + tn;
      float* ws_tile = g.ws + tile_lin * g.splits * BN * BM;
      float* mine = ws_tile + (size_t)z * BN * BM + row;
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(acc.taddr + c, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) __stcg(mine + (size_t)(c + j) * BM, v[j]);
      }
      __threadfence();
      epi_bar();
      if (threadIdx.x == 64) {
        const int prev = atomicAdd(&g.counters[tile_lin], 1);
        const int last = prev == g.splits - 1;
        if (last) g.counters[tile_lin] = 0;
        *last_flag = last;
      }
      epi_bar();
      run = *last_flag != 0;
      __threadfence();
      acc.ws = ws_tile;
    }
    if (run) {
      if (tp) {
        const float ss = run_resid_tp<BN>(g, acc, tm, tn, row, 0, 1, pre, nullptr);
        store_row_sumsq(g, tm, tn, row, ss);
      } else {
        stage_global<BN>(acc, tu, smem, nslot, row);
        epi_bar();   // staged chunks and per-row values visible to every finisher thread
        float ss[4] = {0.f, 0.f, 0.f, 0.f};
        finish<BN, EPI>(g, rw, smem, 1, nslot, tm, tn, 0, 1 << 30, 1, t, &fpre, ss);
        if constexpr (EPI == EPI_RESID) store_ss(g, tm, tn, t, ss);
      }
    }
    if (threadIdx.x == 64) trace_at(g, TR_END);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TCOLS);
  }
}

// ------------------------------------------------------- persistent kernel
// Launches without split-K run persistent: one CTA per SM walks the tiles
// blockIdx.x, blockIdx.x + gridDim.x, ...; the MMA warp alternates between
// two TMEM accumulators, so tile i's epilogue (and, across tensor-parallel
// ranks, its NVLink exchange) overlaps tile i+1's main loop.  The epilogue
// stages 4 chunks at a time in a dedicated shared-memory area (the stage
// ring keeps streaming the next tile) and finishes them with the finisher
// layout.
template <int BN, int STAGES>
struct PersistLayout {
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = STAGES * A_BYTES;
  static constexpr int OFF_STAGE = OFF_B + STAGES * B_BYTES;
  static constexpr int STAGE_CHUNKS = 4;
  static constexpr int OFF_BAR = OFF_STAGE + STAGE_CHUNKS * BM * 16 * 4;
  static constexpr int BAR_BYTES = (2 * STAGES + 4) * 8 + 16 + 4 * BM * 4;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;
  static_assert(SMEM <= 232448, "persistent GEMM shared memory above 227 KiB");
};

// Tile (tm, tn) of linear tile index `tile`: m fastest inside groups of
// group_m row tiles (A tiles of a group stay in L2 while N advances).
__device__ __forceinline__ void tile_coords(const GemmArgs& g, int tile, int& tm, int& tn) {
  const int per_group = g.group_m * g.tiles_n;
  const int first_m = (tile / per_group) * g.group_m;
  const int gsize = min(g.tiles_m - first_m, g.group_m);
  tm = first_m + (tile % per_group) % gsize;
  tn = (tile % per_group) / gsize;
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tma_a,
                           const __grid_constant__ CUtensorMap tma_b, const GemmArgs g) {
  using L = PersistLayout<BN, STAGES>;
  constexpr uint32_t TC = tmem_cols(BN);
  constexpr uint32_t TCOLS = 2 * TC;
  static_assert(TCOLS <= 512, "two accumulators must fit TMEM");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* sA = smem + L::OFF_A;
  uint8_t* sB = smem + L::OFF_B;
  uint8_t* stage = smem + L::OFF_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* row_rs = reinterpret_cast<float*>(tmem_slot + 4);
  int* row_pos = reinterpret_cast<int*>(row_rs + BM);
  int* row_slot = row_pos + BM;
  int* row_dst = row_slot + BM;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = g.tiles_m * g.tiles_n;
  const int num_k = (g.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 1);
    }
    fence_mbar_init();
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TCOLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) {
    pdl_trigger();
    trace_at(g, TR_START);
  }

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer: one continuous ring over all tiles
    pdl_wait();
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      int tm, tn;
      tile_coords(g, tile, tm, tn);
      for (int kb = 0; kb < num_k; ++kb, ++it) {
        const int s = it % STAGES;
        if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], A_BYTES + L::B_BYTES);
        tma_load_2d(sA + s * A_BYTES, &tma_a, &full[s], kb * BK, tm * BM);
        tma_load_2d(sB + s * L::B_BYTES, &tma_b, &full[s], kb * BK, tn * BN);
      }
    }
    trace_at(g, TR_LOADS_ISSUED);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer: accumulator i & 1 for the CTA's i-th tile
    constexpr uint32_t idesc = idesc_bf16_m128(BN);
    int it = 0, i = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++i) {
      const int b = i & 1, use = i >> 1;
      if (use > 0 && !mbar_wait(&acc_empty[b], (use - 1) & 1)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + (uint32_t)(b * TC);
      for (int kb = 0; kb < num_k; ++kb, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * L::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc_mma_bf16(d, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      if (ok) tc_commit(&acc_full[b]);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue: tile by tile, overlapping the next main loop
    const int q = warp & 3;
    const int row = q * 32 + lane;   // TMEM lane of this thread
    const int t = threadIdx.x - 64;  // finisher thread index
    const TileUnits tu = tile_units<BN, EPI>(g);
    const int PG = L::STAGE_CHUNKS / tu.cp;   // pairs per staged group
    const RowStage rw{row_rs, row_pos, row_slot, row_dst};
    const bool tp = EPI == EPI_RESID && g.comm.world > 1;
    AccReader<BN> acc;
    acc.mode = SPLIT_NONE;
    acc.splits = 1;
    acc.z = 0;
    acc.row = row;
    acc.ws = nullptr;
    acc.smem = stage;
    acc.nslot = L::STAGE_CHUNKS;
    pdl_wait();   // the epilogue reads and writes buffers earlier kernels use
    int i = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
      int tm, tn;
      tile_coords(g, tile, tm, tn);
      const int b = i & 1, use = i >> 1;
      epi_bar();   // the previous tile's finisher is done with the per-row arrays
      stage_rows<EPI>(g, rw, tm, row);
      ResidPre pre;
      if constexpr (EPI == EPI_RESID) {
        if (tp) resid_prefetch<BN>(g, tm, tn, row, 0, 1, pre);
      }
      if (!mbar_wait(&acc_full[b], use & 1)) break;
      tc_fence_after();
      acc.taddr = tmem_base + (uint32_t)(b * TC) + ((uint32_t)(q * 32) << 16);
      if (tp) {
        const float ss = run_resid_tp<BN>(g, acc, tm, tn, row, 0, 1, pre, &acc_empty[b]);
        store_row_sumsq(g, tm, tn, row, ss);
        continue;
      }
      float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int p0 = 0; p0 < tu.np; p0 += PG) {
        // stage the group's chunks from TMEM (one row per thread)
        for (int k = 0; k < PG && p0 + k < tu.np; ++k) {
          for (int which = 0; which < tu.cp; ++which) {
            float v[16];
            tmem_ld16(acc.taddr + 16 * tu.chunk(p0 + k, which), v);
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
              *reinterpret_cast<float4*>(stage + stage_off(0, k * tu.cp + which, L::STAGE_CHUNKS,
                                                           row, c4)) =
                  make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
          }
        }
        const bool last = p0 + PG >= tu.np;
        if (last) tc_fence_before();
        epi_bar();   // staged chunks (and, first time, per-row values) visible to all
        if (last && threadIdx.x == 64) mbar_arrive(&acc_empty[b]);   // accumulator reusable
        finish<BN, EPI>(g, rw, stage, 1, L::STAGE_CHUNKS, tm, tn, p0, p0 + PG, 1, t, nullptr, ss);
        epi_bar();   // the staging area is rewritten by the next group
      }
      if constexpr (EPI == EPI_RESID) store_ss(g, tm, tn, t, ss);
    }
    if (threadIdx.x == 64) trace_at(g, TR_END);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TCOLS);
  }
}

// ------------------------------------------------------------------ host side

template <int BN, int STAGES, int EPI>
static int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb_, const GemmArgs& g,
                     cudaStream_t stream) {
  using L = GemmLayout<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES, EPI>;
  static std::atomic<unsigned long long> attr_devs{0};
  if (int rc = smem_attr_once(kern, L::SMEM, attr_devs, "gemm smem attribute")) return rc;
  const int tiles = g.tiles_m * g.tiles_n;
  if (g.splits > 1 && g.ws == nullptr) {  // cluster split-K: a tile's splits are one cluster along x
    const bool paired = EPI == EPI_SWIGLU || (EPI == EPI_QKV && g.head_dim >= 32);
    const int np = paired ? BN / 32 : BN / 16, cp = paired ? 2 : 1;
    if (cluster_region_bytes(np, cp, g.splits) > L::RING)
      return arg_err("cluster split-K: the partial chunks of this (bn, splits) do not fit shared memory");
    return launch_pdl(kern, dim3(tiles * g.splits), dim3(GEMM_THREADS), L::SMEM, stream,
                      g.splits, "gemm cluster launch", ta, tb_, g);
  }
  return launch_pdl(kern, dim3(tiles, g.splits), dim3(GEMM_THREADS), L::SMEM, stream, 1,
                    "gemm launch", ta, tb_, g);
}

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

template <int BN, int STAGES, int EPI>
static int launch_persistent(const CUtensorMap& ta, const CUtensorMap& tb_, const GemmArgs& g,
                             cudaStream_t stream) {
  using L = PersistLayout<BN, STAGES>;
  auto kern = gemm_persistent_kernel<BN, STAGES, EPI>;
  static std::atomic<unsigned long long> attr_devs{0};
  if (int rc = smem_attr_once(kern, L::SMEM, attr_devs, "persistent gemm smem attribute"))
    return rc;
  const int tiles = g.tiles_m * g.tiles_n;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  return launch_pdl(kern, dim3(grid), dim3(GEMM_THREADS), L::SMEM, stream, 1,
                    "gemm persistent launch", ta, tb_, g);
}

template <int EPI>
static int launch_epi(int bn, const CUtensorMap& ta, const CUtensorMap& tb_, const GemmArgs& g,
                      cudaStream_t stream) {
  if (g.splits == 1 && g.ws == nullptr) {   // no split-K: persistent tiles
    switch (bn) {
      case 64: return launch_persistent<64, 7, EPI>(ta, tb_, g, stream);
      case 128: return launch_persistent<128, 5, EPI>(ta, tb_, g, stream);
      case 192: return launch_persistent<192, 4, EPI>(ta, tb_, g, stream);
      case 256: return launch_persistent<256, 3, EPI>(ta, tb_, g, stream);
      default: return arg_err("bn must be 64, 128, 192 or 256");
    }
  }
  switch (bn) {
    case 64: return launch_bn<64, 8, EPI>(ta, tb_, g, stream);
    case 128: return launch_bn<128, 6, EPI>(ta, tb_, g, stream);
    case 192: return launch_bn<192, 5, EPI>(ta, tb_, g, stream);
    case 256: return launch_bn<256, 4, EPI>(ta, tb_, g, stream);
    default: return arg_err("bn must be 64, 128, 192 or 256");
  }
}

template <int BN, int STAGES>
static int max_clusters_bn(int cluster, int* out) {
  using L = GemmLayout<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES, EPI_F32>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  if (e != cudaSuccess) return host_err(e, "gemm smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster * 64, 1, 1);
  cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = L::SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return host_err(cudaOccupancyMaxActiveClusters(out, kern, &cfg), "max active clusters");
}

int gemm_max_active_clusters(int bn, int cluster, int* out) {
  switch (bn) {
    case 64: return max_clusters_bn<64, 8>(cluster, out);
    case 128: return max_clusters_bn<128, 6>(cluster, out);
    case 192: return max_clusters_bn<192, 5>(cluster, out);
    case 256: return max_clusters_bn<256, 4>(cluster, out);
    default: return arg_err("bn must be 64, 128, 192 or 256");
  }
}

unsigned long long* g_debug_trace = nullptr;

int gemm_launch(int epi, int bn, const void* A, int lda, const void* B, int ldb, GemmArgs g,
                cudaStream_t stream) {
  g.trace = g_debug_trace;
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return arg_err("M, N, K must be positive");
  if ((lda * 2) % 16 || (ldb * 2) % 16 || lda < g.K || ldb < g.K)
    return arg_err("lda/ldb: rows must be 16-byte multiples and >= K");
  if (reinterpret_cast<uintptr_t>(A) % 16 || reinterpret_cast<uintptr_t>(B) % 16)
    return arg_err("A and B must be 16-byte aligned");
  const int num_k = (g.K + BK - 1) / BK;
  if (g.splits < 1 || g.splits > num_k) return arg_err("splits must be in [1, ceil(K/64)]");
  if (g.splits > 1 && g.ws == nullptr && g.splits > 8)
    return arg_err("cluster split-K supports at most 8 splits");
  if (g.splits > 1 && (g.ws == nullptr) != (g.counters == nullptr))
    return arg_err("split-K scratch pointers");
  if (g.splits == 1) {   // no split-K: the persistent kernel, no scratch
    g.ws = nullptr;
    g.counters = nullptr;
  }
  g.tiles_m = (g.M + BM - 1) / BM;
  g.tiles_n = (g.N + bn - 1) / bn;
  if (g.group_m <= 0) g.group_m = 16;
  CUtensorMap ta, tbm;
  int rc = make_tmap_2d(&ta, A, g.K, g.M, (uint64_t)lda * 2, BK, BM);
  if (rc) return rc;
  rc = make_tmap_2d(&tbm, B, g.K, g.N, (uint64_t)ldb * 2, BK, bn);
  if (rc) return rc;
  switch (epi) {
    case EPI_F32: return launch_epi<EPI_F32>(bn, ta, tbm, g, stream);
    case EPI_BF16: return launch_epi<EPI_BF16>(bn, ta, tbm, g, stream);
    case EPI_QKV: return launch_epi<EPI_QKV>(bn, ta, tbm, g, stream);
    case EPI_SWIGLU: return launch_epi<EPI_SWIGLU>(bn, ta, tbm, g, stream);
    case EPI_RESID: return launch_epi<EPI_RESID>(bn, ta, tbm, g, stream);
    default: return arg_err("unknown epilogue");
  }
}

}  // namespace tb
