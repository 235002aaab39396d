// tcgen05 GEMM kernel and its host launcher (see gemm.cuh for the design).
#include <stdio.h>

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
                      // CTA parks its partial in its own shared memory and
                      // reduces a slice of columns over DSMEM
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
  static constexpr int BAR_BYTES = (2 * STAGES + 1) * 8 + 16 + BM * 4;  // + per-row sums
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;                // + alignment slack
  // cluster mode parks the fp32 tile [BN/4][BM] float4 over the stage ring
  static_assert(BN * BM * 4 <= OFF_BAR, "stage ring too small for the partial tile");
};

__device__ __forceinline__ float row_scale(const GemmArgs& g, int m) {
  if (g.sq == nullptr || m >= g.M) return 1.f;
  float s = 0.f;
  for (int p = 0; p < g.sq_parts; ++p) s += g.sq[(size_t)p * g.sq_ld + m];
  return rsqrtf(s * g.inv_d + g.eps);
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

__device__ __forceinline__ float4 ld_cluster_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Accumulator access for the epilogue: columns [c, c+W) of this thread's row.
// In SPLIT_NONE / SPLIT_GLOBAL mode it reads TMEM (collective over the warp:
// every lane calls it); in SPLIT_CLUSTER mode it sums the cluster's parked
// partial tiles in rank order.
template <int BN>
struct AccReader {
  uint32_t taddr;   // TMEM address of this warp's lane quarter, column 0
  int mode, splits, z, row;
  const float* ws;  // SPLIT_GLOBAL: this tile's workspace, [splits][BN][128]
  uint32_t red;     // SPLIT_CLUSTER: shared address of the parked tile
  template <int W>
  __device__ __forceinline__ void load(int c, float* v) const {
    if (mode == SPLIT_CLUSTER) {
      // ordered sum over the cluster members, the next member's loads in
      // flight while the current one is added
      const uint32_t off = (uint32_t)(((c / 4) * BM + row) * 16);
      float4 cur[W / 4], nxt[W / 4];
#pragma unroll
      for (int i = 0; i < W / 4; ++i) cur[i] = ld_cluster_v4(cluster_map(red, 0) + off + i * BM * 16);
#pragma unroll
      for (int j = 0; j < W; ++j) v[j] = 0.f;
      for (int s = 0; s < splits; ++s) {
        if (s + 1 < splits) {
          const uint32_t base = cluster_map(red, s + 1) + off;
#pragma unroll
          for (int i = 0; i < W / 4; ++i) nxt[i] = ld_cluster_v4(base + i * BM * 16);
        }
#pragma unroll
        for (int i = 0; i < W / 4; ++i) {
          v[4 * i] += cur[i].x;
          v[4 * i + 1] += cur[i].y;
          v[4 * i + 2] += cur[i].z;
          v[4 * i + 3] += cur[i].w;
          cur[i] = nxt[i];
        }
      }
      return;
    }
    float own[W];
    if constexpr (W == 16) tmem_ld16(taddr + c, own);
    else tmem_ld8(taddr + c, own);
    if (mode == SPLIT_NONE) {
#pragma unroll
      for (int j = 0; j < W; ++j) v[j] = own[j];
      return;
    }
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = 0.f;
    for (int s = 0; s < splits; ++s) {
      if (s == z) {
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] += own[j];
      } else {
        const float* p = ws + ((size_t)s * BN + c) * BM + row;
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] += __ldcg(p + (size_t)j * BM);
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

// 8 bf16 values as fp32, read around L1 (they were written by other GPUs).
__device__ __forceinline__ void ld_bf16x8_cg(const __nv_bfloat16* p, float* v) {
  const uint4 a = __ldcg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(pa[i]);
    v[2 * i] = x.x;
    v[2 * i + 1] = x.y;
  }
}

__device__ __forceinline__ void pack_bf16x16(const float* v, uint4& lo, uint4& hi) {
  lo.x = pack_bf16x2(v[0], v[1]);
  lo.y = pack_bf16x2(v[2], v[3]);
  lo.z = pack_bf16x2(v[4], v[5]);
  lo.w = pack_bf16x2(v[6], v[7]);
  hi.x = pack_bf16x2(v[8], v[9]);
  hi.y = pack_bf16x2(v[10], v[11]);
  hi.z = pack_bf16x2(v[12], v[13]);
  hi.w = pack_bf16x2(v[14], v[15]);
}

// One system fence (cumulative: it orders the CTA's pushes, which the caller
// made visible to this thread with a CTA barrier after each thread's own
// fence), then a relaxed flag store to every rank.
template <class F>
__device__ __forceinline__ void signal_peers(const CommDev& c, F flag_of, uint32_t epoch) {
  fence_sys();
  for (int p = 0; p < c.world; ++p) st_relaxed_sys(flag_of(p), epoch);
}

// Row-parallel epilogue with the all-reduce across tensor-parallel ranks
// fused in (all 128 epilogue threads call it; it synchronises them).
//
//   one-shot  every rank pushes its bf16 partial of the CTA's columns to
//             every rank; each rank sums the world partials in rank order
//   two-shot  every rank pushes each column's partial to the column's owner
//             (rank n / (N / world)); the owner sums them in rank order and
//             pushes the bf16 sum to every rank
// Every rank then adds the same bf16 values to its replicated fp32 residual,
// so h stays bit-identical on all ranks.  A CTA's partners are the CTAs
// with the same index on the other ranks; "delivered" flags carry the call's
// epoch (release stores after a system fence; acquire loads, bounded wait).
//
// Exchange layout: [tile][16-column unit][half][128 rows][8 columns] bf16, the
// epilogue's own thread order (thread = row), so one warp store or load
// instruction moves 512 contiguous bytes over NVLink.
template <int BN>
__device__ __forceinline__ float run_resid_tp(const GemmArgs& g, const AccReader<BN>& acc, int tm,
                                           int tn, int row, int own, int n_own,
                                           const ResidPre& pre) {
  const CommDev& c = g.comm;
  const int m = tm * BM + row;
  const bool valid = m < g.M;
  const int N = g.N;
  const uint32_t epoch = c.state[0] * (uint32_t)c.n_sites + (uint32_t)c.site + 1u;
  const int par = (int)(epoch & 1u);
  // plane: every tile of a max_rows x n_cols output, padded to whole tiles
  const size_t plane = (size_t)((c.max_rows + BM - 1) / BM) * BM * (size_t)(c.n_cols + 256);
  const int cta = blockIdx.x;
  const int per_owner = N / c.world;
  const bool leader = threadIdx.x == 64;
  constexpr int U = BN / 16;
  const size_t tile_base = ((size_t)tm * g.tiles_n + tn) * U;
  auto xoff = [&](int u, int half) {
    return (((tile_base + u) * 2 + half) * BM + row) * 8;
  };
  auto rs_at = [&](int p, int src) { return c.rs[p] + ((size_t)par * c.world + src) * plane; };
  auto flag_at = [&](int p, int kind, int src) {
    return c.flags[p] + ((size_t)((kind * 2 + par) * c.world + src)) * c.max_ctas + cta;
  };
  auto put16 = [&](__nv_bfloat16* base, int u, const float* v) {
    uint4 lo, hi;
    pack_bf16x16(v, lo, hi);
    *reinterpret_cast<uint4*>(base + xoff(u, 0)) = lo;
    *reinterpret_cast<uint4*>(base + xoff(u, 1)) = hi;
  };

  // 1. push this rank's partials
  for (int u = own; u < U; u += n_own) {
    const int n = tn * BN + u * 16;
    if (n >= N) break;
    float v[16];
    acc.template load<16>(u * 16, v);
    if (!valid) continue;
    if (c.two_shot) {
      put16(rs_at(n / per_owner, c.rank), u, v);
    } else {
      for (int p = 0; p < c.world; ++p) put16(rs_at(p, c.rank), u, v);
    }
  }
  fence_sys();
  epi_bar();
  if (leader) {
    trace_at(g, TR_PUSHED);
    signal_peers(c, [&](int p) { return flag_at(p, 0, c.rank); }, epoch);
    for (int s = 0; s < c.world; ++s) wait_flag_sys(flag_at(c.rank, 0, s), epoch);
    trace_at(g, TR_PARTNERS);
  }
  epi_bar();

  // the world partials of unit u summed in rank order; the next rank's loads
  // are in flight while the current rank's are added
  auto sum_partials = [&](int u, float* v) {
    uint4 cur0, cur1, nxt0, nxt1;
    cur0 = __ldcg(reinterpret_cast<const uint4*>(rs_at(c.rank, 0) + xoff(u, 0)));
    cur1 = __ldcg(reinterpret_cast<const uint4*>(rs_at(c.rank, 0) + xoff(u, 1)));
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.f;
    for (int s = 0; s < c.world; ++s) {
      if (s + 1 < c.world) {
        nxt0 = __ldcg(reinterpret_cast<const uint4*>(rs_at(c.rank, s + 1) + xoff(u, 0)));
        nxt1 = __ldcg(reinterpret_cast<const uint4*>(rs_at(c.rank, s + 1) + xoff(u, 1)));
      }
      const __nv_bfloat162* q0 = reinterpret_cast<const __nv_bfloat162*>(&cur0);
      const __nv_bfloat162* q1 = reinterpret_cast<const __nv_bfloat162*>(&cur1);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = __bfloat1622float2(q0[i]);
        const float2 b = __bfloat1622float2(q1[i]);
        v[2 * i] += a.x;
        v[2 * i + 1] += a.y;
        v[8 + 2 * i] += b.x;
        v[8 + 2 * i + 1] += b.y;
      }
      cur0 = nxt0;
      cur1 = nxt1;
    }
  };

  const int dst = (valid && g.row_dst != nullptr) ? g.row_dst[m] : -1;
  float ss = 0.f;
  if (!c.two_shot) {
    // 2. sum the world partials in rank order and apply
    for_resid_units<BN>(g, m, tn, own, n_own, pre,
                        [&](int u, int n, const float* h_old, const uint32_t* g8) {
                          if (!valid) return;
                          float v[16];
                          sum_partials(u, v);
                          ss += resid_update(g, m, n, dst, v, h_old, g8);
                        });
    return ss;
  }

  // 2'. owners reduce their columns and broadcast the bf16 sums
  const size_t ag_off = (size_t)par * plane;
  for (int u = own; u < U; u += n_own) {
    const int n = tn * BN + u * 16;
    if (n >= N) break;
    if (!valid || n / per_owner != c.rank) continue;
    float v[16];
    sum_partials(u, v);
    for (int p = 0; p < c.world; ++p) put16(c.ag[p] + ag_off, u, v);
  }
  fence_sys();
  epi_bar();
  if (leader) {
    signal_peers(c, [&](int p) { return flag_at(p, 1, c.rank); }, epoch);
    for (int s = 0; s < c.world; ++s) wait_flag_sys(flag_at(c.rank, 1, s), epoch);
    trace_at(g, TR_SUMS);
  }
  epi_bar();
  // 3. every rank applies the same reduced sums
  for_resid_units<BN>(g, m, tn, own, n_own, pre,
                      [&](int u, int n, const float* h_old, const uint32_t* g8) {
                        if (!valid) return;
                        float v[16];
                        const __nv_bfloat16* src = c.ag[c.rank] + ag_off;
                        ld_bf16x8_cg(src + xoff(u, 0), v);
                        ld_bf16x8_cg(src + xoff(u, 1), v + 8);
                        ss += resid_update(g, m, n, dst, v, h_old, g8);
                      });
  return ss;
}

// The fused epilogue for this thread's row.  Work is divided in units (a
// 16-column chunk; a head for EPI_QKV); this CTA handles the units u with
// u % n_own == own (all units unless the tile is split over a cluster).
// EPI_RESID returns the row's sum of h^2 over the handled columns.
template <int BN, int EPI>
__device__ __forceinline__ float run_epilogue(const GemmArgs& g, const AccReader<BN>& acc, int tm,
                                              int tn, int row, int own, int n_own,
                                              const ResidPre& pre) {
  const int m = tm * BM + row;
  const bool valid = m < g.M;
  const float rs = row_scale(g, m);
  float ss = 0.f;

  if constexpr (EPI == EPI_F32 || EPI == EPI_BF16) {
    for (int u = own; u < BN / 16; u += n_own) {
      const int c = u * 16;
      const int n = tn * BN + c;
      if (n >= g.N) break;
      float v[16];
      acc.template load<16>(c, v);
      if (!valid) continue;
      if constexpr (EPI == EPI_F32) {
        float* o = reinterpret_cast<float*>(g.out) + (size_t)m * g.ld_out + n;
        if (n + 16 <= g.N) {
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(o + j) =
                make_float4(v[j] * rs, v[j + 1] * rs, v[j + 2] * rs, v[j + 3] * rs);
        } else {
          for (int j = 0; j < 16 && n + j < g.N; ++j) o[j] = v[j] * rs;
        }
      } else {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)m * g.ld_out + n;
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] *= rs;
        if (n + 16 <= g.N) {
          store_bf16x8(o, v);
          store_bf16x8(o + 8, v + 8);
        } else {
          for (int j = 0; j < 16 && n + j < g.N; ++j) o[j] = __float2bfloat16_rn(v[j]);
        }
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // Tile tn holds features [tn*BN/2, (tn+1)*BN/2): gate rows first, up rows second.
    constexpr int HALF = BN / 2;
    for (int u = own; u < HALF / 16; u += n_own) {
      const int c = u * 16;
      const int f = tn * HALF + c;
      if (f >= g.n_feat) break;
      float gv[16], uv[16];
      acc.template load<16>(c, gv);
      acc.template load<16>(HALF + c, uv);
      if (!valid) continue;
      float y[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float a = gv[j] * rs, b = uv[j] * rs;
        y[j] = a / (1.f + __expf(-a)) * b;
      }
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)m * g.ld_out + f;
      store_bf16x8(o, y);
      store_bf16x8(o + 8, y + 8);
    }
  } else if constexpr (EPI == EPI_RESID) {
    if (g.comm.world > 1) return run_resid_tp<BN>(g, acc, tm, tn, row, own, n_own, pre);
    const int dst = (valid && g.row_dst != nullptr) ? g.row_dst[m] : -1;
    for_resid_units<BN>(g, m, tn, own, n_own, pre,
                        [&](int u, int n, const float* h_old, const uint32_t* g8) {
                          float v[16];
                          acc.template load<16>(u * 16, v);
                          if (valid) ss += resid_update(g, m, n, dst, v, h_old, g8);
                        });
  } else if constexpr (EPI == EPI_QKV) {
    const int hd = g.head_dim, half = hd >> 1;
    const int heads_in_tile = BN / hd;
    const int total_heads = g.n_q_heads + 2 * g.n_kv_heads;
    int pos = 0, slot = 0;
    if (valid) {
      pos = g.positions[m];
      slot = g.slots[m];
      if (pos < 0 || pos >= g.max_pos || slot < 0) {
        set_status(ERR_BAD_INDEX);
        pos = 0;
        slot = -1;
      }
    }
    const int blk = slot >= 0 ? slot / g.block_size : 0;
    const int off = slot >= 0 ? slot % g.block_size : 0;
    for (int hh = own; hh < heads_in_tile; hh += n_own) {
      const int head = tn * heads_in_tile + hh;
      if (head >= total_heads) break;
      const int c0 = hh * hd;
      const int n0 = head * hd;
      __nv_bfloat16* dst;
      bool rotate = true;
      if (head < g.n_q_heads) {
        dst = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)m * g.ld_out + (size_t)head * hd;
      } else {
        const int is_v = head >= g.n_q_heads + g.n_kv_heads;
        const int kvh = head - g.n_q_heads - (is_v ? g.n_kv_heads : 0);
        rotate = !is_v;
        dst = g.kv_pool +
              ((((size_t)blk * 2 + is_v) * g.n_kv_heads + kvh) * g.block_size + off) * hd;
      }
      const bool store = valid && (slot >= 0 || head < g.n_q_heads);
      if (rotate) {
        for (int j = 0; j < half; j += 8) {
          float lo[8], hi[8], bl[8], bh[8];
          acc.template load<8>(c0 + j, lo);
          acc.template load<8>(c0 + half + j, hi);
          if (!store) continue;
          load_bf16x8(g.bias + n0 + j, bl);
          load_bf16x8(g.bias + n0 + half + j, bh);
          const float* cs = g.rope_cos + (size_t)pos * half + j;
          const float* sn = g.rope_sin + (size_t)pos * half + j;
          float ol[8], oh[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float x1 = lo[t] * rs + bl[t], x2 = hi[t] * rs + bh[t];
            const float c = cs[t], s = sn[t];
            ol[t] = x1 * c - x2 * s;
            oh[t] = x2 * c + x1 * s;
          }
          store_bf16x8(dst + j, ol);
          store_bf16x8(dst + half + j, oh);
        }
      } else {
        for (int j = 0; j < hd; j += 8) {
          float x[8], b[8];
          acc.template load<8>(c0 + j, x);
          if (!store) continue;
          load_bf16x8(g.bias + n0 + j, b);
#pragma unroll
          for (int t = 0; t < 8; ++t) x[t] = x[t] * rs + b[t];
          store_bf16x8(dst + j, x);
        }
      }
    }
  }
  return ss;
}

// Row sum of h^2 for the whole tile -> sq_out (and sq2 for gathered rows).
__device__ __forceinline__ void store_row_sumsq(const GemmArgs& g, int tm, int tn, int row,
                                                float ss) {
  const int m = tm * BM + row;
  if (m >= g.M) return;
  g.sq_out[(size_t)tn * g.sq_out_ld + m] = ss;
  if (g.row_dst != nullptr) {
    const int dst = g.row_dst[m];
    if (dst >= 0) g.sq2[(size_t)tn * g.sq2_ld + dst] = ss;
  }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a,
                   const __grid_constant__ CUtensorMap tma_b, const GemmArgs g) {
  using L = GemmLayout<BN, STAGES>;
  constexpr uint32_t TCOLS = tmem_cols(BN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + L::OFF_A;
  uint8_t* sB = smem + L::OFF_B;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* row_ss = reinterpret_cast<float*>(tmem_slot + 4);  // [BM] per-row partial sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mode = g.splits == 1 ? SPLIT_NONE : (g.ws != nullptr ? SPLIT_GLOBAL : SPLIT_CLUSTER);

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
  const int row = q * 32 + lane;
  AccReader<BN> acc;
  acc.taddr = tmem_base + ((uint32_t)(q * 32) << 16);
  acc.mode = mode;
  acc.splits = g.splits;
  acc.z = z;
  acc.row = row;
  acc.ws = nullptr;
  acc.red = smem_u32(smem);

  ResidPre pre;
  if (warp >= 2) {
    pdl_wait();   // the epilogue reads and writes buffers earlier kernels use
    if constexpr (EPI == EPI_RESID) {
      if (mode == SPLIT_CLUSTER) resid_prefetch<BN>(g, tm, tn, row, z, g.splits, pre);
      else resid_prefetch<BN>(g, tm, tn, row, 0, 1, pre);
    }
  }
  if (mode == SPLIT_CLUSTER) {
    // 1. park this CTA's fp32 partial over its (idle) stage ring as
    //    float4 [BN/4][BM]; every MMA and TMA write has completed once
    //    `done` fires, so the ring is free
    if (warp >= 2) {
      mbar_wait(done, 0);
      tc_fence_after();
      if (threadIdx.x == 64) trace_at(g, TR_ACC_READY);
      float4* red = reinterpret_cast<float4*>(smem);
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(acc.taddr + c, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          red[(c / 4 + i) * BM + row] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
      if (threadIdx.x == 64) trace_at(g, TR_PARKED);
    }
    cluster_sync_all();
    if (threadIdx.x == 64) trace_at(g, TR_CLUSTER_SYNC);
    // 2. reduce this CTA's share of the columns across the cluster and run
    //    the epilogue on it
    float ss = 0.f;
    if (warp >= 2) ss = run_epilogue<BN, EPI>(g, acc, tm, tn, row, z, g.splits, pre);
    if constexpr (EPI == EPI_RESID) {
      if (warp >= 2) row_ss[row] = ss;
    }
    if (threadIdx.x == 64) trace_at(g, TR_BODY);
    cluster_sync_all();
    // 3. rank 0 of the cluster combines the per-row sums of h^2
    if constexpr (EPI == EPI_RESID) {
      if (warp >= 2 && z == 0) {
        float tot = 0.f;
        const uint32_t a = smem_u32(row_ss + row);
        for (int s = 0; s < g.splits; ++s) tot += ld_cluster_f32(cluster_map(a, s));
        store_row_sumsq(g, tm, tn, row, tot);
      }
    }
    if (threadIdx.x == 64) trace_at(g, TR_COMBINED);
    cluster_sync_all();
    if (threadIdx.x == 64) trace_at(g, TR_END);
  } else if (warp >= 2) {
    mbar_wait(done, 0);
    tc_fence_after();
    if (threadIdx.x == 64) trace_at(g, TR_ACC_READY);
    bool run = true;
    if (mode == SPLIT_GLOBAL) {
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
      const float ss = run_epilogue<BN, EPI>(g, acc, tm, tn, row, 0, 1, pre);
      if constexpr (EPI == EPI_RESID) store_row_sumsq(g, tm, tn, row, ss);
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

// ------------------------------------------------------------------ host side

template <int BN, int STAGES, int EPI>
static int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb_, const GemmArgs& g,
                     cudaStream_t stream) {
  using L = GemmLayout<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    if (e != cudaSuccess) return host_err(e, "gemm smem attribute");
    attr_set = true;
  }
  const int tiles = g.tiles_m * g.tiles_n;
  if (g.splits > 1 && g.ws == nullptr)  // cluster split-K: a tile's splits are one cluster along x
    return launch_pdl(kern, dim3(tiles * g.splits), dim3(GEMM_THREADS), L::SMEM, stream,
                      g.splits, "gemm cluster launch", ta, tb_, g);
  return launch_pdl(kern, dim3(tiles, g.splits), dim3(GEMM_THREADS), L::SMEM, stream, 1,
                    "gemm launch", ta, tb_, g);
}

template <int EPI>
static int launch_epi(int bn, const CUtensorMap& ta, const CUtensorMap& tb_, const GemmArgs& g,
                      cudaStream_t stream) {
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
