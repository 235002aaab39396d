// Tensor-parallel communicator: one device allocation per rank holding the
// all-reduce exchange buffers, the delivery flags and a step counter, shared
// with the other ranks of the node through CUDA IPC (peer-mapped over
// NVLink).  The exchange itself happens inside the row-parallel GEMM
// epilogue (gemm.cu, run_resid_tp); nothing here runs per call except the
// one-thread step-counter kernel.
#include <string.h>

#include "common.cuh"
#include "gemm.cuh"
#include "host.h"

namespace tb {

struct CommHost {
  int rank, world, max_rows, n_cols, max_ctas;
  char* base;           // this rank's allocation
  size_t bytes;
  char* peer[TB_MAX_RANKS];
  bool opened[TB_MAX_RANKS];
  size_t off_rs, off_ag, off_flags, off_state;
  CommDev dev;
};

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Advance the step counter once per forward (every rank, same order), after
// the previous kernel: the last row-parallel GEMM of the previous forward
// has read the old value by then.
__global__ void comm_step_kernel(uint32_t* state) {
  pdl_wait();
  pdl_trigger();
  state[0] += 1u;
}

// Greedy sampling over a vocabulary-parallel LM head.  Row m of `logits`
// holds this rank's n_local vocabulary columns (global columns col0 ...).
// One CTA per row finds the shard's first maximum, stores (value, global
// index) into slot m of every rank's exchange region for this call's epoch
// (plane [parity][source rank]), raises its flag on every rank (lane p
// release-stores to rank p, lane s acquire-polls rank s, bounded), then keeps
// the first maximum over the ranks' candidates in rank order.  Shards are
// ordered by rank, so this is the first maximum of the whole row: the index
// torch.argmax returns.  Every rank computes the same ids.
__global__ void __launch_bounds__(512) tp_argmax_kernel(const float* logits, int ld, int n_local,
                                                        int col0, int* out, CommDev c) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const int m = blockIdx.x;
  const bool vec = (ld % 4 == 0) && (reinterpret_cast<uintptr_t>(logits) % 16 == 0);
  float bv;
  int bi;
  row_argmax(logits + (size_t)m * ld, n_local, vec, bv, bi);
  const uint32_t epoch = c.state[0] * (uint32_t)c.n_sites + (uint32_t)c.site + 1u;
  const int par = (int)(epoch & 1u);
  const size_t plane = (size_t)((c.max_rows + 127) / 128) * 128 * (size_t)(c.n_cols + 256);
  auto slot = [&](int p, int src) {
    return reinterpret_cast<uint2*>(c.rs[p] + ((size_t)par * c.world + src) * plane) + m;
  };
  auto flag_at = [&](int p, int src) {
    return c.flags[p] + ((size_t)(par * c.world + src)) * c.max_ctas + m;
  };
  if (threadIdx.x == 0) {
    const uint2 cand = make_uint2(__float_as_uint(bv),
                                  (uint32_t)(bi == 0x7fffffff ? bi : bi + col0));
    for (int p = 0; p < c.world; ++p) *slot(p, c.rank) = cand;
  }
  __syncthreads();   // the candidate stores precede every lane's release
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32 && lane < c.world) {
    st_release_sys(flag_at(lane, c.rank), epoch);
    wait_flag_sys(flag_at(c.rank, lane), epoch);
  }
  __syncthreads();   // every rank's candidate visible to thread 0
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int s = 0; s < c.world; ++s) {
      const uint2 cs = *slot(c.rank, s);
      better(v, idx, __uint_as_float(cs.x), (int)cs.y);
    }
    out[m] = idx == 0x7fffffff ? 0 : idx;
  }
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_comm_create(int rank, int world, int max_rows, int n_cols, int max_ctas, void** comm_out,
                   void* ipc_handle_out) {
  if (comm_out == nullptr || ipc_handle_out == nullptr) return arg_err("null output pointer");
  if (world < 1 || world > TB_MAX_RANKS || rank < 0 || rank >= world)
    return arg_err("rank/world (world <= 8)");
  if (max_rows <= 0 || n_cols <= 0 || n_cols % (16 * world) || max_ctas <= 0)
    return arg_err("n_cols must be a multiple of 16 * world; sizes positive");
  CommHost* c = new CommHost();
  memset(c, 0, sizeof(*c));
  c->rank = rank;
  c->world = world;
  c->max_rows = max_rows;
  c->n_cols = n_cols;
  c->max_ctas = max_ctas;
  // one exchange plane: every 128 x bn output tile of a max_rows x n_cols
  // result, laid out tile by tile (partial last tiles padded: bn <= 256)
  const size_t plane = (size_t)((max_rows + 127) / 128) * 128 * (size_t)(n_cols + 256) *
                       sizeof(__nv_bfloat16);
  c->off_rs = 0;
  c->off_ag = align256(c->off_rs + 2 * (size_t)world * plane);
  c->off_flags = align256(c->off_ag + 2 * plane);
  c->off_state = align256(c->off_flags + 4 * (size_t)world * max_ctas * sizeof(uint32_t));
  c->bytes = c->off_state + 256;
  int rc = host_err(cudaMalloc(&c->base, c->bytes), "communicator allocation");
  if (rc) {
    delete c;
    return rc;
  }
  rc = host_err(cudaMemset(c->base, 0, c->bytes), "communicator clear");
  if (!rc) rc = host_err(cudaDeviceSynchronize(), "communicator clear");
  if (!rc)
    rc = host_err(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle_out), c->base),
                  "cudaIpcGetMemHandle");
  if (rc) {
    cudaFree(c->base);
    delete c;
    return rc;
  }
  c->peer[rank] = c->base;
  c->opened[rank] = true;
  *comm_out = c;
  return TB_OK;
}

int tb_comm_open(void* comm, const void* ipc_handles) {
  CommHost* c = static_cast<CommHost*>(comm);
  if (c == nullptr || ipc_handles == nullptr) return arg_err("null communicator or handles");
  const cudaIpcMemHandle_t* hs = static_cast<const cudaIpcMemHandle_t*>(ipc_handles);
  for (int p = 0; p < c->world; ++p) {
    if (c->opened[p]) continue;
    void* ptr = nullptr;
    int rc = host_err(cudaIpcOpenMemHandle(&ptr, hs[p], cudaIpcMemLazyEnablePeerAccess),
                      "cudaIpcOpenMemHandle");
    if (rc) return rc;
    c->peer[p] = static_cast<char*>(ptr);
    c->opened[p] = true;
  }
  CommDev& d = c->dev;
  d.rank = c->rank;
  d.world = c->world;
  d.max_rows = c->max_rows;
  d.n_cols = c->n_cols;
  d.max_ctas = c->max_ctas;
  d.state = reinterpret_cast<uint32_t*>(c->base + c->off_state);
  for (int p = 0; p < c->world; ++p) {
    d.rs[p] = reinterpret_cast<__nv_bfloat16*>(c->peer[p] + c->off_rs);
    d.ag[p] = reinterpret_cast<__nv_bfloat16*>(c->peer[p] + c->off_ag);
    d.flags[p] = reinterpret_cast<uint32_t*>(c->peer[p] + c->off_flags);
  }
  return TB_OK;
}

int tb_comm_begin_step(void* comm, void* stream) {
  CommHost* c = static_cast<CommHost*>(comm);
  if (c == nullptr || c->dev.state == nullptr) {
    set_last_error("communicator not opened");
    return TB_ERR_STATE;
  }
  return launch_pdl(comm_step_kernel, dim3(1), dim3(1), 0, static_cast<cudaStream_t>(stream), 1,
                    "communicator step launch", c->dev.state);
}

int tb_comm_destroy(void* comm) {
  CommHost* c = static_cast<CommHost*>(comm);
  if (c == nullptr) return TB_OK;
  int rc = TB_OK;
  for (int p = 0; p < c->world; ++p) {
    if (p != c->rank && c->opened[p]) {
      int r = host_err(cudaIpcCloseMemHandle(c->peer[p]), "cudaIpcCloseMemHandle");
      if (r && !rc) rc = r;
    }
  }
  int r = host_err(cudaFree(c->base), "communicator free");
  if (r && !rc) rc = r;
  delete c;
  return rc;
}

int tb_argmax_vocab_parallel(void* comm, const float* logits, int ld, int M, int n_local,
                             int col0, int* out, int site, int n_sites, void* stream) {
  CommHost* c = static_cast<CommHost*>(comm);
  if (c == nullptr || c->dev.state == nullptr) {
    set_last_error("communicator not opened");
    return TB_ERR_STATE;
  }
  if (M < 0 || n_local < 0 || col0 < 0 || (n_local > 0 && ld < n_local) || out == nullptr)
    return arg_err("argmax shapes");
  if (M > c->max_rows || M > c->max_ctas)
    return arg_err("argmax rows above the communicator's max_rows / max_ctas");
  if (site < 0 || site >= n_sites) return arg_err("site must be in [0, n_sites)");
  if (M == 0) return TB_OK;
  CommDev d = c->dev;
  d.site = site;
  d.n_sites = n_sites;
  return launch_pdl(tp_argmax_kernel, dim3(M), dim3(512), 0, static_cast<cudaStream_t>(stream), 1,
                    "vocab-parallel argmax launch", logits, ld, n_local, col0, out, d);
}

int tb_row_linear_allreduce_residual(const void* x, int ldx, const void* w, int ldw, int M, int N,
                                     int K, float* h, int ld_h, const void* g_next, void* hg,
                                     int ld_hg, float* sq_out, int sq_out_ld, const int* row_dst,
                                     void* hg2, float* sq2, int sq2_ld, void* comm, int site,
                                     int n_sites, int two_shot, int bn, int splits,
                                     const tb_l2_prefetch* next, void* stream) {
  CommHost* c = static_cast<CommHost*>(comm);
  if (c == nullptr || c->dev.state == nullptr) {
    set_last_error("communicator not opened");
    return TB_ERR_STATE;
  }
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256) return arg_err("bn must be 64/128/192/256");
  if (N != c->n_cols || M > c->max_rows || M <= 0) return arg_err("N != communicator n_cols or M > max_rows");
  if (site < 0 || site >= n_sites) return arg_err("site must be in [0, n_sites)");
  if (h == nullptr || g_next == nullptr || hg == nullptr || sq_out == nullptr)
    return arg_err("h / g_next / hg / sq_out");
  if (ld_h < N || ld_h % 4 || ld_hg < N || ld_hg % 8 || sq_out_ld < M)
    return arg_err("ld_h / ld_hg / sq_out_ld");
  if (row_dst != nullptr && (hg2 == nullptr || sq2 == nullptr)) return arg_err("row gather outputs");
  const size_t ctas = (size_t)((M + 127) / 128) * ((N + bn - 1) / bn) * (splits > 1 ? splits : 1);
  if (ctas > (size_t)c->max_ctas) return arg_err("more CTAs than the communicator has flags for");
  GemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.splits = splits;
  g.group_m = 16;
  g.h = h;
  g.ld_h = ld_h;
  g.gnext = static_cast<const __nv_bfloat16*>(g_next);
  g.hg = static_cast<__nv_bfloat16*>(hg);
  g.ld_hg = ld_hg;
  g.sq_out = sq_out;
  g.sq_out_ld = sq_out_ld;
  g.row_dst = row_dst;
  g.hg2 = static_cast<__nv_bfloat16*>(hg2);
  g.sq2 = sq2;
  g.sq2_ld = sq2_ld;
  g.comm = c->dev;
  g.comm.site = site;
  g.comm.n_sites = n_sites;
  g.comm.two_shot = two_shot ? 1 : 0;
  if (c->world == 1) g.comm.world = 0;  // a single rank needs no exchange
  int rc = gemm_set_prefetch(g, next);
  if (rc) return rc;
  // split-K goes through the cluster (no scratch): every CTA reaches the epilogue
  return gemm_launch(EPI_RESID, bn, x, ldx, w, ldw, g, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
