// Tensor-parallel communicator: one device allocation per rank holding the
// all-reduce exchange buffers and the argmax candidate slots, shared with
// the other ranks of the node through CUDA IPC (peer-mapped over NVLink).
// The exchange itself happens inside the row-parallel GEMM epilogue
// (gemm.cu, run_resid_tp) and in tp_argmax_kernel below.  The buffers carry
// no flags: they hold the sentinel word until data lands (common.cuh).
#include <string.h>

#include "common.cuh"
#include "gemm.cuh"
#include "host.h"

namespace tb {

struct CommHost {
  int rank, world, max_rows, n_cols;
  char* base;           // this rank's allocation
  size_t bytes;
  char* peer[TB_MAX_RANKS];
  bool opened[TB_MAX_RANKS];
  size_t off_rs, off_ag, off_am;
  CommDev dev;
};

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Greedy sampling over a vocabulary-parallel LM head.  Row m of `logits`
// holds this rank's n_local vocabulary columns (global columns col0 ...).
// One CTA per row finds the shard's first maximum and stores the candidate
// (value bits, global index) as one 8-byte word into slot m of every rank's
// candidate plane for this call's parity; lane s then polls rank s's word in
// its own plane (bounded), puts the sentinel back, and the warp keeps the
// first maximum over the ranks in rank order.  Shards are ordered by rank,
// so this is the first maximum of the whole row: the index torch.argmax
// returns.  Every rank computes the same ids.  A candidate word is never the
// sentinel: its index half is below 2^31.
__global__ void __launch_bounds__(512) tp_argmax_kernel(const float* logits, int ld, int n_local,
                                                        int col0, int* out, CommDev c) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const int m = blockIdx.x;
  const bool vec = (ld % 4 == 0) && (reinterpret_cast<uintptr_t>(logits) % 16 == 0);
  float bv;
  int bi;
  row_argmax(logits + (size_t)m * ld, n_local, vec, bv, bi);
  auto slot = [&](int p, int src) {
    return c.am[p] + ((size_t)c.par * c.world + src) * c.max_rows + m;
  };
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32) {
    // row_argmax leaves the row's result in thread 0
    bv = __shfl_sync(0xffffffffu, bv, 0);
    bi = __shfl_sync(0xffffffffu, bi, 0);
    const unsigned long long cand =
        (unsigned long long)__float_as_uint(bv) |
        ((unsigned long long)(uint32_t)(bi == 0x7fffffff ? bi : bi + col0) << 32);
    if (lane < c.world) st_word(slot(lane, c.rank), cand);
    float v = -INFINITY;
    int idx = 0x7fffffff;
    if (lane < c.world) {
      unsigned long long w = ld_word(slot(c.rank, lane));
      uint64_t t0 = 0;
      for (uint32_t i = 0; w == TB_SENTINEL; ++i) {
        if ((i & 255u) == 0) {
          const uint64_t now = globaltimer_ns();
          if (t0 == 0) t0 = now;
          else if (now - t0 > PEER_BUDGET_NS) {
            set_status(ERR_PEER_TIMEOUT);
            break;
          }
        }
        w = ld_word(slot(c.rank, lane));
      }
      st_word(slot(c.rank, lane), TB_SENTINEL);
      if (w != TB_SENTINEL) {
        v = __uint_as_float((uint32_t)w);
        idx = (int)(uint32_t)(w >> 32);
      }
    }
    // first maximum over the ranks in rank order (lane order)
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, v, off);
      const int oi = __shfl_down_sync(0xffffffffu, idx, off);
      if (lane + off < 32) better(v, idx, ov, oi);
    }
    if (lane == 0) out[m] = idx == 0x7fffffff ? 0 : idx;
  }
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_comm_create(int rank, int world, int max_rows, int n_cols, void** comm_out,
                   void* ipc_handle_out) {
  if (comm_out == nullptr || ipc_handle_out == nullptr) return arg_err("null output pointer");
  if (world < 1 || world > TB_MAX_RANKS || rank < 0 || rank >= world)
    return arg_err("rank/world (world <= 8)");
  if (max_rows <= 0 || n_cols <= 0 || n_cols % (16 * world))
    return arg_err("n_cols must be a multiple of 16 * world; sizes positive");
  CommHost* c = new CommHost();
  memset(c, 0, sizeof(*c));
  c->rank = rank;
  c->world = world;
  c->max_rows = max_rows;
  c->n_cols = n_cols;
  // one exchange plane: every 128 x bn output tile of a max_rows x n_cols
  // result, laid out tile by tile (partial last tiles padded: bn <= 256)
  const size_t plane = (size_t)((max_rows + 127) / 128) * 128 * (size_t)(n_cols + 256) *
                       sizeof(__nv_bfloat16);
  c->off_rs = 0;
  c->off_ag = align256(c->off_rs + 2 * (size_t)world * plane);
  c->off_am = align256(c->off_ag + 2 * plane);
  c->bytes = align256(c->off_am + 2 * (size_t)world * max_rows * sizeof(unsigned long long));
  int rc = host_err(cudaMalloc(&c->base, c->bytes), "communicator allocation");
  if (rc) {
    delete c;
    return rc;
  }
  // every exchange word starts as the sentinel (all ones)
  rc = host_err(cudaMemset(c->base, 0xFF, c->bytes), "communicator clear");
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
  for (int p = 0; p < c->world; ++p) {
    d.rs[p] = reinterpret_cast<__nv_bfloat16*>(c->peer[p] + c->off_rs);
    d.ag[p] = reinterpret_cast<__nv_bfloat16*>(c->peer[p] + c->off_ag);
    d.am[p] = reinterpret_cast<unsigned long long*>(c->peer[p] + c->off_am);
  }
  return TB_OK;
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

static CommHost* opened(void* comm) {
  CommHost* c = static_cast<CommHost*>(comm);
  if (c == nullptr || c->dev.rs[0] == nullptr) {
    set_last_error("communicator not opened");
    return nullptr;
  }
  return c;
}

int tb_argmax_vocab_parallel(void* comm, const float* logits, int ld, int M, int n_local,
                             int col0, int* out, int seq, void* stream) {
  CommHost* c = opened(comm);
  if (c == nullptr) return TB_ERR_STATE;
  if (M < 0 || n_local < 0 || col0 < 0 || (n_local > 0 && ld < n_local) || out == nullptr)
    return arg_err("argmax shapes");
  if (M > c->max_rows) return arg_err("argmax rows above the communicator's max_rows");
  if (seq < 0) return arg_err("seq must be >= 0");
  if (M == 0) return TB_OK;
  CommDev d = c->dev;
  d.par = seq & 1;
  return launch_pdl(tp_argmax_kernel, dim3(M), dim3(512), 0, static_cast<cudaStream_t>(stream), 1,
                    "vocab-parallel argmax launch", logits, ld, n_local, col0, out, d);
}

int tb_row_linear_allreduce_residual(const void* x, int ldx, const void* w, int ldw, int M, int N,
                                     int K, float* h, int ld_h, const void* g_next, void* hg,
                                     int ld_hg, float* sq_out, int sq_out_ld, const int* row_dst,
                                     void* hg2, float* sq2, int sq2_ld, void* comm, int seq,
                                     int two_shot, unsigned long long* span_ns, int bn,
                                     int splits, void* stream) {
  CommHost* c = opened(comm);
  if (c == nullptr) return TB_ERR_STATE;
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256) return arg_err("bn must be 64/128/192/256");
  if (N != c->n_cols || M > c->max_rows || M <= 0) return arg_err("N != communicator n_cols or M > max_rows");
  if (seq < 0) return arg_err("seq must be >= 0");
  if (h == nullptr || g_next == nullptr || hg == nullptr || sq_out == nullptr)
    return arg_err("h / g_next / hg / sq_out");
  if (ld_h < N || ld_h % 4 || ld_hg < N || ld_hg % 8 || sq_out_ld < M)
    return arg_err("ld_h / ld_hg / sq_out_ld");
  if (row_dst != nullptr && (hg2 == nullptr || sq2 == nullptr)) return arg_err("row gather outputs");
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
  g.comm.par = seq & 1;
  g.comm.two_shot = two_shot ? 1 : 0;
  g.comm.span_ns = span_ns;
  if (c->world == 1) g.comm.world = 0;  // a single rank needs no exchange
  // split-K goes through the cluster (no scratch): every CTA reaches the epilogue
  return gemm_launch(EPI_RESID, bn, x, ldx, w, ldw, g, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
