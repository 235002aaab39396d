// tb_linear_static_scratch: the split-K projection of tb_linear for callers
// that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- inside a
// custom allocator's own callbacks, in a process whose device memory is
// entirely pre-reserved by another framework's pool, or in a host that may
// not call allocation APIs after start-up.  Such a caller still owns its
// inputs and outputs but has no place to put the split-K partial tiles, so
// this variant keeps them in a fixed array that lives in the library itself.
//
// The array is a file-scope __device__ object: every GPU that loads the
// library carries TB_STATIC_SCRATCH_BYTES of it until the process exits.
// Host code cannot use the array's name as a device address (on the host it
// names a shadow object), so the first call on each device, with that
// device current, asks the runtime for the real address with
// cudaGetSymbolAddress and caches it.  Make that first call before any
// stream capture.  The cache remembers the context it was resolved in: after
// a device reset (a new primary context) the next call resolves it again.
//
// All calls on a device share the array and it keeps whatever the last call
// left there.  The arrival counters at its head must start at zero, so each
// call clears the counters it uses (cudaMemsetAsync on the call's stream).
// Two calls that can run at the same time on one device -- different
// streams without ordering between them -- race on the array and may
// corrupt each other's results.
#include <mutex>

#include "gemm.cuh"
#include "host.h"

namespace tb {

// Counter region: one int per output tile (at most 1024 tiles), then the
// fp32 partial tiles.
constexpr size_t STATIC_COUNTER_TILES = 1024;
constexpr size_t STATIC_COUNTER_BYTES = STATIC_COUNTER_TILES * sizeof(int);
static_assert(TB_STATIC_SCRATCH_BYTES > STATIC_COUNTER_BYTES, "scratch too small");

static __device__ __align__(256) unsigned char g_static_scratch[TB_STATIC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
static void* g_static_ptr[MAX_DEVICES] = {};
static unsigned long long g_static_ctx[MAX_DEVICES] = {};
static std::mutex g_static_mu;

// Device address of g_static_scratch on the current device (resolved once
// per device and context).
static int static_scratch_ptr(void** out) {
  int dev = -1;
  int rc = host_err(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= MAX_DEVICES) return arg_err("device index beyond 64");
  unsigned long long ctx = 0;
  if (current_context_id(&ctx) != TB_OK) {
    // no context current on this thread yet: make the device's primary one current
    rc = host_err(cudaSetDevice(dev), "cudaSetDevice");
    if (!rc) rc = current_context_id(&ctx);
    if (rc) return rc;
  }
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_ptr[dev] == nullptr || g_static_ctx[dev] != ctx) {
    void* p = nullptr;
    rc = host_err(cudaGetSymbolAddress(&p, g_static_scratch), "cudaGetSymbolAddress(scratch)");
    if (rc) return rc;
    g_static_ptr[dev] = p;
    g_static_ctx[dev] = ctx;
  }
  *out = g_static_ptr[dev];
  return TB_OK;
}

}  // namespace tb

extern "C" int tb_linear_static_scratch(const void* x, int ldx, const void* w, int ldw, int M,
                                        int N, int K, const float* sq, int sq_parts, int sq_ld,
                                        float inv_d, float eps, void* out, int ld_out,
                                        int out_f32, int bn, int splits, void* stream) {
  using namespace tb;
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256)
    return arg_err("bn must be 64, 128, 192 or 256");
  if (out == nullptr || ld_out < N || (out_f32 ? ld_out % 4 : ld_out % 8))
    return arg_err("out / ld_out");
  if (M <= 0 || N <= 0 || splits < 1) return arg_err("M, N > 0 and splits >= 1 required");
  GemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.splits = splits;
  g.group_m = 16;
  g.sq = sq;
  g.sq_parts = sq_parts;
  g.sq_ld = sq_ld;
  g.inv_d = inv_d;
  g.eps = eps;
  g.out = out;
  g.ld_out = ld_out;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (splits > 1) {
    const size_t tiles = (size_t)((M + 127) / 128) * (size_t)((N + bn - 1) / bn);
    const size_t need = STATIC_COUNTER_BYTES + tiles * splits * bn * 128 * sizeof(float);
    if (tiles > STATIC_COUNTER_TILES || need > TB_STATIC_SCRATCH_BYTES) {
      set_last_error(
          "tb_linear_static_scratch: needs %zu bytes of split-K scratch (%zu tiles x %d "
          "splits); the built-in array holds %zu bytes and 1024 tiles -- use fewer splits "
          "or tb_linear with caller-owned scratch",
          need, tiles, splits, (size_t)TB_STATIC_SCRATCH_BYTES);
      return TB_ERR_ARG;
    }
    void* base = nullptr;
    int rc = static_scratch_ptr(&base);
    if (rc) return rc;
    rc = host_err(cudaMemsetAsync(base, 0, tiles * sizeof(int), st), "clear split-K counters");
    if (rc) return rc;
    g.counters = static_cast<int*>(base);
    g.ws = reinterpret_cast<float*>(static_cast<char*>(base) + STATIC_COUNTER_BYTES);
  }
  return gemm_launch(out_f32 ? EPI_F32 : EPI_BF16, bn, x, ldx, w, ldw, g, st);
}
