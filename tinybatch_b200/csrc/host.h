// Host-side helpers shared by the launchers: error reporting and TMA
// descriptor encoding (through the driver entry point, so the library does
// not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include "../../include/tinybatch_b200.h"

namespace tb {

// Record a failed CUDA call (message readable through tb_last_error) and
// return TB_ERR_CUDA; returns TB_OK for cudaSuccess.
int host_err(cudaError_t e, const char* what);
int arg_err(const char* what);
void set_last_error(const char* fmt, ...);

// Unique id of the calling thread's current CUDA context (changes when a
// device's primary context is reset and created again).
int current_context_id(unsigned long long* id);

// 2-D bf16 tensor map over a row-major [rows, inner] matrix with the given
// row pitch, box {box_inner, box_rows}, 128-byte swizzle (or none, for maps
// only used to prefetch), zero OOB fill.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                 uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_rows,
                 bool swizzle = true);

// Launch `kern` on `stream` with programmatic stream serialisation (PDL) and,
// when cluster_x > 1, a (cluster_x, 1, 1) thread-block cluster.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               int cluster_x, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return host_err(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what);
}

// Kernel attributes are per device: `devs` (one static per kernel at the
// call site) records, one bit per device index, where `kern`'s dynamic
// shared-memory limit (and, with max_carveout, its shared-memory carveout)
// has been set.  Concurrent first calls may both set it, which is harmless.
template <typename... KArgs>
int smem_attr_once(void (*kern)(KArgs...), int bytes, std::atomic<unsigned long long>& devs,
                   const char* what, bool max_carveout = false) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return host_err(e, what);
  const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
  if (bit && (devs.load(std::memory_order_acquire) & bit)) return 0;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && max_carveout)
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return host_err(e, what);
  devs.fetch_or(bit, std::memory_order_release);
  return 0;
}

struct GemmArgs;
int gemm_launch(int epi, int bn, const void* A, int lda, const void* B, int ldb, GemmArgs g,
                cudaStream_t stream);
int gemm_max_active_clusters(int bn, int cluster, int* out);

}  // namespace tb
