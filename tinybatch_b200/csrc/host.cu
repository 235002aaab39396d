// Host helpers: per-thread error message, driver entry point for
// cuTensorMapEncodeTiled, 2-D tensor-map construction.
#include <stdarg.h>
#include <stdio.h>

#include "host.h"

namespace tb {

static thread_local char g_msg[512] = "";

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_msg; }

int host_err(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TB_OK;
  set_last_error("%s: %s", what, cudaGetErrorString(e));
  return TB_ERR_CUDA;
}

int arg_err(const char* what) {
  set_last_error("invalid argument: %s", what);
  return TB_ERR_ARG;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

int current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  if (get_cur == nullptr || get_id == nullptr) {
    void* p = nullptr;
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r1, r2;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r1) != cudaSuccess ||
        r1 != cudaDriverEntryPointSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &q, cudaEnableDefault, &r2) != cudaSuccess ||
        r2 != cudaDriverEntryPointSuccess) {
      set_last_error("cuCtxGetCurrent / cuCtxGetId entry points unavailable");
      return TB_ERR_CUDA;
    }
    get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
    get_id = reinterpret_cast<CtxGetIdFn>(q);
  }
  CUcontext ctx = nullptr;
  if (get_cur(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, id) != CUDA_SUCCESS) {
    set_last_error("no current CUDA context");
    return TB_ERR_CUDA;
  }
  return TB_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                 uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_rows,
                 bool swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_last_error("cuTensorMapEncodeTiled entry point unavailable");
    return TB_ERR_CUDA;
  }
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d): inner=%llu rows=%llu pitch=%llu box=%ux%u",
                   (int)r, (unsigned long long)inner, (unsigned long long)rows,
                   (unsigned long long)row_pitch_bytes, box_inner, box_rows);
    return TB_ERR_CUDA;
  }
  return TB_OK;
}

}  // namespace tb
