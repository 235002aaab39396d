// Host-side helpers shared by the launchers: error reporting and TMA
// descriptor encoding (through the driver entry point, so the library does
// not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/tinybatch_b200.h"

namespace tb {

// Record a failed CUDA call (message readable through tb_last_error) and
// return TB_ERR_CUDA; returns TB_OK for cudaSuccess.
int host_err(cudaError_t e, const char* what);
int arg_err(const char* what);
void set_last_error(const char* fmt, ...);

// 2-D bf16 tensor map over a row-major [rows, inner] matrix with the given
// row pitch, box {box_inner, box_rows}, 128-byte swizzle, zero OOB fill.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                 uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_rows);

struct GemmArgs;
int gemm_launch(int epi, int bn, const void* A, int lda, const void* B, int ldb, GemmArgs g,
                cudaStream_t stream);
size_t gemm_workspace_bytes(int M, int N, int bn, int splits);

}  // namespace tb
