// Embedding gather (+ first-norm prologue) and greedy argmax.
#include "common.cuh"
#include "host.h"

namespace tb {

// One CTA per token row: h = emb[id] (fp32), hg = bf16(h * g), sq = sum h^2.
__global__ void __launch_bounds__(128) embed_kernel(const int* ids, const __nv_bfloat16* emb,
                                                    int ld_emb, int d, int vocab,
                                                    const __nv_bfloat16* g, float* h, int ld_h,
                                                    __nv_bfloat16* hg, int ld_hg, float* sq) {
  __shared__ float red[4];
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const int m = blockIdx.x;
  int id = ids[m];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_status(ERR_BAD_INDEX);
    id = 0;
  }
  const __nv_bfloat16* src = emb + (size_t)id * ld_emb;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
    float v[8], gw[8], o[8];
    load_bf16x8(src + c, v);
    load_bf16x8(g + c, gw);
    float* hp = h + (size_t)m * ld_h + c;
    *reinterpret_cast<float4*>(hp) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(hp + 4) = make_float4(v[4], v[5], v[6], v[7]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ss += v[j] * v[j];
      o[j] = v[j] * gw[j];
    }
    store_bf16x8(hg + (size_t)m * ld_hg + c, o);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) sq[m] = red[0] + red[1] + red[2] + red[3];
}

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// First maximum of row[0, N) over the calling CTA (blockDim.x a multiple of
// 32, at most 512; every thread calls it).  Thread 0 returns the row's
// largest value and its smallest index (torch.argmax semantics); the index
// is 0x7fffffff when no element compares greater than -inf.  `vec`: the row
// may be read as float4 (16-byte aligned row start).
__device__ __forceinline__ void row_argmax(const float* row, int N, bool vec, float& bv, int& bi) {
  __shared__ float sv[16];
  __shared__ int si[16];
  bv = -INFINITY;
  bi = 0x7fffffff;
  if (vec) {
    const int n4 = N / 4;
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int stride = blockDim.x;
    int i = threadIdx.x;
    // eight loads in flight per thread (64 KiB per CTA: one CTA per row has
    // to pull its row at ~1/128 of the HBM bandwidth), then the comparisons
    for (; i + 7 * stride < n4; i += 8 * stride) {
      float4 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __ldcs(r4 + i + k * stride);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int b = 4 * (i + k * stride);
        better(bv, bi, v[k].x, b);
        better(bv, bi, v[k].y, b + 1);
        better(bv, bi, v[k].z, b + 2);
        better(bv, bi, v[k].w, b + 3);
      }
    }
    for (; i < n4; i += stride) {
      const float4 v = r4[i];
      better(bv, bi, v.x, 4 * i);
      better(bv, bi, v.y, 4 * i + 1);
      better(bv, bi, v.z, 4 * i + 2);
      better(bv, bi, v.w, 4 * i + 3);
    }
    for (int j = 4 * n4 + threadIdx.x; j < N; j += blockDim.x) better(bv, bi, row[j], j);
  } else {
    for (int i = threadIdx.x; i < N; i += blockDim.x) better(bv, bi, row[i], i);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, bv, o);
    const int i = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, v, i);
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    bv = sv[0];
    bi = si[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) better(bv, bi, sv[w], si[w]);
  }
}

// One CTA per row; ties go to the smallest index (torch.argmax semantics).
__global__ void __launch_bounds__(512) argmax_kernel(const float* logits, int ld, int N, int* out) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const bool vec = (ld % 4 == 0) && (reinterpret_cast<uintptr_t>(logits) % 16 == 0);
  float bv;
  int bi;
  row_argmax(logits + (size_t)blockIdx.x * ld, N, vec, bv, bi);
  if (threadIdx.x == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
}

int embed_launch(const int* ids, int M, const void* emb, int ld_emb, int d, int vocab,
                 const void* g, float* h, int ld_h, void* hg, int ld_hg, float* sq,
                 cudaStream_t st) {
  if (M < 0 || d <= 0 || d % 8 || ld_emb % 8 || ld_h % 4 || ld_hg % 8) return arg_err("embed shapes");
  if (M == 0) return TB_OK;
  return launch_pdl(embed_kernel, dim3(M), dim3(128), 0, st, 1, "embed launch", ids,
                    (const __nv_bfloat16*)emb, ld_emb, d, vocab, (const __nv_bfloat16*)g, h, ld_h,
                    (__nv_bfloat16*)hg, ld_hg, sq);
}

int argmax_launch(const float* logits, int ld, int M, int N, int* out, cudaStream_t st) {
  if (M < 0 || N <= 0 || ld < N) return arg_err("argmax shapes");
  if (M == 0) return TB_OK;
  return launch_pdl(argmax_kernel, dim3(M), dim3(512), 0, st, 1, "argmax launch", logits, ld, N,
                    out);
}

}  // namespace tb
