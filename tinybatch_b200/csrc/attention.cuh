// Argument block of the paged attention kernels (attention.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace tb {

struct AttnArgs {
  const __nv_bfloat16* q;
  int ld_q;
  __nv_bfloat16* out;
  int ld_out;
  const __nv_bfloat16* pool;
  int num_blocks, n_q_heads, n_kv_heads, block_size;
  const int* block_tables;  // [n_seqs, bt_ld]
  int bt_ld;
  const int* q_start;       // [n_seqs] first row of the sequence in q / out
  const int* q_len;         // [n_seqs]
  const int* ctx_len;       // [n_seqs]
  const int* seq_order;     // decode: [n_seqs] dispatch order of the sequences, or null
  int n_seqs;
  float scale_log2;         // log2(e) / sqrt(head_dim)
  // decode splits
  int split_chunks;         // 16-token chunks per split
  int max_splits;
  float* ws_o;              // [n_seqs, n_kv, max_splits, 16, hd]
  float* ws_lse;            // [n_seqs, n_kv, max_splits, 16]
  int* ws_count;            // [n_seqs, n_kv] split arrivals; zero between calls
  // prefill work list: pairs (seq, row tile)
  const int* work;
  // debug timeline (tb_debug_trace) of the tcgen05 prefill: per CTA 16
  // globaltimer stamps (PT_TR_*), or null
  unsigned long long* trace;
};

int attn_decode(AttnArgs a, int head_dim, cudaStream_t st);
int attn_prefill(AttnArgs a, int head_dim, int n_work, cudaStream_t st);

}  // namespace tb
