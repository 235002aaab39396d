// extern "C" entry points (declared in include/tinybatch_b200.h).
#include "attention.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "host.h"

namespace tb {
extern unsigned long long* g_debug_trace;
const char* last_error();
int embed_launch(const int* ids, int M, const void* emb, int ld_emb, int d, int vocab,
                 const void* g, float* h, int ld_h, void* hg, int ld_hg, float* sq,
                 cudaStream_t st);
int argmax_launch(const float* logits, int ld, int M, int N, int* out, cudaStream_t st);
}  // namespace tb

using namespace tb;

namespace {

constexpr size_t ALIGN = 256;
inline size_t round_up(size_t x) { return (x + ALIGN - 1) / ALIGN * ALIGN; }

// Split-K scratch layout: a fixed region of per-tile arrival counters (kept
// at zero between calls) followed by the fp32 partial tiles.  The counter
// region never moves, so calls with different tile counts can share one
// arena without reading another call's partials as counters.
constexpr size_t COUNTER_TILES = 16384;
constexpr size_t COUNTER_BYTES = COUNTER_TILES * sizeof(int);

size_t tiles_of(int M, int N, int bn) {
  return (size_t)((M + 127) / 128) * (size_t)((N + bn - 1) / bn);
}

// Split the caller's scratch into (counters, partials) for a GEMM.
int gemm_scratch(GemmArgs& g, int bn, void* ws, size_t ws_bytes) {
  g.ws = nullptr;
  g.counters = nullptr;
  if (g.splits <= 1 || ws == nullptr) return TB_OK;  // no scratch: cluster split-K
  const size_t tiles = tiles_of(g.M, g.N, bn);
  if (tiles > COUNTER_TILES) return arg_err("split-K over more than 16384 tiles");
  const size_t need = COUNTER_BYTES + tiles * g.splits * bn * 128 * sizeof(float);
  if (ws == nullptr || ws_bytes < need) return arg_err("split-K scratch too small");
  if (reinterpret_cast<uintptr_t>(ws) % ALIGN) return arg_err("scratch must be 256-byte aligned");
  g.counters = static_cast<int*>(ws);
  g.ws = reinterpret_cast<float*>(static_cast<char*>(ws) + COUNTER_BYTES);
  return TB_OK;
}

GemmArgs base_args(int M, int N, int K, int splits, const float* sq, int sq_parts, int sq_ld,
                   float inv_d, float eps) {
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
  return g;
}

bool valid_bn(int bn) { return bn == 64 || bn == 128 || bn == 192 || bn == 256; }

}  // namespace

extern "C" {

int tb_version(void) { return 1; }

int tb_debug_trace(unsigned long long* buf) {
  g_debug_trace = buf;
  return TB_OK;
}

const char* tb_last_error(void) { return last_error(); }

int tb_status(unsigned int* code_h, int clear) {
  if (code_h == nullptr) return arg_err("code_h is NULL");
  int rc = host_err(cudaDeviceSynchronize(), "status sync");
  if (rc) return rc;
  rc = host_err(cudaMemcpyFromSymbol(code_h, g_status, sizeof(unsigned int)), "status read");
  if (rc || !clear) return rc;
  const unsigned int zero = 0;
  return host_err(cudaMemcpyToSymbol(g_status, &zero, sizeof(unsigned int)), "status clear");
}

int tb_gemm_max_active_clusters(int bn, int cluster, int* out_h) {
  if (out_h == nullptr || cluster < 1 || cluster > 8) return arg_err("cluster must be 1..8");
  return gemm_max_active_clusters(bn, cluster, out_h);
}

size_t tb_gemm_scratch_bytes(int M, int N, int bn, int splits) {
  if (splits <= 1) return 0;
  const size_t tiles = tiles_of(M, N, bn);
  return COUNTER_BYTES + tiles * splits * bn * 128 * sizeof(float);
}

int tb_linear(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
              const float* sq, int sq_parts, int sq_ld, float inv_d, float eps, void* out,
              int ld_out, int out_f32, int bn, int splits, void* ws, size_t ws_bytes,
              void* stream) {
  if (!valid_bn(bn)) return arg_err("bn must be 64, 128, 192 or 256");
  if (out == nullptr || ld_out < N || (out_f32 ? ld_out % 4 : ld_out % 8))
    return arg_err("out / ld_out");
  GemmArgs g = base_args(M, N, K, splits, sq, sq_parts, sq_ld, inv_d, eps);
  g.out = out;
  g.ld_out = ld_out;
  int rc = gemm_scratch(g, bn, ws, ws_bytes);
  if (rc) return rc;
  return gemm_launch(out_f32 ? EPI_F32 : EPI_BF16, bn, x, ldx, w, ldw, g,
                     static_cast<cudaStream_t>(stream));
}

int tb_qkv_rope_kv(const void* x, int ldx, const void* w_qkv, int ldw, const void* bias, int M,
                   int K, int n_q_heads, int n_kv_heads, int head_dim, const float* sq,
                   int sq_parts, int sq_ld, float inv_d, float eps, const float* rope_cos,
                   const float* rope_sin, int max_pos, const int* positions, const int* slots,
                   void* q_out, int ld_q, void* kv_pool, int block_size, int bn, int splits,
                   void* ws, size_t ws_bytes, void* stream) {
  if (!valid_bn(bn) || head_dim <= 0 || head_dim % 16 || bn % head_dim)
    return arg_err("bn must be 64/128/192/256 and a multiple of head_dim (multiple of 16)");
  if (bias == nullptr || rope_cos == nullptr || rope_sin == nullptr || positions == nullptr ||
      slots == nullptr || q_out == nullptr || kv_pool == nullptr)
    return arg_err("null pointer");
  if (ld_q < n_q_heads * head_dim || ld_q % 8 || block_size <= 0 || max_pos <= 0)
    return arg_err("ld_q / block_size / max_pos");
  if (reinterpret_cast<uintptr_t>(rope_cos) % 16 || reinterpret_cast<uintptr_t>(rope_sin) % 16)
    return arg_err("rope_cos / rope_sin must be 16-byte aligned");
  const int N = (n_q_heads + 2 * n_kv_heads) * head_dim;
  GemmArgs g = base_args(M, N, K, splits, sq, sq_parts, sq_ld, inv_d, eps);
  g.out = q_out;
  g.ld_out = ld_q;
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.rope_cos = rope_cos;
  g.rope_sin = rope_sin;
  g.positions = positions;
  g.slots = slots;
  g.kv_pool = static_cast<__nv_bfloat16*>(kv_pool);
  g.n_q_heads = n_q_heads;
  g.n_kv_heads = n_kv_heads;
  g.head_dim = head_dim;
  g.block_size = block_size;
  g.max_pos = max_pos;
  int rc = gemm_scratch(g, bn, ws, ws_bytes);
  if (rc) return rc;
  return gemm_launch(EPI_QKV, bn, x, ldx, w_qkv, ldw, g, static_cast<cudaStream_t>(stream));
}

int tb_gate_up_swiglu(const void* x, int ldx, const void* w_gu, int ldw, int M, int K,
                      int n_feat, const float* sq, int sq_parts, int sq_ld, float inv_d,
                      float eps, void* act, int ld_act, int bn, int splits, void* ws,
                      size_t ws_bytes, void* stream) {
  if (!valid_bn(bn)) return arg_err("bn must be 64, 128, 192 or 256");
  if (n_feat <= 0 || n_feat % 16 || ld_act < n_feat || ld_act % 8 || act == nullptr)
    return arg_err("n_feat must be a multiple of 16; act / ld_act");
  const int half = bn / 2;
  const int N = (n_feat + half - 1) / half * bn;  // interleaved, padded rows
  GemmArgs g = base_args(M, N, K, splits, sq, sq_parts, sq_ld, inv_d, eps);
  g.out = act;
  g.ld_out = ld_act;
  g.n_feat = n_feat;
  int rc = gemm_scratch(g, bn, ws, ws_bytes);
  if (rc) return rc;
  return gemm_launch(EPI_SWIGLU, bn, x, ldx, w_gu, ldw, g, static_cast<cudaStream_t>(stream));
}

int tb_row_linear_residual(const void* x, int ldx, const void* w, int ldw, int M, int N, int K,
                           float* h, int ld_h, const void* g_next, void* hg, int ld_hg,
                           float* sq_out, int sq_out_ld, const int* row_dst, void* hg2,
                           float* sq2, int sq2_ld, int bn, int splits, void* ws,
                           size_t ws_bytes, void* stream) {
  if (!valid_bn(bn)) return arg_err("bn must be 64, 128, 192 or 256");
  if (N % 16 || h == nullptr || g_next == nullptr || hg == nullptr || sq_out == nullptr)
    return arg_err("N must be a multiple of 16; h / g_next / hg / sq_out");
  if (ld_h < N || ld_h % 4 || ld_hg < N || ld_hg % 8 || sq_out_ld < M)
    return arg_err("ld_h / ld_hg / sq_out_ld");
  if (row_dst != nullptr && (hg2 == nullptr || sq2 == nullptr)) return arg_err("row gather outputs");
  GemmArgs g = base_args(M, N, K, splits, nullptr, 0, 0, 0.f, 0.f);
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
  int rc = gemm_scratch(g, bn, ws, ws_bytes);
  if (rc) return rc;
  return gemm_launch(EPI_RESID, bn, x, ldx, w, ldw, g, static_cast<cudaStream_t>(stream));
}

// Split-KV workspace: a fixed 64 KiB region of arrival counters (one int per
// (seq, kv head), at most ATTN_MAX_PAIRS pairs; zero between calls) first, so
// the counters sit at the same offsets whatever the call's size, then the
// per-split outputs and log-sum-exps.
constexpr size_t ATTN_COUNTER_BYTES = 64 << 10;
constexpr int ATTN_MAX_PAIRS = (int)(ATTN_COUNTER_BYTES / sizeof(int));

size_t tb_attention_scratch_bytes(int n_seqs, int n_kv_heads, int head_dim, int max_ctx,
                                  int split_tokens) {
  if (split_tokens <= 0 || max_ctx <= 0) return 0;
  const int chunks = (max_ctx + 15) / 16, per = split_tokens / 16;
  const int splits = per > 0 ? (chunks + per - 1) / per : 0;
  if (splits <= 1) return 0;
  const size_t rows = (size_t)n_seqs * n_kv_heads * splits * 16;
  return ATTN_COUNTER_BYTES + round_up(rows * head_dim * sizeof(float)) +
         round_up(rows * sizeof(float));
}

int tb_paged_attention_decode(const void* q, int ld_q, void* out, int ld_out,
                              const void* kv_pool, int num_blocks, int n_q_heads,
                              int n_kv_heads, int head_dim, int block_size,
                              const int* block_tables, int bt_ld, const int* q_start,
                              const int* q_len, const int* ctx_len, const int* seq_order,
                              int n_seqs, int max_ctx, int split_tokens, void* ws,
                              size_t ws_bytes, void* stream) {
  if (split_tokens <= 0 || split_tokens % 16 || max_ctx <= 0) return arg_err("split_tokens / max_ctx");
  AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.ld_q = ld_q;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ld_out = ld_out;
  a.pool = static_cast<const __nv_bfloat16*>(kv_pool);
  a.num_blocks = num_blocks;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.block_size = block_size;
  a.block_tables = block_tables;
  a.bt_ld = bt_ld;
  a.q_start = q_start;
  a.q_len = q_len;
  a.ctx_len = ctx_len;
  a.seq_order = seq_order;
  a.n_seqs = n_seqs;
  a.split_chunks = split_tokens / 16;
  a.max_splits = ((max_ctx + 15) / 16 + a.split_chunks - 1) / a.split_chunks;
  if (a.max_splits > 1) {
    const size_t need = tb_attention_scratch_bytes(n_seqs, n_kv_heads, head_dim, max_ctx, split_tokens);
    if (ws == nullptr || ws_bytes < need) return arg_err("attention scratch too small");
    if (reinterpret_cast<uintptr_t>(ws) % ALIGN) return arg_err("scratch must be 256-byte aligned");
    if ((long long)n_seqs * n_kv_heads > ATTN_MAX_PAIRS)
      return arg_err("split-KV decode supports at most 16384 (sequence, kv head) pairs");
    const size_t rows = (size_t)n_seqs * n_kv_heads * a.max_splits * 16;
    char* base = static_cast<char*>(ws);
    a.ws_count = reinterpret_cast<int*>(base);
    a.ws_o = reinterpret_cast<float*>(base + ATTN_COUNTER_BYTES);
    a.ws_lse = reinterpret_cast<float*>(base + ATTN_COUNTER_BYTES +
                                        round_up(rows * head_dim * sizeof(float)));
  }
  return attn_decode(a, head_dim, static_cast<cudaStream_t>(stream));
}

int tb_paged_attention_prefill(const void* q, int ld_q, void* out, int ld_out,
                               const void* kv_pool, int num_blocks, int n_q_heads,
                               int n_kv_heads, int head_dim, int block_size,
                               const int* block_tables, int bt_ld, const int* q_start,
                               const int* q_len, const int* ctx_len, int n_seqs,
                               const int* work_pairs, int n_work, void* stream) {
  AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.ld_q = ld_q;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ld_out = ld_out;
  a.pool = static_cast<const __nv_bfloat16*>(kv_pool);
  a.num_blocks = num_blocks;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.block_size = block_size;
  a.block_tables = block_tables;
  a.bt_ld = bt_ld;
  a.q_start = q_start;
  a.q_len = q_len;
  a.ctx_len = ctx_len;
  a.n_seqs = n_seqs;
  a.work = work_pairs;
  if (n_work > 0 && work_pairs == nullptr) return arg_err("work_pairs");
  return attn_prefill(a, head_dim, n_work, static_cast<cudaStream_t>(stream));
}

int tb_embed(const int* ids, int M, const void* emb, int ld_emb, int d, int vocab, const void* g,
             float* h, int ld_h, void* hg, int ld_hg, float* sq, void* stream) {
  return embed_launch(ids, M, emb, ld_emb, d, vocab, g, h, ld_h, hg, ld_hg, sq,
                      static_cast<cudaStream_t>(stream));
}

int tb_argmax(const float* logits, int ld, int M, int N, int* out, void* stream) {
  return argmax_launch(logits, ld, M, N, out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
