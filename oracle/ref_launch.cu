// Host launch wrappers around the reference's own kernels (TEST INFRASTRUCTURE).
//
// oracle/build_ref.py extracts the kernel source strings of the reference's
// src/gpu/kernels.rs into oracle/_ref/ref_kernels.cu and compiles this file,
// which includes them, into oracle/_ref/libqtts_ref.so. Each wrapper launches
// one reference kernel on the legacy default stream with the grid, block and
// dynamic shared memory the reference's Rust launcher uses (cited per
// function); pointers are device pointers. Returns the launch's cudaError_t.
// Only tests call this library, to pin the oracle restatement to outputs of
// the reference's kernels.
#include <cuda_runtime.h>

#include "ref_kernels.cu"

namespace {
inline unsigned blocks_for(int total, unsigned block) { return (unsigned)((total + block - 1) / block); }
}  // namespace

extern "C" {

// launch_rmsnorm_on_stream (src/model/decode.rs:2257-2289): one block of 256 per row.
int ref_rmsnorm(const float* in, const float* gamma, float* out, int rows, int cols, float eps) {
  rmsnorm_f32<<<rows, 256, 256 * sizeof(float)>>>(in, gamma, out, rows, cols, eps);
  return (int)cudaGetLastError();
}

// launch_rope_on_stream (src/model/decode.rs:2356-2395).
int ref_rope(const float* in, float* out, int total, int heads, int steps, int head_dim,
             int offset, float theta) {
  rope_bhsd_f32<<<blocks_for(total, 256), 256>>>(in, out, total, heads, steps, head_dim, offset,
                                                 theta);
  return (int)cudaGetLastError();
}

// launch_write_cache_on_stream (src/model/decode.rs:2421-2462), batch 1.
int ref_write_kv(const float* in, float* cache, int heads, int input_steps, int cache_steps,
                 int head_dim, int offset) {
  const int total = heads * input_steps * head_dim;
  write_kv_cache_f32<<<blocks_for(total, 256), 256>>>(in, cache, 1, heads, input_steps,
                                                      cache_steps, head_dim, offset, total);
  return (int)cudaGetLastError();
}

// launch_attention_scores_cache_on_stream (src/model/decode.rs:2578-2630), batch 1.
int ref_attention_scores_cache(const float* q, const float* k, float* scores, int q_heads,
                               int kv_heads, int query_steps, int key_steps, int cache_steps,
                               int head_dim, int offset, float scale) {
  const int total = q_heads * query_steps * key_steps;
  attention_scores_cache_f32<<<blocks_for(total, 256), 256>>>(
      q, k, scores, 1, q_heads, kv_heads, query_steps, key_steps, cache_steps, head_dim, offset,
      scale, total);
  return (int)cudaGetLastError();
}

// launch_softmax_on_stream (src/model/decode.rs:2642-2671): active_cols = cols.
int ref_softmax(const float* in, float* out, int rows, int cols) {
  masked_softmax_f32<<<rows, 256, 256 * sizeof(float)>>>(in, out, rows, cols, cols);
  return (int)cudaGetLastError();
}

// launch_apply_value_cache_on_stream (src/model/decode.rs:2773-2819), batch 1.
int ref_apply_value_cache(const float* probs, const float* v, float* out, int q_heads,
                          int kv_heads, int query_steps, int key_steps, int cache_steps,
                          int head_dim) {
  const int total = query_steps * q_heads * head_dim;
  attention_apply_value_cache_f32<<<blocks_for(total, 256), 256>>>(
      probs, v, out, 1, q_heads, kv_heads, query_steps, key_steps, cache_steps, head_dim, total);
  return (int)cudaGetLastError();
}

// launch_ternary_on_stream (src/model/decode.rs:2831-2855) with residual_add_f32.
int ref_residual_add(const float* a, const float* b, float* out, int total) {
  residual_add_f32<<<blocks_for(total, 256), 256>>>(a, b, out, total);
  return (int)cudaGetLastError();
}

// launch_ternary_on_stream with swiglu_f32.
int ref_swiglu(const float* gate, const float* up, float* out, int total) {
  swiglu_f32<<<blocks_for(total, 256), 256>>>(gate, up, out, total);
  return (int)cudaGetLastError();
}

// launch_argmax_on_stream (src/model/code_predictor.rs:1006-1026): one row, 256 threads.
int ref_argmax(const float* in, int* out, int cols) {
  argmax_rows_f32<<<1, 256, 256 * (sizeof(float) + sizeof(int))>>>(in, out, 1, cols);
  return (int)cudaGetLastError();
}

// launch_suppress (src/model/talker.rs:571-591).
int ref_suppress(const float* in, float* out, int vocab, int eos) {
  suppress_codec_logits_f32<<<blocks_for(vocab, 256), 256>>>(in, out, vocab, eos);
  return (int)cudaGetLastError();
}

// launch_repetition_penalty (src/model/talker.rs:593-613): a single thread.
int ref_penalty(float* logits, const int* tokens, int count, int vocab, float penalty) {
  apply_repetition_penalty_f32<<<1, 1>>>(logits, tokens, count, vocab, penalty);
  return (int)cudaGetLastError();
}

// launch_sample_topk (src/model/talker.rs:615-643): 1024 threads, the sort
// width the next power of two of the vocab.
int ref_sample_topk(const float* logits, int* token, int vocab, int top_k, float temperature,
                    float u) {
  int sort = 1;
  while (sort < vocab) sort <<= 1;
  const size_t smem = (size_t)sort * (sizeof(float) + sizeof(int));
  sample_topk_f32<<<1, 1024, smem>>>(logits, token, vocab, sort, top_k, temperature, u);
  return (int)cudaGetLastError();
}

}  // extern "C"
