// Host-facing argument blocks and launchers for the sm_100a token-loop kernels.
// All launchers enqueue on `stream` with programmatic dependent launch enabled,
// so they may be captured into one CUDA graph per frame.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace qtts {

// Output transform applied by the projection kernels.
enum Epilogue : int {
  EPI_STORE = 0,      // y = W x
  EPI_RESID = 1,      // y = W x + r          (O-proj / down-proj residual)
  EPI_SWIGLU = 2,     // y[c] = silu(W[c] x) * (W[N + c] x)   (gate|up, N = intermediate)
  EPI_BIAS = 3,       // y = W x + b          (small_to_mtp_projection, text fc2)
  EPI_BIAS_SILU = 4,  // y = silu(W x + b)    (text fc1)
};

struct LinearArgs {
  const __nv_bfloat16* W;  // [rows, K] row-major (PyTorch [out, in])
  const float* x;          // [M, ldx]
  int ldx;
  const float* gamma;      // optional RMSNorm gamma [K]; nullptr = raw input
  float eps;
  float* y;                // [M, ldy]
  int ldy;
  const float* resid;      // EPI_RESID source [M, ldr] (may alias y)
  int ldr;
  const float* bias;       // EPI_BIAS* [N]
  int M, N, K;
  const int* halt;         // optional: kernel is a no-op while *halt != 0
  int trace_id;            // > 0: record entry / dependency-wait / exit times (step trace)
  // EPI_RESID: the residual rows were written at least two launches back, so
  // the kernel may read them before its dependency wait (a kernel starts only
  // after the kernel two places before it has completed).
  int resid_early;
};

// Sampling parameters of one token kind (talker or subtalker).
struct SampleCfg {
  int do_sample;
  int top_k;
  float top_p;
  float temperature;
};

enum RngKind : int { RNG_LCG = 0, RNG_PHILOX = 1 };

// Per-sequence device-resident loop state (one 64-byte block).
struct SeqState {
  int frames;       // frames whose 16 codes are complete
  int semantic;     // semantic token that starts the next frame
  int talker_pos;   // cache position of the next talker decode step
  int prefill_len;  // P
  int n_trailing;   // trailing text rows uploaded
  int halt;         // set once the semantic token is codec EOS
  int error;        // nonzero: device-side invalid state (e.g. no finite logits)
  int rng_kind;
  unsigned long long rng_state;    // LCG state (reference draw order)
  unsigned long long rng_seed;     // Philox key
  unsigned long long rng_counter;  // Philox counter
  int pad[2];
};

enum HeadRole : int {
  ROLE_TALKER_PREFILL = 0,  // token from prefill; no penalty
  ROLE_TALKER_STEP = 1,     // token from a decode step; penalty over history
  ROLE_CP_GROUP = 2,        // CodePredictor group token
  ROLE_LOGITS_ONLY = 3,     // debug: logits only
};

// Widest rows of the precomputed CodePredictor tables a token head copies
// (layer-0 QKV row, projected input row), in floats.
constexpr int kCpQkvTableMax = 4096;
constexpr int kCpXTableMax = 2048;

struct HeadArgs {
  LinearArgs lin;         // M = 1 projection to logits (lin.y = logits)
  unsigned* ticket;       // zero-initialised counter (reset by the last CTA)
  int role;
  SampleCfg cfg;
  SeqState* st;
  // talker
  float penalty;
  const int* history;     // semantic history (length st->frames)
  int eos_token;
  int suppress;           // suppress [V-1024, V) except eos
  const __nv_bfloat16* talker_codec_emb;  // [V, H]
  float* cp_prefix;       // [2, H]: normed hidden, codec_emb[semantic]
  int H;
  // CodePredictor
  int group, last_group;
  const __nv_bfloat16* cp_emb;  // [Vcp, H] embedding of this group
  float* cp_next;          // [H] next group input (pre-projection)
  float* emb_sum;          // [H]
  float* step_in;          // [H] talker decode input (written by the last group)
  const float* trailing;   // [n_trailing, H]
  const float* tts_pad;    // [H]
  int* codes;              // [max_frames, groups]
  int* history_out;        // semantic history
  int groups;
  int* token_out;          // optional: selected token
  int frames_cap;          // > 0: checked bound of the frame counter (codes rows)
  int talker_vocab;        // > 0: checked bound of the semantic token
  // optional: the next group's layer-0 QKV row of every token of this
  // group's vocab ([Vcp, qkv_w]); the selected token's row is copied to qkv_out
  const float* qkv_table;
  float* qkv_out;
  int qkv_w;
  // optional, with qkv_table: the next group's projected input row of every
  // token ([Vcp, x_w], models with the CodePredictor input projection)
  const float* x_table;
  float* x_out;
  int x_w;
};

// Batched heads: per-sequence views of `h` at the given element strides;
// `rms` holds each sequence's RMS scale of its head input row.
struct BatchHeadArgs {
  HeadArgs h;
  const float* logits;     // [B, logits_ld]
  int logits_ld;
  const float* rms;        // [B]
  long long hist_stride, codes_stride, next_stride, step_stride, trail_stride;
  long long qkv_stride, x_stride;  // per-sequence rows of h.qkv_out / h.x_out
};

struct AttnDecodeArgs {
  const float* qkv;        // raw projections of the current position [q_out + 2 kv_out]
  const float* q_gamma;
  const float* k_gamma;
  float eps;
  const float* rope_cos;   // [positions, 64]
  const float* rope_sin;
  KvView kv;
  int layer;
  const int* pos_ptr;      // position = pos_ptr ? *pos_ptr : pos_const
  int pos_const;
  int q_heads;
  float scale;
  float* out;              // [q_heads * 128]
  const int* halt;
  int trace_id;
  // Batched decode (sequence b = blockIdx.y; all zero for one sequence):
  // element strides between sequences of qkv rows and output rows, int
  // strides of the position and halt words, and page-table entries per sequence.
  int qkv_ld, out_ld, pos_stride, halt_stride, pt_stride;
  int batch;               // sequences (0 or 1: one)
  // Fused CodePredictor attention only: when >= 0, the physical page that
  // holds every position of the sequence (no page-table read before the
  // cache reads); -1 reads the table.
  int page0;
};

struct QkPrepArgs {
  const float* qkv;        // [M, q_out + 2 kv_out]
  const float* q_gamma;
  const float* k_gamma;
  float eps;
  const float* rope_cos;
  const float* rope_sin;
  KvView kv;
  int layer;
  int pos0;
  int M;
  int q_heads;
  float* q_out;            // [M, q_heads * 128]
  const int* halt;
};

struct AttnPrefillArgs {
  const float* q;          // [M, q_heads * 128] normed + roped
  KvView kv;
  int layer;
  int pos0;
  int M;
  int q_heads;
  float scale;
  float* out;              // [M, q_heads * 128]
  const int* halt;
};

cudaError_t launch_linear(const LinearArgs& a, Epilogue epi, cudaStream_t stream);
cudaError_t launch_head(const HeadArgs& a, cudaStream_t stream);
// CodePredictor decode attention fused into the O projection (o.x unused,
// o.resid = residual); only for a fixed position below 16 and two q heads per
// kv head (attn_o_fusable).
bool attn_o_fusable(const AttnDecodeArgs& at, const LinearArgs& o);
cudaError_t launch_attn_o(const AttnDecodeArgs& at, const LinearArgs& o, cudaStream_t stream);
cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t stream);
cudaError_t launch_select_batch(const BatchHeadArgs& a, int B, cudaStream_t stream);
// Debugging aid: device pointer of mapped host memory for kernel breadcrumbs.
cudaError_t set_crumbs_kernels(unsigned* host_mapped_dev_ptr);
cudaError_t set_crumbs_gemm(unsigned* host_mapped_dev_ptr);
// Step trace buffer: [8][capacity] u64 indexed by trace_id: globaltimer values
// (first entry, first post-wait, last exit, last post-wait, two kernel-specific
// marks taken by the last CTA) and two kernel-specific durations (max over
// CTAs of the time since the CTA's own dependency wait); nullptr disables.
// Stream-ordered.
cudaError_t set_step_trace(unsigned long long* buf, int capacity, cudaStream_t stream);
// One thread waits (bounded by limit_ns) for *counter >= target; *status = 1
// when the wait ran out, 0 when the target was reached.
cudaError_t launch_wait_selftest(const unsigned long long* counter, unsigned long long target,
                                 unsigned long long limit_ns, int* status, cudaStream_t stream);
cudaError_t launch_qk_prep(const QkPrepArgs& a, cudaStream_t stream);
cudaError_t launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t stream);

// out[r, :] = float(table[ids[r], :])
cudaError_t launch_gather_rows(const __nv_bfloat16* table, const int* ids, int n, int width,
                               float* out, cudaStream_t stream);
// out[r] = proj[proj_index[r]] + (codec_ids[r] >= 0 ? codec[codec_ids[r]] :
//                                  codec_ids[r] == -2 ? xvec : 0)
cudaError_t launch_assemble_rows(const float* proj, const int* proj_index,
                                 const __nv_bfloat16* codec, const int* codec_ids,
                                 const float* xvec, int n, int width, float* out,
                                 cudaStream_t stream);

int max_sample_vocab();
// Sets the dynamic shared-memory limits of every kernel; call once per device
// before the first launch (and before any stream capture).
cudaError_t configure_kernels();

}  // namespace qtts
