// Persistent per-frame kernel: one cooperative launch (one CTA per SM) runs a
// whole 80 ms frame -- the CodePredictor pass of 15 groups and the talker
// decode step, with token selection -- as a fixed list of ops. Ops exchange
// activations through "tagged vectors": every fp32 element is stored together
// with the epoch of the op that wrote it in one 64-bit word, so a reader waits
// on the data itself instead of on a grid barrier.
#pragma once

#include "kernels.h"

namespace qtts {

typedef unsigned long long TV;  // (tag << 32) | float bits

enum FrameOpKind : int {
  FOP_GEMV = 0,         // y = epilogue(W x) over this CTA's row slice
  FOP_ATTN_DECODE = 1,  // QK-norm + RoPE + KV append + attention for one position
  FOP_ATTN_PAIR = 2,    // same for the 2-row CodePredictor prefill (positions 0, 1)
  FOP_HEAD = 3,         // LM-head GEMV, then every CTA selects the same token
};

enum FrameSrc : int {
  FSRC_NONE = 0,
  FSRC_LOCAL = 1,     // the CTA-local vector left by the previous head op
  FSRC_EXT = 2,       // plain fp32 written before this launch
  FSRC_TAG = 3,       // tagged vector written by op `*_op` of this launch
  FSRC_PARTIALS = 4,  // talker attention split partials, combined while staging
};

struct FrameOp {
  int kind;
  int epi;
  int M, N, K;
  int writers;       // CTAs that bump this op's completion counter
  // input vector(s)
  int x_src;
  const float* x_ext;
  const TV* x_tag;
  int ldx;
  int x_op;
  // residual (EPI_RESID)
  int r_src;
  const float* r_ext;
  const TV* r_tag;
  int ldr;
  int r_op;
  const __nv_bfloat16* W;
  const float* gamma;
  float eps;
  const float* bias;
  TV* y;
  int ldy;
  // attention
  const float* q_gamma;
  const float* k_gamma;
  const float* rope_cos;
  const float* rope_sin;
  KvView kv;         // talker: paged bf16 cache (earlier positions from earlier launches)
  TV* cp_cache;      // CodePredictor: tagged cache [layers][2][kv_heads][16][128]
  int layer;
  int q_heads;
  int kv_heads;
  int pos_const;     // >= 0: fixed position; -1: talker position from the loop state
  int nsplit;        // talker: splits over positions (partials), CodePredictor: 1
  float scale;
  // head
  int role;          // ROLE_CP_GROUP or ROLE_TALKER_STEP
  SampleCfg cfg;
  float penalty;
  int suppress;
  int group, last_group;
  const __nv_bfloat16* emb;  // embedding table gathered with the selected token
  TV* next_x;        // tagged input row of the next stack (this CTA writes its slice)
};

struct FrameParams {
  const FrameOp* ops;
  int n_ops;
  SeqState* st;
  unsigned* seq;        // launch counter (epoch high bits); incremented per launch
  int* error;           // [0]: wait timeout code, [1]: op index
  unsigned* counters;   // per-op completion counters (stride 8), zeroed before each launch
  int use_counters;     // 1: wait on counters before loading tagged inputs; 0: tags only
  const __nv_bfloat16* talker_codec_emb;
  int H;                // talker hidden (embedding width)
  int groups;
  int eos_token;
  int* codes;
  int* history;
  const float* trailing;
  const float* tts_pad;
  float* cp_prefix;     // plain [2, H]: next frame's CodePredictor input rows
  // Optional profiling trace: CTA `trace_cta` records clock64() at the start
  // and end of every op ([n_ops][2]); nullptr disables.
  long long* trace;
  int trace_cta;
  int trace_frame;      // frame index traced
};

constexpr int kFrameStages = 10;
constexpr int kFrameStageBytes = 16384;
constexpr int kFrameScratchBytes = 32768;
constexpr int kFrameMaxH = 2048;
constexpr int kFrameThreads = 288;  // 8 consumer warps + 1 producer warp
constexpr int kFrameCpPositions = 16;
constexpr int kFrameSharedTail = 4096;  // mbarriers, flags, current op
constexpr size_t kFrameSmem = (size_t)kFrameStages * kFrameStageBytes + kFrameScratchBytes +
                              2 * kFrameMaxH * sizeof(float) + kFrameSharedTail;

__host__ __device__ inline unsigned frame_tag(unsigned seq, int op) {
  return (seq << 12) | (unsigned)(op + 1);
}

// Rows of one op owned by CTA `b` of `G`.
__host__ __device__ inline void frame_rows(int N, int b, int G, int* r0, int* r1) {
  *r0 = (int)(((long long)N * b) / G);
  *r1 = (int)(((long long)N * (b + 1)) / G);
}

// Rows per ring stage for a K-wide bf16 row (power of two, <= 8).
__host__ __device__ inline int frame_rows_per_stage(int K) {
  const int r = kFrameStageBytes / (2 * K);
  return r >= 8 ? 8 : r >= 4 ? 4 : r >= 2 ? 2 : 1;
}

cudaError_t configure_frame_kernel();
// Enqueues the counter reset and the cooperative frame kernel.
cudaError_t launch_frame(const FrameParams& p, int grid, cudaStream_t stream);
int frame_grid_size(int device);

}  // namespace qtts
