// Persistent CodePredictor pass: one cooperative launch (one CTA per SM) runs
// the whole CodePredictor pass of a frame -- the 2-row prefill, the 14 decode
// groups and the 15 heads with their token selections -- as a fixed list of
// ops (code_predictor.rs:366-471 with project_to_stack, logits_for_hidden).
//
// Each op's weight rows are split over the CTAs; a producer warp streams this
// CTA's rows of the upcoming ops into a shared-memory ring with 1-D bulk
// copies, running ahead of the data dependencies, while eight consumer warps
// compute. Ops that read another op's output wait on one grid-wide arrival
// counter (every CTA adds one per op). Token selection runs in every CTA on
// the same logits, so the next group's embedding row is known CTA-locally
// and the next projection starts without a grid barrier.
#pragma once

#include "kernels.h"

namespace qtts {

enum CpOpKind : int {
  CPOP_GEMV = 0,    // y = epi(W . (gamma * x) * rms) over this CTA's rows
  CPOP_ATTN_O = 1,  // x = attention(qkv, cache) computed in every CTA; y = W_o x + resid
  CPOP_HEAD = 2,    // logits = W (gamma * x) * rms; then every CTA selects the token
};

enum CpSrc : int {
  CPSRC_GLOBAL = 0,  // an fp32 buffer in global memory
  CPSRC_LOCAL = 1,   // the CTA-local embedding row of the last selected token
};

// One op's descriptor (copied into shared memory 16 bytes at a time).
struct __align__(16) CpOp {
  int kind;
  int epi;                 // Epilogue (EPI_STORE, EPI_RESID, EPI_SWIGLU, EPI_BIAS)
  int M;                   // activation rows (2: the prefill, 1: a decode group)
  int N;                   // outputs (channels for EPI_SWIGLU; its weight has 2N rows)
  int K;                   // input width
  const __nv_bfloat16* W;  // [N or 2N, K] row-major
  const float* gamma;      // RMSNorm gamma over the input, or null
  float eps;
  int x_src;               // CpSrc
  const float* x;          // CPSRC_GLOBAL input [M, ldx]
  int ldx;
  float* y;                // output [M, ldy]
  int ldy;
  int r_src;               // CpSrc of the EPI_RESID residual
  const float* resid;
  int ldr;
  const float* bias;
  int wait;                // 1: every CTA must have finished the previous op first
  // CPOP_ATTN_O
  const float* qkv;        // [M, ld_qkv] raw projections of positions pos0..pos0+M-1
  int ld_qkv;
  const float* q_gamma;
  const float* k_gamma;
  int layer;
  int pos0;
  // CPOP_HEAD
  int group;               // codebook group 0..groups-2
  int pad_[3];
};

// The weight rows an op streams: W [nchunk * N (SwiGLU: gate rows then up
// rows), K]; a CTA copies rows [N b / G, N (b + 1) / G) of each chunk.
struct CpLoad {
  const __nv_bfloat16* W;
  int N;
  short K;
  short nchunk;
};

struct CpPassParams {
  const CpOp* ops;
  const CpLoad* loads;          // [n_ops]: the weight table the ring filler reads
  int n_ops;
  unsigned long long* counter;  // grid arrival counter (zeroed at the start of a generation)
  int* error;                   // [0]: first failure code, [1]: op index
  SeqState* st;
  // CodePredictor attention
  int q_heads, kv_heads;
  float scale;
  const float* rope_cos;        // [positions, 64]
  const float* rope_sin;
  __nv_bfloat16* cache;         // [layers][2][kv_heads][kCpPositions][128] bf16
  // embeddings and selection
  int H;                        // talker hidden = embedding width
  int groups;                   // codes per frame (16)
  int vocab;                    // CodePredictor vocab
  const __nv_bfloat16* cp_embs; // [groups-1][vocab][H]
  SampleCfg cfg;                // subtalker sampling
  // frame outputs (written by CTA 0 after the last group)
  int* codes;                   // [frames, groups]
  int* history;                 // semantic history
  const __nv_bfloat16* talker_codec_emb;  // [talker vocab, H]
  const float* trailing;        // [n_trailing, H]
  const float* tts_pad;         // [H]
  float* step_in;               // [H] input of the talker decode step
  unsigned long long* trace;    // optional [n_ops][kCpTraceSlots] globaltimer stamps of CTA 0
  // Parity seam (null in the frame graph): every head's logits
  // [groups-1][vocab] and the final embedding sum [H].
  float* dbg_logits;
  float* emb_sum_out;
};

constexpr int kCpPositions = 16;      // CodePredictor cache positions (prefix 2 + 14 groups)
constexpr int kCpThreads = 256;       // 8 warps; thread 0 also keeps the weight ring filled
constexpr int kCpStageBytes = 24576;  // whole rows for K = 256 .. 6144
constexpr int kCpStages = 6;
constexpr int kCpMaxOps = 512;        // ops of one pass (the weight table lives in shared memory)
constexpr int kCpMaxRows = 128;       // rows of one op per CTA (M = 2 each)
constexpr int kCpMaxH = 2048;
constexpr int kCpScratchBytes = 32768;  // input staging / token selection scratch
// Trace stamps per op (CTA 0, %globaltimer): past the wait, input staged,
// first weight stage ready, rows done, outputs stored, arrival issued, and
// for heads the selection's start and end (other ops: the last weight
// stage ready).
constexpr int kCpTraceSlots = 16;  // slots 8-13: a head's selection phases in clock64 cycles

// Whether the pass kernel supports this CodePredictor / talker shape.
bool cp_pass_supported(int cp_hidden, int intermediate, int q_heads, int kv_heads, int H,
                       int vocab, int sms);
size_t cp_pass_smem();
cudaError_t configure_cp_pass();
// Grid size of the pass on this device (one CTA per SM), 0 when unavailable.
int cp_pass_grid(int device);
cudaError_t launch_cp_pass(const CpPassParams& p, int grid, cudaStream_t stream);
// One thread waits (bounded by limit_ns) for *counter >= target; *status = 1
// when the wait ran out, 0 when the target was reached.
cudaError_t launch_wait_selftest(const unsigned long long* counter, unsigned long long target,
                                 unsigned long long limit_ns, int* status, cudaStream_t stream);

}  // namespace qtts
