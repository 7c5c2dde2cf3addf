// Codec decoder kernels (codes -> 24 kHz waveform), fp32 like the reference's
// HipCodecInitial (src/audio/codec_hip.rs). Activations are channel-major
// [channels][time] throughout, so every linear layer of the pre-transformer
// and the ConvNeXt blocks is a 1x1 convolution and one implicit-GEMM kernel
// serves all of them, the causal / dilated convolutions and (phase by phase)
// the transposed convolutions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qtts {

enum CodecAct : int {
  CACT_NONE = 0,
  CACT_SNAKE = 1,   // x + sin(x * a[c])^2 / (b[c] + 1e-9), a = e^alpha, b = e^beta
  CACT_SWIGLU = 2,  // silu(x[c]) * x[c + up_off]
};
enum CodecEpi : int {
  CEPI_GELU = 1,   // erf GELU after the bias
  CEPI_RESID = 2,  // y = resid + rscale[co] * v (rscale null: 1); resid may alias y
  CEPI_CLAMP = 4,  // clamp to [-1, 1]
  CEPI_SNAKE = 8,  // store snake(v) (out_a / out_b per output channel) instead of v
};

// y[co][t_out] = epi(bias[co] + sum_{ci, k} W[co][ci * taps + k] *
//                    act(x[ci][t + k * dil - pad]))
// for input positions t in [0, lin); t_out = t * ostride + phase with
// phase = 0 .. nphase-1 (transposed convolutions: one packed weight set per
// phase, w + phase * w_phase_stride). x holds `hist` columns of history
// before position 0 (row stride hist + lin; a streaming decoder's carried
// state); inputs outside [-hist, lin) read as 0.
struct CodecConvArgs {
  const float* x;
  int ci, lin;
  const float* w;
  long long w_phase_stride;
  const float* bias;
  int co, taps, dil, pad;
  int act;
  const float* act_a;  // CACT_SNAKE: e^alpha per input channel
  const float* act_b;  //             e^beta per input channel
  int up_off;          // CACT_SWIGLU: row offset of the up half
  float* y;
  int ostride, nphase;
  int epi;
  const float* resid;
  const float* rscale;
  // Output snake (e^alpha, e^beta per output channel): applied to y with
  // CEPI_SNAKE, or written to y2 (same layout) alongside y when y2 is set.
  const float* out_a;
  const float* out_b;
  float* y2;
  int hist;
};

cudaError_t codec_conv(const CodecConvArgs& a, cudaStream_t stream);

// A convolution weight [rows][ci * taps] (fp32, tap fastest; rows
// phase-major for transposed convolutions) repacked for the tensor-core
// path: K tap-major (k = tap * cip + channel, channels zero-padded to cip, a
// multiple of 64, so one 64-wide K step reads one input column) and split
// into bf16 hi + lo, with the TMA maps of both halves.
struct CodecTcWeight {
  __nv_bfloat16* hi = nullptr;
  __nv_bfloat16* lo = nullptr;
  CUtensorMap mh, ml;
  int rows = 0, ci = 0, taps = 0, cip = 0;
};
inline int codec_tc_padded_channels(int ci) { return (ci + 63) / 64 * 64; }
cudaError_t configure_codec_tc();
// Repacks and splits the device weight W into hi / lo (caller-allocated,
// rows * taps * codec_tc_padded_channels(ci) each) and builds the maps.
cudaError_t codec_tc_prepare(const float* W, int rows, int ci, int taps, __nv_bfloat16* hi,
                             __nv_bfloat16* lo, CodecTcWeight* out, cudaStream_t stream);
// Whether codec_conv_tc computes this convolution with this weight.
bool codec_tc_supported(const CodecConvArgs& a, const CodecTcWeight& w);
// Split-K workspace of the tensor-core convolution: partial tiles
// [tiles][splits][128][128] fp32 and one ticket per tile (zero at rest, reset
// by the kernel). `sms`: the device's SM count.
constexpr int kCodecTcMaxSplits = 32;
struct CodecTcSplit {
  float* ws = nullptr;
  size_t ws_floats = 0;
  unsigned* tickets = nullptr;
  int max_tiles = 0;
  int sms = 0;
};
// codec_conv on the tensor cores (tcgen05): bf16 hi + lo splits of the weight
// and of the transformed input, fp32 accumulation; convolutions with few
// output tiles split K over the workspace when `split` is given (the partial
// tiles are summed in a fixed order: results are deterministic). `err`
// receives a nonzero code if a pipeline wait times out.
cudaError_t codec_conv_tc(const CodecConvArgs& a, const CodecTcWeight& w, int* err,
                          const CodecTcSplit* split, cudaStream_t stream);

// first[t][d] = cb_first[code0][d]; rest[t][d] = sum_{g=1..15} cb_rest[g-1][code_g][d]
// (codes taken modulo the codebook size), then
// y[c][t] = sum_d wf[c][d] * first[t][d] + wr[c][d] * rest[t][d]
// (codec_rvq_project_f32, kernels.rs:454-497).
cudaError_t codec_rvq(const int32_t* codes, int frames, int groups, int cb_size, int cb_dim,
                      const float* cb_first, const float* cb_rest, const float* wf,
                      const float* wr, int out_dim, float* first, float* rest, float* y,
                      cudaStream_t stream);

// Per time step over the channel axis of [C][T]: RMSNorm (beta null) or
// LayerNorm (mean / variance, beta added).
cudaError_t codec_chan_norm(const float* x, int C, int T, const float* gamma, const float* beta,
                            float eps, float* y, cudaStream_t stream);

// y[c][t] = b[c] + sum_k w[c][k] * x[c][t + k - (K - 1)] (depthwise, causal);
// x [C][hist + T] carries hist (<= K - 1) history columns, older ones read 0.
cudaError_t codec_dwconv(const float* x, int C, int T, int hist, const float* w, const float* b,
                         int K, float* y, cudaStream_t stream);

// Streaming history of a causal convolution: cat [C][H + n] = the carried
// state [C][H] followed by the new input x [C][n]; state_next [C][H] = the
// last H columns of cat (the state the next chunk starts from).
cudaError_t codec_hist_cat(const float* state_cur, const float* x, int C, int H, int n,
                           float* cat, float* state_next, cudaStream_t stream);

// qkv [3 * heads * hd][T] of positions pos0 .. pos0 + T - 1 -> q [heads][T][hd]
// (RoPE applied) and the caches k (RoPE applied), v [heads][cap][hd] at those
// positions.
cudaError_t codec_qkv_rope(const float* qkv, int heads, int hd, int T, int pos0, int cap,
                           float theta, float* q, float* k, float* v, cudaStream_t stream);

// Causal softmax attention per head of T queries at positions pos0 .. over
// the cached keys / values [heads][cap][hd]; out [heads * hd][T].
cudaError_t codec_attention(const float* q, const float* k, const float* v, int heads, int hd,
                            int T, int pos0, int cap, float scale, float* out,
                            cudaStream_t stream);

// y[i] = expf(x[i]) (snake parameters, computed on the device like the
// reference's per-element expf).
cudaError_t codec_exp(const float* x, int n, float* y, cudaStream_t stream);

}  // namespace qtts
