// Tensor-core (tcgen05) projection for many activation rows: prefill (M = P
// prompt rows), the text MLP and batched decode (M = sequences). Computes the
// same thing as the CUDA-core projection, y[m] = epilogue(rms[m] * W . (gamma
// * x[m])), with weights as the 128-row MMA operand and activation rows as N.
// The kernel itself splits the fp32 activations into bf16 hi + lo parts (two
// MMAs into one fp32 TMEM accumulator), so the product keeps ~16 mantissa
// bits of the activation instead of bf16's 8.
#pragma once

#include <cuda.h>

#include "kernels.h"

namespace qtts {

constexpr int kTcBlockK = 64;     // K per stage: one 128-byte swizzle row of bf16
constexpr int kTcRows = 128;      // weight rows per CTA (MMA M)

// Launch plan of one engine's tensor-core projections.
struct TcPlan {
  int tokens;        // activation rows per CTA tile (MMA N): 64 or 128 (prefill), 16 (batched decode)
  // optional split-K workspace for skinny GEMMs (tc_workspace_floats) and
  // per-tile tickets (zero at rest)
  float* ws;
  size_t ws_floats;
  unsigned* tickets;
  int max_splits;
  int sm_count;
};

// Host: whether the driver's tensor-map encoder is available.
bool tc_available();
// Host: map of a [rows, K] bf16 weight (box 64 x 64 rows). Cached by pointer.
bool tc_weight_map(const __nv_bfloat16* W, int rows, int K, CUtensorMap* out);
size_t tc_workspace_floats(int tokens, int sm_count);

// Whether launch_linear_tc handles this projection.
bool tc_supported(const LinearArgs& a, int epi, const TcPlan& p);
// Enqueues the GEMM; rms_out (optional, [M]) receives each row's RMS scale;
// `err` receives a nonzero code if a pipeline wait times out.
cudaError_t launch_linear_tc(const LinearArgs& a, int epi, const TcPlan& p, float* rms_out,
                             int* err, cudaStream_t stream);
cudaError_t configure_tc_kernels();

}  // namespace qtts
