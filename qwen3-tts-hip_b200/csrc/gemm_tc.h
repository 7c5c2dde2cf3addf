// Tensor-core (tcgen05) projection for many activation rows: prefill (M = P
// prompt rows) and the text MLP. Computes the same thing as the CUDA-core
// projection, y[m] = epilogue(rms[m] * W . (gamma * x[m])), with weights as
// the 128-row MMA operand and activation rows as N. The fp32 activations are
// split into bf16 hi + lo parts (two MMAs into one fp32 TMEM accumulator), so
// the product keeps ~16 mantissa bits of the activation instead of bf16's 8.
#pragma once

#include <cuda.h>

#include "kernels.h"

namespace qtts {

constexpr int kTcBlockK = 64;     // K per stage: one 128-byte swizzle row of bf16
constexpr int kTcRows = 128;      // weight rows per CTA (MMA M)

// Split activations: hi/lo bf16 [rows, ld] of gamma * x, and rms[m] (1 when no gamma).
struct TcActs {
  __nv_bfloat16* hi;
  __nv_bfloat16* lo;
  float* rms;
  int rows_cap;   // rows allocated
  int ld;         // row pitch in elements (>= every K used)
  int box_rows;   // activation rows per CTA tile (MMA N): 128 (prefill) or 16 (batched decode)
  CUtensorMap hi_map, lo_map;  // box: 64 elements x box_rows rows
  // optional split-K workspace (skinny GEMMs): partial tiles and per-tile tickets
  float* ws;
  size_t ws_floats;
  unsigned* tickets;
  int max_splits;
  int sm_count;
};

// Host: builds the maps of an activation buffer pair; false if the driver
// entry point is unavailable.
bool tc_make_acts(TcActs& a);
// Host: map of a [rows, K] bf16 weight (box 64 x 64 rows). Cached by pointer.
bool tc_weight_map(const __nv_bfloat16* W, int rows, int K, CUtensorMap* out);

// Whether launch_linear_tc handles this projection.
bool tc_supported(const LinearArgs& a, int epi, const TcActs& acts);
// Enqueues the split kernel and the tcgen05 GEMM. `err` receives a nonzero
// code if a pipeline wait times out.
cudaError_t launch_linear_tc(const LinearArgs& a, int epi, const TcActs& acts, int* err,
                             cudaStream_t stream);
cudaError_t configure_tc_kernels();

}  // namespace qtts
