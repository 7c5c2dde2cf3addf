// Codec convolutions on the tensor cores (tcgen05, sm_100a) at fp32-level
// accuracy: the same implicit GEMM as k_codec_conv (codec.cu),
//   y[co][t * ostride + ph] = epi(bias[co] + sum_k W[ph][co][k] * act(x)[k][t]),
// with K ordered tap-major here (k = tap * cip + channel, channels padded to
// a multiple of 64), so each 64-wide K step reads 64 channels of one input
// column. W (fp32) is repacked and split once at load into bf16 hi + lo, and
// each activation tile is split the same way while it is built, so every
// product keeps ~16 mantissa bits: D = Wh * [xh; xl] (one MMA with N = 256)
// + Wl * xh (N = 128). The dropped Wl * xl term is below 2^-16 of each
// product.
//
// CTA = 10 warps, one 128-channel x 128-position tile. Warp 0 streams the
// weight tiles of each K step with TMA (hi and lo, two 64-row boxes each,
// 128-byte swizzle); warps 2-9 gather the activation tile of the same step
// (implicit im2col with the input transform: a thread owns one position and
// half the step's channels, the next step's loads in flight while the
// current one is converted) and store hi / lo in the swizzled K-major
// layout; warp 1 owns the TMEM accumulator (256 fp32 columns) and issues the
// MMAs from one thread. A ring of three stages with three mbarriers each
// (weights landed, activations written, MMAs done) decouples the roles;
// every wait is bounded. Afterwards warps 2-9 read TMEM back (each warp its
// 32 lanes, half the positions) and apply the epilogue of k_codec_conv.
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>

#include "codec.h"
#include "common.cuh"
#include "gemm_tc.h"
#include "sm100.cuh"

namespace qtts {
namespace {

constexpr int kCtBuilders = 256;  // 8 warps build the activation tiles
constexpr int kCtThreads = 64 + kCtBuilders;
constexpr int kCtRows = 128;  // output channels per CTA (MMA M)
constexpr int kCtCols = 128;  // positions per CTA (MMA N per half)
constexpr int kCtK = 64;      // K per stage
constexpr int kCtStages = 3;
constexpr int kCtW = kCtRows * kCtK * 2;  // 16 KB: one weight half (hi or lo)
constexpr int kCtX = kCtCols * kCtK * 2;  // 16 KB: one activation half
constexpr int kCtStage = 2 * kCtW + 2 * kCtX;
constexpr size_t kCtSmem = (size_t)kCtStages * kCtStage + 1024 + 256;
constexpr uint32_t kCtTmemCols = 256;
constexpr unsigned long long kCtWaitNs = 2000000000ull;
static_assert(kCtStage % 1024 == 0, "stages keep the 1024-byte swizzle alignment");

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ float snake_f(float x, float a, float b) {
  const float s = sinf(x * a);
  return x + (s * s) / (b + 1.0e-9f);
}

template <int ACT>
__global__ void __launch_bounds__(kCtThreads, 1)
    k_codec_conv_tc(const __grid_constant__ CUtensorMap mh, const __grid_constant__ CUtensorMap ml,
                    CodecConvArgs a, int cip, int* err, CodecTcSplit sp) {
  extern __shared__ uint8_t ct_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(ct_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kCtStages * kCtStage);
  uint64_t* bready = full + kCtStages;
  uint64_t* empty = bready + kCtStages;
  uint64_t* done = empty + kCtStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ph = blockIdx.x % a.nphase;
  const int t0 = (blockIdx.x / a.nphase) * kCtCols;
  const int co0 = blockIdx.y * kCtRows;
  const int wrow = ph * a.co + co0;  // first weight row of this tile (phase-major rows)
  // split K over blockIdx.z: this CTA runs K steps [kb0, kb0 + nk)
  const int nk_all = a.taps * cip / kCtK;
  const int kb0 = (int)((long long)nk_all * blockIdx.z / gridDim.z);
  const int nk = (int)((long long)nk_all * (blockIdx.z + 1) / gridDim.z) - kb0;
  __shared__ int s_last;

  const int pre = min(kCtStages, nk);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kCtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], kCtBuilders / 32);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    for (int i = 0; i < pre; ++i) {
      uint8_t* st = smem + i * kCtStage;
      mbar_expect_tx(&full[i], 2 * kCtW);
      tma_load_2d(st, &mh, (kb0 + i) * kCtK, wrow, &full[i]);
      tma_load_2d(st + kCtW / 2, &mh, (kb0 + i) * kCtK, wrow + kCtRows / 2, &full[i]);
      tma_load_2d(st + kCtW, &ml, (kb0 + i) * kCtK, wrow, &full[i]);
      tma_load_2d(st + kCtW + kCtW / 2, &ml, (kb0 + i) * kCtK, wrow + kCtRows / 2, &full[i]);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, kCtTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    int issued = pre;
    for (int i = pre; i < nk; ++i) {
      const int s = i % kCtStages;
      if (!mbar_wait_ns(&empty[s], ((i / kCtStages) & 1) ^ 1, kCtWaitNs)) {
        atomicExch(err, 1);
        break;
      }
      uint8_t* st = smem + s * kCtStage;
      mbar_expect_tx(&full[s], 2 * kCtW);
      tma_load_2d(st, &mh, (kb0 + i) * kCtK, wrow, &full[s]);
      tma_load_2d(st + kCtW / 2, &mh, (kb0 + i) * kCtK, wrow + kCtRows / 2, &full[s]);
      tma_load_2d(st + kCtW, &ml, (kb0 + i) * kCtK, wrow, &full[s]);
      tma_load_2d(st + kCtW + kCtW / 2, &ml, (kb0 + i) * kCtK, wrow + kCtRows / 2, &full[s]);
      ++issued;
    }
    // No copy may still be landing and no commit still due on a stage barrier
    // when the CTA exits: wait for the last fill of every stage and its release.
    for (int i = (issued > kCtStages ? issued - kCtStages : 0); i < issued; ++i) {
      if (!mbar_wait_ns(&full[i % kCtStages], (i / kCtStages) & 1, kCtWaitNs)) atomicExch(err, 5);
      if (!mbar_wait_ns(&empty[i % kCtStages], (i / kCtStages) & 1, kCtWaitNs)) atomicExch(err, 6);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc2 = umma_idesc_bf16(kCtRows, 2 * kCtCols);  // Wh * [xh; xl]
    constexpr uint32_t idesc1 = umma_idesc_bf16(kCtRows, kCtCols);      // Wl * xh
    for (int i = 0; i < nk; ++i) {
      const int s = i % kCtStages;
      const unsigned par = (i / kCtStages) & 1;
      if (!mbar_wait_ns(&full[s], par, kCtWaitNs) || !mbar_wait_ns(&bready[s], par, kCtWaitNs)) {
        atomicExch(err, 2);
        break;
      }
      tc_fence_after();
      uint8_t* st = smem + s * kCtStage;
      const uint64_t dwh = umma_desc_sw128(st);
      const uint64_t dwl = umma_desc_sw128(st + kCtW);
      const uint64_t dx = umma_desc_sw128(st + 2 * kCtW);
#pragma unroll
      for (int kk = 0; kk < kCtK / 16; ++kk) {  // +32 bytes per 16-element K step
        umma_bf16(tmem, dwh + 2 * kk, dx + 2 * kk, idesc2, (i | kk) != 0);
        umma_bf16(tmem, dwl + 2 * kk, dx + 2 * kk, idesc1, 1u);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);
  } else if (warp >= 2) {
    // builder thread bt: activation row et = bt % 128 (position t0 + et),
    // K half h = bt / 128 (32 of the step's 64 channels)
    const int bt = threadIdx.x - 64;
    const int et = bt & (kCtCols - 1), h = bt >> 7;
    // the activations (and the split-K workspace) come from the previous
    // kernel; the weight tiles above did not wait for it
    pdl_wait();
    if (bt == 0) pdl_trigger();
    const int t = t0 + et;
    const long long ld = (long long)a.lin + a.hist;
    const float* xb = a.x + a.hist;
    constexpr int NU = ACT == CACT_SWIGLU ? 32 : 1;
    // K is tap-major (k = tap * cip + channel), so one step reads 64 channels
    // of a single input column, which is in range or not as a whole
    auto load_step = [&](int i, float (&v)[32], float (&u)[NU]) {
      const int kg = (kb0 + i) * kCtK;
      const int tap = kg / cip;
      const int c0 = kg - tap * cip + 32 * h;
      const int src = t + tap * a.dil - a.pad;
      const bool in = t < a.lin && src >= -a.hist && src < a.lin;
      const float* p = xb + (long long)c0 * ld + src;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const bool ok = in && c0 + q < a.ci;
        v[q] = ok ? __ldg(p + q * ld) : 0.f;
        if (ACT == CACT_SWIGLU) u[q] = ok ? __ldg(p + (q + a.up_off) * ld) : 0.f;
      }
      return c0;
    };
    float cur[32], curu[NU];
    int cch = nk > 0 ? load_step(0, cur, curu) : 0;
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % kCtStages;
      float val[32];
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        float v = cur[q];
        if (ACT == CACT_SNAKE && cch + q < a.ci)
          v = snake_f(v, __ldg(a.act_a + cch + q), __ldg(a.act_b + cch + q));
        else if (ACT == CACT_SWIGLU)
          v = v / (1.0f + expf(-v)) * curu[q % NU];
        val[q] = v;
      }
      if (i + 1 < nk) cch = load_step(i + 1, cur, curu);  // in flight during the stores below
      if (i >= kCtStages && !mbar_wait_ns(&empty[s], ((i / kCtStages) & 1) ^ 1, kCtWaitNs)) {
        atomicExch(err, 4);
        ok = false;
        break;
      }
      uint8_t* xs = smem + s * kCtStage + 2 * kCtW;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c = 4 * h + cc;
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float v0 = val[8 * cc + 2 * q], v1 = val[8 * cc + 2 * q + 1];
          const float h0 = __bfloat162float(__float2bfloat16_rn(v0));
          const float h1 = __bfloat162float(__float2bfloat16_rn(v1));
          hw[q] = pack2(h0, h1);
          lw[q] = pack2(v0 - h0, v1 - h1);
        }
        // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8)
        const int off = et * 128 + ((c ^ (et & 7)) << 4);
        *reinterpret_cast<uint4*>(xs + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(xs + kCtX + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bready[s]);
    }

    // ---- epilogue: TMEM lanes of this warp's quadrant = output channels;
    // warps 2-5 take positions 0-63 of the tile, warps 6-9 positions 64-127
    const int lane_base = 32 * (warp & 3);
    const int cbeg = warp < 6 ? 0 : kCtCols / 2;
    // always wait for the MMAs, even after an error: TMEM must not be freed
    // (nor the CTA exit) while tensor-core work is in flight
    const bool got = mbar_wait_ns(done, 0, 2 * kCtWaitNs) && ok;
    if (!got) atomicExch(err, 3);
    tc_fence_after();
    const int co = co0 + lane_base + lane;
    const long long lout = (long long)a.lin * a.ostride;
    const bool row_ok = co < a.co && got;
    const float b = row_ok && a.bias ? __ldg(a.bias + co) : 0.f;
    const float rs = row_ok && a.rscale ? __ldg(a.rscale + co) : 1.f;
    const float sa = row_ok && a.out_a ? __ldg(a.out_a + co) : 0.f;
    const float sb = row_ok && a.out_a ? __ldg(a.out_b + co) : 0.f;
    // Split K: every CTA of a tile stores its partial tile; the last to
    // finish (ticket) sums all of them in split order, so the result does not
    // depend on which CTA finished last.
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    const int r = lane_base + lane;
    float* part = sp.ws + (((long long)tile * gridDim.z + blockIdx.z) * kCtRows + r) * kCtCols;
    bool final_cta = true;
    if (gridDim.z > 1) {
      for (int c0 = cbeg; c0 < cbeg + kCtCols / 2; c0 += 16) {
        float v[16], w[16];
        tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)c0, v);
        tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(c0 + kCtCols), w);
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          __stcg(reinterpret_cast<float4*>(part + c0 + j),
                 make_float4(v[j] + w[j], v[j + 1] + w[j + 1], v[j + 2] + w[j + 2],
                             v[j + 3] + w[j + 3]));
      }
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kCtBuilders) : "memory");
      if (bt == 0) {
        const unsigned tk = atomicAdd(&sp.tickets[tile], 1u);
        s_last = tk == gridDim.z - 1u;
        if (s_last) sp.tickets[tile] = 0u;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kCtBuilders) : "memory");
      final_cta = s_last != 0;
      if (final_cta) __threadfence();
    }
    if (final_cta) {
      const float* base = sp.ws + ((long long)tile * gridDim.z * kCtRows + r) * kCtCols;
      for (int c0 = cbeg; c0 < cbeg + kCtCols / 2; c0 += 16) {
        if (t0 + c0 >= a.lin) break;  // warp-uniform
        float v[16], w[16];
        if (gridDim.z == 1) {
          tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)c0, v);
          tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(c0 + kCtCols), w);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += w[j];
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
          for (unsigned z = 0; z < gridDim.z; ++z) {
            const float* q = base + (long long)z * kCtRows * kCtCols + c0;
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
              const float4 f = __ldcg(reinterpret_cast<const float4*>(q + j));
              v[j] += f.x; v[j + 1] += f.y; v[j + 2] += f.z; v[j + 3] += f.w;
            }
          }
        }
        if (!row_ok) continue;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int tt = t0 + c0 + j;
          if (tt >= a.lin) break;
          float o = v[j] + b;
          if (a.epi & CEPI_GELU) o = 0.5f * o * (1.0f + erff(o * 0.7071067811865476f));
          const long long at = (long long)co * lout + (long long)tt * a.ostride + ph;
          if (a.epi & CEPI_RESID) o = a.resid[at] + o * rs;
          if (a.epi & CEPI_CLAMP) o = fminf(fmaxf(o, -1.0f), 1.0f);
          if (a.epi & CEPI_SNAKE) {
            a.y[at] = snake_f(o, sa, sb);
          } else {
            a.y[at] = o;
            if (a.y2) a.y2[at] = snake_f(o, sa, sb);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_free(tmem, kCtTmemCols);
}

// W [rows][ci * taps] (tap fastest) -> hi / lo [rows][taps * cip] (tap-major,
// channels padded to cip with zeros).
__global__ void k_split_hi_lo(const float* w, int rows, int ci, int taps, int cip,
                              __nv_bfloat16* hi, __nv_bfloat16* lo) {
  const long long K = (long long)taps * cip;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * K) return;
  const long long r = i / K;
  const int k = (int)(i - r * K), tap = k / cip, c = k - tap * cip;
  const float v = c < ci ? w[r * ci * taps + (long long)c * taps + tap] : 0.f;
  const __nv_bfloat16 hv = __float2bfloat16_rn(v);
  hi[i] = hv;
  lo[i] = __float2bfloat16_rn(v - __bfloat162float(hv));
}

template <int ACT>
cudaError_t launch_ct(const CodecTcWeight& w, const CodecConvArgs& a, int* err,
                      const CodecTcSplit& sp, dim3 grid, cudaStream_t stream) {
  return launch(k_codec_conv_tc<ACT>, grid, dim3(kCtThreads), kCtSmem, stream, w.mh, w.ml, a,
                w.cip, err, sp);
}

template <int ACT>
cudaError_t set_smem() {
  return cudaFuncSetAttribute(k_codec_conv_tc<ACT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kCtSmem);
}

}  // namespace

cudaError_t configure_codec_tc() {
  cudaError_t e;
  if ((e = set_smem<CACT_NONE>()) != cudaSuccess) return e;
  if ((e = set_smem<CACT_SNAKE>()) != cudaSuccess) return e;
  return set_smem<CACT_SWIGLU>();
}

cudaError_t codec_tc_prepare(const float* W, int rows, int ci, int taps, __nv_bfloat16* hi,
                             __nv_bfloat16* lo, CodecTcWeight* out, cudaStream_t stream) {
  if (rows <= 0 || ci <= 0 || taps <= 0) return cudaErrorInvalidValue;
  const int cip = codec_tc_padded_channels(ci);
  const long long n = (long long)rows * taps * cip;
  k_split_hi_lo<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(W, rows, ci, taps, cip, hi, lo);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  out->hi = hi;
  out->lo = lo;
  out->rows = rows;
  out->ci = ci;
  out->taps = taps;
  out->cip = cip;
  if (!tc_weight_map(hi, rows, taps * cip, &out->mh) || !tc_weight_map(lo, rows, taps * cip, &out->ml))
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

bool codec_tc_supported(const CodecConvArgs& a, const CodecTcWeight& w) {
  // one weight set per phase, phase-major rows of the packed [nphase][co][K] layout
  return w.hi && a.co >= 64 && w.ci == a.ci && w.taps == a.taps &&
         (a.nphase == 1 || a.w_phase_stride == (long long)a.co * a.ci * a.taps) &&
         w.rows == a.co * a.nphase && a.act >= CACT_NONE && a.act <= CACT_SWIGLU;
}

cudaError_t codec_conv_tc(const CodecConvArgs& a, const CodecTcWeight& w, int* err,
                          const CodecTcSplit* split, cudaStream_t stream) {
  if (a.ci <= 0 || a.co <= 0 || a.lin <= 0 || a.taps <= 0 || a.nphase <= 0 || a.ostride <= 0 ||
      a.hist < 0 || !codec_tc_supported(a, w))
    return cudaErrorInvalidValue;
  dim3 grid((unsigned)((a.lin + kCtCols - 1) / kCtCols) * a.nphase,
            (unsigned)((a.co + kCtRows - 1) / kCtRows), 1);
  // Few tiles (short inputs: streamed chunks, the pre-transformer) leave most
  // SMs idle while each CTA walks the whole K range: split K so that about
  // one CTA runs per SM, keeping at least two K steps per split.
  CodecTcSplit sp = split ? *split : CodecTcSplit{};
  const int tiles = (int)(grid.x * grid.y);
  const int nk = a.taps * w.cip / kCtK;
  if (sp.ws && sp.tickets && sp.sms > 0 && 2 * tiles <= sp.sms) {
    int splits = std::min({sp.sms / tiles, nk / 2, kCodecTcMaxSplits});
    while (splits > 1 && (size_t)tiles * splits * kCtRows * kCtCols > sp.ws_floats) --splits;
    if (splits > 1 && tiles <= sp.max_tiles) grid.z = splits;
  }
  if (a.act == CACT_SNAKE) return launch_ct<CACT_SNAKE>(w, a, err, sp, grid, stream);
  if (a.act == CACT_SWIGLU) return launch_ct<CACT_SWIGLU>(w, a, err, sp, grid, stream);
  return launch_ct<CACT_NONE>(w, a, err, sp, grid, stream);
}

}  // namespace qtts
