// tcgen05 GEMM for the prefill projections (see gemm_tc.h).
//
// CTA = 6 warps: warp 0 issues TMA loads (weights: two 64-row boxes; split
// activations: hi and lo boxes of kTcTokens rows), warp 1 owns the TMEM
// accumulator (128 lanes x kTcTokens fp32 columns) and issues the MMAs from
// one thread, warps 2-5 read TMEM back (each warp may only touch the 32 lanes
// of its warp-id modulo 4) and apply the epilogue. A kTcStages-deep ring of
// mbarrier pairs (full: TMA bytes landed; empty: the MMAs reading the stage
// completed) decouples loads from MMAs. Every wait is bounded.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "gemm_tc.h"
#include "sm100.cuh"

namespace qtts {
namespace {

constexpr int kTcThreads = 192;
constexpr unsigned kTcSpin = 1u << 22;
constexpr int kStageA = kTcRows * kTcBlockK * 2;  // 16 KB: 128 weight rows x 64 K

// Per token-tile width BN (MMA N): stage ring depth and sizes.
template <int BN>
struct TcCfg {
  static constexpr int kStages = BN >= 128 ? 4 : 8;
  static constexpr int kStageB = BN * kTcBlockK * 2;         // hi or lo
  static constexpr int kStageBytes = kStageA + 2 * kStageB;  // multiple of 1024
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024 /*align*/ + 256;
  static_assert(kStageBytes % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
};

struct TcArgs {
  int M, N, K;
  int epi;
  int up_off;            // SWIGLU: row offset of the up half in W
  float* y;
  int ldy;
  const float* resid;
  int ldr;
  const float* bias;
  const float* rms;
  int* err;
  const int* halt;
  int splits;            // K split over blockIdx.z; > 1 uses ws + tickets
  float* ws;             // [tiles][splits][128][BN] partial tiles
  unsigned* tickets;     // [tiles], zero at rest (reset by the last CTA)
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

template <int BN>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap hmap,
              const __grid_constant__ CUtensorMap lmap, TcArgs a) {
  using Cfg = TcCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool swiglu = a.epi == EPI_SWIGLU;
  const int n0 = blockIdx.x * (swiglu ? kTcRows / 2 : kTcRows);   // first output column
  const int row_a0 = n0;                                          // weight rows, box 0
  const int row_a1 = swiglu ? a.up_off + n0 : n0 + kTcRows / 2;   // box 1
  const int m0 = blockIdx.y * BN;
  const int KB = a.K / kTcBlockK;
  const int kb0 = (int)((long long)KB * blockIdx.z / a.splits);
  const int kb1 = (int)((long long)KB * (blockIdx.z + 1) / a.splits);
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // producer: weight tiles of the first stages do not depend on the previous
    // kernel, so they are requested before the dependency wait.
    const int pre = min(S, nk);
    for (int i = 0; i < pre; ++i) {
      uint8_t* st = smem + i * Cfg::kStageBytes;
      mbar_expect_tx(&full[i], Cfg::kStageBytes);
      const int kx = (kb0 + i) * kTcBlockK;
      tma_load_2d(st, &wmap, kx, row_a0, &full[i]);
      tma_load_2d(st + kStageA / 2, &wmap, kx, row_a1, &full[i]);
    }
    pdl_wait();
    const bool halted = a.halt && __ldcg(a.halt);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      uint8_t* st = smem + s * Cfg::kStageBytes;
      const int kx = (kb0 + i) * kTcBlockK;
      if (i >= S) {
        if (!mbar_wait(&empty[s], ((i / S) & 1) ^ 1, kTcSpin)) {
          atomicExch(a.err, 1);
          break;
        }
        mbar_expect_tx(&full[s], Cfg::kStageBytes);
        tma_load_2d(st, &wmap, kx, row_a0, &full[s]);
        tma_load_2d(st + kStageA / 2, &wmap, kx, row_a1, &full[s]);
      }
      // when halted the activation tiles are still fetched (the stage byte
      // counts must complete) but the epilogue writes nothing
      (void)halted;
      tma_load_2d(st + kStageA, &hmap, kx, m0, &full[s]);
      tma_load_2d(st + kStageA + Cfg::kStageB, &lmap, kx, m0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer
    constexpr uint32_t idesc = umma_idesc_bf16(kTcRows, BN);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(&full[s], (i / S) & 1, kTcSpin)) {
        atomicExch(a.err, 2);
        break;
      }
      tc_fence_after();
      uint8_t* st = smem + s * Cfg::kStageBytes;
      const uint64_t da = umma_desc_sw128(st);
      const uint64_t dh = umma_desc_sw128(st + kStageA);
      const uint64_t dl = umma_desc_sw128(st + kStageA + Cfg::kStageB);
#pragma unroll
      for (int kk = 0; kk < kTcBlockK / 16; ++kk) {
        // +32 bytes per 16-element K step inside the swizzled 128-byte row
        umma_bf16(tmem, da + 2 * kk, dh + 2 * kk, idesc, (i | kk) != 0);
        umma_bf16(tmem, da + 2 * kk, dl + 2 * kk, idesc, 1u);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);  // also fires when nothing was issued
  } else if (warp >= 2) {
    pdl_wait();
    const bool halted = a.halt && __ldcg(a.halt);
    // this warp's 32 TMEM lanes = tile rows lane_base..lane_base+31
    const int lane_base = 32 * (warp & 3);
    const bool got = mbar_wait(done, 0, kTcSpin * 4);
    if (!got) atomicExch(a.err, 3);
    tc_fence_after();
    const int r = lane_base + lane;
    const int cols = min(BN, a.M - m0);
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    bool final_cta = true;
    if (a.splits > 1) {
      // partial tile -> workspace; the last CTA of the tile reduces in split order
      float* part = a.ws + ((long long)tile * a.splits + blockIdx.z) * kTcRows * BN;
      for (int c0 = 0; c0 < BN; c0 += 16) {
        if (c0 >= cols) break;
        float v[16];
        tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)c0, v);
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          __stcg(reinterpret_cast<float4*>(part + r * BN + c0 + j),
                 make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
      }
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (warp == 2 && lane == 0) {
        const unsigned t = atomicAdd(&a.tickets[tile], 1u);
        *last_flag = t == (unsigned)a.splits - 1u;
        if (*last_flag) a.tickets[tile] = 0u;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      final_cta = *last_flag != 0;
      if (final_cta) __threadfence();
    }
    float* xbuf = reinterpret_cast<float*>(smem);  // SWIGLU: up rows, after the mainloop
    for (int c0 = 0; final_cta && c0 < BN; c0 += 16) {
      if (c0 >= cols) break;  // uniform over the epilogue warps
      float v[16];
      if (a.splits > 1) {
        // sum the partial tiles in split order; four splits' loads in flight at once
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.f;
        const float* base = a.ws + (long long)tile * a.splits * kTcRows * BN + r * BN + c0;
        for (int s0 = 0; s0 < a.splits; s0 += 4) {
          float4 q[4][4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int j = 0; j < 4; ++j)
              q[u][j] = s0 + u < a.splits
                            ? __ldcg(reinterpret_cast<const float4*>(
                                  base + (long long)(s0 + u) * kTcRows * BN + 4 * j))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              v[4 * j] += q[u][j].x; v[4 * j + 1] += q[u][j].y;
              v[4 * j + 2] += q[u][j].z; v[4 * j + 3] += q[u][j].w;
            }
        }
      } else {
        tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)c0, v);
      }
      const bool write = got && !halted;
      if (swiglu) {
        if (r >= kTcRows / 2) {
#pragma unroll
          for (int j = 0; j < 16; ++j) xbuf[(r - kTcRows / 2) * BN + c0 + j] = v[j];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (r < kTcRows / 2 && write) {
          const int n = n0 + r;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (c0 + j < cols && n < a.N) {
              const float sc = a.rms ? __ldg(a.rms + m) : 1.0f;
              const float g = v[j] * sc, u = xbuf[r * BN + c0 + j] * sc;
              a.y[(long long)m * a.ldy + n] = g / (1.0f + expf(-g)) * u;
            }
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      } else if (write) {
        const int n = n0 + r;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c0 + j;
          if (c0 + j < cols && n < a.N) {
            float out = v[j] * (a.rms ? __ldg(a.rms + m) : 1.0f);
            if (a.epi == EPI_RESID) out += a.resid[(long long)m * a.ldr + n];
            if (a.epi == EPI_BIAS) out += a.bias[n];
            if (a.epi == EPI_BIAS_SILU) out = silu_f(out + a.bias[n]);
            a.y[(long long)m * a.ldy + n] = out;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, Cfg::kTmemCols);
  }
}

// gamma * x split into bf16 hi + lo, and the per-row RMS scale.
__global__ void __launch_bounds__(256) k_split_rows(const float* x, int ldx, const float* gamma,
                                                    float eps, int K, __nv_bfloat16* hi,
                                                    __nv_bfloat16* lo, int ld, float* rms,
                                                    const int* halt) {
  __shared__ float red[8];
  pdl_wait();
  if (halt && __ldcg(halt)) return;
  const int m = blockIdx.x;
  const float* row = x + (long long)m * ldx;
  float ss = 0.f;
  for (int k = threadIdx.x * 4; k < K; k += 1024) {
    float4 v = *reinterpret_cast<const float4*>(row + k);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    if (gamma) {
      const float4 g = *reinterpret_cast<const float4*>(gamma + k);
      v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
    }
    const float f[4] = {v.x, v.y, v.z, v.w};
    __nv_bfloat16 h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[i] = __float2bfloat16_rn(f[i]);
      l[i] = __float2bfloat16_rn(f[i] - __bfloat162float(h[i]));
    }
    __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(hi + (long long)m * ld + k);
    __nv_bfloat162* lw = reinterpret_cast<__nv_bfloat162*>(lo + (long long)m * ld + k);
    ho[0] = __halves2bfloat162(h[0], h[1]); ho[1] = __halves2bfloat162(h[2], h[3]);
    lw[0] = __halves2bfloat162(l[0], l[1]); lw[1] = __halves2bfloat162(l[2], l[3]);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    rms[m] = gamma ? rsqrtf(t / (float)K + eps) : 1.0f;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_map(const void* base, uint64_t inner, uint64_t rows, uint64_t pitch_bytes,
              uint32_t box_rows, CUtensorMap* out) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBlockK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool tc_make_acts(TcActs& a) {
  return make_map(a.hi, (uint64_t)a.ld, (uint64_t)a.rows_cap, (uint64_t)a.ld * 2,
                  (uint32_t)a.box_rows, &a.hi_map) &&
         make_map(a.lo, (uint64_t)a.ld, (uint64_t)a.rows_cap, (uint64_t)a.ld * 2,
                  (uint32_t)a.box_rows, &a.lo_map);
}

bool tc_weight_map(const __nv_bfloat16* W, int rows, int K, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<const void*, std::pair<long long, CUtensorMap>> cache;
  std::lock_guard<std::mutex> lock(mu);
  const long long key = (long long)rows * 1000003LL + K;
  auto it = cache.find(W);
  if (it != cache.end() && it->second.first == key) {
    *out = it->second.second;
    return true;
  }
  CUtensorMap m;
  if (!make_map(W, (uint64_t)K, (uint64_t)rows, (uint64_t)K * 2, kTcRows / 2, &m)) return false;
  cache[W] = {key, m};
  *out = m;
  return true;
}

bool tc_supported(const LinearArgs& a, int epi, const TcActs& acts) {
  if (!acts.hi || a.M > acts.rows_cap || a.K > acts.ld || a.K % kTcBlockK) return false;
  if (acts.box_rows != 16 && acts.box_rows != 128) return false;
  if (a.ldx % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15)) return false;
  return a.N % (kTcRows / 2) == 0 && (epi != EPI_SWIGLU || a.N >= kTcRows / 2);
}

cudaError_t configure_tc_kernels() {
  cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)TcCfg<128>::kSmem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_gemm_tc<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)TcCfg<16>::kSmem);
}

cudaError_t launch_linear_tc(const LinearArgs& a, int epi, const TcActs& acts, int* err,
                             cudaStream_t stream) {
  if (!tc_supported(a, epi, acts)) return cudaErrorInvalidValue;
  const int w_rows = epi == EPI_SWIGLU ? 2 * a.N : a.N;
  CUtensorMap wmap;
  if (!tc_weight_map(a.W, w_rows, a.K, &wmap)) return cudaErrorInvalidValue;
  cudaError_t e = launch(k_split_rows, dim3(a.M), dim3(256), 0, stream, a.x, a.ldx, a.gamma,
                         a.eps, a.K, acts.hi, acts.lo, acts.ld, acts.rms, a.halt);
  if (e != cudaSuccess) return e;
  const int BN = acts.box_rows;
  const int cols_per_cta = epi == EPI_SWIGLU ? kTcRows / 2 : kTcRows;
  dim3 grid((a.N + cols_per_cta - 1) / cols_per_cta, (a.M + BN - 1) / BN, 1);
  // split K so that a skinny GEMM still spreads over the SMs (deterministic
  // reduction by the last CTA of each tile)
  int splits = 1;
  const int tiles = (int)(grid.x * grid.y);
  if (acts.ws && tiles < acts.sm_count) {
    splits = std::min(acts.sm_count / tiles, (a.K / kTcBlockK) / 4);
    splits = std::max(1, std::min(splits, acts.max_splits));
    while (splits > 1 && (size_t)tiles * splits * kTcRows * BN > acts.ws_floats) --splits;
  }
  grid.z = splits;
  TcArgs t{a.M, a.N, a.K, epi, a.N, a.y, a.ldy, a.resid, a.ldr, a.bias,
           a.gamma ? acts.rms : nullptr, err, a.halt, splits, acts.ws, acts.tickets};
  if (BN == 16)
    return launch(k_gemm_tc<16>, grid, dim3(kTcThreads), TcCfg<16>::kSmem, stream, wmap,
                  acts.hi_map, acts.lo_map, t);
  return launch(k_gemm_tc<128>, grid, dim3(kTcThreads), TcCfg<128>::kSmem, stream, wmap,
                acts.hi_map, acts.lo_map, t);
}

}  // namespace qtts
