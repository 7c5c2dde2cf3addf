// tcgen05 GEMM for projections over many activation rows (see gemm_tc.h).
//
// CTA = 6 warps. Warp 0 streams the weight tile of each K step with TMA (two
// 64-row boxes, 128-byte swizzle). Warps 2-5 build the activation tile of the
// same step in shared memory: they read fp32 rows of x, multiply by gamma,
// split each value into bf16 hi + lo and store both in the swizzled K-major
// layout the MMA reads, accumulating each row's sum of squares on the way (so
// no separate split kernel or launch). Warp 1 owns the TMEM accumulator
// (128 lanes x BN fp32 columns) and issues two MMAs per 16-element K step
// (W * hi, W * lo) from one thread. A ring of stages with three mbarriers
// each (weights landed, activations written, MMAs done) decouples the three
// roles; every wait is bounded, and the producer waits for the final release
// of every stage before the CTA exits. Afterwards warps 2-5 read TMEM back (each warp
// may only touch the 32 lanes of its warp id modulo 4) and apply the RMS scale
// and the epilogue. Skinny shapes split K over blockIdx.z: partial tiles and
// partial sums of squares go to a workspace and the last CTA of each tile
// (ticket) adds them in split order, so results are deterministic.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "gemm_tc.h"
#include "sm100.cuh"

namespace qtts {
__device__ Crumbs g_crumbs;
cudaError_t set_crumbs_gemm(unsigned* host_mapped_dev_ptr) {
  const Crumbs c{host_mapped_dev_ptr};
  return cudaMemcpyToSymbol(g_crumbs, &c, sizeof(c));
}
namespace {

constexpr int kTcThreads = 192;
constexpr unsigned long long kTcWaitNs = 2000000000ull;  // 2 s: a stall, not a slow step
constexpr int kStageA = kTcRows * kTcBlockK * 2;  // 16 KB: 128 weight rows x 64 K

// Per token-tile width BN (MMA N): stage ring depth and sizes.
template <int BN>
struct TcCfg {
  // 16-row tiles: 4 stages (~82 KB) so two CTAs share an SM and split K further
  static constexpr int kStages = 4;
  static constexpr int kStageB = BN * kTcBlockK * 2;         // hi or lo
  static constexpr int kStageBytes = kStageA + 2 * kStageB;  // multiple of 1024
  // accumulator columns: [0, BN) = W * hi, [BN, 2 BN) = W * lo (one MMA with N = 2 BN)
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  // ring + 1024-byte alignment slack + barriers/flags (256 B) + row scales
  static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024 + 256 + BN * sizeof(float);
  static_assert(3 * kStages * 8 + 8 + 8 <= 256, "barrier area");
  static_assert(kStageBytes % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
};

struct TcArgs {
  const float* x;        // [M, ldx] fp32 activations
  int ldx;
  const float* gamma;    // optional RMSNorm gamma [K]
  float eps;
  int M, N, K;
  int epi;
  int up_off;            // SWIGLU: row offset of the up half in W
  float* y;
  int ldy;
  const float* resid;
  int ldr;
  const float* bias;
  float* rms_out;        // optional [M]: the RMS scale of each row (head selection uses it)
  int* err;
  const int* halt;
  int splits;            // K split over blockIdx.z; > 1 uses ws + tickets
  float* ws;             // [tiles][splits][128][BN] partial tiles, then [tiles][splits][BN] sums
  unsigned* tickets;     // [tiles], zero at rest (reset by the last CTA)
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int BN>
__global__ void __launch_bounds__(kTcThreads, BN <= 16 ? 2 : 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap wmap, TcArgs a) {
  using Cfg = TcCfg<BN>;
  constexpr int S = Cfg::kStages;
  QTTS_CRUMB(0, 100000 + BN * 1000 + a.N / 64);
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);  // weights landed
  uint64_t* bready = full + S;                                                // activations written
  uint64_t* empty = bready + S;                                               // MMAs done
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* s_ss = reinterpret_cast<float*>(last_flag + 1);  // [BN] row sums of squares / RMS

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

  // Thread 0 (the weight producer) initialises the barriers and at once
  // requests the first stages' weight tiles: they depend on nothing, and their
  // latency then overlaps the TMEM allocation and the block barrier below.
  const int pre = min(S, nk);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], 4);  // one arrival per activation warp
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    for (int i = 0; i < pre; ++i) {
      uint8_t* st = smem + i * Cfg::kStageBytes;
      mbar_expect_tx(&full[i], kStageA);
      tma_load_2d(st, &wmap, (kb0 + i) * kTcBlockK, row_a0, &full[i]);
      tma_load_2d(st + kStageA / 2, &wmap, (kb0 + i) * kTcBlockK, row_a1, &full[i]);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // weights: they never depend on the previous kernel, so the first stages
    // are requested before the dependency wait
    int issued = pre;
    for (int i = pre; i < nk; ++i) {
      const int s = i % S;
      if (i >= S && !mbar_wait_ns(&empty[s], ((i / S) & 1) ^ 1, kTcWaitNs)) {
        atomicExch(a.err, 1);
        break;
      }
      uint8_t* st = smem + s * Cfg::kStageBytes;
      mbar_expect_tx(&full[s], kStageA);
      const int kx = (kb0 + i) * kTcBlockK;
      tma_load_2d(st, &wmap, kx, row_a0, &full[s]);
      tma_load_2d(st + kStageA / 2, &wmap, kx, row_a1, &full[s]);
      ++issued;
    }
    // Tail: before the CTA exits, no weight copy may still be landing and no
    // tensor-core commit may still be due to arrive on a stage barrier (a late
    // arrival would hit shared memory that the SM has handed to the next CTA).
    // So wait for the last fill of every stage and for its release.
    for (int i = (issued > S ? issued - S : 0); i < issued; ++i) {
      if (!mbar_wait_ns(&full[i % S], (i / S) & 1, kTcWaitNs)) atomicExch(a.err, 5);
      if (!mbar_wait_ns(&empty[i % S], (i / S) & 1, kTcWaitNs)) atomicExch(a.err, 6);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer
    // hi and lo activation tiles are contiguous rows of one K-major operand, so
    // a single MMA with N = 2 BN multiplies both (half the MMA instructions)
    constexpr uint32_t idesc = umma_idesc_bf16(kTcRows, 2 * BN);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      const unsigned ph = (i / S) & 1;
      if (!mbar_wait_ns(&full[s], ph, kTcWaitNs) || !mbar_wait_ns(&bready[s], ph, kTcWaitNs)) {
        atomicExch(a.err, 2);
        break;
      }
      tc_fence_after();
      uint8_t* st = smem + s * Cfg::kStageBytes;
      const uint64_t da = umma_desc_sw128(st);
      const uint64_t db = umma_desc_sw128(st + kStageA);
#pragma unroll
      for (int kk = 0; kk < kTcBlockK / 16; ++kk)  // +32 bytes per 16-element K step
        umma_bf16(tmem, da + 2 * kk, db + 2 * kk, idesc, (i | kk) != 0);
      umma_commit(&empty[s]);
    }
    umma_commit(done);  // also fires when nothing was issued
  } else if (warp >= 2) {
    const int et = threadIdx.x - 64;  // 0..127 over the activation / epilogue warps
    pdl_wait();
    // Dependents may launch once every CTA is past its wait: their weight
    // tiles then stream in while this GEMM runs (they still wait for its end
    // before reading its output).
    if (et == 0) pdl_trigger();
    const bool halted = a.halt && __ldcg(a.halt);
    // ---- activation producer: hi/lo tiles of gamma * x for every K step ----
    // thread et owns 16-byte chunk c = et % 8 (8 consecutive K) of rows et / 8 + 16 j
    constexpr int kRowsPerThread = BN / 16;
    const int c = et & 7;
    float ss[kRowsPerThread];
#pragma unroll
    for (int j = 0; j < kRowsPerThread; ++j) ss[j] = 0.f;
    // rows of the next PF K steps are in flight while one is converted and
    // stored (PF register buffers, rotated by a loop unrolled PF times)
    constexpr int PF = BN <= 16 ? 4 : 1;
    float4 xq[PF][kRowsPerThread][2], gq[PF][2];
    auto load_step = [&](int i, float4 (&xr)[kRowsPerThread][2], float4 (&gr)[2]) {
      const int k = (kb0 + i) * kTcBlockK + 8 * c;
      if (a.gamma) {
        gr[0] = __ldg(reinterpret_cast<const float4*>(a.gamma + k));
        gr[1] = __ldg(reinterpret_cast<const float4*>(a.gamma + k + 4));
      }
#pragma unroll
      for (int j = 0; j < kRowsPerThread; ++j) {
        const int m = m0 + (et >> 3) + 16 * j;
        if (m < a.M) {
          const float* p = a.x + (long long)m * a.ldx + k;
          xr[j][0] = __ldcg(reinterpret_cast<const float4*>(p));
          xr[j][1] = __ldcg(reinterpret_cast<const float4*>(p + 4));
        } else {
          xr[j][0] = xr[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    };
#pragma unroll
    for (int u = 0; u < PF; ++u)
      if (u < nk) load_step(u, xq[u], gq[u]);
    bool ok = true;
    for (int i0 = 0; i0 < nk && ok; i0 += PF) {
#pragma unroll
      for (int u = 0; u < PF; ++u) {
        const int i = i0 + u;
        if (i >= nk || !ok) break;
        const int s = i % S;
        if (i >= S && !mbar_wait_ns(&empty[s], ((i / S) & 1) ^ 1, kTcWaitNs)) {
          atomicExch(a.err, 4);
          ok = false;
          break;
        }
        uint8_t* st = smem + s * Cfg::kStageBytes;
        const float g[8] = {gq[u][0].x, gq[u][0].y, gq[u][0].z, gq[u][0].w,
                            gq[u][1].x, gq[u][1].y, gq[u][1].z, gq[u][1].w};
#pragma unroll
        for (int j = 0; j < kRowsPerThread; ++j) {
          const int r = (et >> 3) + 16 * j;
          float v[8] = {xq[u][j][0].x, xq[u][j][0].y, xq[u][j][0].z, xq[u][j][0].w,
                        xq[u][j][1].x, xq[u][j][1].y, xq[u][j][1].z, xq[u][j][1].w};
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            ss[j] = fmaf(v[q], v[q], ss[j]);
            if (a.gamma) v[q] *= g[q];
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * q]);
            const __nv_bfloat16 h1 = __float2bfloat16_rn(v[2 * q + 1]);
            hw[q] = pack_bf16(__bfloat162float(h0), __bfloat162float(h1));
            lw[q] = pack_bf16(v[2 * q] - __bfloat162float(h0), v[2 * q + 1] - __bfloat162float(h1));
          }
          // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8)
          const int off = r * 128 + ((c ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(st + kStageA + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(st + kStageA + Cfg::kStageB + off) =
              make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        if (i + PF < nk) load_step(i + PF, xq[u], gq[u]);
        // generic-proxy writes -> visible to the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[s]);
      }
    }
    // row sums of squares: the 8 lanes of a row group hold its partial sums
#pragma unroll
    for (int j = 0; j < kRowsPerThread; ++j) {
      ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], 1);
      ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], 2);
      ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], 4);
    }
    if (c == 0) {
#pragma unroll
      for (int j = 0; j < kRowsPerThread; ++j) s_ss[(et >> 3) + 16 * j] = ss[j];
    }

    // ---- epilogue: this warp's 32 TMEM lanes = tile rows lane_base..lane_base+31 ----
    const int lane_base = 32 * (warp & 3);
    // always wait for the MMAs (even after an error above): the CTA must not
    // free TMEM or exit while tensor-core work is in flight
    const bool got = mbar_wait_ns(done, 0, 2 * kTcWaitNs) && ok;
    if (!got) atomicExch(a.err, 3);
    tc_fence_after();
    const int r = lane_base + lane;
    const int cols = min(BN, a.M - m0);
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    bool final_cta = true;
    asm volatile("bar.sync 1, 128;" ::: "memory");  // s_ss complete
    if (a.splits > 1) {
      // partial tile and partial row sums -> workspace; the last CTA of the
      // tile reduces both in split order
      float* part = a.ws + ((long long)tile * a.splits + blockIdx.z) * kTcRows * BN;
      for (int c0 = 0; c0 < BN; c0 += 16) {
        if (c0 >= cols) break;
        float v[16], w[16];
        tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)c0, v);
        tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(c0 + BN), w);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += w[j];
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          __stcg(reinterpret_cast<float4*>(part + r * BN + c0 + j),
                 make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
      }
      float* ssw = a.ws + (long long)gridDim.x * gridDim.y * a.splits * kTcRows * BN;
      if (et < BN) __stcg(ssw + ((long long)tile * a.splits + blockIdx.z) * BN + et, s_ss[et]);
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (et == 0) {
        const unsigned t = atomicAdd(&a.tickets[tile], 1u);
        *last_flag = t == (unsigned)a.splits - 1u;
        if (*last_flag) a.tickets[tile] = 0u;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      final_cta = *last_flag != 0;
      if (final_cta) {
        __threadfence();
        if (et < BN) {
          float t = 0.f;
          for (int s = 0; s < a.splits; ++s)
            t += __ldcg(ssw + ((long long)tile * a.splits + s) * BN + et);
          s_ss[et] = t;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
    }
    // RMS scale per row (1 without gamma), published for the caller if asked
    if (final_cta && et < BN) {
      const float sc = a.gamma ? rsqrtf(s_ss[et] / (float)a.K + a.eps) : 1.0f;
      s_ss[et] = sc;
      if (a.rms_out && blockIdx.x == 0 && m0 + et < a.M && !halted) a.rms_out[m0 + et] = sc;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
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
        float w[16];
        tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)c0, v);
        tmem_ld16(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(c0 + BN), w);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += w[j];
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
              const float sc = s_ss[c0 + j];
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
            float out = v[j] * s_ss[c0 + j];
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
  QTTS_CRUMB(1, 100000 + BN * 1000 + a.N / 64);
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

bool tc_available() { return encode_fn() != nullptr; }

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

bool tc_supported(const LinearArgs& a, int epi, const TcPlan& p) {
  if (p.tokens != 16 && p.tokens != 64 && p.tokens != 128) return false;
  if (a.K % kTcBlockK || a.ldx % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15)) return false;
  return a.N % (kTcRows / 2) == 0 && a.M >= 1;
}

size_t tc_workspace_floats(int tokens, int sm_count) {
  // partial tiles and row sums for up to 4 x sm_count (tile, split) pairs
  return (size_t)4 * sm_count * ((size_t)kTcRows * tokens + tokens);
}

cudaError_t configure_tc_kernels() {
  cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)TcCfg<128>::kSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_gemm_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)TcCfg<64>::kSmem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_gemm_tc<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)TcCfg<16>::kSmem);
}

cudaError_t launch_linear_tc(const LinearArgs& a, int epi, const TcPlan& p, float* rms_out,
                             int* err, cudaStream_t stream) {
  if (!tc_supported(a, epi, p)) return cudaErrorInvalidValue;
  const int w_rows = epi == EPI_SWIGLU ? 2 * a.N : a.N;
  CUtensorMap wmap;
  if (!tc_weight_map(a.W, w_rows, a.K, &wmap)) return cudaErrorInvalidValue;
  const int BN = p.tokens;
  const int cols_per_cta = epi == EPI_SWIGLU ? kTcRows / 2 : kTcRows;
  dim3 grid((a.N + cols_per_cta - 1) / cols_per_cta, (a.M + BN - 1) / BN, 1);
  // split K so that a skinny GEMM still spreads over the SMs (deterministic
  // reduction by the last CTA of each tile)
  int splits = 1;
  const int tiles = (int)(grid.x * grid.y);
  const int slots = p.sm_count * (BN <= 16 ? 2 : 1);  // resident CTAs
  if (p.ws && tiles < slots) {
    splits = std::min(slots / tiles, (a.K / kTcBlockK) / 4);
    splits = std::max(1, std::min(splits, p.max_splits));
    while (splits > 1 &&
           (size_t)tiles * splits * ((size_t)kTcRows * BN + BN) > p.ws_floats)
      --splits;
  }
  grid.z = splits;
  TcArgs t{a.x, a.ldx, a.gamma, a.eps, a.M, a.N, a.K, epi, a.N, a.y, a.ldy, a.resid, a.ldr,
           a.bias, rms_out, err, a.halt, splits, p.ws, p.tickets};
  if (BN == 16)
    return launch(k_gemm_tc<16>, grid, dim3(kTcThreads), TcCfg<16>::kSmem, stream, wmap, t);
  if (BN == 64)
    return launch(k_gemm_tc<64>, grid, dim3(kTcThreads), TcCfg<64>::kSmem, stream, wmap, t);
  return launch(k_gemm_tc<128>, grid, dim3(kTcThreads), TcCfg<128>::kSmem, stream, wmap, t);
}

}  // namespace qtts
