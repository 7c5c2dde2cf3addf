// Fused decode MLP: y = r + down(silu(gate(n)) * up(n)), n = RMSNorm(r) * gamma,
// for one position, in one kernel (decode.rs:1694-1894, post-attention half of
// decode_step_layer_on_stream: post_attention_layernorm, gate|up GEMV, SwiGLU,
// down GEMV + residual).
//
// The two-kernel form (gate|up GEMV, then the down GEMV) costs one extra
// dependent launch per layer. Here CTA j owns intermediate channels
// [j*ni, (j+1)*ni): it streams its gate rows, up rows and the matching rows of
// the TRANSPOSED down matrix (down^T is [I x H], so a channel's down weights
// are contiguous) into shared memory with three bulk copies issued before the
// dependency wait, computes its ni SwiGLU activations, and its partial output
// p_j = down^T[slice]^T * act[slice] over all H columns. The H-wide partials
// are then summed deterministically:
//   1. inside each cluster of CL CTAs (8, 4 or 2) through distributed shared
//      memory, CTA rank r summing columns [r*H/CL, (r+1)*H/CL) over ranks
//      0..CL-1 in order;
//   2. across the 128/CL clusters through a global workspace: each rank-r CTA
//      writes its column slice, takes a ticket, and the last one sums the
//      slices in cluster order, adds the residual and writes y.
// The summation order is fixed, so results are bit-reproducible run to run.
// Included by kernels.cu (shares its step-trace and breadcrumb symbols).
#pragma once
#include "sm100.cuh"

namespace qtts {

namespace {

constexpr int kMlpThreads = 256;
constexpr int kMlpWarps = kMlpThreads / 32;
constexpr unsigned long long kMlpWaitNs = 2000000000ull;  // 2 s

struct MlpSmem {
  // byte offsets within the dynamic shared memory block
  unsigned wg, wu, wd, xs, part, grp, act, red, bar, total;
};

__host__ __device__ inline MlpSmem mlp_smem(int H, int ni) {
  MlpSmem m;
  const unsigned rows = (unsigned)ni * (unsigned)H * 2u;
  m.bar = 0;
  m.wg = 128;
  m.wu = m.wg + rows;
  m.wd = m.wu + rows;
  m.xs = m.wd + rows;
  m.part = m.xs + (unsigned)H * 4u;
  m.grp = m.part + (unsigned)H * 4u;
  m.act = m.grp + kMlpThreads * 16u;
  m.red = m.act + (((unsigned)ni * 4u + 15u) & ~15u);
  m.total = m.red + kMlpWarps * 4u;
  return m;
}

template <int KCH, int CL>
__global__ void __launch_bounds__(kMlpThreads) k_mlp_fused(MlpArgs a) {
  QTTS_CRUMB(0, 20);
  constexpr int H = KCH * 256;
  extern __shared__ __align__(128) unsigned char smem[];
  const int ni = a.I / gridDim.x;
  const MlpSmem L = mlp_smem(H, ni);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
  const __nv_bfloat16* wg = reinterpret_cast<const __nv_bfloat16*>(smem + L.wg);
  const __nv_bfloat16* wu = reinterpret_cast<const __nv_bfloat16*>(smem + L.wu);
  const __nv_bfloat16* wd = reinterpret_cast<const __nv_bfloat16*>(smem + L.wd);
  float* xs = reinterpret_cast<float*>(smem + L.xs);
  float* part = reinterpret_cast<float*>(smem + L.part);
  float* act = reinterpret_cast<float*>(smem + L.act);
  float* red = reinterpret_cast<float*>(smem + L.red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long c0 = (long long)blockIdx.x * ni;
  trace_mark(a.trace_id, 0);

  // Weights never depend on the previous kernel: fetch them before the wait.
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    const unsigned bytes = (unsigned)ni * H * 2u;
    const uint64_t pol = l2_evict_first_policy();
    mbar_expect_tx(bar, 3u * bytes);
    bulk_g2s(smem + L.wg, a.Wgu + c0 * H, bytes, bar, pol);
    bulk_g2s(smem + L.wu, a.Wgu + ((long long)a.I + c0) * H, bytes, bar, pol);
    bulk_g2s(smem + L.wd, a.WdT + c0 * H, bytes, bar, pol);
  }
  if (a.trigger == 0) pdl_trigger();
  pdl_wait();
  trace_mark(a.trace_id, 1);
  const unsigned long long tw = trace_clock(a.trace_id);
  if (a.trigger == 1) pdl_trigger();
  const int halted = a.halt ? __ldcg(a.halt) : 0;

  // Stage gamma * r once; the RMSNorm sum of squares comes from the same pass.
  float ss = 0.f;
#pragma unroll
  for (int k = threadIdx.x * 4; k < H; k += kMlpThreads * 4) {
    float4 v = __ldcg(reinterpret_cast<const float4*>(a.x + k));
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    const float4 g = __ldg(reinterpret_cast<const float4*>(a.gamma + k));
    v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
    *reinterpret_cast<float4*>(xs + k) = v;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kMlpWarps; ++i) t += red[i];
  const float sc = rsqrtf(t / (float)H + a.eps);

  // Every thread waits for the weights (also when halted: no CTA may exit
  // with a bulk copy still landing in its shared memory).
  if (!mbar_wait_ns(bar, 0, kMlpWaitNs)) {
    if (threadIdx.x == 0 && a.err) atomicExch(a.err, 7);
  }
  if (halted) return;  // uniform across the grid: no cluster barrier is skipped by half
  trace_mark(a.trace_id, 4);

  // SwiGLU activations of this CTA's channels: warp w takes channels w, w+8, ...
  float4 x0[KCH], x1[KCH];
#pragma unroll
  for (int j = 0; j < KCH; ++j) {
    x0[j] = *reinterpret_cast<const float4*>(xs + j * 256 + lane * 8);
    x1[j] = *reinterpret_cast<const float4*>(xs + j * 256 + lane * 8 + 4);
  }
  for (int c = warp; c < ni; c += kMlpWarps) {
    float g = 0.f, u = 0.f;
#pragma unroll
    for (int j = 0; j < KCH; ++j) {
      const uint4 wgv = *reinterpret_cast<const uint4*>(wg + (long long)c * H + j * 256 + lane * 8);
      const uint4 wuv = *reinterpret_cast<const uint4*>(wu + (long long)c * H + j * 256 + lane * 8);
      float f[8], e[8];
      unpack8(wgv, f);
      unpack8(wuv, e);
      g = fmaf(f[0], x0[j].x, g); g = fmaf(f[1], x0[j].y, g);
      g = fmaf(f[2], x0[j].z, g); g = fmaf(f[3], x0[j].w, g);
      g = fmaf(f[4], x1[j].x, g); g = fmaf(f[5], x1[j].y, g);
      g = fmaf(f[6], x1[j].z, g); g = fmaf(f[7], x1[j].w, g);
      u = fmaf(e[0], x0[j].x, u); u = fmaf(e[1], x0[j].y, u);
      u = fmaf(e[2], x0[j].z, u); u = fmaf(e[3], x0[j].w, u);
      u = fmaf(e[4], x1[j].x, u); u = fmaf(e[5], x1[j].y, u);
      u = fmaf(e[6], x1[j].z, u); u = fmaf(e[7], x1[j].w, u);
    }
    g = warp_sum(g) * sc;
    u = warp_sum(u) * sc;
    if (lane == 0) act[c] = g / (1.0f + expf(-g)) * u;
  }
  __syncthreads();

  // Partial down projection over this CTA's channels, 4 columns per thread.
  for (int h = threadIdx.x * 4; h < H; h += kMlpThreads * 4) {
    float4 p = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = 0; c < ni; ++c) {
      const float av = act[c];
      const uint2 w = *reinterpret_cast<const uint2*>(wd + (long long)c * H + h);
      p.x = fmaf(av, bf16lo(w.x), p.x); p.y = fmaf(av, bf16hi(w.x), p.y);
      p.z = fmaf(av, bf16lo(w.y), p.z); p.w = fmaf(av, bf16hi(w.y), p.w);
    }
    *reinterpret_cast<float4*>(part + h) = p;
  }

  // 1. Cluster sum through distributed shared memory, ranks in order.
  cluster_arrive();
  cluster_wait();
  const unsigned rank = cluster_rank(), cl = cluster_index();
  constexpr int kCols = H / CL;            // columns this rank reduces
  constexpr int kVec = kCols / 4;          // float4 groups
  constexpr int kNcl = kMlpCtas / CL;      // clusters
  static_assert(kVec <= kMlpThreads, "column slice wider than the CTA");
  if (threadIdx.x < kVec) {
    const int col = rank * kCols + threadIdx.x * 4;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (unsigned r = 0; r < (unsigned)CL; ++r) {
      const float4 v = ld_cluster_f4(cluster_map(part + col, r));
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    __stcg(reinterpret_cast<float4*>(a.ws + (long long)cl * H + col), s);
  }
  // Peers may still be reading this CTA's partials: arrive now, wait at exit.
  cluster_arrive();
  trace_dur(a.trace_id, 6, tw);

  // 2. Cross-cluster sum by the last rank-r CTA to finish its slice.
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.tickets + rank, 1u);
    s_last = prev == kNcl - 1;
  }
  __syncthreads();
  trace_dur(a.trace_id, 7, tw);
  if (s_last) {
    __threadfence();
    // kParts thread groups each sum kPer clusters (all loads in flight at
    // once), then the group sums are added in group order: a fixed tree.
    constexpr int kParts = kMlpThreads / kVec < kNcl ? kMlpThreads / kVec : kNcl;
    constexpr int kPer = kNcl / kParts;
    static_assert(kNcl % kParts == 0, "cluster count must split evenly");
    // (not `part`: cluster peers may still be reading it)
    float4* grp = reinterpret_cast<float4*>(smem + L.grp);
    const int v = threadIdx.x % kVec, g = threadIdx.x / kVec;
    const int col = rank * kCols + v * 4;
    if (g < kParts) {
      float4 vals[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k)
        vals[k] = __ldcg(reinterpret_cast<const float4*>(a.ws + (long long)(g * kPer + k) * H + col));
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        acc.x += vals[k].x; acc.y += vals[k].y; acc.z += vals[k].z; acc.w += vals[k].w;
      }
      grp[g * kVec + v] = acc;
    }
    const float4 r = threadIdx.x < kVec ? __ldcg(reinterpret_cast<const float4*>(a.x + col))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    if (threadIdx.x < kVec) {
      float4 acc = grp[v];
#pragma unroll
      for (int k = 1; k < kParts; ++k) {
        const float4 t4 = grp[k * kVec + v];
        acc.x += t4.x; acc.y += t4.y; acc.z += t4.z; acc.w += t4.w;
      }
      *reinterpret_cast<float4*>(a.y + col) =
          make_float4(r.x + acc.x, r.y + acc.y, r.z + acc.z, r.w + acc.w);
    }
    if (threadIdx.x == 0) a.tickets[rank] = 0u;  // ready for the next launch
  }
  trace_mark(a.trace_id, 2);
  cluster_wait();
}

// dst[c, r] = src[r, c] for a [rows x cols] bf16 matrix (32 x 32 tiles).
__global__ void k_transpose_bf16(const __nv_bfloat16* src, int rows, int cols,
                                 __nv_bfloat16* dst) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = blockIdx.y * 32 + i;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[(long long)r * cols + c];
  }
  __syncthreads();
  const int r = blockIdx.y * 32 + threadIdx.x;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int cc = blockIdx.x * 32 + i;
    if (r < rows && cc < cols) dst[(long long)cc * rows + r] = tile[threadIdx.x][i];
  }
}

template <int KCH, int CL>
cudaError_t launch_mlp_kch(const MlpArgs& a, cudaStream_t stream) {
  const int ni = a.I / kMlpCtas;
  const size_t smem = mlp_smem(KCH * 256, ni).total;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kMlpCtas);
  cfg.blockDim = dim3(kMlpThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = CL;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, k_mlp_fused<KCH, CL>, a);
}

}  // namespace

size_t mlp_fused_smem(int H, int I) { return mlp_smem(H, I / kMlpCtas).total; }

bool mlp_fused_supported(int H, int I) {
  if (H != 256 && H != 512 && H != 1024) return false;
  if (I <= 0 || I % kMlpCtas != 0) return false;
  return mlp_fused_smem(H, I) <= kMlpMaxSmem;
}

template <int CL>
void (*mlp_kernel(int H))(MlpArgs) {
  return H == 256 ? k_mlp_fused<1, CL> : H == 512 ? k_mlp_fused<2, CL> : k_mlp_fused<4, CL>;
}

cudaError_t configure_mlp_fused(int H, int I, int cluster, int* active_clusters) {
  if (!mlp_fused_supported(H, I)) return cudaErrorInvalidValue;
  const int smem = (int)mlp_fused_smem(H, I);
  void (*k)(MlpArgs) = cluster == 8 ? mlp_kernel<8>(H) : cluster == 4 ? mlp_kernel<4>(H)
                       : cluster == 2 ? mlp_kernel<2>(H) : nullptr;
  if (!k) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  if (active_clusters) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kMlpCtas);
    cfg.blockDim = dim3(kMlpThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaOccupancyMaxActiveClusters(active_clusters, k, &cfg);
  }
  return e;
}

cudaError_t launch_mlp_fused(const MlpArgs& a, cudaStream_t stream) {
  if (!mlp_fused_supported(a.H, a.I)) return cudaErrorInvalidValue;
  switch (a.cluster * 4096 + a.H) {
    case 8 * 4096 + 256: return launch_mlp_kch<1, 8>(a, stream);
    case 8 * 4096 + 512: return launch_mlp_kch<2, 8>(a, stream);
    case 8 * 4096 + 1024: return launch_mlp_kch<4, 8>(a, stream);
    case 4 * 4096 + 256: return launch_mlp_kch<1, 4>(a, stream);
    case 4 * 4096 + 512: return launch_mlp_kch<2, 4>(a, stream);
    case 4 * 4096 + 1024: return launch_mlp_kch<4, 4>(a, stream);
    case 2 * 4096 + 256: return launch_mlp_kch<1, 2>(a, stream);
    case 2 * 4096 + 512: return launch_mlp_kch<2, 2>(a, stream);
    case 2 * 4096 + 1024: return launch_mlp_kch<4, 2>(a, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_transpose_bf16(const __nv_bfloat16* src, int rows, int cols,
                                  __nv_bfloat16* dst, cudaStream_t stream) {
  dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  k_transpose_bf16<<<grid, dim3(32, 8), 0, stream>>>(src, rows, cols, dst);
  return cudaGetLastError();
}

}  // namespace qtts
