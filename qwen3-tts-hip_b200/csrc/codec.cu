// Codec decoder kernels for sm_100a (see codec.h). fp32 throughout: the
// reference decoder (src/audio/codec_hip.rs, kernels src/gpu/kernels.rs:453-974)
// is fp32, and the waveform is compared against an fp32 restatement.
#include <math.h>

#include "codec.h"
#include "common.cuh"

namespace qtts {
namespace {

constexpr int kTileT = 128, kTileK = 16, kConvThreads = 256;

template <int ACT>
__device__ __forceinline__ float codec_act(const CodecConvArgs& a, int ci, int src) {
  const long long ld = (long long)a.lin + a.hist;
  const float x = __ldg(a.x + ci * ld + a.hist + src);
  if (ACT == CACT_SNAKE) {
    const float s = sinf(x * __ldg(a.act_a + ci));
    return x + (s * s) / (__ldg(a.act_b + ci) + 1.0e-9f);
  }
  if (ACT == CACT_SWIGLU) {
    const float u = __ldg(a.x + (ci + a.up_off) * ld + a.hist + src);
    return x / (1.0f + expf(-x)) * u;
  }
  return x;
}

__device__ __forceinline__ float snake(float x, float a, float b) {
  const float s = sinf(x * a);
  return x + (s * s) / (b + 1.0e-9f);
}

// BM output channels (64 or 128) x 128 input positions per CTA, K (= ci *
// taps) in chunks of 16 through shared memory, the next chunk's global loads
// held in registers while the current one is multiplied. Thread (ty, tx)
// owns channels MR ty .. MR ty + MR - 1 (MR = BM / 16) and positions
// 4 tx .. 4 tx + 3 and 64 + 4 tx .. 64 + 4 tx + 3, all read from shared
// memory as float4s. The input tile is gathered on the fly (implicit
// im2col) with the input transform applied once per loaded element.
template <int ACT, int TAPS, int BM>  // TAPS 0: taps read at run time
__global__ void __launch_bounds__(kConvThreads) k_codec_conv(CodecConvArgs a) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  constexpr int MR = BM / 16, AL = BM * kTileK / kConvThreads;
  static_assert(AL >= 1 && MR >= 1, "row tile must give every thread an A element");
  const int taps = TAPS ? TAPS : a.taps;
  __shared__ __align__(16) float As[kTileK][BM + 4];  // padded: transposed stores
  __shared__ __align__(16) float Bs[kTileK][kTileT];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  // Phase varies fastest across blockIdx.x: the nphase CTAs of one tile run
  // together, so L2 merges their interleaved (stride-nphase) output columns
  // into whole sectors instead of writing partial ones back to HBM.
  const int ph = blockIdx.x % a.nphase;
  const int t0 = (blockIdx.x / a.nphase) * kTileT, co0 = blockIdx.y * BM;
  const float* W = a.w + (long long)ph * a.w_phase_stride;
  const int K = a.ci * taps;
  float acc[MR][8];
#pragma unroll
  for (int i = 0; i < MR; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  float ra[AL], rb[8];
  auto load = [&](int k0) {
#pragma unroll
    for (int r = 0; r < AL; ++r) {  // A: BM (co) x 16 (kk)
      const int idx = tid + r * kConvThreads;
      const int row = idx >> 4, col = idx & 15;
      const int co = co0 + row, kk = k0 + col;
      ra[r] = (co < a.co && kk < K) ? __ldg(W + (long long)co * K + kk) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {  // B: 16 (kk) x 128 (t)
      const int idx = tid + r * kConvThreads;
      const int row = idx >> 7, col = idx & 127;
      const int kk = k0 + row, t = t0 + col;
      float v = 0.f;
      if (kk < K && t < a.lin) {
        const int ci = kk / taps, tap = kk - ci * taps;
        const int src = t + tap * a.dil - a.pad;
        if (src >= -a.hist && src < a.lin) v = codec_act<ACT>(a, ci, src);
      }
      rb[r] = v;
    }
  };
  auto store = [&]() {
#pragma unroll
    for (int r = 0; r < AL; ++r) {
      const int idx = tid + r * kConvThreads;
      As[idx & 15][idx >> 4] = ra[r];
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int idx = tid + r * kConvThreads;
      Bs[idx >> 7][idx & 127] = rb[r];
    }
  };

  load(0);
  for (int k0 = 0; k0 < K; k0 += kTileK) {
    store();
    __syncthreads();
    if (k0 + kTileK < K) load(k0 + kTileK);  // in flight during the FMAs below
#pragma unroll
    for (int kk = 0; kk < kTileK; ++kk) {
      float ar[MR];
      if constexpr (MR % 4 == 0) {
#pragma unroll
        for (int q = 0; q < MR / 4; ++q) {
          const float4 av = *reinterpret_cast<const float4*>(&As[kk][MR * ty + 4 * q]);
          ar[4 * q] = av.x; ar[4 * q + 1] = av.y; ar[4 * q + 2] = av.z; ar[4 * q + 3] = av.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < MR; ++i) ar[i] = As[kk][MR * ty + i];
      }
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][4 * tx]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][64 + 4 * tx]);
      const float br[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < MR; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }

  const long long lout = (long long)a.lin * a.ostride;
#pragma unroll
  for (int i = 0; i < MR; ++i) {
    const int co = co0 + MR * ty + i;
    if (co >= a.co) continue;
    const float b = a.bias ? __ldg(a.bias + co) : 0.f;
    const float rs = a.rscale ? __ldg(a.rscale + co) : 1.f;
    const float sa = a.out_a ? __ldg(a.out_a + co) : 0.f;
    const float sb = a.out_a ? __ldg(a.out_b + co) : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = t0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + (j - 4));
      if (t >= a.lin) continue;
      float v = acc[i][j] + b;
      if (a.epi & CEPI_GELU) v = 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
      const long long o = (long long)co * lout + (long long)t * a.ostride + ph;
      if (a.epi & CEPI_RESID) v = a.resid[o] + v * rs;
      if (a.epi & CEPI_CLAMP) v = fminf(fmaxf(v, -1.0f), 1.0f);
      if (a.epi & CEPI_SNAKE) {
        a.y[o] = snake(v, sa, sb);
      } else {
        a.y[o] = v;
        if (a.y2) a.y2[o] = snake(v, sa, sb);
      }
    }
  }
}

__global__ void k_codec_rvq_gather(const int32_t* codes, int frames, int groups, int cb_size,
                                   int cb_dim, const float* cb_first, const float* cb_rest,
                                   float* first, float* rest) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  const int t = blockIdx.x;
  if (t >= frames) return;
  auto code_of = [&](int g) {
    int c = codes[t * groups + g] % cb_size;
    return c < 0 ? c + cb_size : c;
  };
  const int c0 = code_of(0);
  for (int d = threadIdx.x; d < cb_dim; d += blockDim.x) {
    first[(long long)t * cb_dim + d] = cb_first[(long long)c0 * cb_dim + d];
    float r = 0.f;
    for (int g = 1; g < groups; ++g)
      r += cb_rest[((long long)(g - 1) * cb_size + code_of(g)) * cb_dim + d];
    rest[(long long)t * cb_dim + d] = r;
  }
}

// One warp per output (channel c, frame t): lanes split the codebook
// dimension (coalesced weight and embedding rows), then a warp reduction.
__global__ void k_codec_rvq_project(const float* first, const float* rest, const float* wf,
                                    const float* wr, int frames, int cb_dim, int out_dim,
                                    float* y) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)frames * out_dim) return;
  const int t = (int)(w % frames), c = (int)(w / frames);
  const float* a = wf + (long long)c * cb_dim;
  const float* b = wr + (long long)c * cb_dim;
  const float* f = first + (long long)t * cb_dim;
  const float* r = rest + (long long)t * cb_dim;
  float s = 0.f;
  for (int d = lane; d < cb_dim; d += 32) s += a[d] * f[d] + b[d] * r[d];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) y[(long long)c * frames + t] = s;
}

// 32 time steps per CTA (one per lane, so every load is a coalesced 128-byte
// row segment) and 32 warps splitting the channels, four loads in flight per
// thread; the per-warp sums meet in shared memory. Short inputs (streamed
// chunks) then still spread a channel sum over 32 warps.
constexpr int kNormWarps = 32;
__global__ void __launch_bounds__(kNormWarps * 32) k_codec_chan_norm(const float* x, int C, int T,
                                                                  const float* gamma,
                                                                  const float* beta, float eps,
                                                                  float* y) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  __shared__ float s_sum[kNormWarps][33], s_sq[kNormWarps][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * 32 + lane;
  const bool on = t < T;
  float s = 0.f, ss = 0.f;
  if (on) {
    int c = warp;
    for (; c + 3 * kNormWarps < C; c += 4 * kNormWarps) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = x[(long long)(c + u * kNormWarps) * T + t];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        s += v[u];
        ss += v[u] * v[u];
      }
    }
    for (; c < C; c += kNormWarps) {
      const float v = x[(long long)c * T + t];
      s += v;
      ss += v * v;
    }
  }
  s_sum[warp][lane] = s;
  s_sq[warp][lane] = ss;
  __syncthreads();
  s = 0.f;
  ss = 0.f;
#pragma unroll 8
  for (int w = 0; w < kNormWarps; ++w) {
    s += s_sum[w][lane];
    ss += s_sq[w][lane];
  }
  if (!on) return;
  if (beta) {  // LayerNorm (codec_layernorm_f32, kernels.rs:613-660)
    const float mean = s / (float)C;
    const float var = fmaxf(ss / (float)C - mean * mean, 0.0f);
    const float inv = rsqrtf(var + eps);
    for (int c = warp; c < C; c += kNormWarps)
      y[(long long)c * T + t] = (x[(long long)c * T + t] - mean) * inv * gamma[c] + beta[c];
  } else {  // RMSNorm (rmsnorm_f32, kernels.rs:2-37)
    const float inv = rsqrtf(ss / (float)C + eps);
    for (int c = warp; c < C; c += kNormWarps)
      y[(long long)c * T + t] = x[(long long)c * T + t] * inv * gamma[c];
  }
}

__global__ void k_codec_dwconv(const float* x, int C, int T, int hist, const float* w,
                               const float* b, int K, float* y) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= C * T) return;
  const int t = idx % T, c = idx / T;
  const float* xr = x + (long long)c * (T + hist) + hist;
  float s = b[c];
  for (int k = 0; k < K; ++k) {
    const int src = t + k - (K - 1);
    if (src >= -hist) s += xr[src] * w[c * K + k];
  }
  y[idx] = s;
}

// cat[c] = [state_cur[c] (H columns) | x[c] (n columns)] and state_next[c] =
// the last H columns of cat[c].
__global__ void k_codec_hist_cat(const float* state_cur, const float* x, int C, int H, int n,
                                 float* cat, float* state_next) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  const long long W = (long long)H + n;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= C * W) return;
  const int c = (int)(idx / W), j = (int)(idx % W);
  const float v = j < H ? state_cur[(long long)c * H + j] : x[(long long)c * n + (j - H)];
  cat[idx] = v;
  if (j >= n) state_next[(long long)c * H + (j - n)] = v;
}

// rope_bhsd_f32 (kernels.rs:40-77): angle = position / theta^(2i/hd),
// rotate-half; positions pos0 .. pos0 + T - 1. k and v land in the caches
// [heads][cap][hd] at those positions.
__global__ void k_codec_qkv_rope(const float* qkv, int heads, int hd, int T, int pos0, int cap,
                                 float theta, float* q, float* k, float* v) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int per = heads * T * hd;
  if (idx >= per) return;
  const int d = idx % hd, t = (idx / hd) % T, h = idx / (hd * T);
  const int half = hd / 2, pair = d % half;
  const float expo = (float)(pair * 2) / (float)hd;
  const float ang = (float)(pos0 + t) / powf(theta, expo);
  const float c = cosf(ang), s = sinf(ang);
  const int qo = heads * hd;
  auto rot = [&](int base) {
    const float first = qkv[(long long)(base + h * hd + pair) * T + t];
    const float second = qkv[(long long)(base + h * hd + pair + half) * T + t];
    return d < half ? first * c - second * s : second * c + first * s;
  };
  q[idx] = rot(0);
  const long long at = ((long long)h * cap + pos0 + t) * hd + d;
  k[at] = rot(qo);
  v[at] = qkv[(long long)(2 * qo + h * hd + d) * T + t];
}

// One warp per (head, query position), keys in chunks of 32 with one key per
// lane: a lane scores its key against the whole query (q in registers), the
// warp updates the online softmax once per chunk, and lane l accumulates
// output dims 2l, 2l + 1 with the chunk's weights broadcast by shuffles.
__global__ void k_codec_attention(const float* q, const float* k, const float* v, int heads,
                                  int T, int pos0, int cap, float scale, float* out) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  constexpr int HD = 64;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= heads * T) return;
  const int h = warp / T, t = warp % T;
  const float4* qr = reinterpret_cast<const float4*>(q + ((long long)h * T + t) * HD);
  float4 qv[HD / 4];
#pragma unroll
  for (int i = 0; i < HD / 4; ++i) {
    qv[i] = __ldg(qr + i);  // the same row in every lane: broadcast
    qv[i].x *= scale; qv[i].y *= scale; qv[i].z *= scale; qv[i].w *= scale;
  }
  const float* kh = k + (long long)h * cap * HD;
  const float* vh = v + (long long)h * cap * HD;
  const int n = pos0 + t + 1;  // keys 0 .. pos0 + t
  float m = -INFINITY, l = 0.f, a0 = 0.f, a1 = 0.f;
  for (int j0 = 0; j0 < n; j0 += 32) {
    const int j = j0 + lane;
    float sc = -INFINITY;
    if (j < n) {
      const float4* kr = reinterpret_cast<const float4*>(kh + (long long)j * HD);
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int i = 0; i < HD / 4; i += 2) {
        const float4 a = __ldg(kr + i), b = __ldg(kr + i + 1);
        s0 = fmaf(qv[i].x, a.x, s0); s0 = fmaf(qv[i].y, a.y, s0);
        s0 = fmaf(qv[i].z, a.z, s0); s0 = fmaf(qv[i].w, a.w, s0);
        s1 = fmaf(qv[i + 1].x, b.x, s1); s1 = fmaf(qv[i + 1].y, b.y, s1);
        s1 = fmaf(qv[i + 1].z, b.z, s1); s1 = fmaf(qv[i + 1].w, b.w, s1);
      }
      sc = s0 + s1;
    }
    float cm = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    const float mn = fmaxf(m, cm);
    const float corr = expf(m - mn);
    const float e = j < n ? expf(sc - mn) : 0.f;
    float es = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) es += __shfl_xor_sync(0xffffffffu, es, o);
    l = l * corr + es;
    a0 *= corr;
    a1 *= corr;
    const int cnt = min(32, n - j0);
    for (int jj = 0; jj < cnt; ++jj) {
      const float w = __shfl_sync(0xffffffffu, e, jj);
      const float2 vv = __ldg(reinterpret_cast<const float2*>(vh + (long long)(j0 + jj) * HD) + lane);
      a0 = fmaf(w, vv.x, a0);
      a1 = fmaf(w, vv.y, a1);
    }
    m = mn;
  }
  const float il = 1.0f / l;
  out[(long long)(h * HD + 2 * lane) * T + t] = a0 * il;
  out[(long long)(h * HD + 2 * lane + 1) * T + t] = a1 * il;
}

__global__ void k_codec_exp(const float* x, int n, float* y) {
  pdl_wait();  // inputs come from the previous kernel on the stream
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = expf(x[i]);
}

inline unsigned blocks(long long n, int per) { return (unsigned)((n + per - 1) / per); }

}  // namespace

// Every codec kernel is launched with programmatic dependent launch: it waits
// for the previous kernel's completion before touching memory and lets the
// next one launch right away, so a decode's ~350 launches do not each pay the
// full launch latency.
template <int BM>
static cudaError_t codec_conv_bm(const CodecConvArgs& a, cudaStream_t stream) {
  const dim3 grid(blocks(a.lin, kTileT) * a.nphase, blocks(a.co, BM), 1);
  const dim3 block(kConvThreads);
  if (a.act == CACT_SNAKE) return launch(k_codec_conv<CACT_SNAKE, 0, BM>, grid, block, 0, stream, a);
  if (a.act == CACT_SWIGLU) return launch(k_codec_conv<CACT_SWIGLU, 0, BM>, grid, block, 0, stream, a);
  switch (a.taps) {  // constant taps: the im2col index split is a multiply, not a divide
    case 1: return launch(k_codec_conv<CACT_NONE, 1, BM>, grid, block, 0, stream, a);
    case 2: return launch(k_codec_conv<CACT_NONE, 2, BM>, grid, block, 0, stream, a);
    case 3: return launch(k_codec_conv<CACT_NONE, 3, BM>, grid, block, 0, stream, a);
    case 7: return launch(k_codec_conv<CACT_NONE, 7, BM>, grid, block, 0, stream, a);
    default: return launch(k_codec_conv<CACT_NONE, 0, BM>, grid, block, 0, stream, a);
  }
}

cudaError_t codec_conv(const CodecConvArgs& a, cudaStream_t stream) {
  if (a.ci <= 0 || a.co <= 0 || a.lin <= 0 || a.taps <= 0 || a.nphase <= 0 || a.ostride <= 0 ||
      a.hist < 0)
    return cudaErrorInvalidValue;
  // 64-channel tiles, except a 16-channel tile for the final 96 -> 1
  // convolution (a 64-row tile would spend 63/64 of its FMAs on padding) and
  // 32-channel tiles for the 96-channel block (three exact tiles, not two
  // 64-row tiles of which a quarter is padding).
  // 128-channel tiles (8 x 8 per thread, ~168 registers, one CTA per SM)
  // measured slower.
  if (a.co <= 16) return codec_conv_bm<16>(a, stream);
  if (a.co % 64 != 0 && a.co % 32 == 0) return codec_conv_bm<32>(a, stream);  // 96 channels
  return codec_conv_bm<64>(a, stream);
}

cudaError_t codec_rvq(const int32_t* codes, int frames, int groups, int cb_size, int cb_dim,
                      const float* cb_first, const float* cb_rest, const float* wf,
                      const float* wr, int out_dim, float* first, float* rest, float* y,
                      cudaStream_t stream) {
  cudaError_t e = launch(k_codec_rvq_gather, dim3(frames), dim3(256), 0, stream, codes, frames,
                         groups, cb_size, cb_dim, cb_first, cb_rest, first, rest);
  if (e != cudaSuccess) return e;
  return launch(k_codec_rvq_project, dim3(blocks((long long)frames * out_dim * 32, 256)),
                dim3(256), 0, stream, (const float*)first, (const float*)rest, wf, wr, frames,
                cb_dim, out_dim, y);
}

cudaError_t codec_chan_norm(const float* x, int C, int T, const float* gamma, const float* beta,
                            float eps, float* y, cudaStream_t stream) {
  return launch(k_codec_chan_norm, dim3(blocks(T, 32)), dim3(kNormWarps * 32), 0, stream, x, C,
                T, gamma, beta, eps, y);
}

cudaError_t codec_dwconv(const float* x, int C, int T, int hist, const float* w, const float* b,
                         int K, float* y, cudaStream_t stream) {
  if (hist < 0 || hist > K - 1) return cudaErrorInvalidValue;
  return launch(k_codec_dwconv, dim3(blocks((long long)C * T, 256)), dim3(256), 0, stream, x, C,
                T, hist, w, b, K, y);
}

cudaError_t codec_hist_cat(const float* state_cur, const float* x, int C, int H, int n,
                           float* cat, float* state_next, cudaStream_t stream) {
  if (C <= 0 || H <= 0 || n <= 0) return cudaErrorInvalidValue;
  return launch(k_codec_hist_cat, dim3(blocks((long long)C * (H + n), 256)), dim3(256), 0,
                stream, state_cur, x, C, H, n, cat, state_next);
}

cudaError_t codec_qkv_rope(const float* qkv, int heads, int hd, int T, int pos0, int cap,
                           float theta, float* q, float* k, float* v, cudaStream_t stream) {
  if (pos0 < 0 || pos0 + T > cap) return cudaErrorInvalidValue;
  return launch(k_codec_qkv_rope, dim3(blocks((long long)heads * T * hd, 256)), dim3(256), 0,
                stream, qkv, heads, hd, T, pos0, cap, theta, q, k, v);
}

cudaError_t codec_attention(const float* q, const float* k, const float* v, int heads, int hd,
                            int T, int pos0, int cap, float scale, float* out,
                            cudaStream_t stream) {
  if (hd != 64 || pos0 < 0 || pos0 + T > cap) return cudaErrorInvalidValue;
  return launch(k_codec_attention, dim3(blocks((long long)heads * T * 32, 256)), dim3(256), 0,
                stream, q, k, v, heads, T, pos0, cap, scale, out);
}

cudaError_t codec_exp(const float* x, int n, float* y, cudaStream_t stream) {
  return launch(k_codec_exp, dim3(blocks(n, 256)), dim3(256), 0, stream, x, n, y);
}

}  // namespace qtts
