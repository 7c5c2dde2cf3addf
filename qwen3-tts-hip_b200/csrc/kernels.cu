// sm_100a kernels for the Qwen3-TTS token loop (talker decode step + CodePredictor pass).
//
// Reference semantics (piedshag/qwen3-tts-hip):
//   projections      rocBLAS sgemm row-major          src/gpu/blas.rs:134-151
//   RMSNorm          rmsnorm_f32                       src/gpu/kernels.rs:2-37
//   RoPE             rope_bhsd_f32 (rotate-half)       src/gpu/kernels.rs:41-76
//   SwiGLU/residual  swiglu_f32 / residual_add_f32     src/gpu/kernels.rs:80-117
//   decode attention scores/softmax/apply (GQA)        src/gpu/kernels.rs:1048-1119,121-173
//   KV write         write_kv_cache_f32                src/gpu/kernels.rs:1121-1144
//   suppression      suppress_codec_logits_f32         src/gpu/kernels.rs:248-263
//   penalty          apply_repetition_penalty_f32      src/gpu/kernels.rs:408-426
//   argmax / top-k   argmax_rows_f32 / sample_topk_f32 src/gpu/kernels.rs:177-220,265-336
//   CPU sampler/LCG  select_token / sample / next_f32  src/model/sampling.rs:40-126
//
// Design: weights are bf16 [out, in] rows streamed once per step with 16-byte
// non-allocating loads; activations stay fp32; the KV cache is paged bf16.
// Norm prologues, QK-norm + RoPE + KV append, residual/SwiGLU/bias epilogues,
// split-K attention combine, and token selection + embedding gathers are fused
// into the kernels that produce their inputs, so one decoder layer is four
// launches and a token head is one.
#include <float.h>

#include "kernels.h"
#include "select.cuh"

namespace qtts {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxVocab = kSelMaxVocab;
constexpr int kXFloats = 12288;  // 48 KB fp32 activation tile per block

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// ---------------------------------------------------------------------------
// Step trace (profiling aid): per launch, the first CTA entry, the first CTA
// past the dependency wait and the last CTA exit, in globaltimer ns; slot 3
// is the last CTA past the wait, slots 4/5 the head's selection start/end.
// ---------------------------------------------------------------------------
__device__ Crumbs g_crumbs;

struct StepTrace {
  unsigned long long* buf;
  int cap;
};
__device__ StepTrace g_trace;

__device__ __forceinline__ void trace_mark(int id, int slot) {
  if (id <= 0 || threadIdx.x != 0) return;
  const StepTrace t = g_trace;
  if (!t.buf || id >= t.cap) return;
  unsigned long long now;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
  if (slot == 1) atomicMax(t.buf + 3 * t.cap + id, now);  // last CTA past the wait
  if (slot >= 2) atomicMax(t.buf + slot * t.cap + id, now);
  else atomicMin(t.buf + slot * t.cap + id, now);
}

__device__ __forceinline__ unsigned long long trace_clock(int id) {
  unsigned long long now = 0;
  if (id > 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
  return now;
}
// Slots 6 and 7: max over CTAs of the time since t0 (the CTA's own wait).
__device__ __forceinline__ void trace_dur(int id, int slot, unsigned long long t0) {
  if (id <= 0 || threadIdx.x != 0) return;
  const StepTrace t = g_trace;
  if (!t.buf || id >= t.cap) return;
  atomicMax(t.buf + slot * t.cap + id, trace_clock(id) - t0);
}

// ---------------------------------------------------------------------------
// Projection body: for the block's M-tile and RPW output columns per warp,
//   acc = W[row] . (gamma * x[m])   then  y = epilogue(inv_rms[m] * acc)
// The RMSNorm scale is a per-row scalar, so it is applied after the dot
// product; gamma is folded into the staged activations.
// ---------------------------------------------------------------------------
template <int MT, int RPW, int EPI>
__device__ __forceinline__ bool linear_body(const LinearArgs& a, float* sx, float* s_inv) {
  constexpr int NR = (EPI == EPI_SWIGLU) ? 2 * RPW : RPW;
  constexpr int KC_MAX = kXFloats / MT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col0 = (blockIdx.x * kWarps + warp) * RPW;
  const int m0 = blockIdx.y * MT;
  const int K = a.K;
  trace_mark(a.trace_id, 0);

  const __nv_bfloat16* wr[NR];
  bool valid[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int c = col0 + r;
    valid[r] = c < a.N;
    const long long cc = valid[r] ? c : 0;
    if (EPI == EPI_SWIGLU) {
      wr[2 * r] = a.W + cc * K;
      wr[2 * r + 1] = a.W + (a.N + cc) * K;
    } else {
      wr[r] = a.W + cc * K;
    }
  }
  // Weights do not depend on the previous kernel: pull this warp's first
  // 16-byte chunks into L2 before waiting on the producer.
#pragma unroll
  for (int r = 0; r < NR; ++r)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(wr[r] + lane * 8));

  pdl_wait();
  trace_mark(a.trace_id, 1);
  if (a.halt && *a.halt) return false;
  const int mcount = min(MT, a.M - m0);

  if (a.gamma) {
    for (int m = warp; m < mcount; m += kWarps) {
      const float4* xr = reinterpret_cast<const float4*>(a.x + (long long)(m0 + m) * a.ldx);
      float ss = 0.f;
      for (int k = lane; k < K / 4; k += 32) {
        float4 v = xr[k];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      ss = warp_sum(ss);
      if (lane == 0) s_inv[m] = rsqrtf(ss / (float)K + a.eps);
    }
  }

  float acc[NR][MT];
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;

  for (int k0 = 0; k0 < K; k0 += KC_MAX) {
    const int kc = min(KC_MAX, K - k0);
    __syncthreads();
    const int kq = kc >> 2;
    for (int i = threadIdx.x; i < MT * kq; i += kThreads) {
      const int m = i / kq, k4 = i - m * kq;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < mcount)
        v = *reinterpret_cast<const float4*>(a.x + (long long)(m0 + m) * a.ldx + k0 + 4 * k4);
      if (a.gamma) {
        const float4 g = *reinterpret_cast<const float4*>(a.gamma + k0 + 4 * k4);
        v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
      }
      *reinterpret_cast<float4*>(sx + m * kc + 4 * k4) = v;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = lane * 8; kk < kc; kk += 256) {
      uint4 wv[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r) wv[r] = ldg_stream(wr[r] + k0 + kk);
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        float wf[8];
        unpack8(wv[r], wf);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const float4 x0 = *reinterpret_cast<const float4*>(sx + m * kc + kk);
          const float4 x1 = *reinterpret_cast<const float4*>(sx + m * kc + kk + 4);
          float t = acc[r][m];
          t = fmaf(wf[0], x0.x, t); t = fmaf(wf[1], x0.y, t);
          t = fmaf(wf[2], x0.z, t); t = fmaf(wf[3], x0.w, t);
          t = fmaf(wf[4], x1.x, t); t = fmaf(wf[5], x1.y, t);
          t = fmaf(wf[6], x1.z, t); t = fmaf(wf[7], x1.w, t);
          acc[r][m] = t;
        }
      }
    }
  }
  pdl_trigger();

#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    if (!valid[r]) continue;  // warp-uniform
    const int c = col0 + r;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m >= mcount) break;
      const float sc = a.gamma ? s_inv[m] : 1.0f;
      float out;
      if (EPI == EPI_SWIGLU) {
        const float g = warp_sum(acc[2 * r][m]) * sc;
        const float u = warp_sum(acc[2 * r + 1][m]) * sc;
        out = g / (1.0f + expf(-g)) * u;
      } else {
        out = warp_sum(acc[r][m]) * sc;
        if (EPI == EPI_RESID) out += a.resid[(long long)(m0 + m) * a.ldr + c];
        if (EPI == EPI_BIAS) out += a.bias[c];
        if (EPI == EPI_BIAS_SILU) out = silu(out + a.bias[c]);
      }
      if (lane == 0) a.y[(long long)(m0 + m) * a.ldy + c] = out;
    }
  }
  trace_mark(a.trace_id, 2);
  return true;
}

template <int MT, int RPW, int EPI>
__global__ void __launch_bounds__(kThreads) k_linear(LinearArgs a) {
  QTTS_CRUMB(0, 10);
  extern __shared__ float4 dyn4[];
  __shared__ float s_inv[MT];
  linear_body<MT, RPW, EPI>(a, reinterpret_cast<float*>(dyn4), s_inv);
}

// CodePredictor attention (at most kCpFusedPositions positions) computed by
// every CTA of the O projection while it stages its input: warp w handles kv
// head w (and w + 8, ...) with its two q heads; lane l holds dims 4l..4l+3.
// QK-RMSNorm, RoPE, the bf16 round of the new K/V row and the softmax follow
// the standalone decode-attention kernel; CTA 0 appends the row to the cache.
constexpr int kCpFusedPositions = 16;

// The cached keys / values of kv head g (positions < pos) and the constant
// norm and RoPE rows one lane needs. The cached rows were written by the
// attention of earlier CodePredictor groups, at least four launches back;
// a kernel only starts once the kernel two places before it has completed
// (every launch triggers its dependents after its own dependency wait), so
// these loads may be issued before this kernel's wait, overlapping its
// predecessor, like the weight loads.
struct CpAttnRows {
  uint2 kc[kCpFusedPositions], vc[kCpFusedPositions];
  float4 qg, kg, rc, rs;
};

__device__ __forceinline__ void load_cp_attention_rows(const AttnDecodeArgs& at, int g,
                                                       CpAttnRows& r) {
  const int lane = threadIdx.x & 31, pos = at.pos_const, d0 = 4 * lane;
  // With a known page the cached rows are read without the table lookup.
  const __nv_bfloat16* kbase =
      at.page0 >= 0 ? at.kv.pool + (long long)at.page0 * at.kv.page_stride +
                          (long long)at.layer * at.kv.layer_stride +
                          ((long long)g << at.kv.page_shift) * kHeadDim
                    : nullptr;
  const long long vofs = ((long long)at.kv.kv_heads << at.kv.page_shift) * kHeadDim;
#pragma unroll
  for (int p = 0; p < kCpFusedPositions; ++p) {
    if (p < pos) {
      const __nv_bfloat16* kp = kbase ? kbase + (long long)p * kHeadDim : kv_ptr(at.kv, at.layer, 0, g, p);
      const __nv_bfloat16* vp = kbase ? kbase + vofs + (long long)p * kHeadDim : kv_ptr(at.kv, at.layer, 1, g, p);
      r.kc[p] = *reinterpret_cast<const uint2*>(kp + d0);
      r.vc[p] = *reinterpret_cast<const uint2*>(vp + d0);
    }
  }
  r.qg = __ldg(reinterpret_cast<const float4*>(at.q_gamma + d0));
  r.kg = __ldg(reinterpret_cast<const float4*>(at.k_gamma + d0));
  r.rc = __ldg(reinterpret_cast<const float4*>(at.rope_cos + pos * 64 + (d0 & 63)));
  r.rs = __ldg(reinterpret_cast<const float4*>(at.rope_sin + pos * 64 + (d0 & 63)));
}

// ---------------------------------------------------------------------------
// Decode GEMV (one activation row). Every lane owns KCH 16-byte chunks of
// each of its NR weight rows and loads all of them into registers before the
// programmatic-dependent-launch wait: weights never depend on the previous
// kernel, so their HBM latency overlaps the producer's tail. After the wait
// the CTA stages gamma * x once in shared memory (the RMSNorm sum of squares
// comes from the same pass) and every warp reads it from there.
// SWIGLU: the warp's two rows are gate row c and up row N + c.
// `xs` holds KCH * 256 floats + 32 words of reduction scratch.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void stage_cp_attention(const AttnDecodeArgs& at, float* xs, int halted,
                                                   int trace_id, unsigned long long tw,
                                                   CpAttnRows& r);

template <int KCH, int NR, bool ATTN = false, int MR = 1>
__device__ __forceinline__ bool gemv1_body(const LinearArgs& a, int epi, float* xs,
                                           float* inv_out, const AttnDecodeArgs* at = nullptr) {
  // MR activation rows (1 for decode, 2 for the CodePredictor's 2-row
  // prefill) share every weight load: MR dot products per weight row.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool swiglu = epi == EPI_SWIGLU;
  const int outs = swiglu ? 1 : NR;
  const int c0 = (blockIdx.x * kWarps + warp) * outs;
  constexpr int K = KCH * 256;
  trace_mark(a.trace_id, 0);
  uint4 w[NR][KCH];
  bool valid[NR];
  const unsigned long long pol = l2_evict_first_policy();
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const int c = swiglu ? c0 : c0 + r;
    valid[r] = c < a.N;
    const long long row = swiglu ? (r == 0 ? c0 : a.N + c0) : c;
    const __nv_bfloat16* src = a.W + (valid[r] ? row : 0) * (long long)K + lane * 8;
#pragma unroll
    for (int j = 0; j < KCH; ++j) w[r][j] = ldg_stream(src + j * 256, pol);
  }
  // residual values of this warp's outputs (lane 0), when known to be final
  const bool early_r = epi == EPI_RESID && a.resid_early;
  float rv[MR][NR];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int r = 0; r < NR; ++r)
      rv[m][r] = early_r && lane == 0 && valid[r] ? __ldcg(a.resid + (long long)m * a.ldr + c0 + r)
                                                  : 0.f;
  CpAttnRows attn_rows;
  if constexpr (ATTN) {
    if (warp < at->kv.kv_heads) load_cp_attention_rows(*at, warp, attn_rows);
  }
  // A branch (never taken) between the weight loads and the dependency wait
  // keeps the two in separate basic blocks, so the SASS scheduler cannot sink
  // the loads past the wait: with both in one block the loads were issued
  // after it and the decode frame measured 9% slower (390 vs 427 frames/s).
  if (a.K < 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(a.W) : "memory");
  pdl_wait();
  trace_mark(a.trace_id, 1);
  const unsigned long long tw = trace_clock(a.trace_id);
  // Dependents launch once this kernel is past its wait: their weight loads
  // then overlap this kernel's staging and compute (measured faster than
  // launching them at entry, which floods the memory queues with several
  // kernels' weights at once, or after staging).
  pdl_trigger();
  // The halt flag is loaded alongside the input (not before it) and only
  // checked before the first write.
  const int halted = a.halt ? __ldcg(a.halt) : 0;
  float* red = xs + MR * K;  // [MR][kWarps] partial sums of squares
  if (ATTN) {
    stage_cp_attention(*at, xs, halted, a.trace_id, tw, attn_rows);
  } else {
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float ss = 0.f;
      for (int k = threadIdx.x * 4; k < K; k += kThreads * 4) {
        float4 v = __ldcg(reinterpret_cast<const float4*>(a.x + (long long)m * a.ldx + k));
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        if (a.gamma) {
          const float4 g = __ldg(reinterpret_cast<const float4*>(a.gamma + k));
          v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
        }
        *reinterpret_cast<float4*>(xs + m * K + k) = v;
      }
      if (a.gamma) {
        ss = warp_sum(ss);
        if (lane == 0) red[m * kWarps + warp] = ss;
      }
    }
  }
  __syncthreads();
  float sc[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    sc[m] = 1.0f;
    if (!ATTN && a.gamma) {
      float t = 0.f;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) t += red[m * kWarps + i];
      sc[m] = rsqrtf(t / (float)K + a.eps);
    }
  }
  if (halted) return false;
  if (inv_out && threadIdx.x == 0) *inv_out = sc[0];
  trace_mark(a.trace_id, 4);
  float acc[MR][NR];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[m][r] = 0.f;
#pragma unroll
  for (int j = 0; j < KCH; ++j) {
    const int k = j * 256 + lane * 8;
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const float4 x0 = *reinterpret_cast<const float4*>(xs + m * K + k);
      const float4 x1 = *reinterpret_cast<const float4*>(xs + m * K + k + 4);
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        float f[8];
        unpack8(w[r][j], f);
        float t = acc[m][r];
        t = fmaf(f[0], x0.x, t); t = fmaf(f[1], x0.y, t);
        t = fmaf(f[2], x0.z, t); t = fmaf(f[3], x0.w, t);
        t = fmaf(f[4], x1.x, t); t = fmaf(f[5], x1.y, t);
        t = fmaf(f[6], x1.z, t); t = fmaf(f[7], x1.w, t);
        acc[m][r] = t;
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[m][r] = warp_sum(acc[m][r]);
  trace_mark(a.trace_id, 5);
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float* y = a.y + (long long)m * a.ldy;
      if (swiglu) {
        if (valid[0]) {
          const float g = acc[m][0] * sc[m], u = acc[m][NR - 1] * sc[m];
          y[c0] = g / (1.0f + expf(-g)) * u;
        }
      } else {
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          if (!valid[r]) continue;
          const int c = c0 + r;
          float out = acc[m][r] * sc[m];
          if (epi == EPI_RESID) out += early_r ? rv[m][r] : __ldcg(a.resid + (long long)m * a.ldr + c);
          if (epi == EPI_BIAS) out += a.bias[c];
          if (epi == EPI_BIAS_SILU) out = silu(out + a.bias[c]);
          y[c] = out;
        }
      }
    }
  }
  trace_mark(a.trace_id, 2);
  return true;
}

// `r` holds kv head `warp`'s rows, loaded before the dependency wait (and
// is reloaded for any further head of the warp).
__device__ __forceinline__ void stage_cp_attention(const AttnDecodeArgs& at, float* xs, int halted,
                                                   int trace_id, unsigned long long tw,
                                                   CpAttnRows& r) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = at.pos_const, T = pos + 1;
  const int kvh = at.kv.kv_heads;
  const int q_out = at.q_heads * kHeadDim, kv_out = kvh * kHeadDim;
  const int d0 = 4 * lane;
  for (int g = warp; g < kvh; g += kWarps) {
    if (g != warp) load_cp_attention_rows(at, g, r);
    const uint2* kc = r.kc;
    const uint2* vc = r.vc;
    const float4 qg = r.qg, kg = r.kg, rc = r.rc, rs = r.rs;
    float4 q[2];
    q[0] = __ldcg(reinterpret_cast<const float4*>(at.qkv + (2 * g) * kHeadDim + d0));
    q[1] = __ldcg(reinterpret_cast<const float4*>(at.qkv + (2 * g + 1) * kHeadDim + d0));
    float4 kk = __ldcg(reinterpret_cast<const float4*>(at.qkv + q_out + g * kHeadDim + d0));
    const float4 vv = __ldcg(reinterpret_cast<const float4*>(at.qkv + q_out + kv_out + g * kHeadDim + d0));
    auto norm_rope = [&](float4 x, float4 gm) {
      const float ss = warp_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
      const float inv = rsqrtf(ss / (float)kHeadDim + at.eps);
      x.x = x.x * inv * gm.x; x.y = x.y * inv * gm.y; x.z = x.z * inv * gm.z; x.w = x.w * inv * gm.w;
      float4 o;
      o.x = __shfl_xor_sync(0xffffffffu, x.x, 16); o.y = __shfl_xor_sync(0xffffffffu, x.y, 16);
      o.z = __shfl_xor_sync(0xffffffffu, x.z, 16); o.w = __shfl_xor_sync(0xffffffffu, x.w, 16);
      if (lane < 16) {
        x.x = x.x * rc.x - o.x * rs.x; x.y = x.y * rc.y - o.y * rs.y;
        x.z = x.z * rc.z - o.z * rs.z; x.w = x.w * rc.w - o.w * rs.w;
      } else {
        x.x = x.x * rc.x + o.x * rs.x; x.y = x.y * rc.y + o.y * rs.y;
        x.z = x.z * rc.z + o.z * rs.z; x.w = x.w * rc.w + o.w * rs.w;
      }
      return x;
    };
    q[0] = norm_rope(q[0], qg);
    q[1] = norm_rope(q[1], qg);
    kk = norm_rope(kk, kg);
    const __nv_bfloat162 kb0 = __floats2bfloat162_rn(kk.x, kk.y), kb1 = __floats2bfloat162_rn(kk.z, kk.w);
    const __nv_bfloat162 vb0 = __floats2bfloat162_rn(vv.x, vv.y), vb1 = __floats2bfloat162_rn(vv.z, vv.w);
    uint2 kcur, vcur;
    kcur.x = *reinterpret_cast<const unsigned*>(&kb0); kcur.y = *reinterpret_cast<const unsigned*>(&kb1);
    vcur.x = *reinterpret_cast<const unsigned*>(&vb0); vcur.y = *reinterpret_cast<const unsigned*>(&vb1);
    if (blockIdx.x == 0 && !halted) {
      *reinterpret_cast<uint2*>(kv_ptr(at.kv, at.layer, 0, g, pos) + d0) = kcur;
      *reinterpret_cast<uint2*>(kv_ptr(at.kv, at.layer, 1, g, pos) + d0) = vcur;
    }
    // partial scores of this lane's 4 dims: d[16 j + p] for q head j, position p
    float d[2 * kCpFusedPositions];
#pragma unroll
    for (int p = 0; p < kCpFusedPositions; ++p) {
      const uint2 ku = p < pos ? kc[p] : kcur;
      const float k0 = bf16lo(ku.x), k1 = bf16hi(ku.x), k2 = bf16lo(ku.y), k3 = bf16hi(ku.y);
#pragma unroll
      for (int j = 0; j < 2; ++j)
        d[kCpFusedPositions * j + p] = (q[j].x * at.scale) * k0 + (q[j].y * at.scale) * k1 +
                                       (q[j].z * at.scale) * k2 + (q[j].w * at.scale) * k3;
    }
    trace_dur(trace_id, 6, tw);  // cached rows and projections in registers
    // Reduce-scatter over the warp (31 shuffles instead of 32 x 5): at each
    // step a lane keeps the half of its values that its lane-id bit selects
    // and adds its partner's copy of that half, so lane l ends with the full
    // score of pair l (q head l / 16, position l % 16).
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
      const bool upper = (lane & w) != 0;
#pragma unroll
      for (int i = 0; i < w; ++i) {
        const float send = upper ? d[i] : d[i + w];
        const float keep = upper ? d[i + w] : d[i];
        d[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
      }
    }
    // softmax over the positions 0..pos of each q head (one half-warp each)
    const int p_own = lane & (kCpFusedPositions - 1);
    const float sc = p_own < T ? d[0] : -INFINITY;
    float m = sc;
#pragma unroll
    for (int o = kCpFusedPositions / 2; o > 0; o >>= 1)
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float e = p_own < T ? expf(sc - m) : 0.f;
    float l = e;
#pragma unroll
    for (int o = kCpFusedPositions / 2; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    const float wgt = e / l;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < kCpFusedPositions; ++p) {
        const float wp = __shfl_sync(0xffffffffu, wgt, kCpFusedPositions * j + p);
        if (p >= T) continue;
        const uint2 vu = p < pos ? vc[p] : vcur;
        acc[0] = fmaf(wp, bf16lo(vu.x), acc[0]); acc[1] = fmaf(wp, bf16hi(vu.x), acc[1]);
        acc[2] = fmaf(wp, bf16lo(vu.y), acc[2]); acc[3] = fmaf(wp, bf16hi(vu.y), acc[3]);
      }
      *reinterpret_cast<float4*>(xs + (2 * g + j) * kHeadDim + d0) =
          make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
  }
  trace_dur(trace_id, 7, tw);  // warp 0's heads done
}

template <int KCH>
__global__ void __maxnreg__(200) k_gemv1_attn(LinearArgs a, AttnDecodeArgs at) {
  QTTS_CRUMB(0, 11);
  __shared__ __align__(16) float xs[KCH * 256 + 32];
  gemv1_body<KCH, 1, true>(a, EPI_RESID, xs, nullptr, &at);
}

template <int KCH, int NR, int MR>
__global__ void __launch_bounds__(kThreads) k_gemv1(LinearArgs a, int epi) {
  QTTS_CRUMB(0, 6);
  __shared__ __align__(16) float xs[MR * KCH * 256 + 32];
  gemv1_body<KCH, NR, false, MR>(a, epi, xs, nullptr);
}

// Token selection and the gathers the next stage needs, for one sequence:
// penalty / suppression, selection, then (talker roles) the CodePredictor
// prefix and halt on EOS, or (CodePredictor groups) the next group input,
// the embedding sum, codes and, after the last group, the talker step input.
// `inv` is the RMS scale of the head input row `a.lin.x`.
__device__ __forceinline__ void head_select_act(const HeadArgs& a, const float* logits, float inv,
                                                float* smem) {
  __shared__ int s_frame, s_sem;
  const unsigned long long t_sel = trace_clock(a.lin.trace_id);

  const int V = a.lin.N;
  Selector<SyncBlock> sel{smem, reinterpret_cast<int*>(smem + kSelMaxVocab)};
  // traced frames: the selection's phase stamps (clock64) land after the
  // trace's eight slots, 16 per head (row 0 the talker, 1 + g CodePredictor group g)
  if (a.lin.trace_id > 0 && g_trace.buf)
    sel.dbg = reinterpret_cast<long long*>(g_trace.buf + 8 * (size_t)g_trace.cap) +
              16 * (a.role == ROLE_CP_GROUP ? 1 + a.group : 0);
  const int tid = threadIdx.x;
  // The RNG state is read alongside the logits (the sampler draws early).
  Rng rng{a.st->rng_kind, a.st->rng_state, a.st->rng_seed, a.st->rng_counter};
  for (int v = tid; v < V; v += kThreads) sel.val[v] = __ldcg(logits + v);
  if (tid == 0) { s_frame = a.st->frames; s_sem = a.st->semantic; }
  __syncthreads();
  trace_dur(a.lin.trace_id, 6, t_sel);  // logits and sequence state reloaded
  // batched heads check the per-sequence state they index with (a fault here
  // would otherwise take the context down): record and skip
  if (a.frames_cap > 0 &&
      (s_frame < 0 || s_frame >= a.frames_cap || s_sem < -1 || s_sem >= a.talker_vocab)) {
    if (tid == 0) {
      a.st->error = 2;
      if (g_crumbs.p) {
        g_crumbs.p[2] = 1000 + a.role;
        g_crumbs.p[3] = (unsigned)s_frame;
        g_crumbs.p[4] = (unsigned)s_sem;
        g_crumbs.p[5] = blockIdx.x;
        __threadfence_system();
      }
    }
    return;
  }
  // The tail's inputs that do not depend on the token are loaded now, so
  // their latency hides under the selection; after it only the token's
  // embedding row is read (4 consecutive elements per thread and pass).
  const int H = a.H;
  constexpr int kIt = 2;  // H <= kIt * 4 * kThreads (checked at engine load)
  const bool cp = a.role == ROLE_CP_GROUP;
  const bool last = cp && a.group == a.last_group;
  const float* tr = nullptr;
  const __nv_bfloat16* se = nullptr;
  if (last) {
    tr = s_frame < __ldcg(&a.st->n_trailing) ? a.trailing + (long long)s_frame * H : a.tts_pad;
    se = a.talker_codec_emb + (long long)s_sem * H;
  }
  // pre_a: CodePredictor running embedding sum / talker normed hidden;
  // pre_b, pre_c: the last group's trailing row and semantic embedding.
  float4 pre_a[kIt], pre_b[kIt];
  uint2 pre_c[kIt];
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    const int i = (it * kThreads + tid) * 4;
    pre_a[it] = pre_b[it] = make_float4(0.f, 0.f, 0.f, 0.f);
    pre_c[it] = make_uint2(0u, 0u);
    if (i >= H) continue;
    if (cp) {
      if (a.group != 0) pre_a[it] = __ldcg(reinterpret_cast<const float4*>(a.emb_sum + i));
      if (last) {
        pre_b[it] = __ldcg(reinterpret_cast<const float4*>(tr + i));
        pre_c[it] = *reinterpret_cast<const uint2*>(se + i);
      }
    } else {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(a.lin.x + i));
      const float4 g = __ldg(reinterpret_cast<const float4*>(a.lin.gamma + i));
      pre_a[it] = make_float4(x.x * inv * g.x, x.y * inv * g.y, x.z * inv * g.z, x.w * inv * g.w);
    }
  }

  if (a.role == ROLE_TALKER_STEP)
    sel.penalise(V, a.history, s_frame, -1, a.penalty, a.suppress, a.eos_token);
  else
    sel.penalise(V, a.history, 0, -1, 1.0f, a.suppress, a.eos_token);
  const int tok = sel.select(V, a.cfg, rng, &a.st->error);
  trace_dur(a.lin.trace_id, 7, t_sel);  // token chosen
  if (tid == 0) {
    a.st->rng_state = rng.state;
    a.st->rng_counter = rng.counter;
  }
  if (a.token_out && tid == 0) *a.token_out = tok;
  if (a.frames_cap > 0 && (tok < 0 || tok >= V)) {
    if (tid == 0) {
      a.st->error = 3;
      if (g_crumbs.p) {
        g_crumbs.p[2] = 2000 + a.role;
        g_crumbs.p[3] = (unsigned)tok;
        g_crumbs.p[4] = (unsigned)V;
        g_crumbs.p[5] = blockIdx.x;
        __threadfence_system();
      }
    }
    return;
  }

  if (a.role == ROLE_TALKER_PREFILL || a.role == ROLE_TALKER_STEP) {
    const __nv_bfloat16* e = a.talker_codec_emb + (long long)tok * H;
    uint2 ev[kIt];
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int i = (it * kThreads + tid) * 4;
      if (i < H) ev[it] = *reinterpret_cast<const uint2*>(e + i);
    }
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int i = (it * kThreads + tid) * 4;
      if (i >= H) continue;
      *reinterpret_cast<float4*>(a.cp_prefix + i) = pre_a[it];
      *reinterpret_cast<float4*>(a.cp_prefix + H + i) =
          make_float4(bf16lo(ev[it].x), bf16hi(ev[it].x), bf16lo(ev[it].y), bf16hi(ev[it].y));
    }
    if (tid == 0) {
      a.st->semantic = tok;
      if (tok == a.eos_token) a.st->halt = 1;
    }
  } else if (cp) {
    // Every read that depends on the token is issued before any store, so
    // the table rows and the embedding row arrive in one memory round trip.
    constexpr int kQIt = kCpQkvTableMax / (4 * kThreads), kXIt = kCpXTableMax / (4 * kThreads);
    float4 qv[kQIt], xv[kXIt];
    const int nq = a.qkv_table ? a.qkv_w / 4 : 0, nx = a.x_table ? a.x_w / 4 : 0;
    if (nq) {
      // the next group's layer-0 projections: a row of the precomputed table
      const float4* src = reinterpret_cast<const float4*>(a.qkv_table + (long long)tok * a.qkv_w);
#pragma unroll
      for (int it = 0; it < kQIt; ++it)
        if (it * kThreads + tid < nq) qv[it] = __ldg(src + it * kThreads + tid);
    }
    if (nx) {
      const float4* src = reinterpret_cast<const float4*>(a.x_table + (long long)tok * a.x_w);
#pragma unroll
      for (int it = 0; it < kXIt; ++it)
        if (it * kThreads + tid < nx) xv[it] = __ldg(src + it * kThreads + tid);
    }
    const __nv_bfloat16* e = a.cp_emb + (long long)tok * H;
    uint2 ev[kIt];
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int i = (it * kThreads + tid) * 4;
      if (i < H) ev[it] = *reinterpret_cast<const uint2*>(e + i);
    }
#pragma unroll
    for (int it = 0; it < kQIt; ++it)
      if (it * kThreads + tid < nq) reinterpret_cast<float4*>(a.qkv_out)[it * kThreads + tid] = qv[it];
#pragma unroll
    for (int it = 0; it < kXIt; ++it)
      if (it * kThreads + tid < nx) reinterpret_cast<float4*>(a.x_out)[it * kThreads + tid] = xv[it];
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int i = (it * kThreads + tid) * 4;
      if (i >= H) continue;
      const float4 ef = make_float4(bf16lo(ev[it].x), bf16hi(ev[it].x), bf16lo(ev[it].y),
                                    bf16hi(ev[it].y));
      const float4 sm = a.group == 0 ? ef
                                     : make_float4(pre_a[it].x + ef.x, pre_a[it].y + ef.y,
                                                   pre_a[it].z + ef.z, pre_a[it].w + ef.w);
      *reinterpret_cast<float4*>(a.cp_next + i) = ef;
      *reinterpret_cast<float4*>(a.emb_sum + i) = sm;
      if (last) {
        const uint2 q = pre_c[it];
        const float4 t = pre_b[it];
        *reinterpret_cast<float4*>(a.step_in + i) =
            make_float4((bf16lo(q.x) + sm.x) + t.x, (bf16hi(q.x) + sm.y) + t.y,
                        (bf16lo(q.y) + sm.z) + t.z, (bf16hi(q.y) + sm.w) + t.w);
      }
    }
    if (tid == 0) {
      a.codes[(long long)s_frame * a.groups + 1 + a.group] = tok;
      if (last) {
        a.codes[(long long)s_frame * a.groups] = s_sem;
        a.history_out[s_frame] = s_sem;
        a.st->talker_pos = a.st->prefill_len + s_frame;
        a.st->frames = s_frame + 1;
      }
    }
  }
}

// Head: final/group RMSNorm + LM head GEMV over all CTAs; the last CTA to
// finish selects the token (head_select_act), so no logits or tokens visit
// the host.
template <int KCH>
__global__ void __launch_bounds__(kThreads) k_head(HeadArgs a) {
  QTTS_CRUMB(0, 7);
  extern __shared__ float4 dyn4[];
  float* smem = reinterpret_cast<float*>(dyn4);
  __shared__ float s_inv[1];
  __shared__ bool s_last;
  if (!gemv1_body<KCH, 1>(a.lin, EPI_STORE, smem, s_inv)) return;
  __syncthreads();  // the selector reuses the staged activation buffer
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x == 0) *a.ticket = 0u;
  __threadfence();
  if (a.role == ROLE_LOGITS_ONLY) return;
  trace_mark(a.lin.trace_id, 4);
  head_select_act(a, a.lin.y, s_inv[0], smem);
  trace_mark(a.lin.trace_id, 5);
}

// Batched heads: the logits of B sequences come from one tensor-core
// projection; CTA b selects sequence b's token (skipped once it has halted).
__global__ void __launch_bounds__(kThreads) k_select_batch(BatchHeadArgs bh) {
  QTTS_CRUMB(0, 3);
  extern __shared__ float4 dyn4[];
  float* smem = reinterpret_cast<float*>(dyn4);
  pdl_wait();
  const int b = blockIdx.x;
  HeadArgs a = bh.h;
  a.st += b;
  if (__ldcg(&a.st->halt)) return;
  a.history += (long long)b * bh.hist_stride;
  a.history_out += (long long)b * bh.hist_stride;
  a.codes += (long long)b * bh.codes_stride;
  if (a.cp_prefix) a.cp_prefix += (long long)b * 2 * a.H;
  a.lin.x += (long long)b * a.lin.ldx;
  if (a.cp_next) a.cp_next += (long long)b * bh.next_stride;
  if (a.emb_sum) a.emb_sum += (long long)b * a.H;
  if (a.step_in) a.step_in += (long long)b * bh.step_stride;
  if (a.trailing) a.trailing += (long long)b * bh.trail_stride;
  if (a.qkv_out) a.qkv_out += (long long)b * bh.qkv_stride;
  if (a.x_out) a.x_out += (long long)b * bh.x_stride;
  a.token_out = nullptr;
  head_select_act(a, bh.logits + (long long)b * bh.logits_ld, __ldcg(bh.rms + b), smem);
}

// ---------------------------------------------------------------------------
// Decode attention: one CTA per kv head, NW warps. The prologue (threads
// < 128) fuses QK-RMSNorm, RoPE and the bf16 KV append of the current
// position. Warp w then owns positions w*8.., (w+NW)*8.., in batches of 8:
// the next batch's K/V rows are loaded while the current batch is scored, the
// 8*G dot products are reduced together, and the online softmax is updated
// once per batch. Warps merge their (max, sum, acc) in shared memory.
// ---------------------------------------------------------------------------
constexpr int kAttnBatch = 8;

template <int G, int NW>
__global__ void __launch_bounds__(NW * 32) k_attn_decode(AttnDecodeArgs a) {
  QTTS_CRUMB(0, 2);
  __shared__ float sq[G][kHeadDim];
  __shared__ float sk[kHeadDim], sv[kHeadDim];
  __shared__ float red[4][G + 1];
  __shared__ float wm[NW][G], wl[NW][G];
  __shared__ float wacc[NW][G][kHeadDim];
  trace_mark(a.trace_id, 0);
  // Before the dependency wait: the halt flag (written only by a frame's last
  // kernel), the position (written by the CodePredictor's last head, at least
  // two launches back), the first batch of cached rows (earlier positions,
  // written by earlier steps) and the constant norm / RoPE rows. A kernel
  // starts only after the kernel two places before it has completed, since
  // every launch triggers its dependents after its own wait; only this
  // step's projections come from the immediately preceding kernel.
  const int seq = blockIdx.y;
  const int halted = a.halt ? __ldcg(a.halt + seq * a.halt_stride) : 0;
  const int h = blockIdx.x, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int pos = a.pos_ptr ? __ldcg(a.pos_ptr + seq * a.pos_stride) : a.pos_const;
  a.qkv += (long long)seq * a.qkv_ld;
  a.out += (long long)seq * a.out_ld;
  a.kv.page_table += (long long)seq * a.pt_stride;
  const int T = pos + 1;
  const int kvh = a.kv.kv_heads;
  const int q_out = a.q_heads * kHeadDim, kv_out = kvh * kHeadDim;
  // Rows before `pos` come from the cache; the current row from shared memory.
  auto load = [&](int p0, uint2 (&ku)[kAttnBatch], uint2 (&vu)[kAttnBatch]) {
#pragma unroll
    for (int i = 0; i < kAttnBatch; ++i) {
      const int p = p0 + i;
      if (p < pos) {
        ku[i] = *reinterpret_cast<const uint2*>(kv_ptr(a.kv, a.layer, 0, h, p) + 4 * lane);
        vu[i] = *reinterpret_cast<const uint2*>(kv_ptr(a.kv, a.layer, 1, h, p) + 4 * lane);
      } else {
        ku[i] = make_uint2(0u, 0u);
        vu[i] = make_uint2(0u, 0u);
      }
    }
  };
  uint2 ku[kAttnBatch], vu[kAttnBatch], nk[kAttnBatch], nv[kAttnBatch];
  int p0 = warp * kAttnBatch;
  if (p0 < T) load(p0, ku, vu);  // cached rows: independent of this step's projections
  float rc = 0.f, rsn = 0.f, qgam = 0.f, kgam = 0.f;
  if (tid < kHeadDim) {
    rc = a.rope_cos[pos * 64 + (tid & 63)];
    rsn = a.rope_sin[pos * 64 + (tid & 63)];
    qgam = a.q_gamma[tid];
    kgam = a.k_gamma[tid];
  }
  // A branch (never taken) keeps the loads above in their own basic block,
  // so the SASS scheduler cannot sink them past the wait.
  if (a.layer < 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(a.qkv) : "memory");
  pdl_wait();
  trace_mark(a.trace_id, 1);
  float qr[G], kr = 0.f, vr = 0.f;
  if (tid < kHeadDim) {
#pragma unroll
    for (int g = 0; g < G; ++g) qr[g] = __ldcg(a.qkv + (h * G + g) * kHeadDim + tid);
    kr = __ldcg(a.qkv + q_out + h * kHeadDim + tid);
    vr = __ldcg(a.qkv + q_out + kv_out + h * kHeadDim + tid);
  }
  if (halted) return;
  if (tid < kHeadDim) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float t = warp_sum(qr[g] * qr[g]);
      if (lane == 0) red[warp][g] = t;
    }
    const float t = warp_sum(kr * kr);
    if (lane == 0) red[warp][G] = t;
  }
  __syncthreads();
  if (tid < kHeadDim) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float ss = red[0][g] + red[1][g] + red[2][g] + red[3][g];
      sq[g][tid] = qr[g] * rsqrtf(ss / (float)kHeadDim + a.eps) * qgam;
    }
    const float ss = red[0][G] + red[1][G] + red[2][G] + red[3][G];
    sk[tid] = kr * rsqrtf(ss / (float)kHeadDim + a.eps) * kgam;
  }
  __syncthreads();
  float rq[G], kroped = 0.f;
  if (tid < kHeadDim) {
    const int pi = tid & 63;
    const float c = rc, sn = rsn;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float x0 = sq[g][pi], x1 = sq[g][pi + 64];
      rq[g] = tid < 64 ? x0 * c - x1 * sn : x1 * c + x0 * sn;
    }
    const float k0 = sk[pi], k1 = sk[pi + 64];
    kroped = tid < 64 ? k0 * c - k1 * sn : k1 * c + k0 * sn;
  }
  __syncthreads();
  if (tid < kHeadDim) {
    const __nv_bfloat16 kb = __float2bfloat16_rn(kroped);
    const __nv_bfloat16 vb = __float2bfloat16_rn(vr);
#pragma unroll
    for (int g = 0; g < G; ++g) sq[g][tid] = rq[g];
    sk[tid] = __bfloat162float(kb);
    sv[tid] = __bfloat162float(vb);
    kv_ptr(a.kv, a.layer, 0, h, pos)[tid] = kb;
    kv_ptr(a.kv, a.layer, 1, h, pos)[tid] = vb;
  }
  __syncthreads();

  float q[G][4], m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) { q[g][j] = sq[g][4 * lane + j] * a.scale; acc[g][j] = 0.f; }
  }
  for (; p0 < T; p0 += NW * kAttnBatch) {
    const int pn = p0 + NW * kAttnBatch;
    if (pn < T) load(pn, nk, nv);
    float kf[kAttnBatch][4], vf[kAttnBatch][4];
#pragma unroll
    for (int i = 0; i < kAttnBatch; ++i) {
      if (p0 + i == pos) {
#pragma unroll
        for (int j = 0; j < 4; ++j) { kf[i][j] = sk[4 * lane + j]; vf[i][j] = sv[4 * lane + j]; }
      } else {
        kf[i][0] = bf16lo(ku[i].x); kf[i][1] = bf16hi(ku[i].x);
        kf[i][2] = bf16lo(ku[i].y); kf[i][3] = bf16hi(ku[i].y);
        vf[i][0] = bf16lo(vu[i].x); vf[i][1] = bf16hi(vu[i].x);
        vf[i][2] = bf16lo(vu[i].y); vf[i][3] = bf16hi(vu[i].y);
      }
    }
    // partial scores of this lane's 4 dims, d[8 g + i] for q head g, position p0 + i
    constexpr int V = G * kAttnBatch;
    static_assert((V & (V - 1)) == 0 && V <= 32, "scores per batch: a power of two <= 32");
    float d[V];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < kAttnBatch; ++i)
        d[kAttnBatch * g + i] =
            q[g][0] * kf[i][0] + q[g][1] * kf[i][1] + q[g][2] * kf[i][2] + q[g][3] * kf[i][3];
    // Reduce-scatter over lane bits below V: a lane keeps the half its bit
    // selects plus its partner's copy, ending with score (lane % V) summed
    // over those lanes; the remaining lane bits finish the sum.
#pragma unroll
    for (int w = V / 2; w >= 1; w >>= 1) {
      const bool upper = (lane & w) != 0;
#pragma unroll
      for (int u = 0; u < w; ++u) {
        const float send = upper ? d[u] : d[u + w];
        const float keep = upper ? d[u + w] : d[u];
        d[u] = keep + __shfl_xor_sync(0xffffffffu, send, w);
      }
    }
    float sc = d[0];
#pragma unroll
    for (int o = V; o < 32; o <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
    const int bi = lane & (kAttnBatch - 1);  // position within the batch of this lane's score
    if (p0 + bi >= T) sc = -INFINITY;
    // per q head (kAttnBatch consecutive lanes): the batch max, then the sum
    float gm = sc;
#pragma unroll
    for (int o = kAttnBatch / 2; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
    const int myg = (lane % V) / kAttnBatch;
    float mbs[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mbs[g] = fmaxf(m[g], __shfl_sync(0xffffffffu, gm, kAttnBatch * g));
    float mine = mbs[0];
#pragma unroll
    for (int g = 1; g < G; ++g)
      if (myg == g) mine = mbs[g];
    const float pe = p0 + bi < T ? expf(sc - mine) : 0.f;
    float ls = pe;
#pragma unroll
    for (int o = kAttnBatch / 2; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float corr = expf(m[g] - mbs[g]);  // m = -inf on the first batch: corr = 0
      l[g] = l[g] * corr + __shfl_sync(0xffffffffu, ls, kAttnBatch * g);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) acc[g][jj] *= corr;
#pragma unroll
      for (int i = 0; i < kAttnBatch; ++i) {
        const float w = __shfl_sync(0xffffffffu, pe, kAttnBatch * g + i);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[g][jj] = fmaf(w, vf[i][jj], acc[g][jj]);
      }
      m[g] = mbs[g];
    }
#pragma unroll
    for (int i = 0; i < kAttnBatch; ++i) { ku[i] = nk[i]; vu[i] = nv[i]; }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int j = 0; j < 4; ++j) wacc[warp][g][4 * lane + j] = acc[g][j];
    if (lane == 0) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
  }
  __syncthreads();
  for (int t = tid; t < G * kHeadDim; t += NW * 32) {
    const int g = t / kHeadDim, dd = t % kHeadDim;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      if (wm[w][g] == -INFINITY) continue;
      const float f = expf(wm[w][g] - M);
      L += wl[w][g] * f;
      A += wacc[w][g][dd] * f;
    }
    a.out[(h * G + g) * kHeadDim + dd] = A / L;
  }
  trace_mark(a.trace_id, 2);
}

// Prefill: QK-RMSNorm + RoPE for M rows at positions pos0.., K/V appended to
// the cache as bf16; Q kept fp32 for the prefill attention.
__global__ void __launch_bounds__(128) k_qk_prep(QkPrepArgs a) {
  QTTS_CRUMB(0, 4);
  __shared__ float sx[kHeadDim];
  __shared__ float red[4];
  pdl_wait();
  if (a.halt && *a.halt) return;
  const int m = blockIdx.x, j = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int kvh = a.kv.kv_heads;
  const int q_out = a.q_heads * kHeadDim, kv_out = kvh * kHeadDim;
  const int ld = q_out + 2 * kv_out;
  const float* row = a.qkv + (long long)m * ld;
  const bool is_q = j < a.q_heads;
  const int hh = is_q ? j : j - a.q_heads;
  const float raw = is_q ? row[hh * kHeadDim + tid] : row[q_out + hh * kHeadDim + tid];
  const float t = warp_sum(raw * raw);
  if (lane == 0) red[warp] = t;
  __syncthreads();
  const float ss = red[0] + red[1] + red[2] + red[3];
  const float* gam = is_q ? a.q_gamma : a.k_gamma;
  sx[tid] = raw * rsqrtf(ss / (float)kHeadDim + a.eps) * gam[tid];
  __syncthreads();
  const int pos = a.pos0 + m;
  const int pi = tid & 63;
  const float c = a.rope_cos[pos * 64 + pi], sn = a.rope_sin[pos * 64 + pi];
  const float x0 = sx[pi], x1 = sx[pi + 64];
  const float r = tid < 64 ? x0 * c - x1 * sn : x1 * c + x0 * sn;
  if (is_q) {
    a.q_out[(long long)m * q_out + hh * kHeadDim + tid] = r;
  } else {
    kv_ptr(a.kv, a.layer, 0, hh, pos)[tid] = __float2bfloat16_rn(r);
    kv_ptr(a.kv, a.layer, 1, hh, pos)[tid] =
        __float2bfloat16_rn(row[q_out + kv_out + hh * kHeadDim + tid]);
  }
}

// Prefill attention: one warp per (query row, q head), causal over the cache.
__global__ void __launch_bounds__(128) k_attn_prefill(AttnPrefillArgs a) {
  QTTS_CRUMB(0, 5);
  pdl_wait();
  if (a.halt && *a.halt) return;
  const int qh = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.y * 4 + warp;
  if (m >= a.M) return;
  const int G = a.q_heads / a.kv.kv_heads;
  const int kh = qh / G;
  const int pos = a.pos0 + m;
  const int q_out = a.q_heads * kHeadDim;
  float q[4], acc[4] = {0.f, 0.f, 0.f, 0.f};
  const float4 qv = *reinterpret_cast<const float4*>(a.q + (long long)m * q_out + qh * kHeadDim + 4 * lane);
  q[0] = qv.x * a.scale; q[1] = qv.y * a.scale; q[2] = qv.z * a.scale; q[3] = qv.w * a.scale;
  float mx = -INFINITY, l = 0.f;
  // positions 0..pos in batches of kAttnBatch: the next batch's K/V rows are
  // loaded while this one is scored, and the softmax is updated once per batch
  auto load = [&](int p0, uint2 (&ku)[kAttnBatch], uint2 (&vu)[kAttnBatch]) {
#pragma unroll
    for (int i = 0; i < kAttnBatch; ++i) {
      const int p = p0 + i;
      if (p <= pos) {
        ku[i] = *reinterpret_cast<const uint2*>(kv_ptr(a.kv, a.layer, 0, kh, p) + 4 * lane);
        vu[i] = *reinterpret_cast<const uint2*>(kv_ptr(a.kv, a.layer, 1, kh, p) + 4 * lane);
      } else {
        ku[i] = vu[i] = make_uint2(0u, 0u);
      }
    }
  };
  uint2 ku[kAttnBatch], vu[kAttnBatch], nk[kAttnBatch], nv[kAttnBatch];
  load(0, ku, vu);
  for (int p0 = 0; p0 <= pos; p0 += kAttnBatch) {
    if (p0 + kAttnBatch <= pos) load(p0 + kAttnBatch, nk, nv);
    float d[kAttnBatch];
#pragma unroll
    for (int i = 0; i < kAttnBatch; ++i)
      d[i] = q[0] * bf16lo(ku[i].x) + q[1] * bf16hi(ku[i].x) + q[2] * bf16lo(ku[i].y) +
             q[3] * bf16hi(ku[i].y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < kAttnBatch; ++i) d[i] += __shfl_xor_sync(0xffffffffu, d[i], o);
    float mb = mx;
#pragma unroll
    for (int i = 0; i < kAttnBatch; ++i) {
      if (p0 + i > pos) d[i] = -INFINITY;
      mb = fmaxf(mb, d[i]);
    }
    const float corr = expf(mx - mb);  // mx = -inf on the first batch: corr = 0
    float ls = 0.f, av[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kAttnBatch; ++i) {
      const float pe = expf(d[i] - mb);
      ls += pe;
      av[0] = fmaf(pe, bf16lo(vu[i].x), av[0]); av[1] = fmaf(pe, bf16hi(vu[i].x), av[1]);
      av[2] = fmaf(pe, bf16lo(vu[i].y), av[2]); av[3] = fmaf(pe, bf16hi(vu[i].y), av[3]);
    }
    l = l * corr + ls;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = acc[j] * corr + av[j];
    mx = mb;
#pragma unroll
    for (int i = 0; i < kAttnBatch; ++i) { ku[i] = nk[i]; vu[i] = nv[i]; }
  }
  const float il = 1.0f / l;
  *reinterpret_cast<float4*>(a.out + (long long)m * q_out + qh * kHeadDim + 4 * lane) =
      make_float4(acc[0] * il, acc[1] * il, acc[2] * il, acc[3] * il);
}

__global__ void k_gather_rows(const __nv_bfloat16* table, const int* ids, int width, float* out) {
  QTTS_CRUMB(0, 8);
  pdl_wait();
  const int r = blockIdx.x;
  const __nv_bfloat16* src = table + (long long)ids[r] * width;
  for (int c = threadIdx.x; c < width; c += blockDim.x)
    out[(long long)r * width + c] = __bfloat162float(src[c]);
}

__global__ void k_assemble_rows(const float* proj, const int* proj_index,
                                const __nv_bfloat16* codec, const int* codec_ids,
                                const float* xvec, int width, float* out) {
  QTTS_CRUMB(0, 9);
  pdl_wait();
  const int r = blockIdx.x;
  const float* p = proj + (long long)proj_index[r] * width;
  const int cid = codec_ids[r];
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float v = p[c];
    if (cid >= 0) v += __bfloat162float(codec[(long long)cid * width + c]);
    if (cid == -2) v += xvec[c];
    out[(long long)r * width + c] = v;
  }
}

// ---------------------------------------------------------------------------

constexpr size_t kLinearSmem = sizeof(float) * (size_t)kXFloats;
constexpr size_t kHeadSmem = sizeof(float) * 2 * (size_t)kMaxVocab;  // selector scratch

template <int MT, int RPW, int EPI>
cudaError_t configure_linear_t() {
  return cudaFuncSetAttribute(k_linear<MT, RPW, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kLinearSmem);
}

template <int EPI>
cudaError_t configure_linear_epi() {
  cudaError_t e;
  if ((e = configure_linear_t<1, 1, EPI>()) != cudaSuccess) return e;
  if ((e = configure_linear_t<1, 2, EPI>()) != cudaSuccess) return e;
  if ((e = configure_linear_t<2, 1, EPI>()) != cudaSuccess) return e;
  if ((e = configure_linear_t<2, 2, EPI>()) != cudaSuccess) return e;
  if ((e = configure_linear_t<8, 1, EPI>()) != cudaSuccess) return e;
  return configure_linear_t<8, 2, EPI>();
}

template <int MT, int RPW, int EPI>
cudaError_t launch_linear_t(const LinearArgs& a, cudaStream_t stream) {
  const size_t smem = kLinearSmem;
  const int per_block = kWarps * RPW;
  dim3 grid((a.N + per_block - 1) / per_block, (a.M + MT - 1) / MT);
  return launch(k_linear<MT, RPW, EPI>, grid, dim3(kThreads), smem, stream, a);
}

template <int MT, int EPI>
cudaError_t launch_linear_mt(const LinearArgs& a, cudaStream_t stream) {
  // Two columns per warp only when that still leaves >= 2 CTAs per SM of work.
  const int blocks2 = (a.N + 2 * kWarps - 1) / (2 * kWarps);
  if (MT == 1 && blocks2 >= 256) return launch_linear_t<MT, 2, EPI>(a, stream);
  return launch_linear_t<MT, 1, EPI>(a, stream);
}

template <int KCH, int NR>
cudaError_t launch_gemv1_t(const LinearArgs& a, int epi, cudaStream_t stream) {
  const int per_block = kWarps * (epi == EPI_SWIGLU ? 1 : NR);
  dim3 grid((a.N + per_block - 1) / per_block);
  if (a.M == 2) {
    if constexpr (KCH <= 12)  // two rows of x must fit the 48 KB of static shared memory
      return launch(k_gemv1<KCH, NR, 2>, grid, dim3(kThreads), 0, stream, a, epi);
    else
      return cudaErrorInvalidValue;
  }
  return launch(k_gemv1<KCH, NR, 1>, grid, dim3(kThreads), 0, stream, a, epi);
}

template <int KCH>
cudaError_t launch_gemv1_k(const LinearArgs& a, int epi, cudaStream_t stream) {
  if (epi == EPI_SWIGLU) return launch_gemv1_t<KCH, 2>(a, epi, stream);
  // two output rows per warp while that still gives >= 256 CTAs (and K is short)
  if (KCH <= 4 && (a.N + 2 * kWarps - 1) / (2 * kWarps) >= 256)
    return launch_gemv1_t<KCH, 2>(a, epi, stream);
  return launch_gemv1_t<KCH, 1>(a, epi, stream);
}

// Decode GEMV dispatch on K (chunks of 256 per lane); false when K is unsupported.
bool launch_gemv1(const LinearArgs& a, int epi, cudaStream_t stream, cudaError_t* err) {
  if (a.M < 1 || a.M > 2 || a.K % 256 != 0) return false;
  if (a.M == 2 && a.K > 12 * 256) return false;  // two rows of x in 48 KB of static smem
  switch (a.K / 256) {
    case 1: *err = launch_gemv1_k<1>(a, epi, stream); return true;
    case 2: *err = launch_gemv1_k<2>(a, epi, stream); return true;
    case 4: *err = launch_gemv1_k<4>(a, epi, stream); return true;
    case 8: *err = launch_gemv1_k<8>(a, epi, stream); return true;
    case 12: *err = launch_gemv1_k<12>(a, epi, stream); return true;
    case 24: *err = launch_gemv1_k<24>(a, epi, stream); return true;
  }
  return false;
}

template <int EPI>
cudaError_t launch_linear_epi(const LinearArgs& a, cudaStream_t stream) {
  if (a.M <= 2) {
    cudaError_t e;
    if (launch_gemv1(a, EPI, stream, &e)) return e;
    if (a.M == 1) return launch_linear_mt<1, EPI>(a, stream);
  }
  if (a.M == 2) return launch_linear_mt<2, EPI>(a, stream);
  return launch_linear_mt<8, EPI>(a, stream);
}

}  // namespace

int max_sample_vocab() { return kMaxVocab; }

cudaError_t launch_linear(const LinearArgs& a, Epilogue epi, cudaStream_t stream) {
  if (a.K % 8 != 0 || a.ldx % 4 != 0 || a.M <= 0 || a.N <= 0) return cudaErrorInvalidValue;
  switch (epi) {
    case EPI_STORE: return launch_linear_epi<EPI_STORE>(a, stream);
    case EPI_RESID: return launch_linear_epi<EPI_RESID>(a, stream);
    case EPI_SWIGLU: return launch_linear_epi<EPI_SWIGLU>(a, stream);
    case EPI_BIAS: return launch_linear_epi<EPI_BIAS>(a, stream);
    case EPI_BIAS_SILU: return launch_linear_epi<EPI_BIAS_SILU>(a, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_head(const HeadArgs& a, cudaStream_t stream) {
  if (a.lin.N > kMaxVocab || a.lin.M != 1 || a.lin.K % 256 != 0) return cudaErrorInvalidValue;
  dim3 grid((a.lin.N + kWarps - 1) / kWarps);
  switch (a.lin.K / 256) {
    case 1: return launch(k_head<1>, grid, dim3(kThreads), kHeadSmem, stream, a);
    case 2: return launch(k_head<2>, grid, dim3(kThreads), kHeadSmem, stream, a);
    case 4: return launch(k_head<4>, grid, dim3(kThreads), kHeadSmem, stream, a);
    case 8: return launch(k_head<8>, grid, dim3(kThreads), kHeadSmem, stream, a);
  }
  return cudaErrorInvalidValue;
}

cudaError_t configure_kernels() {
  cudaError_t e;
  if ((e = configure_linear_epi<EPI_STORE>()) != cudaSuccess) return e;
  if ((e = configure_linear_epi<EPI_RESID>()) != cudaSuccess) return e;
  if ((e = configure_linear_epi<EPI_SWIGLU>()) != cudaSuccess) return e;
  if ((e = configure_linear_epi<EPI_BIAS>()) != cudaSuccess) return e;
  if ((e = configure_linear_epi<EPI_BIAS_SILU>()) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k_head<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHeadSmem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k_head<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHeadSmem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k_head<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHeadSmem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k_select_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHeadSmem)) != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_head<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHeadSmem);
}

bool attn_o_fusable(const AttnDecodeArgs& at, const LinearArgs& o) {
  return !at.pos_ptr && at.pos_const < kCpFusedPositions && at.q_heads == 2 * at.kv.kv_heads &&
         o.M == 1 && o.K == at.q_heads * kHeadDim && !o.gamma &&
         (o.K == 512 || o.K == 1024 || o.K == 2048);
}

cudaError_t launch_attn_o(const AttnDecodeArgs& at, const LinearArgs& o, cudaStream_t stream) {
  if (!attn_o_fusable(at, o)) return cudaErrorInvalidValue;
  dim3 grid((o.N + kWarps - 1) / kWarps);
  if (o.K == 512) return launch(k_gemv1_attn<2>, grid, dim3(kThreads), 0, stream, o, at);
  if (o.K == 1024) return launch(k_gemv1_attn<4>, grid, dim3(kThreads), 0, stream, o, at);
  return launch(k_gemv1_attn<8>, grid, dim3(kThreads), 0, stream, o, at);
}

cudaError_t set_crumbs_kernels(unsigned* host_mapped_dev_ptr) {
  const Crumbs c{host_mapped_dev_ptr};
  return cudaMemcpyToSymbol(g_crumbs, &c, sizeof(c));
}

namespace {
// Self-test of the bounded waits: one thread polls a counter for a target
// that nothing will reach, with an acquire load and a %globaltimer bound, and
// reports the expiry through `status`. Nothing else is in flight in the CTA.
__global__ void k_wait_selftest(const unsigned long long* counter, unsigned long long target,
                                unsigned long long limit_ns, int* status) {
  if (threadIdx.x != 0) return;
  auto now = [] {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
  };
  const unsigned long long t0 = now();
  int expired = 0;
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(counter) : "memory");
    if (v >= target) break;
    if (now() - t0 > limit_ns) {
      expired = 1;
      break;
    }
  }
  *status = expired;
}
}  // namespace

cudaError_t launch_wait_selftest(const unsigned long long* counter, unsigned long long target,
                                 unsigned long long limit_ns, int* status, cudaStream_t stream) {
  k_wait_selftest<<<1, 32, 0, stream>>>(counter, target, limit_ns, status);
  return cudaGetLastError();
}

cudaError_t set_step_trace(unsigned long long* buf, int capacity, cudaStream_t stream) {
  const StepTrace t{buf, buf ? capacity : 0};
  return cudaMemcpyToSymbolAsync(g_trace, &t, sizeof(t), 0, cudaMemcpyHostToDevice, stream);
}

cudaError_t launch_select_batch(const BatchHeadArgs& a, int B, cudaStream_t stream) {
  if (a.h.lin.N > kMaxVocab) return cudaErrorInvalidValue;
  return launch(k_select_batch, dim3(B), dim3(kThreads), kHeadSmem, stream, a);
}

cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t stream) {
  const int G = a.q_heads / a.kv.kv_heads;
  // Fixed positions (CodePredictor, <= 17 rows): 4 warps; a position read on
  // the device (talker): 16 warps (8 with four q heads per kv head).
  const bool small = !a.pos_ptr && a.pos_const < 4 * 4 * kAttnBatch;
  dim3 grid(a.kv.kv_heads, std::max(1, a.batch));
#define QTTS_ATTN(GG)                                                                    \
  return small ? launch(k_attn_decode<GG, 4>, grid, dim3(128), 0, stream, a)             \
               : launch(k_attn_decode<GG, (GG > 2 ? 8 : 16)>, grid,              \
                        dim3(32 * (GG > 2 ? 8 : 16)), 0, stream, a)
  switch (G) {
    case 1: QTTS_ATTN(1);
    case 2: QTTS_ATTN(2);
    case 4: QTTS_ATTN(4);
  }
#undef QTTS_ATTN
  return cudaErrorInvalidValue;
}

cudaError_t launch_qk_prep(const QkPrepArgs& a, cudaStream_t stream) {
  dim3 grid(a.M, a.q_heads + a.kv.kv_heads);
  return launch(k_qk_prep, grid, dim3(128), 0, stream, a);
}

cudaError_t launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t stream) {
  dim3 grid(a.q_heads, (a.M + 3) / 4);
  return launch(k_attn_prefill, grid, dim3(128), 0, stream, a);
}

cudaError_t launch_gather_rows(const __nv_bfloat16* table, const int* ids, int n, int width,
                               float* out, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  return launch(k_gather_rows, dim3(n), dim3(256), 0, stream, table, ids, width, out);
}

cudaError_t launch_assemble_rows(const float* proj, const int* proj_index,
                                 const __nv_bfloat16* codec, const int* codec_ids,
                                 const float* xvec, int n, int width, float* out,
                                 cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  return launch(k_assemble_rows, dim3(n), dim3(256), 0, stream, proj, proj_index, codec,
                codec_ids, xvec, width, out);
}

}  // namespace qtts

