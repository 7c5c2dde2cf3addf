// Persistent per-frame kernel (sm_100a).
//
// One cooperative launch of one CTA per SM runs a whole frame: the 2-row
// CodePredictor prefill, 14 CodePredictor decode steps, the talker decode
// step and the 16 token selections. The op list is static per sampling
// configuration, so every CTA knows in advance which weight rows it needs.
//
// Weight streaming (warp specialisation): warp 8 streams this CTA's weight
// rows for every upcoming op through a ring of shared-memory stages with
// cp.async.bulk (1-D TMA bulk copies completing on mbarriers), running ahead
// of the data dependencies, so HBM reads continue while consumers wait.
//
// Dataflow without grid barriers: activations live in "tagged vectors" --
// 64-bit words holding an fp32 value and the epoch of the op that wrote it,
// written and read as single-copy-atomic 8-byte accesses. A consumer polls the
// words it needs until their tags match, so one L2 round trip both
// synchronises and delivers the data. Buffers are safe to rewrite because
// every op's output depends on every CTA having finished its reads of the
// previous contents (each op's input is produced by all CTAs).
//
// Token selection runs redundantly in every CTA on the same logits, so the
// sampled token, the next embedding and the running embedding sum are known
// CTA-locally. Every wait is bounded: on timeout the CTA records an error,
// finishes the op with garbage, stops at the next uniform check, drains its
// bulk copies and exits.
//
// Reference semantics: decode.rs:1694-1894 (layer), code_predictor.rs:366-471
// (CodePredictor pass), talker.rs:431-496 (head), generation.rs:697-740
// (frame), kernels.rs (per-op math, see kernels.cu).
#include <float.h>

#include "frame_kernel.h"
#include "sm100.cuh"
#include "select.cuh"

namespace qtts {
namespace {

constexpr unsigned kSpinLimit = 1u << 22;
constexpr int kCT = 256;  // consumer threads

__device__ __forceinline__ void tv_st(TV* p, float v, unsigned tag) {
  const TV w = ((TV)tag << 32) | (TV)__float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ TV tv_ld(const TV* p) {
  TV v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void tv_ld2(const TV* p, TV& a, TV& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned tv_tag(TV w) { return (unsigned)(w >> 32); }
__device__ __forceinline__ float tv_val(TV w) { return __uint_as_float((unsigned)w); }

struct Shared {
  uint64_t full[kFrameStages];
  uint64_t empty[kFrameStages];
  int abort;
  int prod_done;
  unsigned issued;
  int talker_pos;
  int frame;
  int sem;
  int halt;
  unsigned seq;
  float inv[2];
  float red[8][4];
  float ml[256];  // talker attention partial (max, sum) pairs, 128 (head, split) entries
  // The current op, copied from global memory once per op: its fields are
  // read after every barrier/fence, which would otherwise re-load them from L2.
  FrameOp op;
};

static_assert(sizeof(Shared) <= kFrameSharedTail, "shared tail too small");

struct Ctx {
  int use_counters;
  const FrameOp* ops;
  unsigned* counters;
  uint8_t* ring;
  float* scratch;
  float* xloc;
  float* esum;
  Shared* sh;
  int* error;
  long long* trace;  // this op's trace slots (CTA trace_cta, thread 0) or nullptr
  int op;
  int stage;
  unsigned round;
  unsigned consumed;
};

__device__ __forceinline__ void csync() { SyncConsumers::sync(); }

__device__ __noinline__ void report_timeout(Ctx& c, int code) {
  if (!*(volatile int*)&c.sh->abort) {
    atomicExch(c.error, code);
    atomicExch(c.error + 1, c.op);
  }
  *(volatile int*)&c.sh->abort = 1;
}

// Re-reads one tagged word until its tag matches (bounded).
__device__ __forceinline__ TV tv_wait1(const TV* p, TV w, unsigned tag, Ctx& c) {
  unsigned it = 0;
  while (tv_tag(w) != tag) {
    if (++it > kSpinLimit || *(volatile int*)&c.sh->abort) {
      report_timeout(c, 3);
      break;
    }
    __nanosleep(128);
    w = tv_ld(p);
  }
  return w;
}
__device__ __forceinline__ void tv_wait2(const TV* p, TV& a, TV& b, unsigned tag, Ctx& c) {
  unsigned it = 0;
  while (tv_tag(a) != tag || tv_tag(b) != tag) {
    if (++it > kSpinLimit || *(volatile int*)&c.sh->abort) {
      report_timeout(c, 3);
      break;
    }
    __nanosleep(128);
    tv_ld2(p, a, b);
  }
}

__device__ __forceinline__ bool wait_stage(Ctx& c) {
  for (unsigned i = 0; i < kSpinLimit; ++i) {
    if (mbar_try(&c.sh->full[c.stage], c.round & 1u)) return true;
    if (*(volatile int*)&c.sh->abort) return false;
    __nanosleep(32);
  }
  report_timeout(c, 2);
  return false;
}

__device__ __forceinline__ void release_stage(Ctx& c, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(&c.sh->empty[c.stage]);
  ++c.consumed;
  if (++c.stage == kFrameStages) { c.stage = 0; ++c.round; }
}

// Waits until every writer CTA of op `j` has bumped its completion counter
// (one polling thread per CTA), then releases the consumer warps.
__device__ __forceinline__ void wait_op(Ctx& c, int j) {
  if (!c.use_counters) return;
  if (threadIdx.x == 0) {
    const unsigned* cnt = c.counters + 8 * j;
    const unsigned need = (unsigned)c.ops[j].writers;
    unsigned it = 0, v;
    while (true) {
      asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
      if (v >= need) break;
      if (++it > kSpinLimit || *(volatile int*)&c.sh->abort) {
        report_timeout(c, 5);
        break;
      }
      __nanosleep(32);
    }
  }
  csync();
}

// Called by thread 0 after the op's outputs were stored by this CTA (and a
// consumer barrier): the data words carry tags, so no fence is needed here.
__device__ __forceinline__ void signal_op(Ctx& c) {
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(c.counters + 8 * c.op) : "memory");
}

// Stages K tagged floats (times gamma) into dst; accumulates the sum of
// squares of the raw values. K even, K <= 6144.
__device__ __forceinline__ void stage_tagged(const TV* src, int K, unsigned tag, const float* gamma, float* dst,
                             float& ss, Ctx& c) {
  const int tid = threadIdx.x;
  for (int j0 = 0; j0 * 512 < K; j0 += 4) {
    TV a[4], b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = tid * 2 + (j0 + j) * 512;
      if (i < K) tv_ld2(src + i, a[j], b[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = tid * 2 + (j0 + j) * 512;
      if (i < K) {
        tv_wait2(src + i, a[j], b[j], tag, c);
        float v0 = tv_val(a[j]), v1 = tv_val(b[j]);
        ss += v0 * v0 + v1 * v1;
        if (gamma) {
          v0 *= __ldg(gamma + i);
          v1 *= __ldg(gamma + i + 1);
        }
        dst[i] = v0;
        dst[i + 1] = v1;
      }
    }
  }
}

// Talker attention input: combine the split partials (max, sum, acc[128]) of
// every q head into the attention output vector (flash-decode merge).
__device__ __forceinline__ void stage_partials(const FrameOp& op, unsigned tag, float* dst, float& ss, Ctx& c) {
  const int tid = threadIdx.x;
  const int NS = op.nsplit, nh = op.q_heads;
  const int stride = 2 + kHeadDim;
  for (int idx = tid; idx < nh * NS; idx += kCT) {
    const TV* p = op.x_tag + (long long)idx * stride;
    TV a, b;
    tv_ld2(p, a, b);
    tv_wait2(p, a, b, tag, c);
    c.sh->ml[2 * idx] = tv_val(a);
    c.sh->ml[2 * idx + 1] = tv_val(b);
  }
  csync();
  const int K = nh * kHeadDim;
  for (int i = tid * 2; i < K; i += 2 * kCT) {
    const int hq = i / kHeadDim, d = i % kHeadDim;
    float M = -INFINITY;
    for (int s = 0; s < NS; ++s) M = fmaxf(M, c.sh->ml[2 * (hq * NS + s)]);
    TV a[4], b[4];
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (s < NS) tv_ld2(op.x_tag + (long long)(hq * NS + s) * stride + 2 + d, a[s], b[s]);
    float L = 0.f, A0 = 0.f, A1 = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if (s >= NS) break;
      tv_wait2(op.x_tag + (long long)(hq * NS + s) * stride + 2 + d, a[s], b[s], tag, c);
      const float mt = c.sh->ml[2 * (hq * NS + s)];
      if (mt == -INFINITY) continue;
      const float f = expf(mt - M);
      L += c.sh->ml[2 * (hq * NS + s) + 1] * f;
      A0 += tv_val(a[s]) * f;
      A1 += tv_val(b[s]) * f;
    }
    const float v0 = A0 / L, v1 = A1 / L;
    ss += v0 * v0 + v1 * v1;
    dst[i] = v0;
    dst[i + 1] = v1;
  }
}

// Consumes this CTA's weight stages of one GEMV op. Warp layout: 256-wide k
// slices; `wpr` warps share a row, each keeping its slices of x in registers
// for the whole op; `NG` row groups split a stage's rows.
template <int MM>
__device__ __forceinline__ void ring_rows(Ctx& c, const float* xs, float* rowacc, int K, int n,
                                          int nseg, int R, int warp, int lane, int tid) {
  constexpr int NTM = MM == 2 ? 2 : 3;  // x slices per warp held in registers
  const int NS = K / 256;
  const int wpr = NS >= 8 ? 8 : NS;
  const int NG = 8 / wpr;
  const int g = warp / wpr, q = warp % wpr;
  float xr[MM][NTM][8];
#pragma unroll
  for (int m = 0; m < MM; ++m)
#pragma unroll
    for (int t = 0; t < NTM; ++t) {
      const int sl = q + t * wpr;
      if (sl < NS) {
        const float4 v0 = *reinterpret_cast<const float4*>(xs + m * K + sl * 256 + lane * 8);
        const float4 v1 = *reinterpret_cast<const float4*>(xs + m * K + sl * 256 + lane * 8 + 4);
        xr[m][t][0] = v0.x; xr[m][t][1] = v0.y; xr[m][t][2] = v0.z; xr[m][t][3] = v0.w;
        xr[m][t][4] = v1.x; xr[m][t][5] = v1.y; xr[m][t][6] = v1.z; xr[m][t][7] = v1.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) xr[m][t][j] = 0.f;
      }
    }
  bool live = true;
  long long t_wait = 0, t_comp = 0;
  for (int seg = 0; seg < nseg; ++seg) {
    for (int ch = 0; ch < n; ch += R) {
      const int rows_here = min(R, n - ch);
      const long long tw0 = clock64();
      if (live && !wait_stage(c)) live = false;  // loop shape stays uniform
      const long long tc0 = clock64();
      t_wait += tc0 - tw0;
      if (!live) continue;
      const __nv_bfloat16* stage =
          reinterpret_cast<const __nv_bfloat16*>(c.ring + c.stage * kFrameStageBytes);
      // four rows per pass so their loads and shuffle reductions overlap
      for (int i0 = g; i0 < rows_here; i0 += 4 * NG) {
        float acc[4][MM];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int m = 0; m < MM; ++m) acc[r][m] = 0.f;
#pragma unroll
        for (int t = 0; t < NTM; ++t) {
          const int sl = q + t * wpr;
          if (sl >= NS) continue;
          uint4 wv[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int i = i0 + r * NG;
            wv[r] = i < rows_here
                        ? *reinterpret_cast<const uint4*>(stage + i * K + sl * 256 + lane * 8)
                        : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            float f[8];
            unpack8(wv[r], f);
#pragma unroll
            for (int m = 0; m < MM; ++m)
#pragma unroll
              for (int j = 0; j < 8; ++j) acc[r][m] = fmaf(f[j], xr[m][t][j], acc[r][m]);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int m = 0; m < MM; ++m) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);
        if (lane == 0) {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int i = i0 + r * NG;
            if (i < rows_here) {
              float* dst = rowacc + ((seg * n + ch + i) * 8 + q) * 2;
#pragma unroll
              for (int m = 0; m < MM; ++m) dst[m] = acc[r][m];
            }
          }
        }
      }
      release_stage(c, lane);
      t_comp += clock64() - tc0;
    }
  }
  if (c.trace && tid == 0) {
    c.trace[5] = t_wait;
    c.trace[6] = t_comp;
  }
}

// ---------------------------------------------------------------------------
// GEMV over this CTA's rows; weights arrive through the ring.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool op_gemv(const FrameOp& op, Ctx& c) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = op.K, M = op.M;
  const unsigned seq = c.sh->seq;
  const unsigned tag_out = frame_tag(seq, c.op);
  float* xs = c.scratch;
  float* rowacc = c.scratch + M * K;
  int r0, r1;
  frame_rows(op.N, blockIdx.x, gridDim.x, &r0, &r1);
  const int n = r1 - r0;
  // residual prefetch (produced at least two ops earlier)
  TV rw = 0;
  float rv = 0.f;
  if (op.epi == EPI_RESID && tid < n * M) {
    const int m = tid / n, j = tid - m * n;
    if (op.r_src == FSRC_TAG) rw = tv_ld(op.r_tag + (long long)m * op.ldr + r0 + j);
    else rv = __ldcg(op.r_ext + (long long)m * op.ldr + r0 + j);
  }
  if (op.x_src == FSRC_TAG || op.x_src == FSRC_PARTIALS) wait_op(c, op.x_op);
  if (c.trace && tid == 0) c.trace[1] = clock64();
  // stage x (times gamma) and its sum of squares
  for (int m = 0; m < M; ++m) {
    float ss = 0.f;
    if (op.x_src == FSRC_TAG) {
      stage_tagged(op.x_tag + (long long)m * op.ldx, K, frame_tag(seq, op.x_op), op.gamma,
                   xs + m * K, ss, c);
    } else if (op.x_src == FSRC_PARTIALS) {
      stage_partials(op, frame_tag(seq, op.x_op), xs, ss, c);
    } else {
      const float* src = op.x_src == FSRC_LOCAL ? c.xloc : op.x_ext + (long long)m * op.ldx;
      for (int i = tid * 4; i < K; i += kCT * 4) {
        float4 v = op.x_src == FSRC_LOCAL ? *reinterpret_cast<const float4*>(src + i)
                                          : __ldcg(reinterpret_cast<const float4*>(src + i));
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        if (op.gamma) {
          const float4 g = __ldg(reinterpret_cast<const float4*>(op.gamma + i));
          v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
        }
        *reinterpret_cast<float4*>(xs + m * K + i) = v;
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) c.sh->red[warp][m] = ss;
  }
  csync();
  if (c.trace && tid == 0) c.trace[2] = clock64();
  if (tid < M) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += c.sh->red[w][tid];
    c.sh->inv[tid] = op.gamma ? rsqrtf(t / (float)K + op.eps) : 1.0f;
  }
  const int nseg = op.epi == EPI_SWIGLU ? 2 : 1;
  const int R = frame_rows_per_stage(K);
  const int wpr = K / 256 >= 8 ? 8 : K / 256;
  if (M == 2)
    ring_rows<2>(c, xs, rowacc, K, n, nseg, R, warp, lane, tid);
  else
    ring_rows<1>(c, xs, rowacc, K, n, nseg, R, warp, lane, tid);
  csync();
  if (c.trace && tid == 0) c.trace[3] = clock64();
  if (*(volatile int*)&c.sh->abort) return false;
  if (tid < n * M) {
    const int m = tid / n, j = tid - m * n;
    const float sc = c.sh->inv[m];
    float acc = 0.f;
    for (int qq = 0; qq < wpr; ++qq) acc += rowacc[(j * 8 + qq) * 2 + m];
    acc *= sc;
    const int row = r0 + j;
    float out;
    if (op.epi == EPI_SWIGLU) {
      float u = 0.f;
      for (int qq = 0; qq < wpr; ++qq) u += rowacc[((n + j) * 8 + qq) * 2 + m];
      u *= sc;
      out = acc / (1.0f + expf(-acc)) * u;
    } else {
      out = acc;
      if (op.epi == EPI_RESID) {
        if (op.r_src == FSRC_TAG) {
          const TV* rp = op.r_tag + (long long)m * op.ldr + row;
          rv = tv_val(tv_wait1(rp, rw, frame_tag(seq, op.r_op), c));
        }
        out += rv;
      }
      if (op.epi == EPI_BIAS) out += __ldg(op.bias + row);
      if (op.epi == EPI_BIAS_SILU) {
        out += __ldg(op.bias + row);
        out = out / (1.0f + expf(-out));
      }
    }
    tv_st(op.y + (long long)m * op.ldy + row, out, tag_out);
  }
  if (c.trace && tid == 0) c.trace[7] = clock64();
  return true;
}

__device__ __forceinline__ TV* cp_cache_at(const FrameOp& op, int kind, int h, int pos) {
  return op.cp_cache +
         ((((long long)op.layer * 2 + kind) * op.kv_heads + h) * kFrameCpPositions + pos) *
             kHeadDim;
}

// ---------------------------------------------------------------------------
// Decode attention, one CTA per (q head, split). QK-RMSNorm + RoPE of the
// current position, KV append, online softmax over positions; the talker
// writes split partials (merged by the O-proj staging), the CodePredictor
// writes the final output.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void op_attn_decode(const FrameOp& op, Ctx& c) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int items = op.q_heads * op.nsplit;
  if ((int)blockIdx.x >= items) return;
  wait_op(c, op.x_op);
  const int G = op.q_heads / op.kv_heads;
  const int qh = blockIdx.x / op.nsplit, s = blockIdx.x % op.nsplit, h = qh / G;
  const unsigned seq = c.sh->seq;
  const unsigned tag_in = frame_tag(seq, op.x_op), tag_out = frame_tag(seq, c.op);
  const bool talker = op.pos_const < 0;
  const int pos = talker ? c.sh->talker_pos : op.pos_const;
  const int T = pos + 1;
  const int q_out = op.q_heads * kHeadDim, kv_out = op.kv_heads * kHeadDim;
  float* sq = c.scratch;            // [128]
  float* sk = sq + kHeadDim;        // [128]
  float* sv = sk + kHeadDim;        // [128]
  float* wm = sv + kHeadDim;        // [8]
  float* wl = wm + 8;               // [8]
  float* wacc = wl + 8;             // [8][128]
  float qr = 0.f, kr = 0.f, vr = 0.f;
  if (tid < kHeadDim) {
    const TV* pq = op.x_tag + qh * kHeadDim + tid;
    const TV* pk = op.x_tag + q_out + h * kHeadDim + tid;
    const TV* pv = op.x_tag + q_out + kv_out + h * kHeadDim + tid;
    TV wq = tv_ld(pq), wk = tv_ld(pk), wv = tv_ld(pv);
    qr = tv_val(tv_wait1(pq, wq, tag_in, c));
    kr = tv_val(tv_wait1(pk, wk, tag_in, c));
    vr = tv_val(tv_wait1(pv, wv, tag_in, c));
    const float a = warp_sum(qr * qr), b = warp_sum(kr * kr);
    if (lane == 0) { c.sh->red[warp][0] = a; c.sh->red[warp][1] = b; }
  }
  csync();
  if (tid < kHeadDim) {
    const float ssq = c.sh->red[0][0] + c.sh->red[1][0] + c.sh->red[2][0] + c.sh->red[3][0];
    const float ssk = c.sh->red[0][1] + c.sh->red[1][1] + c.sh->red[2][1] + c.sh->red[3][1];
    sq[tid] = qr * rsqrtf(ssq / (float)kHeadDim + op.eps) * __ldg(op.q_gamma + tid);
    sk[tid] = kr * rsqrtf(ssk / (float)kHeadDim + op.eps) * __ldg(op.k_gamma + tid);
  }
  csync();
  float rq = 0.f, rk = 0.f;
  if (tid < kHeadDim) {
    const int pi = tid & 63;
    const float cs = __ldg(op.rope_cos + pos * 64 + pi), sn = __ldg(op.rope_sin + pos * 64 + pi);
    const float x0 = sq[pi], x1 = sq[pi + 64];
    rq = tid < 64 ? x0 * cs - x1 * sn : x1 * cs + x0 * sn;
    const float k0 = sk[pi], k1 = sk[pi + 64];
    rk = tid < 64 ? k0 * cs - k1 * sn : k1 * cs + k0 * sn;
  }
  csync();
  if (tid < kHeadDim) {
    const __nv_bfloat16 kb = __float2bfloat16_rn(rk), vb = __float2bfloat16_rn(vr);
    sq[tid] = rq;
    sk[tid] = __bfloat162float(kb);
    sv[tid] = __bfloat162float(vb);
    if (qh % G == 0 && s == 0) {
      if (talker) {
        kv_ptr(op.kv, op.layer, 0, h, pos)[tid] = kb;
        kv_ptr(op.kv, op.layer, 1, h, pos)[tid] = vb;
      } else {
        tv_st(cp_cache_at(op, 0, h, pos) + tid, sk[tid], tag_out);
        tv_st(cp_cache_at(op, 1, h, pos) + tid, sv[tid], tag_out);
      }
    }
  }
  csync();
  const int chunk = (T + op.nsplit - 1) / op.nsplit;
  const int start = s * chunk, end = min(T, start + chunk);
  float q[4], acc[4] = {0.f, 0.f, 0.f, 0.f}, m = -INFINITY, l = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) q[j] = sq[4 * lane + j];
  for (int p0 = start + warp; p0 < end; p0 += 16) {
    float kf[2][4], vf[2][4];
    // issue the loads of up to two positions before using any
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int pp = p0 + 8 * u;
      if (pp >= end) continue;
      if (pp == pos) {
#pragma unroll
        for (int j = 0; j < 4; ++j) { kf[u][j] = sk[4 * lane + j]; vf[u][j] = sv[4 * lane + j]; }
      } else if (talker) {
        const uint2 ku = __ldcg(reinterpret_cast<const uint2*>(kv_ptr(op.kv, op.layer, 0, h, pp) + 4 * lane));
        const uint2 vu = __ldcg(reinterpret_cast<const uint2*>(kv_ptr(op.kv, op.layer, 1, h, pp) + 4 * lane));
        kf[u][0] = bf16lo(ku.x); kf[u][1] = bf16hi(ku.x); kf[u][2] = bf16lo(ku.y); kf[u][3] = bf16hi(ku.y);
        vf[u][0] = bf16lo(vu.x); vf[u][1] = bf16hi(vu.x); vf[u][2] = bf16lo(vu.y); vf[u][3] = bf16hi(vu.y);
      } else {
        const TV* kp = cp_cache_at(op, 0, h, pp) + 4 * lane;
        const TV* vp = cp_cache_at(op, 1, h, pp) + 4 * lane;
        TV w[8];
        tv_ld2(kp, w[0], w[1]);
        tv_ld2(kp + 2, w[2], w[3]);
        tv_ld2(vp, w[4], w[5]);
        tv_ld2(vp + 2, w[6], w[7]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const TV* src = j < 4 ? kp + j : vp + j - 4;
          unsigned it = 0;
          while ((tv_tag(w[j]) >> 12) != (seq & 0xFFFFFu)) {  // written in this launch
            if (++it > kSpinLimit || *(volatile int*)&c.sh->abort) { report_timeout(c, 4); break; }
            __nanosleep(128);
            w[j] = tv_ld(src);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) { kf[u][j] = tv_val(w[j]); vf[u][j] = tv_val(w[4 + j]); }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (p0 + 8 * u >= end) break;
      float d = q[0] * kf[u][0] + q[1] * kf[u][1] + q[2] * kf[u][2] + q[3] * kf[u][3];
      d = warp_sum(d) * op.scale;
      const float mn = fmaxf(m, d);
      const float corr = expf(m - mn), pe = expf(d - mn);
      l = l * corr + pe;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = acc[j] * corr + pe * vf[u][j];
      m = mn;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) wacc[warp * kHeadDim + 4 * lane + j] = acc[j];
  if (lane == 0) { wm[warp] = m; wl[warp] = l; }
  csync();
  if (tid < kHeadDim) {
    float M = -INFINITY;
    for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < 8; ++w) {
        if (wm[w] == -INFINITY) continue;
        const float f = expf(wm[w] - M);
        L += wl[w] * f;
        A += wacc[w * kHeadDim + tid] * f;
      }
    }
    if (op.nsplit == 1) {
      tv_st(op.y + qh * kHeadDim + tid, A / L, tag_out);
    } else {
      TV* part = op.y + (long long)(qh * op.nsplit + s) * (2 + kHeadDim);
      if (tid == 0) { tv_st(part, M, tag_out); tv_st(part + 1, L, tag_out); }
      tv_st(part + 2 + tid, A, tag_out);
    }
  }
}

// 2-row CodePredictor prefill attention at positions 0 and 1: row 0 attends
// to itself, row 1 to both (decode.rs:1077-1298 with prefix_steps = 2).
__device__ __forceinline__ void op_attn_pair(const FrameOp& op, Ctx& c) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if ((int)blockIdx.x >= op.q_heads) return;
  wait_op(c, op.x_op);
  const int G = op.q_heads / op.kv_heads;
  const int qh = blockIdx.x, h = qh / G;
  const unsigned seq = c.sh->seq;
  const unsigned tag_in = frame_tag(seq, op.x_op), tag_out = frame_tag(seq, c.op);
  const int q_out = op.q_heads * kHeadDim, kv_out = op.kv_heads * kHeadDim;
  const int ld = q_out + 2 * kv_out;
  float* nq = c.scratch;            // [2][128] normalised q
  float* nk = nq + 2 * kHeadDim;    // [2][128] normalised k
  float raw_q[2] = {0.f, 0.f}, raw_k[2] = {0.f, 0.f}, raw_v[2] = {0.f, 0.f};
  if (tid < kHeadDim) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const TV* row = op.x_tag + (long long)r * ld;
      const TV* pq = row + qh * kHeadDim + tid;
      const TV* pk = row + q_out + h * kHeadDim + tid;
      const TV* pv = row + q_out + kv_out + h * kHeadDim + tid;
      TV wq = tv_ld(pq), wk = tv_ld(pk), wv = tv_ld(pv);
      raw_q[r] = tv_val(tv_wait1(pq, wq, tag_in, c));
      raw_k[r] = tv_val(tv_wait1(pk, wk, tag_in, c));
      raw_v[r] = tv_val(tv_wait1(pv, wv, tag_in, c));
      const float a = warp_sum(raw_q[r] * raw_q[r]), b = warp_sum(raw_k[r] * raw_k[r]);
      if (lane == 0) { c.sh->red[warp][2 * r] = a; c.sh->red[warp][2 * r + 1] = b; }
    }
  }
  csync();
  if (tid < kHeadDim) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float a = 0.f, b = 0.f;
      for (int w = 0; w < 4; ++w) { a += c.sh->red[w][2 * r]; b += c.sh->red[w][2 * r + 1]; }
      nq[r * kHeadDim + tid] = raw_q[r] * rsqrtf(a / (float)kHeadDim + op.eps) * __ldg(op.q_gamma + tid);
      nk[r * kHeadDim + tid] = raw_k[r] * rsqrtf(b / (float)kHeadDim + op.eps) * __ldg(op.k_gamma + tid);
    }
  }
  csync();
  float kb[2], vb[2], q1 = 0.f;
  if (tid < kHeadDim) {
    const int pi = tid & 63;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float cs = __ldg(op.rope_cos + r * 64 + pi), sn = __ldg(op.rope_sin + r * 64 + pi);
      const float k0 = nk[r * kHeadDim + pi], k1 = nk[r * kHeadDim + pi + 64];
      const float rk = tid < 64 ? k0 * cs - k1 * sn : k1 * cs + k0 * sn;
      kb[r] = bf16_round(rk);
      vb[r] = bf16_round(raw_v[r]);
      if (r == 1) {
        const float x0 = nq[kHeadDim + pi], x1 = nq[kHeadDim + pi + 64];
        q1 = tid < 64 ? x0 * cs - x1 * sn : x1 * cs + x0 * sn;
      }
      if (qh % G == 0) {
        tv_st(cp_cache_at(op, 0, h, r) + tid, kb[r], tag_out);
        tv_st(cp_cache_at(op, 1, h, r) + tid, vb[r], tag_out);
      }
    }
    const float d0 = warp_sum(q1 * kb[0]), d1 = warp_sum(q1 * kb[1]);
    if (lane == 0) { c.sh->red[warp][0] = d0; c.sh->red[warp][1] = d1; }
  }
  csync();
  if (tid < kHeadDim) {
    const float s0 = (c.sh->red[0][0] + c.sh->red[1][0] + c.sh->red[2][0] + c.sh->red[3][0]) * op.scale;
    const float s1 = (c.sh->red[0][1] + c.sh->red[1][1] + c.sh->red[2][1] + c.sh->red[3][1]) * op.scale;
    const float mx = fmaxf(s0, s1);
    const float e0 = expf(s0 - mx), e1 = expf(s1 - mx);
    tv_st(op.y + qh * kHeadDim + tid, vb[0], tag_out);  // softmax over one key is exactly 1
    tv_st(op.y + q_out + qh * kHeadDim + tid, (e0 * vb[0] + e1 * vb[1]) / (e0 + e1), tag_out);
  }
}

// LM head over this CTA's vocab rows, then the same token selection in every
// CTA, then the embedding bookkeeping of the role.
__device__ __forceinline__ bool op_head(const FrameOp& op, const FrameParams& p, Ctx& c, Rng& rng) {
  const int tid = threadIdx.x;
  const int H = p.H;
  if (!op_gemv(op, c)) return false;
  long long* tr = (c.trace != nullptr)
                      ? p.trace + 8 * p.n_ops + 4 * op.group + (op.role == ROLE_TALKER_STEP ? 64 : 0)
                      : nullptr;
  if (tr) tr[0] = clock64();
  const bool talker = op.role == ROLE_TALKER_STEP;
  if (talker && blockIdx.x == 0) {
    // normalised talker hidden = next frame's CodePredictor input row 0
    const float inv = c.sh->inv[0];
    for (int i = tid; i < H; i += kCT) p.cp_prefix[i] = c.scratch[i] * inv;
  }
  csync();
  if (tid == 0) signal_op(c);
  wait_op(c, c.op);
  const int V = op.N;
  const unsigned tag_out = frame_tag(c.sh->seq, c.op);
  Selector<SyncConsumers> sel{c.scratch, reinterpret_cast<int*>(c.scratch + kSelMaxVocab)};
  float ss = 0.f;
  stage_tagged(op.y, V, tag_out, nullptr, sel.val, ss, c);
  csync();
  if (tr) tr[1] = clock64();
  if (*(volatile int*)&c.sh->abort) return false;
  const int frame = c.sh->frame, sem = c.sh->sem;
  if (talker)
    sel.penalise(V, p.history, frame, sem, op.penalty, op.suppress, p.eos_token);
  else
    sel.penalise(V, p.history, 0, -1, 1.0f, op.suppress, p.eos_token);
  const int tok = sel.select(V, op.cfg, rng, &p.st->error);
  if (tr) tr[2] = clock64();
  int r0, r1;
  frame_rows(H, blockIdx.x, gridDim.x, &r0, &r1);
  if (!talker) {
    const __nv_bfloat16* e = op.emb + (long long)tok * H;
    const bool last = op.group == op.last_group;
    const float* tr = nullptr;
    const __nv_bfloat16* se = nullptr;
    if (last) {
      tr = frame < __ldcg(&p.st->n_trailing) ? p.trailing + (long long)frame * H : p.tts_pad;
      se = p.talker_codec_emb + (long long)sem * H;
    }
    for (int i = tid; i < H; i += kCT) {
      const float ev = __bfloat162float(e[i]);
      const float sum = op.group == 0 ? ev : c.esum[i] + ev;
      c.esum[i] = sum;
      c.xloc[i] = last ? (__bfloat162float(se[i]) + sum) + __ldcg(tr + i) : ev;
    }
    csync();
    for (int i = r0 + tid; i < r1; i += kCT) tv_st(op.next_x + i, c.xloc[i], tag_out);
    if (blockIdx.x == 0 && tid == 0) {
      p.codes[(long long)frame * p.groups + 1 + op.group] = tok;
      if (last) {
        p.codes[(long long)frame * p.groups] = sem;
        p.history[frame] = sem;
      }
    }
  } else if (blockIdx.x == 0) {
    const __nv_bfloat16* e = p.talker_codec_emb + (long long)tok * H;
    for (int i = tid; i < H; i += kCT) p.cp_prefix[H + i] = __bfloat162float(e[i]);
    if (tid == 0) {
      p.st->semantic = tok;
      if (tok == p.eos_token) p.st->halt = 1;
    }
  }
  csync();
  if (tr) tr[3] = clock64();
  return true;
}

__device__ __forceinline__ void producer(const FrameParams& p, Ctx& c) {
  const int lane = threadIdx.x & 31;
  if (lane != 0) return;
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  int stage = 0;
  unsigned round = 0, issued = 0;
  for (int oi = 0; oi < p.n_ops; ++oi) {
    // fields loaded once into registers (the loop below has memory clobbers)
    const int kind = __ldg(&p.ops[oi].kind);
    if (kind != FOP_GEMV && kind != FOP_HEAD) continue;
    const int N = __ldg(&p.ops[oi].N), K = __ldg(&p.ops[oi].K), epi = __ldg(&p.ops[oi].epi);
    const __nv_bfloat16* W = p.ops[oi].W;
    int r0, r1;
    frame_rows(N, blockIdx.x, gridDim.x, &r0, &r1);
    const int n = r1 - r0;
    const int nseg = epi == EPI_SWIGLU ? 2 : 1;
    const int R = frame_rows_per_stage(K);
    for (int seg = 0; seg < nseg; ++seg) {
      const long long base = seg == 0 ? r0 : (long long)N + r0;
      for (int ch = 0; ch < n; ch += R) {
        const int rows = min(R, n - ch);
        const unsigned bytes = (unsigned)rows * K * 2u;
        bool ok = false;
        for (unsigned i = 0; i < kSpinLimit; ++i) {
          if (mbar_try(&c.sh->empty[stage], (round & 1u) ^ 1u)) { ok = true; break; }
          if (*(volatile int*)&c.sh->abort) break;
          __nanosleep(256);  // a full ring can stay full for microseconds
        }
        if (!ok) {
          // consumers turn a stall into an abort at a uniform point; the
          // producer only stops issuing
          *(volatile unsigned*)&c.sh->issued = issued;
          __threadfence_block();
          *(volatile int*)&c.sh->prod_done = 1;
          return;
        }
        mbar_expect_tx(&c.sh->full[stage], bytes);
        bulk_g2s(c.ring + stage * kFrameStageBytes, W + (base + ch) * K, bytes,
                 &c.sh->full[stage], policy);
        ++issued;
        if (++stage == kFrameStages) { stage = 0; ++round; }
      }
    }
  }
  *(volatile unsigned*)&c.sh->issued = issued;
  __threadfence_block();
  *(volatile int*)&c.sh->prod_done = 1;
}

// After an abort: wait (bounded) for the producer to stop, then for every copy
// it issued to land, so no bulk copy targets shared memory after exit.
__device__ __forceinline__ void drain(Ctx& c) {
  if (threadIdx.x != 0) return;
  for (unsigned i = 0; i < kSpinLimit && !*(volatile int*)&c.sh->prod_done; ++i) __nanosleep(64);
  const unsigned issued = *(volatile unsigned*)&c.sh->issued;
  while (c.consumed < issued) {
    for (unsigned i = 0; i < kSpinLimit; ++i)
      if (mbar_try(&c.sh->full[c.stage], c.round & 1u)) break;
    ++c.consumed;
    if (++c.stage == kFrameStages) { c.stage = 0; ++c.round; }
  }
}

__global__ void __launch_bounds__(kFrameThreads, 1) k_frame(FrameParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  Ctx c;
  c.ring = smem;
  c.scratch = reinterpret_cast<float*>(smem + kFrameStages * kFrameStageBytes);
  c.xloc = reinterpret_cast<float*>(smem + kFrameStages * kFrameStageBytes + kFrameScratchBytes);
  c.esum = c.xloc + kFrameMaxH;
  c.sh = reinterpret_cast<Shared*>(c.esum + kFrameMaxH);
  c.error = p.error;
  c.ops = p.ops;
  c.use_counters = p.use_counters;
  c.counters = p.counters;
  c.trace = nullptr;
  c.op = -1;
  c.stage = 0;
  c.round = 0;
  c.consumed = 0;
  const int tid = threadIdx.x;
  if (tid == 0) {
    const SeqState* st = p.st;
    c.sh->halt = __ldcg(&st->halt);
    c.sh->frame = __ldcg(&st->frames);
    c.sh->sem = __ldcg(&st->semantic);
    c.sh->talker_pos = __ldcg(&st->prefill_len) + c.sh->frame;
    c.sh->seq = __ldcg(p.seq) & 0xFFFFFu;
    c.sh->abort = 0;
    c.sh->prod_done = 0;
    c.sh->issued = 0;
    for (int s = 0; s < kFrameStages; ++s) {
      mbar_init(&c.sh->full[s], 1);
      mbar_init(&c.sh->empty[s], 8);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (c.sh->halt) return;
  if (tid >= kCT) {
    producer(p, c);
    return;
  }
  Rng rng{p.st->rng_kind, __ldcg(&p.st->rng_state), __ldcg(&p.st->rng_seed),
          __ldcg(&p.st->rng_counter)};
  const bool tracing = p.trace && (int)blockIdx.x == p.trace_cta && tid == 0 &&
                       c.sh->frame == p.trace_frame;
  bool ok = true;
  for (int oi = 0; oi < p.n_ops && ok; ++oi) {
    {
      constexpr int kWords = sizeof(FrameOp) / 4;
      const int* src = reinterpret_cast<const int*>(p.ops + oi);
      int* dst = reinterpret_cast<int*>(&c.sh->op);
      for (int i = tid; i < kWords; i += kCT) dst[i] = __ldg(src + i);
      csync();
    }
    const FrameOp& op = c.sh->op;
    c.op = oi;
    c.trace = tracing ? p.trace + 8 * oi : nullptr;
    if (tracing) { p.trace[8 * oi] = clock64(); p.trace[8 * oi + 5] = 0; p.trace[8 * oi + 6] = 0; }
    switch (op.kind) {
      case FOP_GEMV: ok = op_gemv(op, c); break;
      case FOP_HEAD: ok = op_head(op, p, c, rng); break;
      case FOP_ATTN_DECODE: op_attn_decode(op, c); break;
      case FOP_ATTN_PAIR: op_attn_pair(op, c); break;
    }
    if (!ok) *(volatile int*)&c.sh->abort = 1;
    csync();
    ok = !*(volatile int*)&c.sh->abort;
    if (ok && tid == 0 && op.kind != FOP_HEAD &&
        (op.kind == FOP_GEMV || (int)blockIdx.x < op.writers))
      signal_op(c);
    if (tracing) p.trace[8 * oi + 4] = clock64();
  }
  if (!ok) {
    drain(c);
    return;
  }
  if (blockIdx.x == 0 && tid == 0) {
    p.st->rng_state = rng.state;
    p.st->rng_counter = rng.counter;
    p.st->frames = c.sh->frame + 1;
    p.st->talker_pos = c.sh->talker_pos + 1;
    *p.seq = (c.sh->seq + 1u) & 0xFFFFFu;
  }
}

}  // namespace

cudaError_t configure_frame_kernel() {
  return cudaFuncSetAttribute(k_frame, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kFrameSmem);
}

int frame_grid_size(int device) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_frame, kFrameThreads, kFrameSmem) !=
      cudaSuccess)
    return 0;
  return per_sm >= 1 ? sms : 0;
}

cudaError_t launch_frame(const FrameParams& p, int grid, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(p.counters, 0, sizeof(unsigned) * 8 * (size_t)p.n_ops, stream);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFrameThreads);
  cfg.dynamicSmemBytes = kFrameSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_frame, p);
}

}  // namespace qtts
