// Persistent CodePredictor pass (sm_100a): one cooperative launch per frame.
//
// Reference semantics: generate_inner[_sampled] (code_predictor.rs:366-471):
// a 2-row prefill at positions 0, 1, head 0, then groups g = 1..14 decoded
// at position g + 1, each followed by lm_heads[g] and a token; the decoder
// layer is decode_step_layer_on_stream (decode.rs:1694-1894), the 1.7B input
// projection project_to_stack (code_predictor.rs:754-817), the head
// logits_for_hidden (code_predictor.rs:819-862), and the frame tail
// build_step_input (talker.rs:320-356). Per-op arithmetic (RMSNorm folded into
// the projection, QK-norm + RoPE + bf16 KV, softmax, SwiGLU, token selection)
// is the same as the per-op kernels in kernels.cu.
//
// Structure: eight warps per CTA, one CTA per SM. Thread 0 keeps a ring of
// shared-memory stages filled with this CTA's weight rows of the upcoming ops
// (cp.async.bulk, completion on mbarriers): after each op it refills the
// stages that op consumed, so the copies of later ops run while this one
// waits on its data dependencies. An op that reads another CTA's output first
// waits for the grid arrival counter to show every CTA done with the previous
// op; it stages its input, multiplies this CTA's rows from the ring, stores,
// and adds one to the counter. The next op's descriptor is prefetched into
// shared memory (cp.async) while the current op runs.
//
// Every wait is bounded (2 s of %globaltimer): on expiry the CTA records an
// error, stops, lets its bulk copies land and exits; the host reads the error.
#include <float.h>

#include "cp_pass.h"
#include "select.cuh"
#include "sm100.cuh"

namespace qtts {
namespace {

constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr int kCW = 8;            // consumer warps
constexpr int kCT = kCW * 32;     // consumer threads

struct CpShared {
  uint64_t full[kCpStages];
  unsigned long long base;  // arrival count before this launch
  int abort;
  int frame, sem, n_trailing, prefill_len;
  float inv[2];
  float red[kCW][2];
};

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __noinline__ void cp_fail(CpShared* sh, int* err, int code, int op) {
  if (atomicCAS(err, 0, code) == 0) atomicExch(err + 1, op);
  *(volatile int*)&sh->abort = 1;
}

// Thread 0 of the consumers: waits until `target` arrivals are counted.
__device__ __forceinline__ void grid_wait(const CpPassParams& p, CpShared* sh,
                                          unsigned long long target, int op) {
  if (ld_acquire64(p.counter) >= target) return;
  const unsigned long long t0 = gtime();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (ld_acquire64(p.counter) >= target) return;
    if (*(volatile int*)&sh->abort) return;
    if (gtime() - t0 > kWaitNs) {
      cp_fail(sh, p.error, 1, op);
      return;
    }
  }
}

__device__ __forceinline__ bool stage_wait(CpShared* sh, uint64_t* bar, unsigned parity,
                                           int* err, int code, int op) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtime();
  for (;;) {
    for (int i = 0; i < 16; ++i)
      if (mbar_try(bar, parity)) return true;
    if (*(volatile int*)&sh->abort) return false;
    if (gtime() - t0 > kWaitNs) {
      cp_fail(sh, err, code, op);
      return false;
    }
  }
}

// This CTA's weight rows of an op: one contiguous chunk, two for SwiGLU
// (gate rows, then the same channels' up rows).
struct Slice {
  const char* src[2];
  int rows;     // rows per chunk
  int nchunk;
  int row_bytes;
  int r0;       // first output row / channel
};

__device__ __forceinline__ Slice op_slice(const CpOp& op, int b, int G) {
  Slice s;
  s.r0 = op.N * b / G;  // N * G < 2^31 for every supported shape
  const int r1 = op.N * (b + 1) / G;
  s.rows = r1 - s.r0;
  s.row_bytes = op.K * 2;
  s.nchunk = op.epi == EPI_SWIGLU ? 2 : 1;
  s.src[0] = reinterpret_cast<const char*>(op.W + (long long)s.r0 * op.K);
  s.src[1] = reinterpret_cast<const char*>(op.W + (long long)(op.N + s.r0) * op.K);
  return s;
}

__device__ __forceinline__ int rows_per_stage(int row_bytes) {
  return kCpStageBytes / row_bytes;
}

__device__ __forceinline__ int rows_per_stage_of(const CpLoad& w) {
  return kCpStageBytes / (2 * w.K);
}

// Thread 0's view of the ring: the next piece to copy (op, chunk, first row)
// and how many pieces were issued; pieces are consumed in the same order.
struct Filler {
  int op, chunk, row;
  unsigned issued;
};

// Issues copies for free stages (the consumers have read every issued piece
// up to `consumed`) until the ring is full or every op's rows are issued.
__device__ __forceinline__ void top_up(const CpPassParams& p, CpShared* sh, char* ring,
                                       const CpLoad* loads, Filler& f, unsigned consumed,
                                       unsigned long long pol) {
  const int G = gridDim.x;
  while (f.op < p.n_ops && f.issued - consumed < (unsigned)kCpStages) {
    const CpLoad w = loads[f.op];
    const int r0 = w.N * (int)blockIdx.x / G;
    const int r1 = w.N * ((int)blockIdx.x + 1) / G;
    const int rows = r1 - r0, rps = rows_per_stage_of(w);
    if (f.row >= rows) {  // this chunk is done (or empty)
      f.row = 0;
      if (++f.chunk >= w.nchunk) {
        f.chunk = 0;
        ++f.op;
      }
      continue;
    }
    const int n = min(rps, rows - f.row);
    const int stage = (int)(f.issued % kCpStages);
    const size_t row_bytes = (size_t)w.K * 2;
    const char* src = reinterpret_cast<const char*>(w.W) +
                      ((size_t)(f.chunk ? w.N : 0) + r0 + f.row) * row_bytes;
    const unsigned bytes = (unsigned)(n * row_bytes);
    mbar_expect_tx(&sh->full[stage], bytes);
    bulk_g2s(ring + (size_t)stage * kCpStageBytes, src, bytes, &sh->full[stage], pol);
    ++f.issued;
    f.row += n;
  }
}

// Before the CTA exits: every issued copy must have landed (waiting for the
// last fill of each stage covers the earlier ones).
__device__ __forceinline__ void drain(const CpPassParams& p, CpShared* sh, const Filler& f) {
  for (int s = 0; s < kCpStages; ++s) {
    if ((unsigned)s >= f.issued) break;
    const unsigned last = f.issued - 1u - ((f.issued - 1u - (unsigned)s) % kCpStages);
    const unsigned parity = (last / kCpStages) & 1u;
    const unsigned long long t0 = gtime();
    while (!mbar_try(&sh->full[s], parity)) {
      if (gtime() - t0 > kWaitNs) {
        cp_fail(sh, p.error, 3, -1);
        return;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Consumers
// ---------------------------------------------------------------------------
struct Ring {
  char* base;
  unsigned consumed;  // pieces read so far (stage = consumed % kCpStages)
};

// Dot products of weight row `wr` (bf16, K wide, in shared memory) with the
// staged input rows: lane l covers k = 8l + 256j.
template <int M>
__device__ __forceinline__ void row_dot(const __nv_bfloat16* wr, const float* xs, int K, int lane,
                                        float (&acc)[2]) {
#pragma unroll 4
  for (int k = lane * 8; k < K; k += 256) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(wr + k), f);
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float4 a0 = *reinterpret_cast<const float4*>(xs + m * K + k);
      const float4 a1 = *reinterpret_cast<const float4*>(xs + m * K + k + 4);
      float t = acc[m];
      t = fmaf(f[0], a0.x, t); t = fmaf(f[1], a0.y, t);
      t = fmaf(f[2], a0.z, t); t = fmaf(f[3], a0.w, t);
      t = fmaf(f[4], a1.x, t); t = fmaf(f[5], a1.y, t);
      t = fmaf(f[6], a1.z, t); t = fmaf(f[7], a1.w, t);
      acc[m] = t;
    }
  }
}

// Multiplies this CTA's rows of `op` (arriving through the ring) with the
// staged input rows xs[M][K]; out[row * 2 + m] = dot product (pre-scale).
// Each warp takes two rows at a time so their loads and reductions overlap.
template <int M>
__device__ __forceinline__ bool op_rows(const CpPassParams& p, CpShared* sh, Ring& rg,
                                        const CpOp& op, const Slice& sl, const float* xs,
                                        float* out, int j, unsigned long long* tr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = op.K;
  const int rps = rows_per_stage(sl.row_bytes);
  bool ok = true, first = true;
  for (int c = 0; c < sl.nchunk; ++c) {
    for (int r = 0; r < sl.rows; r += rps) {
      const int n = min(rps, sl.rows - r);
      const int stage = (int)(rg.consumed % kCpStages);
      const unsigned parity = (rg.consumed / kCpStages) & 1u;
      if (ok && !stage_wait(sh, &sh->full[stage], parity, p.error, 4, j)) ok = false;
      if (first && tr) tr[2] = gtime();
      if (tr && op.kind != CPOP_HEAD) tr[6] = gtime();  // the last piece's arrival
      first = false;
      if (ok) {
        const __nv_bfloat16* wst =
            reinterpret_cast<const __nv_bfloat16*>(rg.base + (size_t)stage * kCpStageBytes);
        for (int i = warp; i < n; i += 2 * kCW) {
          const int i2 = i + kCW;
          float a[2] = {0.f, 0.f}, b[2] = {0.f, 0.f};
          row_dot<M>(wst + (size_t)i * K, xs, K, lane, a);
          if (i2 < n) row_dot<M>(wst + (size_t)i2 * K, xs, K, lane, b);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
              a[m] += __shfl_xor_sync(0xffffffffu, a[m], o);
              b[m] += __shfl_xor_sync(0xffffffffu, b[m], o);
            }
          }
          if (lane == 0) {
            const int row = c * sl.rows + r + i;
#pragma unroll
            for (int m = 0; m < M; ++m) out[row * 2 + m] = a[m];
            if (i2 < n)
#pragma unroll
              for (int m = 0; m < M; ++m) out[(row + kCW) * 2 + m] = b[m];
          }
        }
      }
      ++rg.consumed;
    }
  }
  return ok;
}

// Stages M input rows (times gamma) into xs and their RMS scales into sh->inv.
__device__ __forceinline__ void stage_input(const CpOp& op, CpShared* sh, const float* loc_e,
                                            float* xs) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = op.K;
  for (int m = 0; m < op.M; ++m) {
    float ss = 0.f;
    for (int k = tid * 4; k < K; k += kCT * 4) {
      float4 v = op.x_src == CPSRC_LOCAL
                     ? *reinterpret_cast<const float4*>(loc_e + k)
                     : __ldcg(reinterpret_cast<const float4*>(op.x + (long long)m * op.ldx + k));
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      if (op.gamma) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(op.gamma + k));
        v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
      }
      *reinterpret_cast<float4*>(xs + m * K + k) = v;
    }
    ss = warp_sum(ss);
    if (lane == 0) sh->red[warp][m] = ss;
  }
  csync();
  if (tid < op.M) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kCW; ++w) t += sh->red[w][tid];
    sh->inv[tid] = op.gamma ? rsqrtf(t / (float)K + op.eps) : 1.0f;
  }
}

// CodePredictor attention of positions pos0 .. pos0 + M - 1 (every CTA
// computes all heads). Warp w handles kv head w (and w + 8, ...) with its two
// q heads; lane l holds dims 4l .. 4l + 3. Cached rows of earlier positions
// come from the bf16 cache; the new rows are QK-normed, roped and rounded to
// bf16 like the cache entries, and CTA 0 appends them. M is a template
// parameter so that every per-row array stays in registers.
template <int M>
__device__ __forceinline__ void stage_attention(const CpPassParams& p, const CpOp& op, float* xs,
                                                bool write_cache) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = p.kv_heads;
  const int q_out = p.q_heads * kHeadDim, kv_out = kvh * kHeadDim;
  const int d0 = 4 * lane;
  const int pos0 = op.pos0;
  const long long hs = (long long)kCpPositions * kHeadDim;  // one head's rows
  const float4 qg = __ldg(reinterpret_cast<const float4*>(op.q_gamma + d0));
  const float4 kg = __ldg(reinterpret_cast<const float4*>(op.k_gamma + d0));
  for (int g = warp; g < kvh; g += kCW) {
    __nv_bfloat16* kbase = p.cache + ((long long)(op.layer * 2 + 0) * kvh + g) * hs;
    __nv_bfloat16* vbase = p.cache + ((long long)(op.layer * 2 + 1) * kvh + g) * hs;
    // every load of this head first: cached rows, then the new rows
    uint2 kc[kCpPositions], vc[kCpPositions];
#pragma unroll
    for (int q = 0; q < kCpPositions; ++q) {
      kc[q] = make_uint2(0u, 0u);
      vc[q] = make_uint2(0u, 0u);
      if (q < pos0) {
        kc[q] = __ldcg(reinterpret_cast<const uint2*>(kbase + q * kHeadDim + d0));
        vc[q] = __ldcg(reinterpret_cast<const uint2*>(vbase + q * kHeadDim + d0));
      }
    }
    float4 qr[M][2], kr[M], vr[M];
#pragma unroll
    for (int t = 0; t < M; ++t) {
      const float* row = op.qkv + (long long)t * op.ld_qkv;
      qr[t][0] = __ldcg(reinterpret_cast<const float4*>(row + (2 * g) * kHeadDim + d0));
      qr[t][1] = __ldcg(reinterpret_cast<const float4*>(row + (2 * g + 1) * kHeadDim + d0));
      kr[t] = __ldcg(reinterpret_cast<const float4*>(row + q_out + g * kHeadDim + d0));
      vr[t] = __ldcg(reinterpret_cast<const float4*>(row + q_out + kv_out + g * kHeadDim + d0));
    }
    uint2 kn[M], vn[M];
#pragma unroll
    for (int t = 0; t < M; ++t) {
      const int pos = pos0 + t;
      const float4 rc = __ldg(reinterpret_cast<const float4*>(p.rope_cos + pos * 64 + (d0 & 63)));
      const float4 rs = __ldg(reinterpret_cast<const float4*>(p.rope_sin + pos * 64 + (d0 & 63)));
      auto norm_rope = [&](float4 x, float4 gm) {
        const float ss = warp_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
        const float inv = rsqrtf(ss / (float)kHeadDim + op.eps);
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
      qr[t][0] = norm_rope(qr[t][0], qg);
      qr[t][1] = norm_rope(qr[t][1], qg);
      const float4 kk = norm_rope(kr[t], kg);
      const float4 vv = vr[t];
      const __nv_bfloat162 kb0 = __floats2bfloat162_rn(kk.x, kk.y), kb1 = __floats2bfloat162_rn(kk.z, kk.w);
      const __nv_bfloat162 vb0 = __floats2bfloat162_rn(vv.x, vv.y), vb1 = __floats2bfloat162_rn(vv.z, vv.w);
      kn[t].x = *reinterpret_cast<const unsigned*>(&kb0); kn[t].y = *reinterpret_cast<const unsigned*>(&kb1);
      vn[t].x = *reinterpret_cast<const unsigned*>(&vb0); vn[t].y = *reinterpret_cast<const unsigned*>(&vb1);
      if (write_cache) {
        *reinterpret_cast<uint2*>(kbase + pos * kHeadDim + d0) = kn[t];
        *reinterpret_cast<uint2*>(vbase + pos * kHeadDim + d0) = vn[t];
      }
    }
#pragma unroll
    for (int t = 0; t < M; ++t) {
      const int T = pos0 + t + 1;  // keys 0 .. pos0 + t
      // key q: cached below pos0, else new row q - pos0 (0 or 1)
      auto key_at = [&](int q, const uint2* c, const uint2* nw) {
        return q < pos0 ? c[q] : (M == 2 && q > pos0 ? nw[M - 1] : nw[0]);
      };
      float d[2][kCpPositions];
#pragma unroll
      for (int q = 0; q < kCpPositions; ++q) {
        const uint2 ku = key_at(q, kc, kn);
        const float k0 = bf16lo(ku.x), k1 = bf16hi(ku.x), k2 = bf16lo(ku.y), k3 = bf16hi(ku.y);
#pragma unroll
        for (int h = 0; h < 2; ++h)
          d[h][q] = (qr[t][h].x * p.scale) * k0 + (qr[t][h].y * p.scale) * k1 +
                    (qr[t][h].z * p.scale) * k2 + (qr[t][h].w * p.scale) * k3;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int q = 0; q < kCpPositions; ++q)
            d[h][q] += __shfl_xor_sync(0xffffffffu, d[h][q], o);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float mx = -INFINITY;
#pragma unroll
        for (int q = 0; q < kCpPositions; ++q)
          if (q < T) mx = fmaxf(mx, d[h][q]);
        float l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < kCpPositions; ++q) {
          if (q >= T) continue;
          const float e = expf(d[h][q] - mx);
          const uint2 vu = key_at(q, vc, vn);
          l += e;
          acc[0] = fmaf(e, bf16lo(vu.x), acc[0]); acc[1] = fmaf(e, bf16hi(vu.x), acc[1]);
          acc[2] = fmaf(e, bf16lo(vu.y), acc[2]); acc[3] = fmaf(e, bf16hi(vu.y), acc[3]);
        }
        const float il = 1.0f / l;
        *reinterpret_cast<float4*>(xs + t * q_out + (2 * g + h) * kHeadDim + d0) =
            make_float4(acc[0] * il, acc[1] * il, acc[2] * il, acc[3] * il);
      }
    }
  }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_all;" ::: "memory");
}

__device__ void run_pass(const CpPassParams& p, CpShared* sh, char* ring, float* xs, float* loc_e,
                         float* emb_sum, float* out, const CpLoad* loads, CpOp* desc) {
  const int tid = threadIdx.x;
  const int G = gridDim.x;
  const bool cta0 = blockIdx.x == 0;
  const unsigned long long pol = l2_evict_first_policy();
  constexpr int kDescChunks = (int)(sizeof(CpOp) / 16);
  Ring rg{ring, 0u};
  Filler fill{0, 0, 0, 0u};
  if (tid == 0) top_up(p, sh, ring, loads, fill, 0u, pol);
  Rng rng{p.st->rng_kind, p.st->rng_state, p.st->rng_seed, p.st->rng_counter};
  int* sel_err = cta0 ? &p.st->error : nullptr;
  int dummy_err = 0;
  // descriptor of op 0
  if (tid < kDescChunks) cp_async16(reinterpret_cast<char*>(desc) + 16 * tid,
                                    reinterpret_cast<const char*>(p.ops) + 16 * tid);
  for (int j = 0; j < p.n_ops; ++j) {
    if (tid < kDescChunks) cp_async_commit_wait();
    csync();
    const CpOp op = desc[j & 1];
    if (j + 1 < p.n_ops && tid < kDescChunks)  // next descriptor, behind this op
      cp_async16(reinterpret_cast<char*>(desc + ((j + 1) & 1)) + 16 * tid,
                 reinterpret_cast<const char*>(p.ops + j + 1) + 16 * tid);
    if (*(volatile int*)&sh->abort) break;
    if (op.wait) {
      if (tid == 0) grid_wait(p, sh, sh->base + (unsigned long long)j * G, j);
      csync();
      if (*(volatile int*)&sh->abort) break;
    }
    unsigned long long* tr = (p.trace && cta0 && tid == 0) ? p.trace + kCpTraceSlots * j : nullptr;
    if (tr) tr[0] = gtime();
    if (op.kind == CPOP_ATTN_O) {
      if (op.M == 2) stage_attention<2>(p, op, xs, cta0);
      else stage_attention<1>(p, op, xs, cta0);
      if (tid < 2) sh->inv[tid] = 1.0f;
    } else {
      stage_input(op, sh, loc_e, xs);
    }
    csync();
    if (tr) tr[1] = gtime();
    const Slice sl = op_slice(op, blockIdx.x, G);
    const bool ok = op.M == 2 ? op_rows<2>(p, sh, rg, op, sl, xs, out, j, tr)
                              : op_rows<1>(p, sh, rg, op, sl, xs, out, j, tr);
    csync();
    if (!ok || *(volatile int*)&sh->abort) break;
    if (tr) tr[3] = gtime();
    // epilogue: this CTA's outputs
    const int n = sl.rows;
    for (int t = tid; t < n * op.M; t += kCT) {
      const int m = t / n, jj = t - m * n;
      const int row = sl.r0 + jj;
      const float sc = sh->inv[m];
      const float a = out[jj * 2 + m] * sc;
      float v;
      if (op.epi == EPI_SWIGLU) {
        const float u = out[(n + jj) * 2 + m] * sc;
        v = a / (1.0f + expf(-a)) * u;
      } else {
        v = a;
        if (op.epi == EPI_RESID)
          v += op.r_src == CPSRC_LOCAL ? loc_e[row]
                                       : __ldcg(op.resid + (long long)m * op.ldr + row);
        if (op.epi == EPI_BIAS) v += __ldg(op.bias + row);
      }
      op.y[(long long)m * op.ldy + row] = v;
      if (op.kind == CPOP_HEAD && p.dbg_logits) p.dbg_logits[(long long)op.group * p.vocab + row] = v;
    }
    csync();
    if (tid == 0) {
      // every thread's stores precede this release (barrier above)
      if (tr) tr[4] = gtime();
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(p.counter) : "memory");
      if (tr) tr[5] = gtime();
      // Every warp is past this op's stages (barriers above): refill them
      // with later ops' rows while the other CTAs finish this op.
      top_up(p, sh, ring, loads, fill, rg.consumed, pol);
      if (tr && op.kind != CPOP_HEAD) tr[8] = gtime() - tr[5];
    }
    if (op.kind != CPOP_HEAD) continue;

    // ---- token of group op.group, in every CTA on the same logits ----
    if (tid == 0) grid_wait(p, sh, sh->base + (unsigned long long)(j + 1) * G, j);
    csync();
    if (*(volatile int*)&sh->abort) break;
    const int V = op.N;
    Selector<SyncConsumers> sel{xs, reinterpret_cast<int*>(xs + kSelMaxVocab)};
    __shared__ long long s_selclk[16];
    if (tr) sel.dbg = s_selclk;
    for (int v = tid; v < V; v += kCT) sel.val[v] = __ldcg(op.y + v);
    csync();
    if (tr) tr[6] = gtime();
    const int tok = sel.select(V, p.cfg, rng, sel_err ? sel_err : &dummy_err);
    if (tr) {
      tr[7] = gtime();
      for (int q = 10; q < 16; ++q) tr[8 + (q - 10)] = (unsigned long long)(s_selclk[q] - s_selclk[10]);
    }
    // next group's input row and the running embedding sum (CTA-local)
    const __nv_bfloat16* e = p.cp_embs + ((long long)op.group * p.vocab + tok) * p.H;
    for (int i = tid * 4; i < p.H; i += kCT * 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(e + i);
      const float4 ef = make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
      float4 sm = ef;
      if (op.group != 0) {
        const float4 s0 = *reinterpret_cast<const float4*>(emb_sum + i);
        sm = make_float4(s0.x + ef.x, s0.y + ef.y, s0.z + ef.z, s0.w + ef.w);
      }
      *reinterpret_cast<float4*>(loc_e + i) = ef;
      *reinterpret_cast<float4*>(emb_sum + i) = sm;
    }
    if (cta0 && tid == 0) p.codes[(long long)sh->frame * p.groups + 1 + op.group] = tok;
  }
  if (tid < kDescChunks) cp_async_commit_wait();
  csync();
  if (tid == 0) drain(p, sh, fill);
  if (*(volatile int*)&sh->abort || !cta0) return;
  // ---- frame tail (CTA 0): codes, history, state, talker step input ----
  const int frame = sh->frame, sem = sh->sem;
  const float* trow = frame < sh->n_trailing ? p.trailing + (long long)frame * p.H : p.tts_pad;
  const __nv_bfloat16* se = p.talker_codec_emb + (long long)sem * p.H;
  for (int i = tid * 4; i < p.H; i += kCT * 4) {
    const uint2 q = *reinterpret_cast<const uint2*>(se + i);
    const float4 sm = *reinterpret_cast<const float4*>(emb_sum + i);
    const float4 t = __ldcg(reinterpret_cast<const float4*>(trow + i));
    *reinterpret_cast<float4*>(p.step_in + i) =
        make_float4((bf16lo(q.x) + sm.x) + t.x, (bf16hi(q.x) + sm.y) + t.y,
                    (bf16lo(q.y) + sm.z) + t.z, (bf16hi(q.y) + sm.w) + t.w);
    if (p.emb_sum_out) *reinterpret_cast<float4*>(p.emb_sum_out + i) = sm;
  }
  if (tid == 0) {
    p.codes[(long long)frame * p.groups] = sem;
    p.history[frame] = sem;
    p.st->talker_pos = sh->prefill_len + frame;
    p.st->frames = frame + 1;
    p.st->rng_state = rng.state;
    p.st->rng_counter = rng.counter;
  }
}

__global__ void __launch_bounds__(kCpThreads, 1) k_cp_pass(CpPassParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  char* ring = reinterpret_cast<char*>(smem);
  float* xs = reinterpret_cast<float*>(smem + (size_t)kCpStages * kCpStageBytes);
  float* loc_e = xs + kCpScratchBytes / 4;
  float* emb_sum = loc_e + kCpMaxH;
  float* out = emb_sum + kCpMaxH;
  CpLoad* loads = reinterpret_cast<CpLoad*>(out + 2 * kCpMaxRows);
  CpOp* desc = reinterpret_cast<CpOp*>(loads + kCpMaxOps);
  CpShared* sh = reinterpret_cast<CpShared*>(desc + 2);
  const int tid = threadIdx.x;
  // EOS already selected: the frame is a no-op. After a failed pass (an
  // expired wait) the remaining frames of the burst are no-ops too; the host
  // reports the failure once the burst ends.
  if (__ldcg(&p.st->halt) || __ldcg(p.error)) return;
  for (int i = tid; i < p.n_ops; i += kCT) loads[i] = p.loads[i];
  if (tid == 0) {
    for (int s = 0; s < kCpStages; ++s) mbar_init(&sh->full[s], 1);
    fence_mbar_init();
    sh->abort = 0;
    const unsigned long long per = (unsigned long long)p.n_ops * gridDim.x;
    const unsigned long long c = ld_acquire64(p.counter);
    sh->base = c - c % per;
    sh->frame = p.st->frames;
    sh->sem = p.st->semantic;
    sh->n_trailing = p.st->n_trailing;
    sh->prefill_len = p.st->prefill_len;
  }
  __syncthreads();
  run_pass(p, sh, ring, xs, loc_e, emb_sum, out, loads, desc);
}

// Self-test of the bounded waits: one thread polls a counter for a target
// that nothing will reach, with the same acquire loads and %globaltimer
// bound as the pass's grid waits, and reports the expiry through `status`.
// Nothing else is in flight in the CTA.
__global__ void k_wait_selftest(const unsigned long long* counter, unsigned long long target,
                                unsigned long long limit_ns, int* status) {
  if (threadIdx.x != 0) return;
  const unsigned long long t0 = gtime();
  int expired = 0;
  while (ld_acquire64(counter) < target) {
    if (gtime() - t0 > limit_ns) {
      expired = 1;
      break;
    }
  }
  *status = expired;
}

}  // namespace

cudaError_t launch_wait_selftest(const unsigned long long* counter, unsigned long long target,
                                 unsigned long long limit_ns, int* status, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, k_wait_selftest, counter, target, limit_ns, status);
}

size_t cp_pass_smem() {
  return (size_t)kCpStages * kCpStageBytes + kCpScratchBytes + 2 * kCpMaxH * sizeof(float) +
         2 * kCpMaxRows * sizeof(float) + kCpMaxOps * sizeof(CpLoad) + 2 * sizeof(CpOp) +
         sizeof(CpShared);
}

bool cp_pass_supported(int cp_hidden, int intermediate, int q_heads, int kv_heads, int H,
                       int vocab, int sms) {
  if (sms < 64) return false;
  if (q_heads != 2 * kv_heads) return false;
  if (cp_hidden % 256 || intermediate % 256 || H % 256 || H > kCpMaxH) return false;
  const int qkv = (q_heads + 2 * kv_heads) * kHeadDim;
  const int widths[] = {cp_hidden, intermediate, q_heads * kHeadDim, H};
  for (int k : widths)
    if (k * 2 > kCpStageBytes || k > kCpScratchBytes / 8) return false;  // 2 rows staged
  if (vocab > kSelMaxVocab) return false;
  auto per_cta = [&](int n) { return (n + sms - 1) / sms; };
  return per_cta(qkv) <= kCpMaxRows && 2 * per_cta(intermediate) <= kCpMaxRows &&
         per_cta(vocab) <= kCpMaxRows && per_cta(cp_hidden) <= kCpMaxRows;
}

cudaError_t configure_cp_pass() {
  return cudaFuncSetAttribute(k_cp_pass, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)cp_pass_smem());
}

int cp_pass_grid(int device) {
  int sms = 0, coop = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop)
    return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_cp_pass, kCpThreads,
                                                    cp_pass_smem()) != cudaSuccess ||
      per_sm < 1)
    return 0;
  return sms;
}

cudaError_t launch_cp_pass(const CpPassParams& p, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kCpThreads);
  cfg.dynamicSmemBytes = cp_pass_smem();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_cp_pass, p);
}

}  // namespace qtts
