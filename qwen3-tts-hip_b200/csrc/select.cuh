// Block-wide token selection shared by the standalone head kernel and the
// persistent frame kernel. 256 threads; `Sync` is the block barrier in use
// (all threads, or the 8 consumer warps of a warp-specialised CTA).
//
// Semantics follow the reference:
//   greedy      argmax_rows_f32 (src/gpu/kernels.rs:177-220): start -FLT_MAX,
//               lowest index wins ties
//   device path sample_topk_f32 (src/gpu/kernels.rs:265-336), taken when
//               0 < top_k <= 256 and top_p >= 0.999999 (sampling.rs:28-37):
//               non-finite -> -FLT_MAX, descending order, softmax((l-max)/T)
//               over min(top_k, V), inverse CDF on u * sum, one draw always
//   CPU path    sample (src/model/sampling.rs:53-118): finite entries only,
//               stable descending order, top-k, softmax, top-p renormalised,
//               inverse CDF on u; no draw when the sum is not finite/positive
// Ties inside a sort are ordered by lowest index (stable order). The
// probability sum is accumulated sequentially in rank order, as the
// reference's single-thread loop does.
#pragma once

#include <float.h>

#include "kernels.h"

namespace qtts {

constexpr int kSelThreads = 256;
constexpr int kSelMaxVocab = 4096;
constexpr int kSelSmallK = 256;

struct SyncBlock {
  __device__ static void sync() { __syncthreads(); }
};
struct SyncConsumers {  // named barrier 1 over the 8 consumer warps
  __device__ static void sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
};

__device__ __forceinline__ unsigned order_key(float f) {
  const unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 64-bit LCG (sampling.rs:120-126) or Philox-4x32-10 (Salmon et al., SC'11)
// counter mode; both return top-24-bit uniforms.
struct Rng {
  int kind;
  unsigned long long state, seed, counter;

  __device__ float next() {
    if (kind == RNG_LCG) {
      state = state * 6364136223846793005ull + 1442695040888963407ull;
      return (float)(unsigned)(state >> 40) / 16777216.0f;
    }
    unsigned c0 = (unsigned)counter, c1 = (unsigned)(counter >> 32), c2 = 0u, c3 = 0u;
    unsigned k0 = (unsigned)seed, k1 = (unsigned)(seed >> 32);
#pragma unroll
    for (int i = 0; i < 10; ++i) {
      const unsigned hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
      const unsigned hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
      const unsigned n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
      c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
      k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
    counter += 1ull;
    return (float)(c0 >> 8) / 16777216.0f;
  }
};

// Shared scratch: val[kSelMaxVocab] floats + aux[kSelMaxVocab] ints (32 KB).
template <typename Sync>
struct Selector {
  float* val;
  int* aux;
  long long* dbg = nullptr;  // optional phase timestamps (thread 0)
  __device__ __forceinline__ void stamp(int i) {
    if (dbg && threadIdx.x == 0) dbg[i] = clock64();
  }

  __device__ __forceinline__ int scan_excl(int v, int* total) {
    __shared__ int s_w[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += n;
    }
    Sync::sync();
    if (lane == 31) s_w[warp] = inc;
    Sync::sync();
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const int t = s_w[w];
      if (w < warp) before += t;
      all += t;
    }
    *total = all;
    return before + inc - v;
  }

  // Repetition penalty once per occurrence (kernels.rs:408-426) over
  // hist[0..n_hist) plus an optional extra token, then codec suppression of
  // [V-1024, V) except eos (kernels.rs:248-263).
  __device__ __forceinline__ void penalise(int V, const int* hist, int n_hist, int extra_tok, float penalty,
                           int suppress, int eos) {
    const int tid = threadIdx.x;
    if (penalty != 1.0f && (n_hist > 0 || extra_tok >= 0)) {
      for (int v = tid; v < V; v += kSelThreads) aux[v] = 0;
      Sync::sync();
      for (int i = tid; i < n_hist; i += kSelThreads) {
        const int t = __ldcg(hist + i);
        if (t >= 0 && t < V) atomicAdd(&aux[t], 1);
      }
      if (tid == 0 && extra_tok >= 0 && extra_tok < V) atomicAdd(&aux[extra_tok], 1);
      Sync::sync();
      for (int v = tid; v < V; v += kSelThreads) {
        float x = val[v];
        for (int c = aux[v]; c > 0; --c) x = x < 0.f ? x * penalty : x / penalty;
        val[v] = x;
      }
    }
    if (suppress)
      for (int v = max(0, V - 1024) + tid; v < V; v += kSelThreads)
        if (v != eos) val[v] = -__int_as_float(0x7f800000);
    Sync::sync();
  }

  // Returns the token to every thread; *error set when no finite logits.
  // Only thread 0 draws from `rng`.
  __device__ __forceinline__ int select(int V, const SampleCfg& cfg, Rng& rng, int* error) {
    __shared__ int s_res;
    __shared__ unsigned s_hist[256];
    __shared__ unsigned s_prefix;
    __shared__ int s_rem;
    __shared__ float cval[kSelSmallK], sval[kSelSmallK], prob[kSelSmallK];
    __shared__ int cidx[kSelSmallK], sidx[kSelSmallK];
    __shared__ float s_bv[8];
    __shared__ int s_bi[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (!cfg.do_sample) {
      float bv = -FLT_MAX;
      int bi = 0;
      for (int v = tid; v < V; v += kSelThreads) {
        const float x = val[v];
        if (x > bv) { bv = x; bi = v; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) { s_bv[warp] = bv; s_bi[warp] = bi; }
      Sync::sync();
      if (tid == 0) {
        float b = s_bv[0];
        int i0 = s_bi[0];
        for (int w = 1; w < 8; ++w)
          if (s_bv[w] > b || (s_bv[w] == b && s_bi[w] < i0)) { b = s_bv[w]; i0 = s_bi[w]; }
        s_res = i0;
      }
      Sync::sync();
      return s_res;
    }

    const bool device_path = cfg.top_k > 0 && cfg.top_k <= 256 && cfg.top_p >= 0.999999f;
    stamp(0);
    int nfin = 0;
    for (int v = tid; v < V; v += kSelThreads) {
      const float x = val[v];
      const bool fin = isfinite(x);
      if (device_path && !fin) val[v] = -FLT_MAX;
      nfin += fin ? 1 : 0;
    }
    int n_elig;
    scan_excl(nfin, &n_elig);
    if (device_path) n_elig = V;
    if (n_elig == 0) {
      if (tid == 0) *error = 1;
      Sync::sync();
      return 0;
    }
    const int K = device_path ? min(cfg.top_k, V)
                              : ((cfg.top_k > 0 && cfg.top_k < n_elig) ? cfg.top_k : n_elig);
    const float* sv;
    const int* si;
    if (K <= kSelSmallK) {
      // Radix select (8-bit digits, MSB first) of the K-th largest key, with
      // warp-aggregated histogram updates (many keys share the top digits).
      stamp(1);
      if (tid == 0) { s_prefix = 0u; s_rem = K; }
      unsigned mask = 0u;
      for (int shift = 24; shift >= 0; shift -= 8) {
        s_hist[tid] = 0u;
        Sync::sync();
        const unsigned prefix = s_prefix;
        for (int v0 = 0; v0 < V; v0 += kSelThreads) {
          const int v = v0 + tid;
          int bin = -1;
          if (v < V) {
            const float x = val[v];
            if (device_path || isfinite(x)) {
              const unsigned key = order_key(x);
              if ((key & mask) == prefix) bin = (int)((key >> shift) & 255u);
            }
          }
          const unsigned peers = __match_any_sync(0xffffffffu, bin);
          if (bin >= 0 && (__ffs(peers) - 1) == lane) atomicAdd(&s_hist[bin], __popc(peers));
        }
        Sync::sync();
        const int digit = 255 - tid;
        const int cnt = (int)s_hist[digit];
        int tot;
        const int before = scan_excl(cnt, &tot);
        const int rem = s_rem;
        Sync::sync();
        if (before < rem && rem <= before + cnt) {
          s_prefix = prefix | ((unsigned)digit << shift);
          s_rem = rem - before;
        }
        mask |= 255u << shift;
        Sync::sync();
      }
      stamp(2);
      const unsigned thr = s_prefix;
      const int take_eq = s_rem;
      const int per = (V + kSelThreads - 1) / kSelThreads;
      const int lo = tid * per, hi = min(V, lo + per);
      int gt = 0, eq = 0;
      for (int v = lo; v < hi; ++v) {
        const float x = val[v];
        if (!device_path && !isfinite(x)) continue;
        const unsigned key = order_key(x);
        gt += key > thr;
        eq += key == thr;
      }
      int tot;
      const int eq_before = scan_excl(eq, &tot);
      const int eq_take = max(0, min(eq, take_eq - eq_before));
      int o = scan_excl(gt + eq_take, &tot);
      for (int v = lo, e = 0; v < hi; ++v) {
        const float x = val[v];
        if (!device_path && !isfinite(x)) continue;
        const unsigned key = order_key(x);
        bool take = key > thr;
        if (key == thr) { take = e < eq_take; ++e; }
        if (take) { cval[o] = x; cidx[o] = v; ++o; }
      }
      Sync::sync();
      stamp(3);
      if (tid < K) {
        const float vi = cval[tid];
        const int ii = cidx[tid];
        int rank = 0;
        for (int j = 0; j < K; ++j) {
          const float vj = cval[j];
          rank += (vj > vi) || (vj == vi && cidx[j] < ii);
        }
        sval[rank] = vi;
        sidx[rank] = ii;
      }
      Sync::sync();
      // exponentials in parallel; the sum stays sequential (thread 0)
      stamp(4);
      if (tid < K) prob[tid] = expf((sval[tid] - sval[0]) / cfg.temperature);
      Sync::sync();
      stamp(5);
      sv = sval;
      si = sidx;
    } else {
      // Large K (CPU-sampler path only): bitonic sort of the whole vocab,
      // descending value then ascending index; non-finite entries last.
      int n2 = 1;
      while (n2 < V) n2 <<= 1;
      for (int v = tid; v < n2; v += kSelThreads) {
        float x = v < V ? val[v] : -INFINITY;
        if (!isfinite(x)) x = -INFINITY;
        val[v] = x;
        aux[v] = v;
      }
      Sync::sync();
      for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int i = tid; i < n2; i += kSelThreads) {
            const int j = i ^ stride;
            if (j > i) {
              const float a = val[i], b = val[j];
              const int ia = aux[i], ib = aux[j];
              const bool a_first = a > b || (a == b && ia < ib);
              const bool desc = (i & size) == 0;
              if (desc ? !a_first : a_first) {
                val[i] = b; val[j] = a;
                aux[i] = ib; aux[j] = ia;
              }
            }
          }
          Sync::sync();
        }
      }
      sv = val;
      si = aux;
    }

    if (tid == 0) {
      const float mx = sv[0];
      const float temp = cfg.temperature;
      auto p_at = [&](int i) { return K <= kSelSmallK ? prob[i] : expf((sv[i] - mx) / temp); };
      float sum = 0.f;
      for (int i = 0; i < K; ++i) sum += p_at(i);
      int tok;
      if (device_path) {
        const float u = rng.next();  // drawn before the kernel in the reference
        if (!isfinite(sum) || sum <= 0.f) {
          tok = si[0];
        } else {
          float target = u * sum;
          tok = si[K - 1];
          for (int i = 0; i < K; ++i) {
            const float pi = p_at(i);
            if (target <= pi) { tok = si[i]; break; }
            target -= pi;
          }
        }
      } else if (!isfinite(sum) || sum <= 0.f) {
        tok = si[0];  // no draw (sampling.rs:79-81)
      } else {
        int keep = K;
        float ks = 1.0f;
        if (cfg.top_p < 1.0f) {
          float cum = 0.f;
          keep = 0;
          for (int i = 0; i < K; ++i) {
            ++keep;
            cum += p_at(i) / sum;
            if (cum >= cfg.top_p) break;
          }
          keep = max(keep, 1);
          ks = 0.f;
          for (int i = 0; i < keep; ++i) ks += p_at(i) / sum;
          if (!(ks > 0.f)) ks = 1.0f;
        }
        float target = rng.next();
        tok = si[keep - 1];
        for (int i = 0; i < keep; ++i) {
          float pi = p_at(i) / sum;
          if (cfg.top_p < 1.0f) pi /= ks;
          if (target <= pi) { tok = si[i]; break; }
          target -= pi;
        }
      }
      s_res = tok;
    }
    stamp(6);
    Sync::sync();
    return s_res;
  }
};

}  // namespace qtts
