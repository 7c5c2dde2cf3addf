// Block-wide token selection of the head kernels (the last CTA of k_head,
// one CTA per sequence in k_select_batch). 256 threads; `Sync` is the block
// barrier in use.
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
  long long* dbg = nullptr;  // optional phase timestamps (thread 0): clock64 at slots
                             // 0-6 (general path) and 10-15 (fast path)
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

  // Device-path sampling for 0 < K <= kFastK: the same selection as the
  // general path below, with fewer block barriers. The K-th largest key is
  // found by an MSB-first radix select over 4-bit digits: each thread counts
  // its keys per digit in packed 8-bit fields of two registers (no shared
  // atomics), warps reduce them with __reduce_add_sync, and one barrier per
  // digit publishes the eight warp counts, from which every warp derives the
  // same bucket. Once at most kFastCand keys lie at or above the bucket they
  // are compacted with ballots, ranked exactly (value descending, index
  // ascending), and thread 0 sums their probabilities and walks the inverse
  // CDF in rank order. Returns -1 (uniformly) when more than kFastCand keys
  // tie at the threshold; the caller then runs the general path.
  static constexpr int kFastK = 64;
  static constexpr int kFastCand = 128;
  // PER: keys per thread (V <= PER * 256); the CodePredictor's 2048-entry
  // vocab needs 8, the talker's 3072 needs 16.
  template <int PER>
  __device__ __forceinline__ int select_fast(int V, const SampleCfg& cfg, float u) {
    __shared__ unsigned s_wc[2][kSelThreads / 32][16];
    __shared__ int s_wn[kSelThreads / 32];
    __shared__ __align__(16) unsigned long long s_cand[kFastCand];
    __shared__ float s_val[kFastK];
    __shared__ int s_idx[kFastK];
    __shared__ __align__(16) float s_prob[kFastK];
    __shared__ int s_res, s_cnt;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int kPer = PER;
    const int K = min(cfg.top_k, V);
    unsigned key[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int v = j * kSelThreads + tid;
      unsigned k = 0u;  // 0: no entry (no float maps to 0)
      if (v < V) {
        float x = val[v];
        if (!isfinite(x)) {  // the device path ranks non-finite logits as -FLT_MAX
          x = -FLT_MAX;
          val[v] = x;
        }
        k = order_key(x);
      }
      key[j] = k;
    }
    stamp(10);
    unsigned prefix = 0u, mask = 0u, lower = 0u;
    int above = 0, rem = K, buf = 0;
    bool done = false;
    for (int shift = 28; shift >= 0; shift -= 4) {
      unsigned long long c_lo = 0ull, c_hi = 0ull;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const unsigned k = key[j];
        if (k != 0u && (k & mask) == prefix) {
          const unsigned d = (k >> shift) & 15u;
          if (d < 8u) c_lo += 1ull << (8u * d);
          else c_hi += 1ull << (8u * (d - 8u));
        }
      }
      unsigned mine = 0u;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        const unsigned c = (unsigned)((d < 8 ? c_lo >> (8 * d) : c_hi >> (8 * (d - 8))) & 255ull);
        const unsigned w = __reduce_add_sync(0xffffffffu, c);
        if (lane == d) mine = w;
      }
      if (lane < 16) s_wc[buf][warp][lane] = mine;
      Sync::sync();
      // every warp derives the bucket: lane d < 16 holds digit d's total
      unsigned tot = 0u;
      if (lane < 16)
#pragma unroll
        for (int w = 0; w < kSelThreads / 32; ++w) tot += s_wc[buf][w][lane];
      unsigned incl = tot;  // keys in digits >= lane
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        const unsigned n = __shfl_down_sync(0xffffffffu, incl, o);
        if (lane + o < 16) incl += n;
      }
      const unsigned excl = incl - tot;  // keys in digits > lane
      const bool hit = lane < 16 && (int)excl < rem && (int)incl >= rem;
      const int digit = __ffs(__ballot_sync(0xffffffffu, hit)) - 1;
      const int ex = (int)__shfl_sync(0xffffffffu, excl, digit);
      const int in_bucket = (int)__shfl_sync(0xffffffffu, tot, digit);
      prefix |= (unsigned)digit << shift;
      mask |= 15u << shift;
      above += ex;
      rem -= ex;
      buf ^= 1;
      if (above + in_bucket <= kFastCand) {
        lower = prefix;
        done = true;
        break;
      }
    }
    stamp(11);
    if (!done) return -1;  // more than kFastCand keys equal the threshold (uniform)
    // compaction: keys at or above `lower`, per-warp ballots, warp order
    auto take = [&](unsigned k) { return k != 0u && k >= lower; };
    int wc = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) wc += __popc(__ballot_sync(0xffffffffu, take(key[j])));
    if (lane == 0) s_wn[warp] = wc;
    Sync::sync();
    int base = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kSelThreads / 32; ++w) {
      const int c = s_wn[w];
      base += w < warp ? c : 0;
      total += c;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const bool t = take(key[j]);
      const unsigned bal = __ballot_sync(0xffffffffu, t);
      if (t)
        s_cand[base + __popc(bal & ((1u << lane) - 1u))] =
            ((unsigned long long)key[j] << 32) |
            (unsigned)(0xffffffffu - (unsigned)(j * kSelThreads + tid));
      base += __popc(bal);
    }
    // zero keys pad the list to a multiple of 16 (no candidate ranks below 0)
    const int total16 = (total + 15) & ~15;
    if (tid >= total && tid < total16) s_cand[tid] = 0ull;
    Sync::sync();
    stamp(12);
    // exact rank of each candidate: larger key first, then lower index
    if (tid < total) {
      const unsigned long long me = s_cand[tid];
      int rank = 0;
      // 16 keys per step: the broadcast shared-memory reads overlap
      for (int i = 0; i < total16; i += 16) {
#pragma unroll
        for (int u = 0; u < 16; u += 2) {
          const ulonglong2 q = *reinterpret_cast<const ulonglong2*>(s_cand + i + u);
          rank += (q.x > me) + (q.y > me);
        }
      }
      if (rank < K) {
        const int idx = (int)(0xffffffffu - (unsigned)me);
        s_val[rank] = val[idx];
        s_idx[rank] = idx;
      }
    }
    Sync::sync();
    stamp(13);
    if (tid < K) s_prob[tid] = expf((s_val[tid] - s_val[0]) / cfg.temperature);
    Sync::sync();
    stamp(14);
    if (tid == 0) {
      // sum and inverse-CDF walk in rank order (sample_topk_f32's sequence)
      float p[kFastK];
#pragma unroll
      for (int i = 0; i < kFastK; i += 4) {
        const float4 q = *reinterpret_cast<const float4*>(s_prob + i);
        p[i] = q.x; p[i + 1] = q.y; p[i + 2] = q.z; p[i + 3] = q.w;
      }
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < kFastK; ++i)
        if (i < K) sum += p[i];
      int pick = 0;
      if (isfinite(sum) && sum > 0.f) {
        float target = u * sum;
        pick = K - 1;
#pragma unroll
        for (int i = 0; i < kFastK; ++i) {
          if (i < K) {
            if (target <= p[i]) {
              pick = i;
              break;
            }
            target -= p[i];
          }
        }
      }
      s_res = s_idx[pick];
      s_cnt = total;
    }
    Sync::sync();
    stamp(15);
    return s_res;
  }

  // Returns the token to every thread; *error set when no finite logits.
  // Only thread 0 draws from `rng`.
  __device__ __forceinline__ int select(int V, const SampleCfg& cfg, Rng& rng, int* error) {
    __shared__ int s_res;
    __shared__ unsigned s_prefix;
    __shared__ int s_rem;
    __shared__ unsigned s_above, s_lower;
    __shared__ int s_done, s_cnt, s_ties, s_wcnt[kSelThreads / 32];
    __shared__ __align__(16) unsigned long long cand[kSelSmallK];
    __shared__ float sval[kSelSmallK];
    __shared__ __align__(16) float prob[kSelSmallK];
    __shared__ int sidx[kSelSmallK];
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
    // The device path always draws once (drawn before the kernel in the
    // reference), so the draw can run here, off the serial tail.
    float u_dev = 0.f;
    if (device_path && tid == 0) u_dev = rng.next();
    if (device_path && min(cfg.top_k, V) <= kFastK) {
      const int r = V <= 8 * kSelThreads ? select_fast<8>(V, cfg, u_dev)
                                         : select_fast<kSelMaxVocab / kSelThreads>(V, cfg, u_dev);
      if (r >= 0) return r;
    }
    stamp(0);
    // Keys of this thread's entries (v = j * 256 + tid) stay in registers;
    // 0 marks an ineligible entry (no finite float maps to 0). The device
    // path maps non-finite logits to -FLT_MAX, in `val` too.
    constexpr int kPer = kSelMaxVocab / kSelThreads;
    unsigned key[kPer];
    int nfin = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int v = j * kSelThreads + tid;
      unsigned k = 0u;
      if (v < V) {
        const float x = val[v];
        if (isfinite(x)) {
          k = order_key(x);
          ++nfin;
        } else if (device_path) {
          val[v] = -FLT_MAX;
          k = order_key(-FLT_MAX);
        }
      }
      key[j] = k;
    }
    int n_elig = V;
    if (!device_path) scan_excl(nfin, &n_elig);
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
      // Radix select over 8-bit digits, MSB first, that stops as soon as the
      // keys at or above the current bucket fit the candidate buffer; those
      // candidates are compacted and ranked exactly (value desc, index asc).
      stamp(1);
      if (tid == 0) { s_prefix = 0u; s_rem = K; s_lower = 0u; s_done = 0; s_above = 0u; s_ties = 0; }
      Sync::sync();  // every thread reads the initial prefix in the first pass
      // Stop once at most `stop` keys are at or above the bucket: ranking is
      // quadratic in the candidate count.
      const int stop = min(kSelSmallK, max(2 * K, 64));
      unsigned* whist = reinterpret_cast<unsigned*>(aux) + warp * 256;  // per-warp bins
      unsigned mask = 0u;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = lane; i < 256; i += 32) whist[i] = 0u;
        __syncwarp();
        const unsigned prefix = s_prefix;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          if (j * kSelThreads >= V) break;
          const unsigned k = key[j];
          const int bin = (k != 0u && (k & mask) == prefix) ? (int)((k >> shift) & 255u) : -1;
          if (bin >= 0) atomicAdd(&whist[bin], 1u);  // (__match_any_sync costs ~200 cycles here)
        }
        Sync::sync();
        const int digit = 255 - tid;
        int cnt = 0;
#pragma unroll
        for (int w = 0; w < kSelThreads / 32; ++w) cnt += (int)aux[w * 256 + digit];
        int tot;
        const int before = scan_excl(cnt, &tot);
        const int rem = s_rem;
        const int above = (int)s_above;
        Sync::sync();
        if (before < rem && rem <= before + cnt) {
          const unsigned p = prefix | ((unsigned)digit << shift);
          s_prefix = p;
          s_rem = rem - before;
          // keys >= p (bits below `shift` zero) = everything above this bucket plus it
          if (above + before + cnt <= stop || shift == 0) {
            s_lower = p;
            s_done = 1;
            s_ties = above + before + cnt > kSelSmallK;  // many equal keys at the threshold
          }
          s_above = above + before;
        }
        mask |= 255u << shift;
        Sync::sync();
        if (s_done) break;
      }
      stamp(2);
      const unsigned lower = s_lower;
      const bool ties = s_ties;
      // Compaction from the register keys: per-warp ballots give each warp's
      // count, a prefix over warps gives its first slot (no atomics).
      auto take = [&](unsigned k) { return k != 0u && (ties ? k > lower : k >= lower); };
      int wc = 0;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (j * kSelThreads >= V) break;
        wc += __popc(__ballot_sync(0xffffffffu, take(key[j])));
      }
      stamp(8);
      if (lane == 0) s_wcnt[warp] = wc;
      Sync::sync();
      stamp(9);
      constexpr int nw = kSelThreads / 32;
      int base = 0, total = 0;
#pragma unroll
      for (int w = 0; w < nw; ++w) {
        const int c = s_wcnt[w];
        base += w < warp ? c : 0;
        total += c;
      }
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (j * kSelThreads >= V) break;
        const bool t = take(key[j]);
        const unsigned bal = __ballot_sync(0xffffffffu, t);
        if (t)
          cand[base + __popc(bal & ((1u << lane) - 1u))] =
              ((unsigned long long)key[j] << 32) |
              (unsigned)(0xffffffffu - (unsigned)(j * kSelThreads + tid));
        base += __popc(bal);
      }
      stamp(10);
      if (tid == 0) s_cnt = total;
      Sync::sync();
      if (ties) {
        // Keys equal to the threshold, lowest indices first, until K are held.
        const int greater = s_cnt;
        const int per = (V + kSelThreads - 1) / kSelThreads;
        const int lo = tid * per, hi = min(V, lo + per);
        int eq = 0;
        for (int v = lo; v < hi; ++v) {
          const float x = val[v];
          if ((device_path || isfinite(x)) && order_key(x) == lower) ++eq;
        }
        int tot;
        int o = scan_excl(eq, &tot);
        for (int v = lo; v < hi && greater + o < K; ++v) {
          const float x = val[v];
          if ((device_path || isfinite(x)) && order_key(x) == lower)
            cand[greater + o++] = ((unsigned long long)lower << 32) | (0xffffffffu - (unsigned)v);
        }
        Sync::sync();
        if (tid == 0) s_cnt = min(greater + tot, K);
        Sync::sync();
      }
      stamp(3);
      const int C = s_cnt;
      if (tid < C) {
        const unsigned long long me = cand[tid];
        int rank = 0;
        int j = 0;
        for (; j + 4 <= C; j += 4) {
          const ulonglong2 p0 = *reinterpret_cast<const ulonglong2*>(cand + j);
          const ulonglong2 p1 = *reinterpret_cast<const ulonglong2*>(cand + j + 2);
          rank += (p0.x > me) + (p0.y > me) + (p1.x > me) + (p1.y > me);
        }
        for (; j < C; ++j) rank += cand[j] > me;
        if (rank < K) {
          const int idx = (int)(0xffffffffu - (unsigned)me);
          sval[rank] = val[idx];
          sidx[rank] = idx;
        }
      }
      Sync::sync();
      // exponentials in parallel; the sum stays sequential (thread 0)
      stamp(4);
      if (tid < K) prob[tid] = expf((sval[tid] - sval[0]) / cfg.temperature);
      else if (tid < ((K + 3) & ~3)) prob[tid] = 0.f;  // pads the float4 reads below
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

    if (device_path && tid == 0) {
      // Sequential sum and inverse-CDF walk in rank order, 4 entries per load
      // (adding the zero padding leaves the sum unchanged).
      const float4* p4 = reinterpret_cast<const float4*>(prob);
      const int K4 = (K + 3) >> 2;
      const float u = u_dev;
      float sum = 0.f;
#pragma unroll 8
      for (int c = 0; c < K4; ++c) {
        const float4 q = p4[c];
        sum += q.x; sum += q.y; sum += q.z; sum += q.w;
      }
      int pick = 0;
      if (isfinite(sum) && sum > 0.f) {
        float target = u * sum;
        pick = K - 1;
        float4 q = p4[0];
        for (int c = 0; c < K4; ++c) {
          const float4 nq = p4[c + 1 < K4 ? c + 1 : c];  // next group's read in flight
          const float pv[4] = {q.x, q.y, q.z, q.w};
          bool found = false;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int i = 4 * c + j;
            if (!found && i < K) {
              if (target <= pv[j]) { pick = i; found = true; }
              else target -= pv[j];
            }
          }
          if (found) break;
          q = nq;
        }
      }
      s_res = si[pick];
    } else if (tid == 0) {
      const float mx = sv[0];
      const float temp = cfg.temperature;
      auto p_at = [&](int i) { return K <= kSelSmallK ? prob[i] : expf((sv[i] - mx) / temp); };
      float sum = 0.f;
      for (int i = 0; i < K; ++i) sum += p_at(i);
      int tok;
      if (device_path) {
        const float u = u_dev;
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
