// Shared device helpers for the sm_100a Qwen3-TTS token-loop kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qtts {

constexpr int kHeadDim = 128;  // Qwen3-TTS talker and CodePredictor head_dim

// ---- programmatic dependent launch (PDL) --------------------------------
// Every kernel calls pdl_wait() before it touches memory written by the
// previous kernel on the stream; weights may be fetched before it.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 16-byte streaming load of constant weights: non-coherent path, no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// L2 policy for weights streamed once per use: evicted first, so a frame's
// gigabytes of weights do not push kernel code and activations out of L2.
__device__ __forceinline__ unsigned long long l2_evict_first_policy() {
  unsigned long long pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint4 ldg_stream(const void* p, unsigned long long pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ void unpack8(uint4 u, float f[8]) {
  f[0] = bf16lo(u.x); f[1] = bf16hi(u.x);
  f[2] = bf16lo(u.y); f[3] = bf16hi(u.y);
  f[4] = bf16lo(u.z); f[5] = bf16hi(u.z);
  f[6] = bf16lo(u.w); f[7] = bf16hi(u.w);
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Paged bf16 KV cache view. A physical page holds `1 << page_shift` positions
// of every layer: [layer][k|v][kv_head][page_pos][head_dim].
struct KvView {
  __nv_bfloat16* pool;
  const int* page_table;  // logical page -> physical page
  int page_shift;
  int kv_heads;
  long long page_stride;   // elements per physical page
  long long layer_stride;  // elements per layer inside a page
};

__device__ __forceinline__ __nv_bfloat16* kv_ptr(const KvView& v, int layer, int kind,
                                                 int head, int pos) {
  const int page = v.page_table[pos >> v.page_shift];
  const int inpage = pos & ((1 << v.page_shift) - 1);
  return v.pool + (long long)page * v.page_stride + (long long)layer * v.layer_stride +
         ((long long)((kind * v.kv_heads + head) << v.page_shift) + inpage) * kHeadDim;
}

// Debugging aid (QTTS_CRUMBS=1): each kernel's first thread records its id in
// mapped host memory at entry ([0]) and exit ([1]), so after a device fault
// the host can still tell which kernel was running. Null when off.
struct Crumbs {
  volatile unsigned* p;
};
#define QTTS_CRUMB(slot, id)                                                         \
  do {                                                                               \
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 &&  \
        g_crumbs.p) {                                                                \
      g_crumbs.p[slot] = (unsigned)(id);                                             \
      __threadfence_system();                                                        \
    }                                                                                \
  } while (0)

// Kernel launch with programmatic dependent launch allowed (the kernel's
// griddepcontrol.wait orders it after its predecessor; work before the wait
// may overlap the predecessor's tail).
template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

}  // namespace qtts
