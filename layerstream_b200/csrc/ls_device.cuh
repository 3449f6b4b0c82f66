// Device helpers shared by the CUDA translation units of layerstream_b200.
#pragma once
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <string>

#include "ls_internal.h"

namespace ls {

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// signed int8 byte k of a word -> float, exact: 0x4B0000xx is 2^23 + xx.
__device__ __forceinline__ float s8_to_f(uint32_t wx /* word ^ 0x80808080 */, int k) {
  return __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7440u + k)) - 8388736.0f;
}
// nibble (value + 8 stored) -> float value, exact.
__device__ __forceinline__ float u4_to_f(uint32_t w, int shift) {
  return __uint_as_float(((w >> shift) & 0xFu) | 0x4B000000u) - 8388616.0f;
}

__device__ __forceinline__ bool arg_better(float v2, uint32_t i2, float v1, uint32_t i1) {
  return v2 > v1 || (v2 == v1 && i2 < i1);
}

__device__ __forceinline__ void warp_argmax(float& v, uint32_t& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    uint32_t i2 = __shfl_xor_sync(0xffffffffu, i, o);
    if (arg_better(v2, i2, v, i)) {
      v = v2;
      i = i2;
    }
  }
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

// Last-CTA election: every thread has finished its global writes; returns true in exactly one CTA
// (the last of `total` to arrive), which then reads the others' writes. Resets the ticket.
__device__ __forceinline__ bool last_cta(unsigned* ticket, unsigned total) {
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t = atomicAdd(ticket, 1u);
    s_last = (t == total - 1);
    if (s_last) *ticket = 0u;
  }
  __syncthreads();
  if (s_last) __threadfence();
  return s_last != 0;
}

// Programmatic dependent launch: the next kernel in the stream may start its prologue (weight
// prefetch) while this one finishes; griddepcontrol.wait blocks until the previous grid has
// completed and its writes are visible. Both are no-ops without the launch attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  // bulk L2 prefetch: address and size multiples of 16
  if (bytes >= 16) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes & ~15u) : "memory");
}


constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;

// Reduces the per-CTA argmax parts of every token (first-maximum rule), then applies the
// acceptance rule of src/spec.rs:121-125 (verify) or records the next token (forward).
// Run by one whole CTA of at most GEMV_THREADS threads.
__device__ __noinline__ static void argmax_finalize_block(const ArgPart* parts, int nparts, int M, Ctl* ctl) {
  __shared__ float s_v[GEMV_THREADS];
  __shared__ uint32_t s_i[GEMV_THREADS];
  const int per = (int)blockDim.x / M;  // threads per token (M <= blockDim.x)
  const int t = threadIdx.x % M, j = threadIdx.x / M;
  float v = -CUDART_INF_F;
  uint32_t idx = 0xffffffffu;
  if (j < per) {
#pragma unroll 8
    for (int k = j; k < nparts; k += per) {
      const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(parts + (size_t)k * M + t));
      const float pv = __uint_as_float(raw.x);
      if (arg_better(pv, raw.y, v, idx)) {
        v = pv;
        idx = raw.y;
      }
    }
  }
  s_v[threadIdx.x] = v;
  s_i[threadIdx.x] = idx;
  __syncthreads();
  if (threadIdx.x < M) {
    for (int jj = 1; jj < per; jj++) {
      const int q = jj * M + threadIdx.x;
      if (arg_better(s_v[q], s_i[q], v, idx)) {
        v = s_v[q];
        idx = s_i[q];
      }
    }
    ctl->argmax[threadIdx.x] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (ctl->mode == 1) {
      // longest prefix of guesses the target agrees with, then the correction (or bonus) token;
      // the cache keeps [a, d_1 .. d_m]
      int m = 0;
      while (m < M - 1 && ctl->argmax[m] == ctl->tokens[m + 1]) m++;
      ctl->m = m;
      ctl->next = ctl->argmax[m];
      ctl->pos0 += m + 1;
    } else {
      ctl->m = 0;
      ctl->next = ctl->argmax[M - 1];
      ctl->pos0 += ctl->M;
      if (ctl->mode == 2) ctl->tokens[0] = ctl->next;
    }
  }
}

// Raises a kernel's dynamic shared-memory limit (per device) before a launch that needs it. The
// default 48 KB limit covers static plus dynamic shared memory, so the static part is counted.
template <class K>
static void ensure_smem(K kernel, size_t dyn) {
  struct Entry {
    size_t configured;
    size_t static_bytes;
  };
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, Entry> seen;  // (kernel, device)
  int dev = 0;
  LS_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  auto it = seen.find(key);
  if (it == seen.end()) {
    cudaFuncAttributes fa;
    LS_CUDA(cudaFuncGetAttributes(&fa, kernel));
    it = seen.emplace(key, Entry{0, fa.sharedSizeBytes}).first;
  }
  if (dyn + it->second.static_bytes > 48 * 1024 && dyn > it->second.configured) {
    LS_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn));
    it->second.configured = dyn;
  }
}

template <class K, class... Args>
static void launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  LS_CUDA(cudaLaunchKernelEx(&cfg, kernel, args...));
}

}  // namespace ls
