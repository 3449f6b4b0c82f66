// Device helpers shared by the CUDA translation units of layerstream_b200.
#pragma once
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

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


}  // namespace ls
