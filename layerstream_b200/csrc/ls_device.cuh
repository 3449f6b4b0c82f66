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


namespace tc {

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_poll(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase completes (or ~20 us pass)
// instead of spinning, leaving the issue slots to the warps doing the work.
__device__ __forceinline__ bool mbar_try_sleep(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
// Bounded wait without a suspend hint: try_wait blocks for a short hardware-defined time per call,
// so a completed phase is seen with the least delay (for the short hand-offs inside a K loop).
// Bounded by an iteration count (well under a few seconds); false (and the CTA's abort flag) on
// timeout.
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* b, uint32_t parity, volatile int* abort) {
  if (mbar_poll(b, parity)) return true;
  for (uint32_t i = 0; i < (1u << 22); i++) {
    if (mbar_try(b, parity)) return true;
    if ((i & 63) == 63 && *abort) return false;
  }
  *abort = 1;
  return false;
}
// Bounded wait on an mbarrier phase (about a second at most). Returns false (and raises the CTA's
// abort flag) on timeout. A non-blocking test first: a completed phase costs no suspension.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  if (mbar_poll(b, parity)) return true;
  for (uint32_t i = 0; i < (1u << 16); i++) {
    if (mbar_try_sleep(b, parity)) return true;
    if (*abort) return false;
  }
  *abort = 1;
  return false;
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}
// A and B both from shared memory (descriptors).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}
// 3-D tiled TMA load of one box into shared memory, completing bytes on an mbarrier (no multicast).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(su32(bar))
      : "memory");
}
// Plain (untiled) bulk copy global -> shared memory, completing bytes on an mbarrier.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src),
               "r"(bytes), "r"(su32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}
// Adds expected bytes to the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar)) : "memory");
}
// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core matrices, LBO =
// byte distance between the two K halves of a k16 step, SBO = byte distance between 8-row groups.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
// Instruction descriptor: kind::f16, A = B = f16, D = f32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t h2_sub_mul(uint32_t v, uint32_t sub, uint32_t scale) {
  __half2 a = *reinterpret_cast<__half2*>(&v);
  const __half2 b = *reinterpret_cast<const __half2*>(&sub);
  const __half2 c = *reinterpret_cast<const __half2*>(&scale);
  a = __hmul2(__hsub2(a, b), c);
  return *reinterpret_cast<uint32_t*>(&a);
}
// High nibble of a byte pair already placed as 1024 + 16 u (f16x2): (x / 16 - 72) = u - 8 exactly
// in one fused multiply-add, then times the scale (the same single rounding as h2_sub_mul).
__device__ __forceinline__ uint32_t h2_hi_mul(uint32_t v, uint32_t scale) {
  const uint32_t sixteenth = 0x2C002C00u, m72 = 0xD480D480u;  // 1/16, -72 as f16x2
  __half2 a = *reinterpret_cast<__half2*>(&v);
  a = __hfma2(a, *reinterpret_cast<const __half2*>(&sixteenth), *reinterpret_cast<const __half2*>(&m72));
  a = __hmul2(a, *reinterpret_cast<const __half2*>(&scale));
  return *reinterpret_cast<uint32_t*>(&a);
}
__device__ __forceinline__ uint32_t h2_splat(float s) {
  const __half h = __float2half_rn(s);
  const uint16_t u = __half_as_ushort(h);
  return (uint32_t)u | ((uint32_t)u << 16);
}

}  // namespace tc

// K elements per A block: one group for int4 groups of 128, else 64.
__host__ __device__ constexpr int tc_kb(int bits, int group) { return (bits == 4 && group > 64) ? group : 64; }
// (bf16 weights, bits 16, have no group scales: one unused slot keeps the arrays non-empty)
// Group scales one row needs per A block.
__host__ __device__ constexpr int tc_ns(int bits, int group) {
  return bits == 16 ? 1 : tc_kb(bits, group) >= group ? tc_kb(bits, group) / group : 1;
}

// The MMA operand parts of one dequantized weight: int4 weights (q - 8) * scale have at most 4 + 8
// significant bits and are exact in f16 (one part); int8 weights q * scale have up to 7 + 8 and
// enter the MMA as two f16 parts, hi = f16(q * scale) and lo = q * scale - hi (exact in f16 for
// scales >= 2^-17: the remainder has at most 5 significant bits), whose products the tensor core
// adds into the same f32 accumulator, so the weights it multiplies are the exact dequantized ones.
__host__ __device__ constexpr int tc_parts(int bits) { return bits == 8 ? 2 : 1; }

namespace tc {
// hi = v * s rounded to f16, lo = v * s - hi in one fused multiply-add (exact, see tc_parts)
__device__ __forceinline__ void h2_mul_split(uint32_t v, uint32_t sub, uint32_t scale, uint32_t& hi, uint32_t& lo) {
  __half2 a = *reinterpret_cast<__half2*>(&v);
  a = __hsub2(a, *reinterpret_cast<const __half2*>(&sub));  // the exact integer q
  const __half2 sc = *reinterpret_cast<const __half2*>(&scale);
  const __half2 h = __hmul2(a, sc);
  const __half2 l = __hfma2(a, sc, __hneg2(h));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}
}  // namespace tc

// int8 K block -> hi parts in a[0 .. KB/2) and lo parts in lo[0 .. KB/2) (f16 pairs in K order).
template <int G>
__device__ __forceinline__ void tc_dequant_block_i8(const uint4* wv, const uint32_t* scur, uint32_t* a, uint32_t* lo) {
  constexpr int KB = 64, NS = tc_ns(8, G), CPB = KB / 16;
#pragma unroll
  for (int q = 0; q < CPB; q++) {
    const uint32_t wd[4] = {wv[q].x, wv[q].y, wv[q].z, wv[q].w};
    const uint32_t s2 = scur[(NS > 1) ? (q * 16) / G : 0];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t p0 = (__byte_perm(wd[k], 0u, 0x4140u) ^ 0x00800080u) | 0x64006400u;
      const uint32_t p1 = (__byte_perm(wd[k], 0u, 0x4342u) ^ 0x00800080u) | 0x64006400u;
      tc::h2_mul_split(p0, 0x64806480u, s2, a[q * 8 + 2 * k], lo[q * 8 + 2 * k]);
      tc::h2_mul_split(p1, 0x64806480u, s2, a[q * 8 + 2 * k + 1], lo[q * 8 + 2 * k + 1]);
    }
  }
}

// One 16-byte chunk per CPB of a row's packed K block (tc_kb(BITS, G) weights) -> f16 pairs in K
// order, each weight (q - 8) * scale (int4, stored q = w + 8; group >= 32: low nibbles are K j,
// high nibbles K j + G/2 of the group) or q * scale (int8). scur[s]: f16x2 splat of the block's
// s-th group scale. Exact in f16 products of the int and the bf16 scale rounded to f16.
template <int BITS, int G>
__device__ __forceinline__ void tc_dequant_block(const uint4* wv, const uint32_t* scur, uint32_t* a) {
  if constexpr (BITS == 16) {
    // bf16 weights: 8 per chunk, converted to f16 pairs in K order. The conversion is exact for
    // |w| >= 2^-17 (below that, f16 keeps multiples of 2^-24); no scales.
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const uint32_t wd[4] = {wv[q].x, wv[q].y, wv[q].z, wv[q].w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const __half2 h = __floats2half2_rn(__uint_as_float(wd[k] << 16), __uint_as_float(wd[k] & 0xFFFF0000u));
        a[q * 4 + k] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    return;
  }
  constexpr int KB = tc_kb(BITS, G);
  constexpr int NS = tc_ns(BITS, G);
  constexpr int CPB = KB / (128 / BITS);
  const uint32_t sub8 = BITS == 8 ? 0x64806480u : 0x64086408u;  // 1152 | 1032 as f16x2
#pragma unroll
  for (int q = 0; q < CPB; q++) {
    const uint32_t wd[4] = {wv[q].x, wv[q].y, wv[q].z, wv[q].w};
    if constexpr (BITS == 8) {
      const uint32_t s2 = scur[(NS > 1) ? (q * 16) / G : 0];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const uint32_t p0 = (__byte_perm(wd[k], 0u, 0x4140u) ^ 0x00800080u) | 0x64006400u;
        const uint32_t p1 = (__byte_perm(wd[k], 0u, 0x4342u) ^ 0x00800080u) | 0x64006400u;
        a[q * 8 + 2 * k] = tc::h2_sub_mul(p0, sub8, s2);
        a[q * 8 + 2 * k + 1] = tc::h2_sub_mul(p1, sub8, s2);
      }
    } else if constexpr (G == 16) {
      // bytes 0..7: group 2q (low -> K 32q+j, high -> 32q+8+j); bytes 8..15: group 2q+1
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const uint32_t sc = scur[2 * q + (k < 2 ? 0 : 1)];
        const int base = q * 16 + (k < 2 ? 0 : 8);
        const int j = (k & 1) * 4;
        const uint32_t p0 = __byte_perm(wd[k], 0u, 0x4140u), p1 = __byte_perm(wd[k], 0u, 0x4342u);
        a[base + j / 2] = tc::h2_sub_mul((p0 & 0x000F000Fu) | 0x64006400u, sub8, sc);
        a[base + j / 2 + 1] = tc::h2_sub_mul((p1 & 0x000F000Fu) | 0x64006400u, sub8, sc);
        a[base + 4 + j / 2] = tc::h2_hi_mul((p0 & 0x00F000F0u) | 0x64006400u, sc);
        a[base + 4 + j / 2 + 1] = tc::h2_hi_mul((p1 & 0x00F000F0u) | 0x64006400u, sc);
      }
    } else {
      // group >= 32: chunk q holds bytes j0..j0+15 of its group; low nibbles are K j0+j,
      // high nibbles K j0+j+G/2 (relative to the group start)
      constexpr int HALF = G / 2;
      const uint32_t sc = scur[(NS > 1) ? (q * 32) / G : 0];
      const int j0 = (q * 16) % HALF;
      const int gbase = ((q * 32) / G) * G;  // group start relative to the block start
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const uint32_t p0 = __byte_perm(wd[k], 0u, 0x4140u), p1 = __byte_perm(wd[k], 0u, 0x4342u);
        const int lo = (gbase + j0 + 4 * k) / 2, hi = (gbase + j0 + HALF + 4 * k) / 2;
        a[lo] = tc::h2_sub_mul((p0 & 0x000F000Fu) | 0x64006400u, sub8, sc);
        a[lo + 1] = tc::h2_sub_mul((p1 & 0x000F000Fu) | 0x64006400u, sub8, sc);
        a[hi] = tc::h2_hi_mul((p0 & 0x00F000F0u) | 0x64006400u, sc);
        a[hi + 1] = tc::h2_hi_mul((p1 & 0x00F000F0u) | 0x64006400u, sc);
      }
    }
  }
}

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;

// Reduces the per-CTA argmax parts of every token (first-maximum rule), then applies the
// acceptance rule of src/spec.rs:121-125 (verify) or records the next token (forward).
// Run by one whole CTA (its first GEMV_THREADS threads do the reduction).
__device__ __noinline__ static void argmax_finalize_block(const ArgPart* parts, int nparts, int M, Ctl* ctl) {
  __shared__ float s_v[GEMV_THREADS];
  __shared__ uint32_t s_i[GEMV_THREADS];
  const int nth = (int)blockDim.x < GEMV_THREADS ? (int)blockDim.x : GEMV_THREADS;
  const int per = nth / M;  // threads per token (M <= nth)
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
  if ((int)threadIdx.x < nth) {
    s_v[threadIdx.x] = v;
    s_i[threadIdx.x] = idx;
  }
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
