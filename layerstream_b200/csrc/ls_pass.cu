// Persistent verify-pass kernel: one cooperative launch runs a whole forward pass of up to 48 tokens
// (embedding, 24 x [QKV, attention, O, gate/up, down], LM head, argmax + acceptance).
//
// Why: a pass is ~120 dependent steps whose data are small (0.5 MB .. 5 MB of weights each), so
// separate kernels spend most of their time in launch and dependency latency. Here each CTA (one
// per SM) keeps its tensor memory, mbarriers and load ring for the whole pass, phases are separated
// by a grid barrier, and before waiting at a barrier every CTA starts streaming the weights of its
// first item of the next phase (weights never depend on the previous phase).
//
// Split-K partial sums and residual adds accumulate in 64-bit fixed point (2^-32 resolution):
// integer addition is associative, so the result does not depend on the order in which CTAs
// finish — the pass stays deterministic and every token's result is independent of how many
// tokens share the pass.
//
// GEMV phases: a CTA has PK_NWG dequantizing warpgroups, each owning one 128-row tile of the
// current 256-row item, and one issuer warp. Every K block of 64 columns, each warpgroup turns its
// int4/int8 rows into f16 (scale applied) and stores them to its A buffer in tensor memory; the
// issuer warp runs the tcgen05 MMAs of all warpgroups against the activations staged in shared
// memory. A and the f32 accumulators are double-buffered in tensor memory, so dequantization, MMA
// issue and the accumulator read-back of the previous item overlap.
//
// Every wait is bounded (grid barrier spins, mbarrier polls); on a timeout the CTA records an
// error in the control block, the other CTAs see it at their next wait, tensor memory is released
// and the kernel returns.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "ls_device.cuh"
#include "ls_internal.h"

namespace ls {

constexpr int PK_NWG = 2;                    // dequantizing warpgroups per CTA
constexpr int PK_CT = PK_NWG * 128;           // their threads
constexpr int PK_ISSUER = PK_CT / 32;           // warp of warpgroup g's MMA issuer: PK_ISSUER + g
constexpr int PK_PRODUCER = PK_ISSUER + PK_NWG;  // warp index of the weight-stream (TMA) producer
constexpr int PK_STAGERS = PK_CT + 32 * PK_NWG;  // compute warps + issuers: the B-operand staging group
constexpr int PK_THREADS = PK_STAGERS + 32;
constexpr int PK_NW = PK_THREADS / 32;
constexpr int kMaxSlots = 16;  // attention slots per head (context tiles split across CTAs)
// Weight stream: STAGES stages of one 256-row box of ~16 KB of packed weights (+ its scales),
// filled by TMA. Bulk copies of >= 16 KB per stage stream at HBM bandwidth with one CTA per SM
// (per-thread 16-byte copies top out near a third of it).
constexpr int PK_MAX_STAGES = 8;  // the launch's stage count (a.stages) fills the shared memory left
constexpr int PK_STAGE_DATA = 16384;
constexpr int PK_TMEM_COLS = 512;  // one CTA per SM: the whole tensor memory
constexpr int PK_ABUF = 4;         // A buffers per warpgroup (dequantizers run ahead of the MMAs)

// Named barrier over the compute warps and the issuer (the producer never joins it, so it can
// wait on the ring while the others stage activations).
__device__ __forceinline__ void stagers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(PK_STAGERS) : "memory"); }

__device__ __forceinline__ long long to_fix(float v) {
  v = fminf(fmaxf(v, -1.0e9f), 1.0e9f);
  return __float2ll_rn(v * 4294967296.0f);
}
// One conversion, rounded to nearest, then an exact power-of-two scale: for |f| < 2^53 (|value| <
// 2^21) the same float as converting through double and scaling there, without the two
// double-precision operations per value (the activations' staging runs tens of thousands of these
// per phase).
__device__ __forceinline__ float from_fix(long long f) { return __ll2float_rn(f) * 2.3283064365386962890625e-10f; }
__device__ __forceinline__ void fix_add(long long* p, float v) {
  atomicAdd(reinterpret_cast<unsigned long long*>(p), (unsigned long long)to_fix(v));
}
__device__ __forceinline__ long long ldcg_ll(const long long* p) { return __ldcg(p); }

__device__ __forceinline__ unsigned gtimer() {
  unsigned t;
  asm volatile("mov.u32 %0, %%globaltimer_lo;" : "=r"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier over a counter zeroed before the launch, taken by every thread of every CTA
// (also after a failure, so that the CTA barriers inside always match). Bounded: after `limit`
// polls the CTA records error 3; returns false when any CTA has recorded an error (including this
// one timing out) or this CTA has aborted.
__device__ bool grid_barrier(unsigned* bar, unsigned target, int* err, unsigned limit, const volatile int* local_abort) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    // release: the CTA's writes (ordered before this thread's by the CTA barrier) are visible to
    // whoever acquires the count; no round trip is waited for
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(bar), "r"(1u) : "memory");
    int ok = 1;
    for (uint32_t i = 0;; i++) {
      if (ld_acquire(bar) >= target) break;
      if (*(volatile int*)err || *local_abort) {
        ok = 0;
        break;
      }
      if (i > limit) {
        atomicExch(err, 3);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    s_ok = ok;  // the acquiring load orders the other CTAs' writes before this CTA's reads
  }
  __syncthreads();
  return s_ok != 0;
}

// ---------------------------------------------------------------------------------------------
// The tensor-core GEMV of one item: rows [256 t256, 256 t256 + 256) over K blocks [kb0, kb1).
// The producer warp streams the item's weights (and group scales) as 256-row TMA boxes of NB K
// blocks into a ring of `nst` stages (full / empty mbarriers); each compute warpgroup dequantizes its
// 128 rows block by block into its A buffer in tensor memory; the issuer warp runs the MMAs.
// State is kept across items and phases; all roles walk the same item / block sequence.
// Tensor memory columns: A buffer (b, g) at (b PK_NWG + g) ACOLS, accumulator (d, g) at
// PK_ABUF PK_NWG ACOLS + (d PK_NWG + g) NT.
// ---------------------------------------------------------------------------------------------
template <int BITS, int G>
struct Stream {
  static constexpr int KB = tc_kb(BITS, G), NS = tc_ns(BITS, G), CPB = KB / (128 / BITS);
  static constexpr int NB = (PK_STAGE_DATA / (8 * CPB * 512)) < 1 ? 1 : PK_STAGE_DATA / (8 * CPB * 512);
  static constexpr uint32_t kData = 8 * CPB * NB * 512, kScales = 8 * NS * NB * 64, kStage = kData + kScales;
};

// Weight-stream load: each weight byte is read once per pass, so the copy is marked first to be
// evicted from L2, which keeps the pass's activations and small per-layer tensors there.
__device__ __forceinline__ void tma_load3(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(tc::su32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(tc::su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Instrumentation policy of the GEMV core: mark(point, block) is called at fixed points of the
// K loop; the product instance does nothing (microbenchmarks pass a recording one).
struct NoMarks {
  __device__ __forceinline__ void mark(int, uint32_t) const {}
};

template <int BITS, int G, int NT, class Marks = NoMarks>
struct TcGemv {
  using S = Stream<BITS, G>;
  Marks marks;
  // one K block: its f16 pairs (two per column), for int8 its exact hi then lo parts
  static constexpr int KB = S::KB, NS = S::NS, CPB = S::CPB, NB = S::NB, HC = KB / 2, ACOLS = HC * tc_parts(BITS);
  // One A buffer holds a whole stream stage (NB K blocks side by side): one hand-off per stage.
  static constexpr int AC = NB * ACOLS, AB = (256 / (PK_NWG * AC)) < PK_ABUF ? 256 / (PK_NWG * AC) : PK_ABUF;
  static_assert(AB >= 2 && AB * PK_NWG * AC + 2 * PK_NWG * NT <= PK_TMEM_COLS, "tensor memory");
  uint32_t tmem;
  uint8_t* ring;
  uint64_t *full, *empty;        // [nst] weight stream
  int nst;
  uint64_t *bar_a, *bar_full;    // [PK_NWG][AB] A buffers: MMAs done / A written
  uint64_t *bar_d, *bar_dfree;   // [PK_NWG][2] accumulators: ready / read
  int* abort;
  uint32_t blk, itc, rpos;  // A hand-offs (stages), items and stream stages consumed so far

  __device__ uint32_t a_col(int b, int g) const { return tmem + (uint32_t)((b * PK_NWG + g) * AC); }
  __device__ uint32_t d_col(int d, int g) const { return tmem + (uint32_t)(AB * PK_NWG * AC + (d * PK_NWG + g) * NT); }

  // Compute threads: the K loop of an item over the streamed stages, then the accumulators.
  // false on a timeout.
  __device__ bool run(int kb0, int kb1, float (&tot)[NT]) {
    const int g = threadIdx.x >> 7, warp8 = threadIdx.x >> 5, warp = warp8 & 3, lane = threadIdx.x & 31;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t sub8 = BITS == 8 ? 0x64806480u : 0x64086408u;
    // The tensor-memory stores of stage j complete while stage j + 1's first block is dequantized;
    // only then is stage j handed to the issuer (pend = its A buffer's barrier, or null).
    uint64_t* pend = nullptr;
    auto hand_off = [&]() {
      if (pend == nullptr) return;
      tc::wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::su32(pend)) : "memory");
      pend = nullptr;
    };
    for (int kbs = kb0; kbs < kb1; kbs += NB) {
      const int slot = rpos % nst;
      bool fail = !tc::mbar_wait_fast(&full[slot], (rpos / nst) & 1, abort);
      if (__any_sync(0xffffffffu, fail)) {
        tc::wait_st();
        return false;
      }
      marks.mark(0, blk);
      rpos++;
      const uint8_t* st = ring + (size_t)slot * S::kStage;
      const int nb = min(NB, kb1 - kbs);
      // the stage's blocks go to one A buffer side by side (block bi at column bi ACOLS); each
      // block's store is issued as soon as it is dequantized, the stage is handed off once
      const int b = blk % AB;
#pragma unroll
      for (int bi = 0; bi < NB; bi++) {
        if (bi >= nb) break;
        // this warp's 32 rows (row group warp8 of the box): chunk (bi CPB + q), group (bi NS + s)
        uint4 wv[CPB];
#pragma unroll
        for (int q = 0; q < CPB; q++)
          wv[q] = *reinterpret_cast<const uint4*>(st + ((size_t)(warp8 * CPB * NB + bi * CPB + q)) * 512 + lane * 16);
        uint32_t sc[NS];
#pragma unroll
        for (int q = 0; q < NS; q++)
          sc[q] = tc::h2_splat(bf16f(reinterpret_cast<const uint16_t*>(st + S::kData + (size_t)(warp8 * NS * NB + bi * NS + q) * 64)[lane]));
        uint32_t a[ACOLS];
        if constexpr (BITS == 8) tc_dequant_block_i8<G>(wv, sc, a, a + HC);
#pragma unroll
        for (int q = 0; q < CPB; q++) {
          const uint32_t wd[4] = {wv[q].x, wv[q].y, wv[q].z, wv[q].w};
          if constexpr (BITS == 8) {
          } else if constexpr (G == 16) {
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const uint32_t s2 = sc[2 * q + (k < 2 ? 0 : 1)];
              const int base = q * 16 + (k < 2 ? 0 : 8), j = (k & 1) * 4;
              const uint32_t p0 = __byte_perm(wd[k], 0u, 0x4140u), p1 = __byte_perm(wd[k], 0u, 0x4342u);
              a[base + j / 2] = tc::h2_sub_mul((p0 & 0x000F000Fu) | 0x64006400u, sub8, s2);
              a[base + j / 2 + 1] = tc::h2_sub_mul((p1 & 0x000F000Fu) | 0x64006400u, sub8, s2);
              a[base + 4 + j / 2] = tc::h2_sub_mul(((p0 >> 4) & 0x000F000Fu) | 0x64006400u, sub8, s2);
              a[base + 4 + j / 2 + 1] = tc::h2_sub_mul(((p1 >> 4) & 0x000F000Fu) | 0x64006400u, sub8, s2);
            }
          } else {
            constexpr int HALF = G / 2;
            const uint32_t s2 = sc[(NS > 1) ? (q * 32) / G : 0];
            const int j0 = (q * 16) % HALF, gbase = ((q * 32) / G) * G;
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const uint32_t p0 = __byte_perm(wd[k], 0u, 0x4140u), p1 = __byte_perm(wd[k], 0u, 0x4342u);
              const int lo = (gbase + j0 + 4 * k) / 2, hi = (gbase + j0 + HALF + 4 * k) / 2;
              a[lo] = tc::h2_sub_mul((p0 & 0x000F000Fu) | 0x64006400u, sub8, s2);
              a[lo + 1] = tc::h2_sub_mul((p1 & 0x000F000Fu) | 0x64006400u, sub8, s2);
              a[hi] = tc::h2_sub_mul(((p0 >> 4) & 0x000F000Fu) | 0x64006400u, sub8, s2);
              a[hi + 1] = tc::h2_sub_mul(((p1 >> 4) & 0x000F000Fu) | 0x64006400u, sub8, s2);
            }
          }
        }
        if (bi == 0) {
          marks.mark(1, blk + (a[ACOLS - 1] == 0x7fffffffu ? 1u : 0u));
          hand_off();  // the previous stage
          // A buffer b is free once the MMAs of hand-off blk - AB have completed
          const uint32_t u = blk / AB;
          fail = u > 0 && !tc::mbar_wait_fast(&bar_a[g * AB + b], (u - 1) & 1, abort);
          if (__any_sync(0xffffffffu, fail)) {
            tc::wait_st();
            return false;
          }
          marks.mark(2, blk);
          tc::fence_after();
        }
#pragma unroll
        for (int q = 0; q < ACOLS / 16; q++) tc::st16(a_col(b, g) + bi * ACOLS + lane_base + q * 16, a + q * 16);
      }
      __syncwarp();  // this warp is done with the stage: the producer may refill it
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::su32(&empty[slot])) : "memory");
      pend = &bar_full[g * AB + b];
      marks.mark(3, blk);
      blk++;
    }
    hand_off();  // the item's last stage
    const int d = itc & 1;
    const uint32_t v = itc >> 1;
    itc++;
    bool fail = !tc::mbar_wait_fast(&bar_d[g * 2 + d], v & 1, abort);
    if (__any_sync(0xffffffffu, fail)) return false;
    tc::fence_after();
#pragma unroll
    for (int q = 0; q < NT / 16; q++) {
      uint32_t r[16];
      tc::ld16(d_col(d, g) + lane_base + q * 16, r);
      tc::wait_ld();
#pragma unroll
      for (int e = 0; e < 16; e++) tot[q * 16 + e] = __uint_as_float(r[e]);
    }
    tc::fence_before();
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::su32(&bar_dfree[g * 2 + d])) : "memory");
    return true;
  }

  // Issuer warp of warpgroup g (lane 0 issues): the MMAs of an item, B = the staged activations.
  // Descriptors are formed once per item and advanced by adds. false on a timeout.
  __device__ bool issue(int g, int kb0, int kb1, uint32_t xb_addr, uint32_t sbo) {
    const int lane = threadIdx.x & 31;
    const int d = itc & 1;
    const uint32_t v = itc >> 1;
    itc++;
    const uint32_t idesc = tc::idesc_f16(NT);
    bool fail = false;
    if (lane == 0) {
      // accumulator d is free once the compute threads have read item itc - 2
      if (v > 0 && !tc::mbar_wait_fast(&bar_dfree[g * 2 + d], (v - 1) & 1, abort)) fail = true;
      const uint64_t bd0 = tc::sdesc(xb_addr, 128u, sbo);  // start address field: 16-byte units
      const uint32_t dcol = d_col(d, g);
      for (int kbs = kb0; kbs < kb1 && !fail; kbs += NB) {
        const int nb = min(NB, kb1 - kbs);
        const int b = blk % AB;
        const uint32_t u = blk / AB;
        blk++;
        if (!tc::mbar_wait_fast(&bar_full[g * AB + b], u & 1, abort)) {
          fail = true;
          break;
        }
        marks.mark(4, blk - 1);
        tc::fence_after();
        const uint32_t acol = a_col(b, g);
        for (int bi = 0; bi < nb; bi++) {
          const uint64_t bdk = bd0 + (uint64_t)((kbs + bi - kb0) * KB);  // K column kpos sits kpos / 8 * 128 bytes in
#pragma unroll
          for (int j = 0; j < KB / 16; j++) {
            tc::mma_f16_ts(dcol, acol + bi * ACOLS + j * 8, bdk + (uint64_t)(j * 16), idesc,
                           (kbs + bi > kb0 || j > 0) ? 1u : 0u);
            if constexpr (BITS == 8) tc::mma_f16_ts(dcol, acol + bi * ACOLS + HC + j * 8, bdk + (uint64_t)(j * 16), idesc, 1u);
          }
        }
        tc::commit(&bar_a[g * AB + b]);
        marks.mark(5, blk - 1);
      }
      if (!fail) tc::commit(&bar_d[g * 2 + d]);
    } else {
      blk += (kb1 - kb0 + NB - 1) / NB;
    }
    blk = __shfl_sync(0xffffffffu, blk, 0);
    return !__any_sync(0xffffffffu, fail);
  }
};

// Item split of a GEMV phase: item i -> (K slice, 256-row tile), slices outermost.
struct Split {
  int tiles, ks, nblk;
  __device__ int items() const { return tiles * ks; }
  __device__ void item(int i, int* t256, int* kb0, int* kb1) const {
    const int k = i / tiles;
    *t256 = i - k * tiles;
    *kb0 = (int)((long long)k * nblk / ks);
    *kb1 = (int)((long long)(k + 1) * nblk / ks);
  }
};

template <int BITS, int G>
__device__ __forceinline__ Split make_split(const QMat& w, int ks) {
  Split s;
  s.tiles = (w.rows_pad / 32 + 4 * PK_NWG - 1) / (4 * PK_NWG);
  s.ks = ks;
  s.nblk = w.cols / tc_kb(BITS, G);
  return s;
}

// Producer (lane 0 of warp PK_PRODUCER): issues the stages of the CTA's items of a GEMV phase, in
// the order the compute warps consume them, each a 256-row box of NB K blocks plus its scales.
template <int BITS, int G>
struct Producer {
  using S = Stream<BITS, G>;
  uint8_t* ring;
  uint64_t *full, *empty;
  int nst;
  int* abort;
  uint32_t lpos;  // stages issued so far
  const QMaps* maps;
  Split sp;
  int i, kb, kb1, t256;

  __device__ void begin(const QMaps* m, const Split& s) {
    maps = m;
    sp = s;
    i = blockIdx.x;
    if (i < sp.items()) {
      int kb0;
      sp.item(i, &t256, &kb0, &kb1);
      kb = kb0;
    }
  }
  __device__ bool done() const { return i >= sp.items(); }
  // Issues the next stage. wait == false: returns false at once when its slot is still in use.
  // A timeout also returns false (and raises *abort).
  __device__ bool issue_one(bool wait) {
    const int slot = lpos % nst;
    const uint32_t use = lpos / nst;
    if (use > 0) {
      if (!wait) {
        if (!mbar_test(&empty[slot], (use - 1) & 1)) return false;
      } else if (!tc::mbar_wait(&empty[slot], (use - 1) & 1, abort)) {
        return false;
      }
    }
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::su32(&full[slot])), "r"(S::kStage)
                 : "memory");
    const uint32_t dst = tc::su32(ring + (size_t)slot * S::kStage);
    const uint64_t pol = evict_first_policy();
    tma_load3(dst, &maps->data, 0, kb * S::CPB, t256 * 8, &full[slot], pol);
    tma_load3(dst + S::kData, &maps->scales, 0, kb * S::NS, t256 * 8, &full[slot], pol);
    lpos++;
    kb += S::NB;
    if (kb >= kb1) {
      i += gridDim.x;
      if (i < sp.items()) {
        int kb0;
        sp.item(i, &t256, &kb0, &kb1);
        kb = kb0;
      }
    }
    return true;
  }
};

// Writes activations (already f32) for tokens t < T, K columns [col0, col0 + ncol) into the
// canonical K-major f16 layout; value(t, col) is a callable.
template <int NT, class F>
__device__ __forceinline__ void stage_b(uint8_t* xb, uint32_t sbo, int T, int col0, int ncol, F value) {
  const int n8 = ncol / 8;
#pragma unroll 4
  for (int i = threadIdx.x; i < NT * n8; i += PK_STAGERS) {
    const int t = i / n8, kc = i - t * n8;
    uint32_t w4[4] = {0u, 0u, 0u, 0u};
    if (t < T) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const __half2 h = __floats2half2_rn(value(t, col0 + kc * 8 + 2 * e), value(t, col0 + kc * 8 + 2 * e + 1));
        w4[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(xb + (size_t)(t / 8) * sbo + (size_t)kc * 128 + (t % 8) * 16) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1 / rms of the first T rows of x (fixed point, n columns, n even) into s_inv. The rows are copied
// into shared memory (buf, buf_bytes) with cp.async, every 16-byte chunk in flight at once (as many
// rows per round as fit; one round trip to L2 for a verify block of a small model), then warp w sums
// the squares of row t's columns (lane l: column pairs l, l + 32, ...) in a fixed order that
// depends only on n, so a token's statistics do not depend on its place in the pass.
__device__ __forceinline__ void rms_stats(const long long* x, int T, int n, float eps, float* s_inv, uint8_t* buf,
                                          size_t buf_bytes) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, np = n >> 1;
  const int per = max(1, (int)(buf_bytes / ((size_t)n * 8)));
  const longlong2* rows = reinterpret_cast<const longlong2*>(buf);
  for (int t0 = 0; t0 < T; t0 += per) {
    const int tn = min(per, T - t0);
    const longlong2* src = reinterpret_cast<const longlong2*>(x + (size_t)t0 * n);
    for (int i = threadIdx.x; i < tn * np; i += PK_THREADS) tc::cp_async16(tc::su32(buf + (size_t)i * 16), src + i);
    tc::cp_commit();
    tc::cp_wait<0>();
    __syncthreads();
    for (int t = warp; t < tn; t += PK_NW) {
      const longlong2* r = rows + (size_t)t * np;
      float ss = 0.f;
      for (int p = lane; p < np; p += 32) {
        const longlong2 v = r[p];
        const float f0 = from_fix(v.x), f1 = from_fix(v.y);
        ss = fmaf(f0, f0, ss);
        ss = fmaf(f1, f1, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) s_inv[t0 + t] = 1.0f / sqrtf(ss / (float)n + eps);
    }
    __syncthreads();
  }
}

// The same statistics (same sums in the same order), the rows loaded into registers and kept in
// shared memory as f32 (xs: [T][n]) together with the norm weights (wn: [n], from bf16 nb or f32
// nf), so that the staging of every K slice of the phase reads shared memory only. Warp w takes
// rows w, w + PK_NW, ...; lane l its column pairs l, l + 32, ..., loaded 16 at a time.
__device__ __forceinline__ void rms_rows(const long long* x, int T, int n, float eps, float* s_inv, float* xs, float* wn,
                                         const uint16_t* nb, const float* nf) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, np = n >> 1;
  for (int c = threadIdx.x; c < n; c += PK_THREADS) wn[c] = nb ? bf16f(nb[c]) : nf[c];
  for (int t = warp; t < T; t += PK_NW) {
    const longlong2* r = reinterpret_cast<const longlong2*>(x + (size_t)t * n);
    float2* o = reinterpret_cast<float2*>(xs + (size_t)t * n);
    float ss = 0.f;
    for (int p0 = 0; p0 < np; p0 += 32 * 16) {
      longlong2 v[16];
#pragma unroll
      for (int k = 0; k < 16; k++) {
        const int p = p0 + lane + 32 * k;
        v[k] = p < np ? __ldcg(r + p) : make_longlong2(0, 0);
      }
#pragma unroll
      for (int k = 0; k < 16; k++) {
        const int p = p0 + lane + 32 * k;
        if (p < np) {
          const float f0 = from_fix(v[k].x), f1 = from_fix(v[k].y);
          o[p] = make_float2(f0, f1);
          ss = fmaf(f0, f0, ss);
          ss = fmaf(f1, f1, ss);
        }
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) s_inv[t] = 1.0f / sqrtf(ss / (float)n + eps);
  }
  __syncthreads();
}

__device__ __forceinline__ void zero_ll(long long* p, size_t n) {
  for (size_t i = (size_t)blockIdx.x * PK_THREADS + threadIdx.x; i < n; i += (size_t)gridDim.x * PK_THREADS) p[i] = 0;
}

// Attention. The context is cut into chunks of PK_CHUNK positions; chunk c belongs to slot c % S
// (S slots per query head, one CTA item each). A slot visits its chunks in tiles of pk_at(hd) rows
// (several chunks side by side, in increasing position order), so which positions a tile holds and
// the order in which they are summed depend only on absolute positions: a token's result does not
// depend on how many tokens share the pass. Items write their slot state (m, l, acc); the O phase
// merges the slots while staging its activations.
constexpr int PK_CHUNK = 32;
__host__ __device__ constexpr int pk_at(int hd) { return hd <= 64 ? 128 : 64; }
// K/V tile row stride (halves): rows start on 16-byte boundaries (cp.async targets) and the
// per-position 16-byte reads of a quarter warp hit distinct banks.
__host__ __device__ constexpr int pk_hpk(int hd) { return hd + 8; }
// Dedicated K/V tile region: K then V, [pk_at][pk_hpk] f16 each.
__host__ __device__ constexpr size_t pk_kv_smem(int hd) { return 2 * (size_t)pk_at(hd) * pk_hpk(hd) * 2; }
// Attention scratch in the B-operand region: q [T][HD] f32, running state [T][HD + 2] f32 (m, l,
// acc), probabilities [PK_NW][pk_at] f32.
__host__ __device__ constexpr size_t pk_att_smem(int T, int hd) {
  return (size_t)T * hd * 4 + (size_t)T * (hd + 2) * 4 + (size_t)PK_NW * pk_at(hd) * 4;
}

// Context position of row r of tile ti of slot `slot` (S slots, CPT chunks per tile).
__device__ __forceinline__ int att_row_pos(int slot, int S, int ti, int cpt, int r) {
  return (slot + S * (ti * cpt + r / PK_CHUNK)) * PK_CHUNK + r % PK_CHUNK;
}

// Starts the cp.async copies of the cached K/V rows (positions < pos0, which no phase of this pass
// writes) of tile 0 of item (hh, slot) into the K/V region, spread over `nthr` threads (this one
// is `tid`); each of them commits one group, which attention_item's wait covers.
__device__ void attention_prefetch(const PassArgs& a, int pos0, int l, int hh, int slot, uint8_t* kvb, int tid, int nthr) {
  const int HD = a.hd, HPK = pk_hpk(HD), AT = pk_at(HD), c8 = HD / 8;
  const int g = hh / (a.heads / a.kv_heads);
  const uint16_t* kc = a.kc + (size_t)l * a.kv_layer;
  const uint16_t* vc = a.vc + (size_t)l * a.kv_layer;
  __half* Ks = reinterpret_cast<__half*>(kvb);
  __half* Vs = Ks + AT * HPK;
  for (int i = tid; i < AT * c8; i += nthr) {
    const int r = i / c8, ch = i - r * c8;
    const int p = att_row_pos(slot, a.slots, 0, AT / PK_CHUNK, r);
    if (p < pos0) {
      const size_t row = kv_row(a.pages, a.page_shift, a.num_pages, g, p) * HD + ch * 8;
      tc::cp_async16(tc::su32(Ks + r * HPK + ch * 8), kc + row);
      tc::cp_async16(tc::su32(Vs + r * HPK + ch * 8), vc + row);
    }
  }
  tc::cp_commit();
}

// Attention item: query head hh over the chunks of `slot`; writes the slot state (m, l, acc) of
// every token to att_part. prefetched: tile 0's cached rows were started by attention_prefetch.
// sub (optional, profiling): globaltimer stamps of thread 0, sub[0] after the query rows are
// staged, sub[stride] after the first tile is in shared memory, sub[2 stride] once the slot state
// is written.
template <int PPL>
__device__ void attention_item(const PassArgs& a, int pos0, int l, int hh, int slot, uint8_t* sm, uint8_t* kvb,
                               bool prefetched, unsigned* sub, int stride) {
  constexpr int AT = 32 * PPL, CPT = AT / PK_CHUNK;
  const int HD = a.hd, HALF = HD / 2, HP = HD + 2, HPK = HD + 8, T = a.T, S = a.slots;
  const int group = a.heads / a.kv_heads, g = hh / group;
  const int total = pos0 + T;
  const int nch = (total + PK_CHUNK - 1) / PK_CHUNK;
  const int H = a.heads * HD, KV = a.kv_heads * HD, QS = H + 2 * KV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint16_t* kc = a.kc + (size_t)l * a.kv_layer;  // this layer's page pools
  uint16_t* vc = a.vc + (size_t)l * a.kv_layer;
  float* qs = reinterpret_cast<float*>(sm);   // [T][HD]
  float* st = qs + T * HD;                    // [T][HP]
  float* es = st + T * HP;                    // [PK_NW][AT]
  __half* Ks = reinterpret_cast<__half*>(kvb);  // [AT][HPK]
  __half* Vs = Ks + AT * HPK;
  const float scale = 1.0f / sqrtf((float)HD);
  for (int i = threadIdx.x; i < T * HALF; i += PK_THREADS) {
    const int t = i / HALF, d = i - t * HALF;
    const float2 cs = a.rope[(size_t)(pos0 + t) * HALF + d];
    const long long* q = a.qkv + (size_t)t * QS + hh * HD;
    const float x1 = from_fix(ldcg_ll(q + d)), x2 = from_fix(ldcg_ll(q + d + HALF));
    qs[t * HD + d] = x1 * cs.x - x2 * cs.y;
    qs[t * HD + d + HALF] = x2 * cs.x + x1 * cs.y;
  }
  for (int i = threadIdx.x; i < T * HP; i += PK_THREADS) st[i] = (i % HP == 0) ? -CUDART_INF_F : 0.f;
  if (sub && threadIdx.x == 0) sub[0] = gtimer();
  const bool writer = (hh % group) == 0;
  const int c8 = HD / 8;
  for (int ti = 0; slot + S * ti * CPT < nch; ti++) {
    if (ti > 0 || !prefetched) {
      __syncthreads();  // the previous tile's readers are done
      for (int i = threadIdx.x; i < AT * c8; i += PK_THREADS) {
        const int r = i / c8, ch = i - r * c8;
        const int p = att_row_pos(slot, S, ti, CPT, r);
        if (p < pos0) {
          const size_t row = kv_row(a.pages, a.page_shift, a.num_pages, g, p) * HD + ch * 8;
          tc::cp_async16(tc::su32(Ks + r * HPK + ch * 8), kc + row);
          tc::cp_async16(tc::su32(Vs + r * HPK + ch * 8), vc + row);
        }
      }
      tc::cp_commit();
    }
    // rows of this pass's block (rotated, rounded to f16, appended to the cache) and zero padding
    for (int i = threadIdx.x; i < AT * HALF; i += PK_THREADS) {
      const int r = i / HALF, d = i - r * HALF, p = att_row_pos(slot, S, ti, CPT, r);
      if (p < pos0) continue;
      __half k1 = __float2half_rn(0.f), k2 = k1, v1 = k1, v2 = k1;
      if (p < total) {
        const int t = p - pos0;
        const long long* kr = a.qkv + (size_t)t * QS + H + g * HD;
        const long long* vr = a.qkv + (size_t)t * QS + H + KV + g * HD;
        const float2 cs = a.rope[(size_t)p * HALF + d];
        const float x1 = from_fix(ldcg_ll(kr + d)), x2 = from_fix(ldcg_ll(kr + d + HALF));
        k1 = __float2half_rn(x1 * cs.x - x2 * cs.y);
        k2 = __float2half_rn(x2 * cs.x + x1 * cs.y);
        v1 = __float2half_rn(from_fix(ldcg_ll(vr + d)));
        v2 = __float2half_rn(from_fix(ldcg_ll(vr + d + HALF)));
        if (writer) {
          const size_t row = kv_row(a.pages, a.page_shift, a.num_pages, g, p) * HD;
          kc[row + d] = __half_as_ushort(k1);
          kc[row + d + HALF] = __half_as_ushort(k2);
          vc[row + d] = __half_as_ushort(v1);
          vc[row + d + HALF] = __half_as_ushort(v2);
        }
      }
      Ks[r * HPK + d] = k1;
      Ks[r * HPK + d + HALF] = k2;
      Vs[r * HPK + d] = v1;
      Vs[r * HPK + d + HALF] = v2;
    }
    tc::cp_wait<0>();
    __syncthreads();
    if (sub && ti == 0 && threadIdx.x == 0) sub[stride] = gtimer();
    float* ew = es + warp * AT;
    for (int t = warp; t < T; t += PK_NW) {
      // valid rows: a prefix of the tile (positions grow with the row)
      const int ctx = pos0 + t + 1;
      int lim = 0;
      for (int k = 0; k < CPT; k++) {
        const int c0 = (slot + S * (ti * CPT + k)) * PK_CHUNK;
        if (c0 >= ctx) break;
        lim = k * PK_CHUNK + min(PK_CHUNK, ctx - c0);
      }
      if (lim == 0) continue;
      // scores of rows lane + 32 j: 16-byte K reads, two FMA chains per row
      float sa[PPL], sb[PPL];
#pragma unroll
      for (int j = 0; j < PPL; j++) sa[j] = sb[j] = 0.f;
      const float* q = qs + t * HD;
      for (int d = 0; d < HD; d += 8) {
        const float4 qa = *reinterpret_cast<const float4*>(q + d), qb = *reinterpret_cast<const float4*>(q + d + 4);
#pragma unroll
        for (int j = 0; j < PPL; j++) {
          if (32 * j >= lim) break;
          const uint4 kv = *reinterpret_cast<const uint4*>(Ks + (lane + 32 * j) * HPK + d);
          const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kv.x));
          const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kv.y));
          const float2 k2 = __half22float2(*reinterpret_cast<const __half2*>(&kv.z));
          const float2 k3 = __half22float2(*reinterpret_cast<const __half2*>(&kv.w));
          sa[j] = fmaf(qa.x, k0.x, sa[j]);
          sb[j] = fmaf(qa.y, k0.y, sb[j]);
          sa[j] = fmaf(qa.z, k1.x, sa[j]);
          sb[j] = fmaf(qa.w, k1.y, sb[j]);
          sa[j] = fmaf(qb.x, k2.x, sa[j]);
          sb[j] = fmaf(qb.y, k2.y, sb[j]);
          sa[j] = fmaf(qb.z, k3.x, sa[j]);
          sb[j] = fmaf(qb.w, k3.y, sb[j]);
        }
      }
      float sc[PPL], tmax = -CUDART_INF_F;
#pragma unroll
      for (int j = 0; j < PPL; j++) {
        sc[j] = (lane + 32 * j < lim) ? (sa[j] + sb[j]) * scale : -CUDART_INF_F;
        tmax = fmaxf(tmax, sc[j]);
      }
      tmax = warp_max(tmax);
      float* Sx = st + t * HP;
      const float m_old = Sx[0], m_new = fmaxf(m_old, tmax);
      const float corr = (m_old == -CUDART_INF_F) ? 0.f : expf(m_old - m_new);
      float esum = 0.f;
#pragma unroll
      for (int j = 0; j < PPL; j++) {
        const float e = (sc[j] == -CUDART_INF_F) ? 0.f : expf(sc[j] - m_new);
        ew[lane + 32 * j] = e;
        esum += e;
      }
      const float lsum = warp_sum(esum);
      __syncwarp();
      // values: lane owns columns d0 + 2 lane, d0 + 2 lane + 1; even and odd rows in two chains
      for (int d0 = 0; d0 < HD; d0 += 64) {
        const int d = d0 + 2 * lane;
        if (d < HD) {
          float ax = 0.f, ay = 0.f, bx = 0.f, by = 0.f;
          int p = 0;
          for (; p + 1 < lim; p += 2) {
            const float e0 = ew[p], e1 = ew[p + 1];
            const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(Vs + p * HPK + d));
            const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(Vs + (p + 1) * HPK + d));
            ax = fmaf(e0, v0.x, ax);
            ay = fmaf(e0, v0.y, ay);
            bx = fmaf(e1, v1.x, bx);
            by = fmaf(e1, v1.y, by);
          }
          if (p < lim) {
            const float e0 = ew[p];
            const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(Vs + p * HPK + d));
            ax = fmaf(e0, v0.x, ax);
            ay = fmaf(e0, v0.y, ay);
          }
          Sx[2 + d] = fmaf(Sx[2 + d], corr, ax + bx);
          Sx[3 + d] = fmaf(Sx[3 + d], corr, ay + by);
        }
      }
      __syncwarp();
      if (lane == 0) {
        Sx[1] = fmaf(Sx[1], corr, lsum);
        Sx[0] = m_new;
      }
      __syncwarp();
    }
  }
  if (prefetched && slot >= nch) tc::cp_wait<0>();  // no tile: the prefetch group (empty) retires here
  __syncthreads();
  float* part = a.att_part + ((size_t)hh * S + slot) * T * HP;
  for (int i = threadIdx.x; i < T * HP; i += PK_THREADS) part[i] = st[i];
  if (sub && threadIdx.x == 0) sub[2 * (size_t)stride] = gtimer();
}

// O-phase staging of attention columns [col0, col0 + ncol): merges the S slot states. A warp makes
// 32 adjacent column pairs of one token (a whole warp always shares the token and, for head widths
// that are multiples of 64, the head: then lane s computes slot s's weight e^(m_s - m*) / L once and
// the warp shares it). Every lane loads the two values of each slot at once (one round trip) and
// sums in slot order. Rows T..NT-1 are zero.
template <int NT>
__device__ __forceinline__ void stage_attention(const PassArgs& a, uint8_t* xb, uint32_t sbo, int col0, int ncol) {
  const int HD = a.hd, HP = HD + 2, S = a.slots, T = a.T, np = ncol / 2;
  const int lane = threadIdx.x & 31;
  const size_t sstride = (size_t)T * HP;  // between the slots of one head
  auto put = [&](int t, int c, float ox, float oy) {
    const int kc = (c - col0) / 8, e = (c - col0) % 8;
    *reinterpret_cast<__half2*>(xb + (size_t)(t / 8) * sbo + (size_t)kc * 128 + (t % 8) * 16 + e * 2) =
        __floats2half2_rn(ox, oy);
  };
  // np is a multiple of 32 (K slices are whole 64-column blocks) and so is PK_STAGERS: a warp's 32
  // pairs never straddle a token
#pragma unroll 1
  for (int i0 = threadIdx.x - lane; i0 < T * np; i0 += PK_STAGERS) {
    const int i = i0 + lane, t = i / np, c = col0 + 2 * (i - t * np);
    const int hh = c / HD, d = c - hh * HD;
    const float* base = a.att_part + (size_t)hh * S * sstride + (size_t)t * HP;
    float2 v[kMaxSlots];
#pragma unroll
    for (int s2 = 0; s2 < kMaxSlots; s2++)
      v[s2] = s2 < S ? __ldcg(reinterpret_cast<const float2*>(base + s2 * sstride + 2 + d)) : make_float2(0.f, 0.f);
    // the slot (m, l) pair of lane `lane` < S, loaded with the values (one L2 round trip); used
    // when the warp's 32 pairs lie in one head
    const float2 ml = lane < S ? __ldcg(reinterpret_cast<const float2*>(base + lane * sstride)) : make_float2(-CUDART_INF_F, 0.f);
    const bool one_head = __all_sync(0xffffffffu, hh == __shfl_sync(0xffffffffu, hh, 0));
    float ox = 0.f, oy = 0.f;
    if (one_head) {
      const float mx = warp_max(ml.x);
      const float e = (ml.x == -CUDART_INF_F) ? 0.f : __expf(ml.x - mx);
      const float w = __fdividef(e, warp_sum(ml.y * e));
#pragma unroll
      for (int s2 = 0; s2 < kMaxSlots; s2++) {
        const float ws = __shfl_sync(0xffffffffu, w, s2);
        if (s2 < S) {
          ox = fmaf(v[s2].x, ws, ox);
          oy = fmaf(v[s2].y, ws, oy);
        }
      }
    } else {  // head widths that are not multiples of 64: every lane weighs its own head's slots
      float2 ml[kMaxSlots];
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int s2 = 0; s2 < kMaxSlots; s2++) {
        ml[s2] = s2 < S ? __ldcg(reinterpret_cast<const float2*>(base + s2 * sstride)) : make_float2(-CUDART_INF_F, 0.f);
        mx = fmaxf(mx, ml[s2].x);
      }
      float L = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < kMaxSlots; s2++) {
        ml[s2].x = (ml[s2].x == -CUDART_INF_F) ? 0.f : __expf(ml[s2].x - mx);
        L = fmaf(ml[s2].y, ml[s2].x, L);
      }
#pragma unroll
      for (int s2 = 0; s2 < kMaxSlots; s2++) {
        const float ws = __fdividef(ml[s2].x, L);
        ox = fmaf(v[s2].x, ws, ox);
        oy = fmaf(v[s2].y, ws, oy);
      }
    }
    put(t, c, ox, oy);
  }
  for (int i = T * np + threadIdx.x; i < NT * np; i += PK_STAGERS) {
    const int t = i / np;
    put(t, col0 + 2 * (i - t * np), 0.f, 0.f);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// The pass kernel
// ---------------------------------------------------------------------------------------------
template <int BITS, int G, int NT>
__global__ void __launch_bounds__(PK_THREADS, 1) pass_kernel(const PassArgs a) {
  using Gemv = TcGemv<BITS, G, NT>;
  using Str = Stream<BITS, G>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t bar_a[PK_NWG * PK_ABUF], bar_full[PK_NWG * PK_ABUF], bar_d[PK_NWG * 2], bar_dfree[PK_NWG * 2],
      bar_fin[PK_NWG];
  __shared__ uint64_t s_full[PK_MAX_STAGES], s_empty[PK_MAX_STAGES];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort, s_pos0;
  __shared__ float s_inv[NT];
  __shared__ float s_bv[PK_NW][NT];
  __shared__ uint32_t s_bi[PK_NW][NT];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool compute = threadIdx.x < PK_CT;
  const int T = a.T, h = a.hidden, I = a.inter;
  const int kvd = a.kv_heads * a.hd, QS = h + 2 * kvd;
  int* err = &a.ctl->err;
  // shared memory: [weight-stream ring (1 KB aligned)][B operand, or attention scratch, or rms sums]
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int nst = a.stages;
  uint8_t* xb = ring + (size_t)nst * Str::kStage;
  uint8_t* kvb = xb + a.kv_off;  // attention K/V tiles
  // the B operand and K/V regions are contiguous: the RMS statistics copy rows of x into both
  const size_t rms_bytes = (size_t)a.kv_off + pk_kv_smem(a.hd);
  // or (a.xs) they keep the rows as f32 and the norm weights after the K/V region for the staging
  float* xs = a.xs ? reinterpret_cast<float*>(kvb + pk_kv_smem(a.hd)) : nullptr;
  float* wn = xs ? xs + (size_t)NT * h : nullptr;
  const uint32_t xb_addr = tc::su32(xb);

  if (threadIdx.x == 0) {
    for (int i = 0; i < PK_NWG * PK_ABUF; i++) {
      tc::mbar_init(&bar_a[i], 1);
      tc::mbar_init(&bar_full[i], 4);  // one arrival per compute warp of the warpgroup
    }
    for (int i = 0; i < PK_NWG * 2; i++) {
      tc::mbar_init(&bar_d[i], 1);
      tc::mbar_init(&bar_dfree[i], 4);
    }
    for (int i = 0; i < nst; i++) {
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&s_empty[i], PK_NWG * 4);
    }
    for (int i = 0; i < PK_NWG; i++) tc::mbar_init(&bar_fin[i], 1);
    s_abort = 0;
    s_pos0 = a.ctl->pos0;  // the pass's start position: only CTA 0 advances it, after the last barrier
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::su32(&s_tmem)),
                 "r"(PK_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  tc::fence_after();
  const int pos0 = s_pos0;
  Gemv gm;
  gm.tmem = s_tmem;
  gm.ring = ring;
  gm.nst = nst;
  gm.full = s_full;
  gm.empty = s_empty;
  gm.bar_a = bar_a;
  gm.bar_full = bar_full;
  gm.bar_d = bar_d;
  gm.bar_dfree = bar_dfree;
  gm.abort = &s_abort;
  gm.blk = gm.itc = gm.rpos = 0;
  Producer<BITS, G> pr;
  pr.ring = ring;
  pr.nst = nst;
  pr.full = s_full;
  pr.empty = s_empty;
  pr.abort = &s_abort;
  pr.lpos = 0;
  pr.i = 1 << 30;
  pr.sp.tiles = pr.sp.ks = pr.sp.nblk = 0;
  const bool producer = warp == PK_PRODUCER && lane == 0;

  // Profiling timeline: slot 0 = start, 2b - 1 / 2b = arrival at / departure from barrier b.
  auto stamp = [&](unsigned slot) {
    if (a.trace && threadIdx.x == 0) a.trace[(size_t)slot * gridDim.x + blockIdx.x] = gtimer();
  };
  stamp(0);
  unsigned nbar = 0;
  bool ok = true;
  auto barrier = [&]() {
    nbar++;
    if (a.trace) {
      __syncthreads();
      stamp(2 * nbar - 1);
    }
    // a test hook (stall_barrier) makes one barrier wait for an arrival that never comes, so that
    // its bounded wait runs out
    const unsigned target = nbar * gridDim.x + (nbar == (unsigned)a.stall_barrier ? 1u : 0u);
    if (!grid_barrier(a.bar, target, err, a.poll_limit, &s_abort)) ok = false;
    if (s_abort) ok = false;
    stamp(2 * nbar);
    return ok;
  };
  // Stamps inside the phase that follows barrier nbar (thread 0's progress): 0 = phase prepared
  // (RMS statistics), 1 = first item staged, 2 = first item done, 3 = last item done.
  auto sub_ptr = [&](int k) -> unsigned* {
    return a.trace ? a.trace + ((size_t)a.trace_sub + 4 * nbar + k) * gridDim.x + blockIdx.x : nullptr;
  };
  auto sub = [&](int k) {
    if (a.trace && threadIdx.x == 0) *sub_ptr(k) = gtimer();
  };
  // Starts the weight stream of this CTA's items of the next GEMV phase (before the barrier):
  // as many stages as the ring has free, without waiting.
  auto prefetch = [&](const QMat& w, const QMaps* maps, int ks) {
    if (!producer) return;
    pr.begin(maps, make_split<BITS, G>(w, ks));
    while (!pr.done() && pr.issue_one(false)) {
    }
  };
  // Runs the items of a GEMV phase (its weights streaming since the prefetch): stage(col0, ncol,
  // sbo) fills the B operand of a K slice, epi(row, ks_index, tot) consumes the accumulators. The
  // producer finishes the phase's stream; the others walk the same item sequence (so the staging
  // barriers match even after a failure, when the work is skipped and bounded waits return).
  auto gemv_phase = [&](const QMat& w, int ks, auto stage, auto epi) {
    const Split sp = make_split<BITS, G>(w, ks);
    sub(0);
    if (warp == PK_PRODUCER) {
      if (producer) {
        while (ok && !pr.done()) {
          if (!pr.issue_one(true)) {
            ok = false;
            s_abort = 1;
            atomicCAS(err, 0, 1);
          }
        }
      }
      return;
    }
    int staged = -1;
    for (int i = blockIdx.x; i < sp.items(); i += gridDim.x) {
      const bool first = i == (int)blockIdx.x;
      int t256, kb0, kb1;
      sp.item(i, &t256, &kb0, &kb1);
      const int kslice = i / sp.tiles;
      const int col0 = kb0 * Gemv::KB, ncol = (kb1 - kb0) * Gemv::KB;
      const uint32_t sbo = (uint32_t)(ncol / 8) * 128u;
      if (kslice != staged) {
        stagers_sync();
        if (ok) stage(col0, ncol, sbo);
        stagers_sync();
        staged = kslice;
      }
      if (first) sub(1);
      if (!ok) continue;
      if (compute) {
        float tot[NT];
        if (!gm.run(kb0, kb1, tot)) {
          ok = false;
        } else {
          const int t32 = t256 * 8 + warp;
          if (t32 < w.rows_pad / 32) epi(t32 * 32 + lane, kslice, tot);
          if (first) sub(2);
          sub(3);
        }
      } else if (!gm.issue(warp - PK_ISSUER, kb0, kb1, xb_addr, sbo)) {
        ok = false;
      }
      if (!ok) {
        s_abort = 1;
        if (lane == 0) atomicCAS(err, 0, 1);  // the other CTAs stop at their next wait
      }
    }
  };

  // ---- embedding rows into the residual stream; zero the q|k|v accumulators ----
  {
    const QMat& e = a.embed;
    const int nch = e.chunks();
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
      const uint32_t tok = a.ctl->tokens[t];
      if (tok >= (uint32_t)a.vocab) {
        if (threadIdx.x == 0) atomicExch(err, 2);
        continue;
      }
      const uint8_t* row = e.data + ((size_t)(tok / 32) * nch) * 512 + (tok % 32) * 16;
      const uint16_t* sc = e.scales + (size_t)(tok / 32) * e.groups() * 32 + (tok % 32);
      for (int c = threadIdx.x; c < h; c += PK_THREADS) {
        const int gi = c / e.group;
        float q;
        if (e.bits == 8) {
          q = (float)(int8_t)row[(size_t)(c / 16) * 512 + c % 16];
        } else {
          const int half = e.group / 2, j = c % e.group;
          const int bi = gi * half + (j < half ? j : j - half);
          const uint8_t by = row[(size_t)(bi / 16) * 512 + bi % 16];
          q = (float)((j < half ? (by & 15) : (by >> 4)) - 8);
        }
        a.x[(size_t)t * h + c] = to_fix(q * bf16f(sc[(size_t)gi * 32]));
      }
    }
    zero_ll(a.qkv, (size_t)T * QS);
  }
  prefetch(a.layers[0].qkv, &a.layers[0].maps[0], a.ks_qkv);
  barrier();

  for (int l = 0; l < a.L && ok; l++) {
    const PassLayer& W = a.layers[l];
    // ---- QKV: RMSNorm(x) -> q|k|v sums (+ bias once) ----
    if (xs) rms_rows(a.x, T, h, a.eps, s_inv, xs, wn, W.in_norm, nullptr);
    else rms_stats(a.x, T, h, a.eps, s_inv, xb, rms_bytes);
    // cached K/V rows of this CTA's first attention item: they stream in during the QKV phase,
    // issued by the producer warp's lanes 1..31 (idle while lane 0 streams the weights), so their
    // page-table lookups stay off the phase's critical path
    if ((int)blockIdx.x < a.heads * a.slots && warp == PK_PRODUCER && lane != 0)
      attention_prefetch(a, pos0, l, blockIdx.x / a.slots, blockIdx.x % a.slots, kvb, lane - 1, 31);
    gemv_phase(
        W.qkv, a.ks_qkv,
        [&](int col0, int ncol, uint32_t sbo) {
          stage_b<NT>(xb, sbo, T, col0, ncol, [&](int t, int c) {
            return xs ? xs[(size_t)t * h + c] * s_inv[t] * wn[c]
                      : from_fix(ldcg_ll(a.x + (size_t)t * h + c)) * s_inv[t] * bf16f(W.in_norm[c]);
          });
        },
        [&](int r, int kslice, float (&tot)[NT]) {
          if (r >= QS) return;
          const float b = kslice == 0 ? bf16f(W.qkv_bias[r]) : 0.f;
#pragma unroll
          for (int t = 0; t < NT; t++)
            if (t < T) fix_add(a.qkv + (size_t)t * QS + r, tot[t] + b);
        });
    if (!barrier()) break;

    // ---- attention slot states (the block's K/V appended to the cache); zero the gate/up sums ----
    for (int it = blockIdx.x; it < a.heads * a.slots; it += gridDim.x) {
      __syncthreads();
      const bool first = it == (int)blockIdx.x;
      if (a.hd <= 64)
        attention_item<4>(a, pos0, l, it / a.slots, it % a.slots, xb, kvb, first, first ? sub_ptr(0) : nullptr, (int)gridDim.x);
      else
        attention_item<2>(a, pos0, l, it / a.slots, it % a.slots, xb, kvb, first, first ? sub_ptr(0) : nullptr, (int)gridDim.x);
      sub(3);
    }
    zero_ll(a.gu, (size_t)T * 2 * I);
    prefetch(W.o, &W.maps[1], a.ks_o);
    if (!barrier()) break;

    // ---- O: residual add into x ----
    gemv_phase(
        W.o, a.ks_o, [&](int col0, int ncol, uint32_t sbo) { stage_attention<NT>(a, xb, sbo, col0, ncol); },
        [&](int r, int, float (&tot)[NT]) {
          if (r >= h) return;
#pragma unroll
          for (int t = 0; t < NT; t++)
            if (t < T) fix_add(a.x + (size_t)t * h + r, tot[t]);
        });
    zero_ll(a.qkv, (size_t)T * QS);
    prefetch(W.gu, &W.maps[2], a.ks_gu);
    if (!barrier()) break;

    // ---- gate/up: RMSNorm(x) -> gate/up sums ----
    if (xs) rms_rows(a.x, T, h, a.eps, s_inv, xs, wn, W.post_norm, nullptr);
    else rms_stats(a.x, T, h, a.eps, s_inv, xb, rms_bytes);
    gemv_phase(
        W.gu, a.ks_gu,
        [&](int col0, int ncol, uint32_t sbo) {
          stage_b<NT>(xb, sbo, T, col0, ncol, [&](int t, int c) {
            return xs ? xs[(size_t)t * h + c] * s_inv[t] * wn[c]
                      : from_fix(ldcg_ll(a.x + (size_t)t * h + c)) * s_inv[t] * bf16f(W.post_norm[c]);
          });
        },
        [&](int r, int, float (&tot)[NT]) {
          if (r >= 2 * I) return;
#pragma unroll
          for (int t = 0; t < NT; t++)
            if (t < T) fix_add(a.gu + (size_t)t * 2 * I + r, tot[t]);
        });
    prefetch(W.down, &W.maps[3], a.ks_down);
    if (!barrier()) break;

    // ---- down: SwiGLU while staging, residual add into x ----
    gemv_phase(
        W.down, a.ks_down,
        [&](int col0, int ncol, uint32_t sbo) {
          stage_b<NT>(xb, sbo, T, col0, ncol, [&](int t, int j) {
            const long long* row = a.gu + (size_t)t * 2 * I + (j / 16) * 32 + (j % 16);
            const float gt = from_fix(ldcg_ll(row)), up = from_fix(ldcg_ll(row + 16));
            return gt * __frcp_rn(1.0f + __expf(-gt)) * up;
          });
        },
        [&](int r, int, float (&tot)[NT]) {
          if (r >= h) return;
#pragma unroll
          for (int t = 0; t < NT; t++)
            if (t < T) fix_add(a.x + (size_t)t * h + r, tot[t]);
        });
    if (l + 1 < a.L) prefetch(a.layers[l + 1].qkv, &a.layers[l + 1].maps[0], a.ks_qkv);
    else if (a.n_logits > 0) prefetch(a.embed, a.embed_maps, 1);
    if (!barrier()) break;
  }

  // ---- LM head on the last n_logits rows: final RMSNorm, per-CTA argmax parts ----
  if (ok && a.n_logits > 0) {
    const int n = a.n_logits, r0 = T - n;
    for (int i = threadIdx.x; i < PK_NW * NT; i += PK_THREADS) {
      (&s_bv[0][0])[i] = -CUDART_INF_F;
      (&s_bi[0][0])[i] = 0xffffffffu;
    }
    if (xs) rms_rows(a.x + (size_t)r0 * h, n, h, a.eps, s_inv, xs, wn, nullptr, a.final_norm);
    else rms_stats(a.x + (size_t)r0 * h, n, h, a.eps, s_inv, xb, rms_bytes);
    gemv_phase(
        a.embed, 1,
        [&](int col0, int ncol, uint32_t sbo) {
          stage_b<NT>(xb, sbo, n, col0, ncol, [&](int t, int c) {
            return xs ? xs[(size_t)t * h + c] * s_inv[t] * wn[c]
                      : from_fix(ldcg_ll(a.x + (size_t)(r0 + t) * h + c)) * s_inv[t] * a.final_norm[c];
          });
        },
        [&](int r, int, float (&tot)[NT]) {
#pragma unroll
          for (int t = 0; t < NT; t++) {
            if (t < n) {
              float v = (r < a.vocab) ? tot[t] : -CUDART_INF_F;
              uint32_t idx = (uint32_t)r;
              if (a.logits && r < a.vocab) a.logits[(size_t)t * a.vocab + r] = tot[t];
              warp_argmax(v, idx);
              if (lane == 0 && arg_better(v, idx, s_bv[warp][t], s_bi[warp][t])) {
                s_bv[warp][t] = v;
                s_bi[warp][t] = idx;
              }
            }
          }
        });
    __syncthreads();
    if (threadIdx.x < n) {
      const int t = threadIdx.x;
      float v = s_bv[0][t];
      uint32_t idx = s_bi[0][t];
      for (int w = 1; w < PK_NW; w++)
        if (arg_better(s_bv[w][t], s_bi[w][t], v, idx)) {
          v = s_bv[w][t];
          idx = s_bi[w][t];
        }
      a.arg_parts[(size_t)blockIdx.x * n + t] = ArgPart{v, idx};
    }
    if (barrier() && blockIdx.x == 0) argmax_finalize_block(a.arg_parts, gridDim.x, n, a.ctl);
  } else if (ok && blockIdx.x == 0 && threadIdx.x == 0) {
    a.ctl->pos0 += a.ctl->M;
  }
  __syncthreads();
  stamp(2 * nbar + 1);

  tc::cp_wait<0>();  // an attention prefetch left by an aborted layer
  // ---- release tensor memory (after the issuer's MMAs and the stream's copies have all
  // completed, also after an abort) ----
  if (warp >= PK_ISSUER && warp < PK_ISSUER + PK_NWG && lane == 0) {
    volatile int no_abort = 0;
    tc::commit(&bar_fin[warp - PK_ISSUER]);
    tc::mbar_wait(&bar_fin[warp - PK_ISSUER], 0, &no_abort);
  }
  if (producer) {
    volatile int no_abort = 0;
    for (uint32_t p = pr.lpos > (uint32_t)nst ? pr.lpos - nst : 0; p < pr.lpos; p++)
      tc::mbar_wait(&s_full[p % nst], (p / nst) & 1, &no_abort);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(s_tmem), "r"(PK_TMEM_COLS) : "memory");
  }
  if (s_abort && threadIdx.x == 0) atomicCAS(err, 0, 1);
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------

int pass_kernel_nt(int T) { return T <= 16 ? 16 : T <= 32 ? 32 : 48; }

bool pass_kernel_supported(const WeightFormat& body, const WeightFormat& embed, int T, int hd) {
  if (!(body == embed) || T < 1 || T > 48 || hd % 8 || hd > 128) return false;
  return (body.bits == 8 && (body.group == 32 || body.group == 64)) || (body.bits == 4 && (body.group == 16 || body.group == 32));
}

int pass_kernel_stage_blocks(const WeightFormat& f) {
  const int cpb = tc_kb(f.bits, f.group) / (128 / f.bits);
  return std::max(1, PK_STAGE_DATA / (8 * cpb * 512));
}

static size_t pass_stage_bytes(const WeightFormat& f) {
  const int kb = tc_kb(f.bits, f.group), cpb = kb / (128 / f.bits), ns = kb >= f.group ? kb / f.group : 1;
  const int nb = pass_kernel_stage_blocks(f);
  return (size_t)8 * cpb * nb * 512 + (size_t)8 * ns * nb * 64;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link needed).
void pass_encode_maps(const QMat& w, QMaps* out) {
  WeightFormat f;
  f.bits = w.bits;
  f.group = w.group;
  const int kb = tc_kb(w.bits, w.group), cpb = kb / (128 / w.bits), ns = kb >= w.group ? kb / w.group : 1;
  const int nb = pass_kernel_stage_blocks(f);
  encode_qmat_maps(w, cpb * nb, ns * nb, 8, out);
}

void encode_qmat_maps(const QMat& w, int box_chunks, int box_groups, int box_rowgroups, QMaps* out) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                              const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    LS_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn) LS_THROW(-3, "cuTensorMapEncodeTiled is not available from the driver");
    encode = reinterpret_cast<Encode>(fn);
  }
  const cuuint64_t tiles32 = (cuuint64_t)w.rows_pad / 32, nch = (cuuint64_t)w.chunks(), ngr = (cuuint64_t)w.groups();
  const cuuint32_t es[3] = {1, 1, 1};
  if (box_chunks < 1 || box_chunks > 256 || box_groups < 1 || box_groups > 256 || box_rowgroups < 1 || box_rowgroups > 256)
    LS_THROW(-3, "tensor map box out of range");
  {
    const cuuint64_t dims[3] = {128, nch, tiles32};
    const cuuint64_t strides[2] = {512, nch * 512};
    const cuuint32_t box[3] = {128, (cuuint32_t)box_chunks, (cuuint32_t)box_rowgroups};
    const CUresult r = encode(&out->data, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(w.data), dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) LS_THROW(-3, "cuTensorMapEncodeTiled (weights) failed: " + std::to_string((int)r));
  }
  {
    const cuuint64_t dims[3] = {32, ngr, tiles32};
    const cuuint64_t strides[2] = {64, ngr * 64};
    const cuuint32_t box[3] = {32, (cuuint32_t)box_groups, (cuuint32_t)box_rowgroups};
    const CUresult r = encode(&out->scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint16_t*>(w.scales), dims, strides, box,
                              es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) LS_THROW(-3, "cuTensorMapEncodeTiled (scales) failed: " + std::to_string((int)r));
  }
}

// Bytes of the B-operand region (rounded to 128): the attention K/V region follows it.
size_t pass_kernel_kv_off(const WeightFormat& f, int T, int hidden, int inter, int hd, int ks_down) {
  const int NT = pass_kernel_nt(T);
  const int kb = tc_kb(f.bits, f.group);
  // largest B operand: the full hidden width (QKV, O, gate/up, head) or a K slice of down
  const int nblk_down = inter / kb;
  const int down_cols = ((nblk_down + ks_down - 1) / ks_down) * kb;
  size_t b = (size_t)NT * std::max(hidden, down_cols) * 2;
  b = std::max(b, pk_att_smem(T, hd));
  return (b + 127) & ~(size_t)127;
}

// The x copy after the K/V region: [NT][hidden] f32 rows, then [hidden] f32 norm weights.
size_t pass_kernel_xs_bytes(int T, int hidden) { return ((size_t)pass_kernel_nt(T) + 1) * hidden * 4; }

size_t pass_kernel_smem(const WeightFormat& f, int T, int hidden, int inter, int hd, int ks_down, int stages, bool xs) {
  return 1024 + (size_t)stages * pass_stage_bytes(f) + pass_kernel_kv_off(f, T, hidden, inter, hd, ks_down) +
         pk_kv_smem(hd) + (xs ? pass_kernel_xs_bytes(T, hidden) : 0);  // 1 KB for aligning the ring
}

// The deepest weight ring (2 .. PK_MAX_STAGES stages) whose shared memory fits `budget` bytes; 0 if
// none does. A deeper ring keeps more bytes in flight per SM (the LM head streams at the ring's
// depth over the memory latency).
int pass_kernel_stages(const WeightFormat& f, int T, int hidden, int inter, int hd, int ks_down, size_t budget, bool xs) {
  for (int st = PK_MAX_STAGES; st >= 2; st--)
    if (pass_kernel_smem(f, T, hidden, inter, hd, ks_down, st, xs) <= budget) return st;
  return 0;
}

template <int BITS, int G, int NT>
static void launch_pass_t(const PassArgs& a, size_t smem, int grid, cudaStream_t s) {
  ensure_smem(pass_kernel<BITS, G, NT>, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(PK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  LS_CUDA(cudaLaunchKernelEx(&cfg, pass_kernel<BITS, G, NT>, a));
}

void launch_pass(const PassArgs& a, const WeightFormat& f, size_t smem, int grid, cudaStream_t s) {
  const int NT = pass_kernel_nt(a.T);
#define LS_PK(B, GG)                                                   \
  if (f.bits == B && f.group == GG) {                                  \
    if (NT == 16) return launch_pass_t<B, GG, 16>(a, smem, grid, s);  \
    if (NT == 32) return launch_pass_t<B, GG, 32>(a, smem, grid, s);  \
    return launch_pass_t<B, GG, 48>(a, smem, grid, s);                \
  }
  LS_PK(8, 32)
  LS_PK(8, 64)
  LS_PK(4, 16)
  LS_PK(4, 32)
#undef LS_PK
  LS_THROW(-1, "format not supported by the pass kernel");
}

// Dynamic shared memory a pass-kernel launch for T tokens may use: the device's per-block opt-in
// limit less the kernel's static shared memory (mbarriers, per-token sums, argmax parts).
size_t pass_kernel_smem_budget(const WeightFormat& f, int T) {
  const int NT = pass_kernel_nt(T);
  int dev = 0, optin = 0;
  LS_CUDA(cudaGetDevice(&dev));
  LS_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  cudaFuncAttributes fa{};
#define LS_PKA(B, GG)                                                                  \
  if (f.bits == B && f.group == GG) {                                                  \
    if (NT == 16) LS_CUDA(cudaFuncGetAttributes(&fa, pass_kernel<B, GG, 16>));         \
    else if (NT == 32) LS_CUDA(cudaFuncGetAttributes(&fa, pass_kernel<B, GG, 32>));    \
    else LS_CUDA(cudaFuncGetAttributes(&fa, pass_kernel<B, GG, 48>));                  \
  }
  LS_PKA(8, 32)
  LS_PKA(8, 64)
  LS_PKA(4, 16)
  LS_PKA(4, 32)
#undef LS_PKA
  return (size_t)optin > fa.sharedSizeBytes ? (size_t)optin - fa.sharedSizeBytes : 0;
}

// CTAs of the token tile of T that are resident per SM at once (the cooperative launch needs the
// whole grid resident), capped at max_per_sm and at one (each CTA allocates all tensor memory).
int pass_kernel_blocks_per_sm(const WeightFormat& f, int T, size_t smem, int max_per_sm) {
  const int NT = pass_kernel_nt(T);
  int per_sm = 0;
  auto q = [&](auto kern) {
    ensure_smem(kern, smem);
    LS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, PK_THREADS, smem));
  };
#define LS_PKO(B, GG)                                 \
  if (f.bits == B && f.group == GG) {                 \
    if (NT == 16) q(pass_kernel<B, GG, 16>);          \
    else if (NT == 32) q(pass_kernel<B, GG, 32>);     \
    else q(pass_kernel<B, GG, 48>);                   \
  }
  LS_PKO(8, 32)
  LS_PKO(8, 64)
  LS_PKO(4, 16)
  LS_PKO(4, 32)
#undef LS_PKO
  if (getenv("LS_PASS_VERBOSE")) fprintf(stderr, "pass kernel T=%d smem %zu: %d CTAs/SM resident\n", T, smem, per_sm);
  // the CTA takes the whole tensor memory of its SM
  return std::min(std::min(per_sm, max_per_sm), 1);
}

}  // namespace ls
