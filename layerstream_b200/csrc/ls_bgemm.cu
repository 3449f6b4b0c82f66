// Batched weight GEMM (tcgen05) of the verify / prefill pass: y[t][r] = sum_k W[r][k] * x[t][k]
// for the M token rows of a pass (batches of sequences x (k + 1) verify rows, prefill chunks)
// through int4 / int8 group-quantized planes.
//
// One CTA per (128-row weight tile, group of up to 256 tokens, K slice):
//   warp 8  producer: per stage of kstage 64-wide K blocks, one 3-D TMA box of the tile's packed
//           rows (4 x 32-row planes), one of their group scales, and one plain bulk copy of the token
//           group's activations (f16, already in the B-operand layout, one contiguous block) into a
//           ring of shared-memory stages (full / empty mbarriers)
//   warps 0-7 two warpgroups taking alternate K blocks, one weight row per thread: dequantise the
//           block ((q - 8) * s or q * s, f16; int8 as exact hi + lo parts) into one of the A buffers
//           in tensor memory (four for int4, two for int8's double width; tcgen05.st),
//           dequantising the next block while the store of this one completes
//   warps 9-10 one thread each issues tcgen05.mma for alternate stages (A = weights in tensor
//           memory, B = activations in shared memory, N = the token group, f32 accumulator of its own
//           in tensor memory), then commits the stage and the A buffer back to their producers; one
//           issuer's commits and waits overlap the other's MMAs, and the two accumulators are summed
//           in the epilogue (plan options: one issuer with four int8 buffers, or the two issuers
//           splitting the tokens of one accumulator; both measured slower on config 4's shapes)
//   epilogue warps 0-7 read D (tcgen05.ld; thread = weight row, warpgroup = half of the tokens) and
//           store, add the residual, add the bias, apply SwiGLU into the next GEMM's f16 operand,
//           or take per-token argmax parts.
// Each weight tile is dequantised once per pass for all tokens of the group. Small matrices split
// K over CTAs; the last CTA of a tile sums the slices in order. Every wait is bounded: on a timeout
// the kernel records the error and returns after releasing tensor memory.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "ls_device.cuh"
#include "ls_internal.h"

// Profiling (g.trace): clock() stamps of pipeline events of CTA (0, 0, 0) — 0 producer issued stage
// i, 1 issuer saw K block i's A buffer written, 2 its MMAs issued, 3 dequantiser warp 0 has block
// i's data, 4 its A store issued, 5 its store complete, 6 issuer waits for block i, 7 epilogue (0:
// start, 1: end) — and every CTA's start / end.
#define BG_STAMP(kind, i)                                                                    \
  do {                                                                                       \
    if (g.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)                  \
      g.trace[(kind) * 64 + min((int)(i), 63)] = (unsigned)clock();                        \
  } while (0)
#define BG_CTA_TIME(k)                                                                                    \
  do {                                                                                                    \
    if (g.trace)                                                                                          \
      g.trace[BG_TRACE_CTA + 2 * (blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)) + (k)] = \
          (unsigned)clock();                                                                              \
  } while (0)

namespace ls {

constexpr int BG_DEQ_WARPS = 4;   // warps of one dequantising warpgroup (and of the epilogue)
constexpr int BG_WG = 2;          // dequantising warpgroups: warpgroup g takes the K blocks i % 2 == g
constexpr int BG_PRODUCER = 8;    // warp index
constexpr int BG_ISSUER = 9;      // warps 9, 10: issuer g takes the stages s % 2 == g into accumulator g
constexpr int BG_NISS = 2;  // issuer warps (a plan uses 1 or 2 of them)
constexpr int BG_THREADS = 352;
constexpr int BG_MAX_STAGES = 8;
constexpr int BG_MAX_N = 192;  // two accumulators of N columns next to the A buffers (<= 512 columns)

namespace {

// The eight epilogue (dequantising) warps only (the producer and issuer warps may have left).
__device__ __forceinline__ void deq_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

}  // namespace

template <int BITS, int G>
struct BgShape {
  static constexpr int KB = tc_kb(BITS, G), NS = tc_ns(BITS, G), CPB = KB / (128 / BITS);
  // one A buffer: a K block's f16 pairs (two per column), for int8 its exact hi then lo parts
  static constexpr int HCOLS = KB / 2, ACOLS = HCOLS * tc_parts(BITS);
  // per K block: 128 rows of packed ints, their group scales, N tokens of f16 activations
  static constexpr uint32_t W_KB = 4u * CPB * 512u;
  static constexpr uint32_t S_KB = 4u * NS * 64u;
  __host__ __device__ static uint32_t x_kb(int N) { return (uint32_t)N * KB * 2u; }
};

template <int BITS, int G>
#ifndef BG_MIN_BLOCKS
#define BG_MIN_BLOCKS 2
#endif
__global__ void __launch_bounds__(BG_THREADS, BG_MIN_BLOCKS)
    bgemm_kernel(const __grid_constant__ BgemmLaunch g, const __grid_constant__ BgemmPlan p, const __grid_constant__ QMaps maps) {
  using SH = BgShape<BITS, G>;
  constexpr int KB = SH::KB, NS = SH::NS, CPB = SH::CPB, ACOLS = SH::ACOLS, HCOLS = SH::HCOLS;
  const int ABUF = p.abuf, NISS = p.niss;  // A buffers (2 or 4), issuers (1 or 2)
  const bool NSPLIT = p.n0 > 0;  // issuers split the tokens (each takes every K block) instead of the K blocks
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[BG_MAX_STAGES], empty[BG_MAX_STAGES], bar_a[4], bar_af[4], bar_d, bar_fin[BG_NISS];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_epi_fail;  // written only by the epilogue warps before they agree on it
  __shared__ float s_bv[BG_DEQ_WARPS][BG_MAX_N];
  __shared__ uint32_t s_bi[BG_DEQ_WARPS][BG_MAX_N];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);

  const int N = p.N, S = p.stages, KST = p.kstage;
  // stage: [W: 4 planes x CPB*KST chunks x 512 B][S: 4 x NS*KST groups x 64 B][X: KST x KB/8 chunks x N x 16 B]
  const uint32_t W_ST = SH::W_KB * KST, S_ST = SH::S_KB * KST, X_KB = SH::x_kb(N);
  const uint32_t STAGE = W_ST + S_ST + X_KB * KST;
  const int t128 = blockIdx.x, grp = blockIdx.y, ks = blockIdx.z;
  const int tiles32 = g.w.rows_pad / 32;
  const int m0 = grp * N, Mloc = min(N, g.M - m0);
  const int K = g.w.cols, nblk = g.w.chunks() / CPB;
  const int kb0 = (int)((long long)ks * nblk / p.ks), kb1 = (int)((long long)(ks + 1) * nblk / p.ks);
  const int nkb = kb1 - kb0, nst = (nkb + KST - 1) / KST;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) BG_CTA_TIME(0);
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], NSPLIT ? 2 : 1);
    }
    for (int b = 0; b < ABUF; b++) {
      tc::mbar_init(&bar_a[b], NSPLIT ? 2 : 1);
      tc::mbar_init(&bar_af[b], BG_DEQ_WARPS);
    }
    tc::mbar_init(&bar_d, NISS);
    for (int q = 0; q < BG_NISS; q++) tc::mbar_init(&bar_fin[q], 1);
    s_abort = 0;
    s_epi_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::su32(&s_tmem)), "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t d_col = tmem + ABUF * ACOLS;
  bool failed = false;
  // everything but the producer's early weight loads waits for the previous kernel (no-op without
  // the launch attribute)
  if (warp != BG_PRODUCER) pdl_wait();

  if (warp == BG_PRODUCER) {
    if (lane == 0) {
      int issued = 0;
      const uint16_t* xg = g.x + bt_off(m0, 0, K, N);  // this token group's block
      // the weights do not depend on the previous kernel: the first ring of stages starts loading
      // before griddepcontrol.wait (programmatic dependent launch), the activations after it
      auto load_w = [&](int i) {
        const int s = i % S, kb = kb0 + i * KST;
        const uint32_t st = tc::su32(smem + (size_t)s * STAGE);
        tc::mbar_expect_tx_only(&full[s], W_ST + S_ST);
        tc::tma_load_3d(st, &maps.data, 0, kb * CPB, t128 * 4, &full[s]);
        tc::tma_load_3d(st + W_ST, &maps.scales, 0, kb * NS, t128 * 4, &full[s]);
      };
      const int npre = min(S, nst);
      for (int i = 0; i < npre; i++) load_w(i);
      pdl_wait();
      for (int i = 0; i < nst; i++) {
        const int s = i % S, kb = kb0 + i * KST, nv = min(KST, kb1 - kb);
        if (i >= S) {
          if (!tc::mbar_wait_fast(&empty[s], ((i / S) & 1) ^ 1, &s_abort)) {
            failed = true;
            break;
          }
          load_w(i);
        }
        const uint32_t st = tc::su32(smem + (size_t)s * STAGE);
        tc::mbar_expect_tx(&full[s], X_KB * nv);  // the stage's arrival, with its activation bytes
        tc::bulk_load(st + W_ST + S_ST, xg + (size_t)kb * (KB / 8) * N * 8, X_KB * nv, &full[s]);
        BG_STAMP(0, i);
        issued = i + 1;
      }
      // no copy may still be landing when the CTA leaves (error path): wait, bounded, for every
      // stage issued that the consumers may not have waited for
      volatile int no_abort = 0;
      for (int i = max(0, issued - S); i < issued; i++) tc::mbar_wait(&full[i % S], (i / S) & 1, &no_abort);
    }
  } else if (warp >= BG_ISSUER + NISS && warp < BG_ISSUER + BG_NISS) {
    // an issuer warp the plan does not use
  } else if (warp >= BG_ISSUER && warp < BG_ISSUER + NISS) {
    if (lane == 0) {
      const int ig = warp - BG_ISSUER;
      // token split: issuer ig runs tokens [ig n0, ...) of every K block into its columns of the one
      // accumulator; K split: alternate stages into an accumulator of its own
      const int ncols = NSPLIT ? (ig == 0 ? p.n0 : N - p.n0) : N;
      const uint32_t idesc = tc::idesc_f16(ncols);
      const uint32_t dacc = d_col + (NSPLIT ? ig * p.n0 : ig * N);
      const uint32_t xoff = NSPLIT ? (uint32_t)(ig * p.n0) * 16u : 0u;  // the first of its tokens' 16-byte rows
      bool first = true;
      for (int st_i = NSPLIT ? 0 : ig; st_i < nst && !failed; st_i += NSPLIT ? 1 : NISS) {
        const int s = st_i % S;
        if (!tc::mbar_wait_fast(&full[s], (st_i / S) & 1, &s_abort)) {
          failed = true;
          break;
        }
        const int i_end = min(nkb, (st_i + 1) * KST);
        for (int i = st_i * KST; i < i_end; i++) {
          const int j = i - st_i * KST, b = i % ABUF;
          BG_STAMP(6, i);
          if (!tc::mbar_wait_fast(&bar_af[b], (i / ABUF) & 1, &s_abort)) {
            failed = true;
            break;
          }
          BG_STAMP(1, i);
          tc::fence_after();
          const uint32_t xa = tc::su32(smem + (size_t)s * STAGE + W_ST + S_ST) + (uint32_t)j * X_KB;
#pragma unroll
          for (int jj = 0; jj < KB / 16; jj++) {
            const uint64_t bd = tc::sdesc(xa + xoff + jj * 2u * N * 16u, (uint32_t)N * 16u, 128u);
            tc::mma_f16_ts(dacc, tmem + b * ACOLS + jj * 8, bd, idesc, (!first || jj > 0) ? 1u : 0u);
            if constexpr (ACOLS > HCOLS) tc::mma_f16_ts(dacc, tmem + b * ACOLS + HCOLS + jj * 8, bd, idesc, 1u);
          }
          first = false;
          tc::commit(&bar_a[b]);  // the A buffer is free once these MMAs have read it
          BG_STAMP(2, i);
        }
        if (!failed) tc::commit(&empty[s]);  // and so is the stage
      }
      if (!failed) tc::commit(&bar_d);
      // every MMA this thread issued has completed before tensor memory is released
      volatile int no_abort = 0;
      tc::commit(&bar_fin[ig]);
      tc::mbar_wait(&bar_fin[ig], 0, &no_abort);
    }
  } else {
    // ---- dequantising warpgroups: one weight row per thread, alternate K blocks ----
    const int wq = warp & 3, wg = warp >> 2;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    // block i's packed ints of this row, dequantised into a (waits for its stage on the first
    // block this warpgroup takes from it)
    auto load_block = [&](int i, uint32_t* a) -> bool {
      const int st_i = i / KST, j = i - st_i * KST, s = st_i % S;
      if (j < 2 && !tc::mbar_wait_fast(&full[s], (st_i / S) & 1, &s_abort)) return false;
      const uint8_t* st = smem + (size_t)s * STAGE;
      uint4 wv[CPB];
#pragma unroll
      for (int q = 0; q < CPB; q++)
        wv[q] = *reinterpret_cast<const uint4*>(st + ((wq * KST + j) * CPB + q) * 512 + lane * 16);
      uint32_t scur[NS];
#pragma unroll
      for (int q = 0; q < NS; q++)
        scur[q] = tc::h2_splat(bf16f(*reinterpret_cast<const uint16_t*>(st + W_ST + ((wq * KST + j) * NS + q) * 64 + lane * 2)));
      if constexpr (ACOLS > HCOLS) tc_dequant_block_i8<G>(wv, scur, a, a + HCOLS);
      else tc_dequant_block<BITS, G>(wv, scur, a);
      if (wq == 0 && lane == 0) BG_STAMP(3, i);
      return true;
    };
    uint32_t acur[ACOLS], anext[ACOLS];
    int i = wg;
    bool have = i < nkb;
    if (have && !load_block(i, acur)) failed = true;
    while (have && !__any_sync(0xffffffffu, failed)) {
      const int b = i % ABUF;
      if (i >= ABUF && !tc::mbar_wait_fast(&bar_a[b], ((i / ABUF) & 1) ^ 1, &s_abort)) failed = true;
      if (__any_sync(0xffffffffu, failed)) break;
      tc::fence_after();
#pragma unroll
      for (int q = 0; q < ACOLS / 16; q++) tc::st16(tmem + lane_base + b * ACOLS + q * 16, acur + q * 16);
      if (wq == 0 && lane == 0) BG_STAMP(4, i);
      const int inext = i + BG_WG;
      have = inext < nkb;
      if (have && !load_block(inext, anext)) failed = true;  // overlaps the tensor-memory store
      tc::wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bar_af[b]);
      if (wq == 0 && lane == 0) BG_STAMP(5, i);
      i = inext;
#pragma unroll
      for (int q = 0; q < ACOLS; q++) acur[q] = anext[q];
    }
    failed = __any_sync(0xffffffffu, failed);
    {
    // ---- epilogue: both warpgroups, warpgroup wg taking tokens [n_lo, n_hi) of every row (the
    // eight warps agree on failure before their named barriers) ----
    const int nh = (N / 16 + 1) / 2 * 16;
    const int n_lo = wg ? nh : 0, n_hi = wg ? N : nh;
    if (!failed && !tc::mbar_wait_fast(&bar_d, 0, &s_abort)) failed = true;
    failed = __any_sync(0xffffffffu, failed);
    if (failed && lane == 0) s_epi_fail = 1;
    deq_sync();
    if (s_epi_fail == 0) {
      tc::fence_after();
      if (warp == 0 && lane == 0) BG_STAMP(7, 0);
      // columns [16 n16, 16 n16 + 16) of this thread's row: the issuers' accumulators summed in order
      auto acc_load = [&](int n16, float* v) {
        uint32_t u[16];
        if (!NSPLIT && NISS > 1 && nst > 1) {  // both accumulators' loads in flight before one wait
          uint32_t* u2 = reinterpret_cast<uint32_t*>(v);
          tc::ld16(d_col + lane_base + n16 * 16, u);
          tc::ld16(d_col + N + lane_base + n16 * 16, u2);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 16; e++) v[e] = __uint_as_float(u[e]) + __uint_as_float(u2[e]);
          return;
        }
        tc::ld16(d_col + lane_base + n16 * 16, u);
        tc::wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e++) v[e] = __uint_as_float(u[e]);
      };
      const int t32 = t128 * 4 + wq;
      const bool row_valid = t32 < tiles32;
      const int r = t32 * 32 + lane;
      if (p.ks > 1) {
        // this slice's accumulators; the last slice's CTA sums them all (after the teardown)
        float* part = g.partial + (((size_t)t128 * p.ngroups + grp) * p.ks + ks) * (size_t)N * 128;
        for (int n16 = n_lo / 16; n16 < n_hi / 16; n16++) {
          float v[16];
          acc_load(n16, v);
#pragma unroll
          for (int e = 0; e < 16; e++) part[(size_t)(n16 * 16 + e) * 128 + wq * 32 + lane] = v[e];
        }
      }
      if (p.ks == 1) {
        for (int n16 = n_lo / 16; n16 < n_hi / 16; n16++) {
          if (n16 * 16 >= Mloc) break;
          float v16[16];
          acc_load(n16, v16);
#pragma unroll
          for (int e = 0; e < 16; e++) {
            const int n = n16 * 16 + e;  // warp-uniform
            if (n >= Mloc) break;
            const float v = v16[e];
            const int t = m0 + n;
            if (g.epi == EPI_ARGMAX) {
              float bv = (row_valid && r < g.n_valid_rows) ? v : -CUDART_INF_F;
              uint32_t bi = (uint32_t)(r + g.row_offset);
              warp_argmax(bv, bi);
              if (lane == 0) {
                s_bv[wq][n] = bv;
                s_bi[wq][n] = bi;
              }
            } else if (g.epi == EPI_SWIGLU_H) {
              const float u = __shfl_down_sync(0xffffffffu, v, 16);
              if (row_valid && lane < 16) {
                const float h = v / (1.0f + expf(-v)) * u;
                g.yh[bt_off(t, t32 * 16 + lane, g.w.rows / 2, N)] = __half_as_ushort(__float2half_rn(h));
              }
            } else if (row_valid && r < g.w.rows) {
              float* dst = g.y + (size_t)t * g.y_stride + r;
              if (g.epi == EPI_RESID) *dst += v;
              else if (g.epi == EPI_BIAS_STORE) *dst = v + bf16f(g.bias[r]);
              else *dst = v;
            }
          }
        }
        if (g.epi == EPI_ARGMAX) {
          deq_sync();
          for (int n = threadIdx.x; n < Mloc; n += 2 * BG_DEQ_WARPS * 32) {
            float bv = s_bv[0][n];
            uint32_t bi = s_bi[0][n];
            for (int w = 1; w < BG_DEQ_WARPS; w++)
              if (arg_better(s_bv[w][n], s_bi[w][n], bv, bi)) {
                bv = s_bv[w][n];
                bi = s_bi[w][n];
              }
            g.arg_parts[(size_t)(t128 + g.part_tile_offset) * g.M + m0 + n] = ArgPart{bv, bi};
          }
        }
      }
    } else {
      failed = true;
    }
    }  // epilogue
  }

  // ---- release tensor memory (also on the error path) ----
  if (threadIdx.x == 0) BG_STAMP(7, 1);
  tc::fence_before();
  failed = __syncthreads_or(failed || s_abort);
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
  }
  if (failed && threadIdx.x == 0 && g.err) atomicExch(g.err, 1);
  if (!failed && p.ks > 1 && last_cta(g.tickets + (size_t)t128 * p.ngroups + grp, (unsigned)p.ks)) {
    // ---- split-K: the slices summed in order by the whole CTA, 4 rows x 1 token per item ----
    const float* part = g.partial + ((size_t)t128 * p.ngroups + grp) * p.ks * (size_t)N * 128;
    auto slice_sum = [&](int n, int rl) -> float4 {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k0 = 0; k0 < p.ks; k0 += 4) {
        float4 t[4];
#pragma unroll
        for (int q = 0; q < 4; q++)
          t[q] = (k0 + q < p.ks) ? __ldcg(reinterpret_cast<const float4*>(part + ((size_t)(k0 + q) * N + n) * 128 + rl))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          acc.x += t[q].x;
          acc.y += t[q].y;
          acc.z += t[q].z;
          acc.w += t[q].w;
        }
      }
      return acc;
    };
    if (g.epi == EPI_SWIGLU_H) {
      // 16 gate rows then their 16 up rows in every 32-row group
      for (int item = threadIdx.x; item < Mloc * 16; item += BG_THREADS) {
        const int n = item >> 4, q = item & 15, t32 = t128 * 4 + (q >> 2), rl = (q >> 2) * 32 + (q & 3) * 4;
        if (t32 >= tiles32) continue;
        const float4 gt = slice_sum(n, rl), up = slice_sum(n, rl + 16);
        const float h0 = gt.x / (1.0f + expf(-gt.x)) * up.x, h1 = gt.y / (1.0f + expf(-gt.y)) * up.y;
        const float h2 = gt.z / (1.0f + expf(-gt.z)) * up.z, h3 = gt.w / (1.0f + expf(-gt.w)) * up.w;
        const __half2 a = __floats2half2_rn(h0, h1), b = __floats2half2_rn(h2, h3);
        *reinterpret_cast<uint2*>(g.yh + bt_off(m0 + n, t32 * 16 + (q & 3) * 4, g.w.rows / 2, N)) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
      }
    } else {
      for (int item = threadIdx.x; item < Mloc * 32; item += BG_THREADS) {
        const int n = item >> 5, rl = (item & 31) * 4, r0 = t128 * 128 + rl;
        const float4 v4 = slice_sum(n, rl);
        const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int r = r0 + e;
          if (r >= g.w.rows) break;
          float* dst = g.y + (size_t)(m0 + n) * g.y_stride + r;
          if (g.epi == EPI_RESID) *dst += vv[e];
          else if (g.epi == EPI_BIAS_STORE) *dst = vv[e] + bf16f(g.bias[r]);
          else *dst = vv[e];
        }
      }
    }
  }
  if (threadIdx.x == 0) BG_CTA_TIME(1);
}

// ---- activations into the bt layout ----

void bgemm_groups(int M, int* N, int* ngroups) {
  const int ng = std::max(1, (M + BG_MAX_N - 1) / BG_MAX_N);
  *ngroups = ng;
  *N = std::max(16, ((M + ng - 1) / ng + 15) / 16 * 16);
}

size_t bt_elems(int M, int K) {
  int N = 16, ng = 1;
  bgemm_groups(M, &N, &ng);
  return (size_t)ng * N * K;
}

// One CTA per row of the padded token groups (rows M .. ng * N are zero).
__global__ void bt_prep_kernel(const float* __restrict__ x, int x_stride, int M, int K, int N, const uint16_t* __restrict__ nb,
                               const float* __restrict__ nf, float eps, uint16_t* __restrict__ out) {
  const int t = blockIdx.x;
  __shared__ float s_red[4];
  __shared__ float s_inv;
  pdl_trigger();
  pdl_wait();  // x is the previous kernel's output
  const float* xr = x + (size_t)t * x_stride;
  const bool live = t < M;
  const bool norm = nb != nullptr || nf != nullptr;
  if (live && norm) {
    float ss = 0.f;
    for (int c4 = threadIdx.x; c4 < K / 4; c4 += blockDim.x) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(xr) + c4);
      ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); w++) tot += s_red[w];
      s_inv = 1.0f / sqrtf(tot / (float)K + eps);
    }
    __syncthreads();
  }
  const float inv = (live && norm) ? s_inv : 1.f;
  for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
    uint4 o = make_uint4(0, 0, 0, 0);
    if (live) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(xr + c * 8));
      const float4 b = __ldg(reinterpret_cast<const float4*>(xr + c * 8) + 1);
      float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int k = c * 8 + e;
        if (norm) v[e] = v[e] * inv * (nb ? bf16f(nb[k]) : nf[k]);
      }
      uint32_t w4[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const __half2 h = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
        w4[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      o = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
    *reinterpret_cast<uint4*>(out + bt_off(t, c * 8, K, N)) = o;
  }
}

void launch_bt_prep(const float* x, int x_stride, int M, int K, const uint16_t* norm_bf16, const float* norm_f32, float eps,
                    uint16_t* out, cudaStream_t s) {
  if (M <= 0) return;
  if (K % 8) LS_THROW(-1, "the bt layout needs K to be a multiple of 8");
  int N = 16, ng = 1;
  bgemm_groups(M, &N, &ng);
  launch_pdl(bt_prep_kernel, dim3(ng * N), dim3(128), 0, s, x, x_stride, M, K, N, norm_bf16, norm_f32, eps, out);
}

// ---- host side ----

bool bgemm_supported(const QMat& w) {
  // (an int8 K block is 64 columns: its scales are whole groups only for groups of at most 64)
  const bool fmt = (w.bits == 8 && (w.group == 16 || w.group == 32 || w.group == 64)) ||
                   (w.bits == 4 && (w.group == 16 || w.group == 32 || w.group == 64 || w.group == 128));
  return fmt && (w.cols % tc_kb(w.bits, w.group)) == 0 && w.rows_pad % 32 == 0;
}

BgemmPlan bgemm_plan(const QMat& w, int M, int num_sms, bool argmax) {
  BgemmPlan p;
  if (M <= 0) return p;
  bgemm_groups(M, &p.N, &p.ngroups);
  const int KB = tc_kb(w.bits, w.group), NS = tc_ns(w.bits, w.group), CPB = KB / (128 / w.bits);
  const int tiles128 = (w.rows_pad / 32 + 3) / 4, nblk = w.cols / KB;
  const int base = tiles128 * p.ngroups;
  p.ks = 1;
  if (!argmax && base < num_sms) p.ks = std::min({(num_sms + base - 1) / base, std::max(1, nblk / 4), 16});
  // Tensor memory: A buffers of aw columns (4 for int4, 2 for int8's hi + lo parts) and one
  // N-column accumulator per issuer. Two issuers measured faster than one with 4 int8 buffers
  // (config 4's gate/up, N = 160: 45 vs 50 us); LS_BGEMM_ISSUERS=1 selects one issuer (4 buffers).
  const int aw = KB / 2 * tc_parts(w.bits);
  static const int issuers = [] {
    const char* e = getenv("LS_BGEMM_ISSUERS");
    return (e && std::string(e) == "1") ? 1 : 2;
  }();
  p.niss = issuers;
  p.abuf = (issuers == 1 || aw <= 32) ? 4 : 2;
  p.tmem_cols = p.abuf * aw + p.niss * p.N <= 256 ? 256 : 512;
  // Opt-in (LS_BGEMM_NSPLIT = the smallest N that splits; default 0 = never): the two issuers split
  // the tokens (multiples of 16) of one N-column accumulator, each issuing every K block's MMAs,
  // which leaves tensor memory for four A buffers. Measured slower than the K split on config 4's
  // gate/up (N = 160: 45.9 against 40.4 us): both issuers then pay their per-block commit and wait
  // overhead at the same time, while alternating K blocks overlaps one's overhead with the other's
  // MMAs.
  static const int nsplit_min = [] {
    const char* e = getenv("LS_BGEMM_NSPLIT");
    return e ? atoi(e) : 0;
  }();
  if (issuers == 2 && nsplit_min > 0 && p.N >= std::max(32, nsplit_min)) {
    const int n0 = (p.N / 2 + 15) / 16 * 16;
    if (p.N - n0 >= 16 && 4 * aw + p.N <= 512) {
      p.n0 = n0;
      p.abuf = 4;
      p.tmem_cols = 4 * aw + p.N <= 256 ? 256 : 512;
    }
  }
  // stages of kstage K blocks (~24 KB each, within the slice); two CTAs per SM when tensor memory
  // allows it: keep the ring near 96 KB, else up to ~200 KB
  const uint32_t per_kb = 4u * CPB * 512u + 4u * NS * 64u + (uint32_t)p.N * KB * 2u;
  const int min_slice = nblk / p.ks;
  p.kstage = (int)std::max<uint32_t>(1, std::min<uint32_t>({8u, 24u * 1024 / per_kb, (uint32_t)std::max(1, min_slice)}));
  // K block i uses A buffer i % ABUF, and two issuers take alternate stages of kstage blocks:
  // blocks i and i + ABUF (consecutive uses of a buffer) must belong to the same issuer, which
  // waits for the buffer's mbarrier phases in order (a parity wait two phases ahead would read
  // the stale phase as complete). That holds when kstage divides ABUF / 2 (one issuer: always).
  if (p.niss == 2 && p.n0 == 0)
    while ((p.abuf / 2) % p.kstage) p.kstage--;
  const uint32_t st = per_kb * p.kstage;
  const uint32_t budget = p.tmem_cols == 256 ? 96u * 1024 : 200u * 1024;
  p.stages = (int)std::max<uint32_t>(2, std::min<uint32_t>(BG_MAX_STAGES, budget / st));
  p.smem = (size_t)p.stages * st + 1024;
  p.partial_floats = p.ks > 1 ? (size_t)tiles128 * p.ngroups * p.ks * p.N * 128 : 0;
  p.tickets = (size_t)tiles128 * p.ngroups;
  return p;
}

// Tensor maps of a matrix's planes for a stage size, encoded once per (planes, shape, stage) on
// the host (encoding is a driver call: far slower than a launch).
static const QMaps& bg_maps(const QMat& w, int kstage, int cpb, int ns) {
  struct Key {
    const void *d, *s;
    int rows_pad, cols, bits, group, kstage;
    bool operator<(const Key& o) const {
      return std::tie(d, s, rows_pad, cols, bits, group, kstage) < std::tie(o.d, o.s, o.rows_pad, o.cols, o.bits, o.group, o.kstage);
    }
  };
  static std::mutex mu;
  static std::map<Key, QMaps> cache;
  const Key k{w.data, w.scales, w.rows_pad, w.cols, w.bits, w.group, kstage};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(k);
  if (it == cache.end()) {
    if (cache.size() > 4096) cache.clear();  // planes of released models
    QMaps m;
    encode_qmat_maps(w, cpb * kstage, ns * kstage, 4, &m);
    it = cache.emplace(k, m).first;
  }
  return it->second;
}

template <int BITS, int G>
static void launch_bg_t(const BgemmLaunch& g, const BgemmPlan& p, cudaStream_t s) {
  using SH = BgShape<BITS, G>;
  const QMaps maps = bg_maps(g.w, p.kstage, SH::CPB, SH::NS);
  ensure_smem(bgemm_kernel<BITS, G>, p.smem);
  const dim3 grid((g.w.rows_pad / 32 + 3) / 4, p.ngroups, p.ks);
  launch_pdl(bgemm_kernel<BITS, G>, grid, dim3(BG_THREADS), p.smem, s, g, p, maps);
}

void launch_bgemm(const BgemmLaunch& g, const BgemmPlan& p, cudaStream_t s) {
  if (g.M <= 0) return;
  if (!bgemm_supported(g.w)) LS_THROW(-1, "format not supported by the batched GEMM");
  if (p.N % 16 || p.N > BG_MAX_N || p.ngroups * p.N < g.M) LS_THROW(-1, "batched GEMM plan does not cover the tokens");
  if (p.stages < 2 || p.stages > BG_MAX_STAGES || p.kstage < 1) LS_THROW(-1, "batched GEMM plan: bad stage count");
  if ((p.abuf != 2 && p.abuf != 4) || (p.niss != 1 && p.niss != 2) ||
      p.abuf * (tc_kb(g.w.bits, g.w.group) / 2 * tc_parts(g.w.bits)) + (p.n0 ? 1 : p.niss) * p.N > p.tmem_cols ||
      (p.niss == 2 && p.n0 == 0 && (p.abuf / 2) % p.kstage) ||
      (p.n0 && (p.niss != 2 || p.n0 % 16 || (p.N - p.n0) < 16 || (p.N - p.n0) % 16)))
    LS_THROW(-1, "batched GEMM plan: bad tensor-memory split");
  {
    int N = 0, ng = 0;
    bgemm_groups(g.M, &N, &ng);
    if (N != p.N || ng != p.ngroups) LS_THROW(-1, "batched GEMM plan does not match the activation layout");
  }
  if (p.ks > 1 && (!g.partial || !g.tickets)) LS_THROW(-1, "a split batched GEMM needs partial-sum scratch");
  if (g.epi == EPI_ARGMAX && p.ks != 1) LS_THROW(-1, "the argmax epilogue needs whole dot products (no K split)");
  if (g.epi == EPI_SWIGLU_H && (!g.yh || (g.w.rows / 2) % 8)) LS_THROW(-1, "SwiGLU output needs an f16 buffer");
  if (g.w.bits == 8) {
    switch (g.w.group) {
      case 16: return launch_bg_t<8, 16>(g, p, s);
      case 32: return launch_bg_t<8, 32>(g, p, s);
      case 64: return launch_bg_t<8, 64>(g, p, s);
      default: return launch_bg_t<8, 128>(g, p, s);
    }
  }
  switch (g.w.group) {
    case 16: return launch_bg_t<4, 16>(g, p, s);
    case 32: return launch_bg_t<4, 32>(g, p, s);
    case 64: return launch_bg_t<4, 64>(g, p, s);
    default: return launch_bg_t<4, 128>(g, p, s);
  }
}

}  // namespace ls
