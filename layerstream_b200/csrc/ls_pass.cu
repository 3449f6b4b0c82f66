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
// Every wait is bounded (grid barrier spins, mbarrier polls); on a timeout the CTA records an
// error in the control block, the other CTAs see it at their next wait, tensor memory is released
// and the kernel returns.
#include <algorithm>

#include "ls_device.cuh"
#include "ls_internal.h"

namespace ls {

constexpr int PK_THREADS = 128;
constexpr int PK_NW = PK_THREADS / 32;
constexpr int PK_STAGES = 6;
constexpr int PK_ATT_TILE = 64;

__device__ __forceinline__ long long to_fix(float v) {
  v = fminf(fmaxf(v, -1.0e9f), 1.0e9f);
  return __float2ll_rn(v * 4294967296.0f);
}
__device__ __forceinline__ float from_fix(long long f) { return (float)((double)f * 2.3283064365386962890625e-10); }
__device__ __forceinline__ void fix_add(long long* p, float v) {
  atomicAdd(reinterpret_cast<unsigned long long*>(p), (unsigned long long)to_fix(v));
}
__device__ __forceinline__ long long ldcg_ll(const long long* p) { return __ldcg(p); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier over a counter zeroed before the launch. Bounded: returns false when any CTA
// has recorded an error (including this one timing out).
__device__ bool grid_barrier(unsigned* bar, unsigned target, int* err) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
    int ok = 1;
    for (uint32_t i = 0;; i++) {
      if (ld_acquire(bar) >= target) break;
      if (*(volatile int*)err) {
        ok = 0;
        break;
      }
      if (i > (1u << 21)) {
        atomicExch(err, 3);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// ---------------------------------------------------------------------------------------------
// The tensor-core GEMV of one 128-row tile over K blocks [kb0, kb1), as in gemv_tc_kernel, with
// state kept across items: each thread owns one weight row and leaves its NT accumulators in tot.
// ---------------------------------------------------------------------------------------------
template <int BITS, int G, int NT>
struct TcGemv {
  static constexpr int KB = tc_kb(BITS, G), NS = tc_ns(BITS, G), WPC = 128 / BITS, CPB = KB / WPC, ACOLS = KB / 2;
  static constexpr uint32_t kStage = PK_THREADS * CPB * 16;
  uint32_t tmem, ring_addr;
  uint8_t* ring;
  uint64_t *bar_a, *bar_full, *bar_d;
  int* abort;
  uint32_t uses0, uses1, dphase;

  __device__ void prologue(const QMat& w, int t128, int kb0, int kb1) const {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t32 = t128 * 4 + warp;
    const bool valid = t32 < w.rows_pad / 32;
    const uint8_t* db = w.data + ((size_t)(valid ? t32 : 0) * w.chunks()) * 512 + lane * 16;
#pragma unroll
    for (int s = 0; s < PK_STAGES - 1; s++) {
      const int kb = kb0 + s;
      if (kb < kb1 && valid) {
#pragma unroll
        for (int q = 0; q < CPB; q++) tc::cp_async16(ring_addr + s * kStage + q * 16, db + (size_t)(kb * CPB + q) * 512);
      }
      tc::cp_commit();
    }
  }

  // Runs the K loop (prologue already issued) and reads the accumulators. false on a timeout.
  __device__ bool run(const QMat& w, int t128, int kb0, int kb1, uint32_t xb_addr, uint32_t sbo, float (&tot)[NT]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles32 = w.rows_pad / 32, nch = w.chunks(), ngr = w.groups();
    const int t32 = t128 * 4 + warp;
    const bool row_valid = t32 < tiles32;
    const uint8_t* db = w.data + ((size_t)(row_valid ? t32 : 0) * nch) * 512 + lane * 16;
    const uint16_t* sb = w.scales + (size_t)(row_valid ? t32 : 0) * ngr * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t d_col = tmem + 2 * ACOLS;
    const uint32_t idesc = tc::idesc_f16(NT);
    const uint32_t sub8 = BITS == 8 ? 0x64806480u : 0x64086408u;
    auto load_scales = [&](int kb, uint16_t (&sc)[NS]) {
#pragma unroll
      for (int s = 0; s < NS; s++) sc[s] = (row_valid && kb < kb1) ? sb[(size_t)((kb * KB) / G + s) * 32] : (uint16_t)0;
    };
    uint16_t sr0[NS], sr1[NS], sr2[NS];
    load_scales(kb0, sr0);
    load_scales(kb0 + 1, sr1);
    bool failed = false;
    for (int kb = kb0; kb < kb1; kb++) {
      const int it = kb - kb0;
      {
        const int kn = kb + PK_STAGES - 1, sn = (it + PK_STAGES - 1) % PK_STAGES;
        if (kn < kb1 && row_valid) {
#pragma unroll
          for (int q = 0; q < CPB; q++) tc::cp_async16(ring_addr + sn * kStage + q * 16, db + (size_t)(kn * CPB + q) * 512);
        }
        tc::cp_commit();
      }
      load_scales(kb + 2, sr2);
      uint32_t sc[NS];
#pragma unroll
      for (int q = 0; q < NS; q++) sc[q] = tc::h2_splat(bf16f(sr0[q]));
      tc::cp_wait<PK_STAGES - 1>();
      uint4 wv[CPB];
      const uint8_t* rs = ring + (size_t)(it % PK_STAGES) * kStage + (size_t)threadIdx.x * CPB * 16;
#pragma unroll
      for (int q = 0; q < CPB; q++) wv[q] = row_valid ? *reinterpret_cast<const uint4*>(rs + q * 16) : make_uint4(0, 0, 0, 0);
      uint32_t a[ACOLS];
#pragma unroll
      for (int q = 0; q < CPB; q++) {
        const uint32_t wd[4] = {wv[q].x, wv[q].y, wv[q].z, wv[q].w};
        if constexpr (BITS == 8) {
          const uint32_t s2 = sc[(NS > 1) ? (q * 16) / G : 0];
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const uint32_t p0 = (__byte_perm(wd[k], 0u, 0x4140u) ^ 0x00800080u) | 0x64006400u;
            const uint32_t p1 = (__byte_perm(wd[k], 0u, 0x4342u) ^ 0x00800080u) | 0x64006400u;
            a[q * 8 + 2 * k] = tc::h2_sub_mul(p0, sub8, s2);
            a[q * 8 + 2 * k + 1] = tc::h2_sub_mul(p1, sub8, s2);
          }
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
#pragma unroll
      for (int q = 0; q < NS; q++) {
        sr0[q] = sr1[q];
        sr1[q] = sr2[q];
      }
      const int b = it & 1;
      const uint32_t ub = b ? uses1 : uses0;
      if (ub > 0 && !tc::mbar_wait(&bar_a[b], (ub - 1) & 1, abort)) failed = true;
      if (__any_sync(0xffffffffu, failed)) {
        failed = true;
        break;
      }
      tc::fence_after();
      __syncwarp();
#pragma unroll
      for (int q = 0; q < ACOLS / 16; q++) tc::st16(tmem + lane_base + b * ACOLS + q * 16, a + q * 16);
      tc::wait_st();
      tc::fence_before();
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::su32(&bar_full[b])) : "memory");
      if (threadIdx.x == 0) {
        if (!tc::mbar_wait(&bar_full[b], ub & 1, abort)) {
          failed = true;
        } else {
          tc::fence_after();
#pragma unroll
          for (int j = 0; j < KB / 16; j++) {
            const uint32_t kpos = (uint32_t)(it * KB + j * 16);
            const uint64_t bd = tc::sdesc(xb_addr + (kpos / 8) * 128u, 128u, sbo);
            tc::mma_f16_ts(d_col, tmem + b * ACOLS + j * 8, bd, idesc, (it > 0 || j > 0) ? 1u : 0u);
          }
          tc::commit(&bar_a[b]);
        }
      }
      __syncwarp();
      if (b) uses1++;
      else uses0++;
      if (__any_sync(0xffffffffu, failed)) {
        failed = true;
        break;
      }
    }
    tc::cp_wait<0>();
    if (failed) return false;
    if (threadIdx.x == 0) tc::commit(bar_d);
    if (!tc::mbar_wait(bar_d, dphase & 1, abort)) failed = true;
    if (__any_sync(0xffffffffu, failed)) return false;
    dphase++;
    tc::fence_after();
#pragma unroll
    for (int q = 0; q < NT / 16; q++) {
      uint32_t v[16];
      tc::ld16(d_col + lane_base + q * 16, v);
      tc::wait_ld();
#pragma unroll
      for (int e = 0; e < 16; e++) tot[q * 16 + e] = __uint_as_float(v[e]);
    }
    tc::fence_before();
    return true;
  }
};

// Item split of a GEMV phase: item i -> (K slice, 128-row tile), slices outermost.
struct Split {
  int tiles128, ks, nblk;
  __device__ int items() const { return tiles128 * ks; }
  __device__ void item(int i, int* t128, int* kb0, int* kb1) const {
    const int k = i / tiles128;
    *t128 = i - k * tiles128;
    *kb0 = (int)((long long)k * nblk / ks);
    *kb1 = (int)((long long)(k + 1) * nblk / ks);
  }
};

template <int BITS, int G>
__device__ __forceinline__ Split make_split(const QMat& w, int ks) {
  Split s;
  s.tiles128 = (w.rows_pad / 32 + 3) / 4;
  s.ks = ks;
  s.nblk = w.cols / tc_kb(BITS, G);
  return s;
}

// Writes activations (already f32) for tokens t < T, K columns [col0, col0 + ncol) into the
// canonical K-major f16 layout; value(t, col) is a callable.
template <int NT, class F>
__device__ __forceinline__ void stage_b(uint8_t* xb, uint32_t sbo, int T, int col0, int ncol, F value) {
  const int n8 = ncol / 8;
#pragma unroll 4
  for (int i = threadIdx.x; i < NT * n8; i += PK_THREADS) {
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

// 1 / rms of the first T rows of x (fixed point, n columns) into s_inv (one warp per token).
__device__ __forceinline__ void rms_stats(const long long* x, int T, int n, float eps, float* s_inv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = warp; t < T; t += PK_NW) {
    float ss = 0.f;
#pragma unroll 8
    for (int c = lane; c < n; c += 32) {
      const float v = from_fix(ldcg_ll(x + (size_t)t * n + c));
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) s_inv[t] = 1.0f / sqrtf(ss / (float)n + eps);
  }
}

__device__ __forceinline__ void zero_ll(long long* p, size_t n) {
  for (size_t i = (size_t)blockIdx.x * PK_THREADS + threadIdx.x; i < n; i += (size_t)gridDim.x * PK_THREADS) p[i] = 0;
}

// ---------------------------------------------------------------------------------------------
// Attention item: query head hh over context tiles {slot, slot + S, ...}; writes (m, l, acc).
// ---------------------------------------------------------------------------------------------
__device__ void attention_item(const PassArgs& a, int l, int hh, int slot, float* sm) {
  const int HD = a.hd, HALF = HD / 2, HP = HD + 1, T = a.T, S = a.slots;
  const int group = a.heads / a.kv_heads, g = hh / group;
  const int pos0 = a.ctl->pos0, total = pos0 + T;
  const int ntiles = (total + PK_ATT_TILE - 1) / PK_ATT_TILE;
  const int H = a.heads * HD, KV = a.kv_heads * HD, QS = H + 2 * KV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t lstride = (size_t)a.kv_heads * a.max_ctx * HD;
  uint16_t* kc = a.kc + (size_t)l * lstride;
  uint16_t* vc = a.vc + (size_t)l * lstride;
  float* qs = sm;                    // [T][HD]
  float* Ks = qs + T * HD;           // [64][HP]
  float* Vs = Ks + PK_ATT_TILE * HP;
  float* st = Vs + PK_ATT_TILE * HP;  // [T][HD + 2]
  const float scale = 1.0f / sqrtf((float)HD);
  for (int i = threadIdx.x; i < T * HALF; i += PK_THREADS) {
    const int t = i / HALF, d = i - t * HALF;
    const float2 cs = a.rope[(size_t)(pos0 + t) * HALF + d];
    const long long* q = a.qkv + (size_t)t * QS + hh * HD;
    const float x1 = from_fix(ldcg_ll(q + d)), x2 = from_fix(ldcg_ll(q + d + HALF));
    qs[t * HD + d] = x1 * cs.x - x2 * cs.y;
    qs[t * HD + d + HALF] = x2 * cs.x + x1 * cs.y;
  }
  for (int i = threadIdx.x; i < T * (HD + 2); i += PK_THREADS) st[i] = (i % (HD + 2) == 0) ? -CUDART_INF_F : 0.f;
  const bool writer = (hh % group) == 0;
  for (int tile = slot; tile < ntiles; tile += S) {
    const int p0 = tile * PK_ATT_TILE;
    __syncthreads();
    for (int i = threadIdx.x; i < PK_ATT_TILE * HALF; i += PK_THREADS) {
      const int pl = i / HALF, d = i - pl * HALF, p = p0 + pl;
      float k1 = 0.f, k2 = 0.f, v1 = 0.f, v2 = 0.f;
      if (p < pos0) {
        const size_t base = ((size_t)g * a.max_ctx + p) * HD;
        k1 = __half2float(__ushort_as_half(kc[base + d]));
        k2 = __half2float(__ushort_as_half(kc[base + d + HALF]));
        v1 = __half2float(__ushort_as_half(vc[base + d]));
        v2 = __half2float(__ushort_as_half(vc[base + d + HALF]));
      } else if (p < total) {
        const int t = p - pos0;
        const long long* kr = a.qkv + (size_t)t * QS + H + g * HD;
        const long long* vr = a.qkv + (size_t)t * QS + H + KV + g * HD;
        const float2 cs = a.rope[(size_t)p * HALF + d];
        const float x1 = from_fix(ldcg_ll(kr + d)), x2 = from_fix(ldcg_ll(kr + d + HALF));
        k1 = __half2float(__float2half_rn(x1 * cs.x - x2 * cs.y));
        k2 = __half2float(__float2half_rn(x2 * cs.x + x1 * cs.y));
        v1 = __half2float(__float2half_rn(from_fix(ldcg_ll(vr + d))));
        v2 = __half2float(__float2half_rn(from_fix(ldcg_ll(vr + d + HALF))));
        if (writer) {
          const size_t base = ((size_t)g * a.max_ctx + p) * HD;
          kc[base + d] = __half_as_ushort(__float2half_rn(k1));
          kc[base + d + HALF] = __half_as_ushort(__float2half_rn(k2));
          vc[base + d] = __half_as_ushort(__float2half_rn(v1));
          vc[base + d + HALF] = __half_as_ushort(__float2half_rn(v2));
        }
      }
      Ks[pl * HP + d] = k1;
      Ks[pl * HP + d + HALF] = k2;
      Vs[pl * HP + d] = v1;
      Vs[pl * HP + d + HALF] = v2;
    }
    __syncthreads();
    for (int t = warp; t < T; t += PK_NW) {
      const int ctx = pos0 + t + 1;
      if (p0 >= ctx) continue;
      const float* q = qs + t * HD;
      float s0 = -CUDART_INF_F, s1 = -CUDART_INF_F;
      if (p0 + lane < ctx) {
        float acc = 0.f;
        for (int d = 0; d < HD; d++) acc = fmaf(q[d], Ks[lane * HP + d], acc);
        s0 = acc * scale;
      }
      if (p0 + 32 + lane < ctx) {
        float acc = 0.f;
        for (int d = 0; d < HD; d++) acc = fmaf(q[d], Ks[(lane + 32) * HP + d], acc);
        s1 = acc * scale;
      }
      const float tmax = warp_max(fmaxf(s0, s1));
      float* Sx = st + t * (HD + 2);
      const float m_old = Sx[0], m_new = fmaxf(m_old, tmax);
      const float corr = (m_old == -CUDART_INF_F) ? 0.f : expf(m_old - m_new);
      const float e0 = (s0 == -CUDART_INF_F) ? 0.f : expf(s0 - m_new);
      const float e1 = (s1 == -CUDART_INF_F) ? 0.f : expf(s1 - m_new);
      const float lsum = warp_sum(e0 + e1);
      for (int d0 = 0; d0 < HD; d0 += 32) {
        const int d = d0 + lane;
        float acc = (d < HD) ? Sx[2 + d] * corr : 0.f;
        for (int pl = 0; pl < 32; pl++) {
          const float e = __shfl_sync(0xffffffffu, e0, pl);
          if (d < HD) acc = fmaf(e, Vs[pl * HP + d], acc);
        }
        for (int pl = 0; pl < 32; pl++) {
          const float e = __shfl_sync(0xffffffffu, e1, pl);
          if (d < HD) acc = fmaf(e, Vs[(pl + 32) * HP + d], acc);
        }
        if (d < HD) Sx[2 + d] = acc;
      }
      __syncwarp();
      if (lane == 0) {
        Sx[1] = Sx[1] * corr + lsum;
        Sx[0] = m_new;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  float* part = a.att_part + ((size_t)hh * S + slot) * T * (HD + 2);
  for (int i = threadIdx.x; i < T * (HD + 2); i += PK_THREADS) part[i] = st[i];
}

// ---------------------------------------------------------------------------------------------
// The pass kernel
// ---------------------------------------------------------------------------------------------
template <int BITS, int G, int NT>
__global__ void __launch_bounds__(PK_THREADS, 1) pass_kernel(const PassArgs a) {
  using Gemv = TcGemv<BITS, G, NT>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar_a[2], bar_full[2], bar_d;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ float s_inv[NT];
  __shared__ float s_bv[PK_NW][NT];
  __shared__ uint32_t s_bi[PK_NW][NT];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = a.T, h = a.hidden, I = a.inter;
  const int kvd = a.kv_heads * a.hd, QS = h + 2 * kvd;
  int* err = &a.ctl->err;
  // shared memory: [load ring][B operand or attention scratch]
  uint8_t* ring = smem;
  uint8_t* xb = smem + (size_t)PK_STAGES * Gemv::kStage;
  const uint32_t xb_addr = tc::su32(xb);

  if (threadIdx.x == 0) {
    tc::mbar_init(&bar_a[0], 1);
    tc::mbar_init(&bar_a[1], 1);
    tc::mbar_init(&bar_full[0], PK_THREADS);
    tc::mbar_init(&bar_full[1], PK_THREADS);
    tc::mbar_init(&bar_d, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::su32(&s_tmem)), "r"(128)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  tc::fence_after();
  Gemv gm;
  gm.tmem = s_tmem;
  gm.ring = ring;
  gm.ring_addr = tc::su32(ring) + (uint32_t)threadIdx.x * Gemv::CPB * 16;
  gm.bar_a = bar_a;
  gm.bar_full = bar_full;
  gm.bar_d = &bar_d;
  gm.abort = &s_abort;
  gm.uses0 = gm.uses1 = gm.dphase = 0;

  unsigned nbar = 0;
  bool ok = true;
  auto barrier = [&]() {
    nbar++;
    if (ok && !grid_barrier(a.bar, nbar * gridDim.x, err)) ok = false;
    if (s_abort) ok = false;
    return ok;
  };
  // Starts the weight stream of this CTA's first item of a GEMV phase (before the barrier).
  auto prefetch = [&](const QMat& w, int ks) {
    const Split sp = make_split<BITS, G>(w, ks);
    if ((int)blockIdx.x < sp.items()) {
      int t128, kb0, kb1;
      sp.item(blockIdx.x, &t128, &kb0, &kb1);
      gm.prologue(w, t128, kb0, kb1);
    }
  };
  // Runs the items of a GEMV phase: stage(kb0, kb1) fills the B operand of a K slice,
  // epi(t128, ks_index, tot) consumes the accumulators.
  auto gemv_phase = [&](const QMat& w, int ks, auto stage, auto epi) {
    const Split sp = make_split<BITS, G>(w, ks);
    int staged = -1;
    bool first = true;
    for (int i = blockIdx.x; i < sp.items() && ok; i += gridDim.x) {
      int t128, kb0, kb1;
      sp.item(i, &t128, &kb0, &kb1);
      const int kslice = i / sp.tiles128;
      const int col0 = kb0 * Gemv::KB, ncol = (kb1 - kb0) * Gemv::KB;
      const uint32_t sbo = (uint32_t)(ncol / 8) * 128u;
      if (kslice != staged) {
        __syncthreads();
        stage(col0, ncol, sbo);
        __syncthreads();
        staged = kslice;
      }
      if (!first) gm.prologue(w, t128, kb0, kb1);
      first = false;
      float tot[NT];
      if (!gm.run(w, t128, kb0, kb1, xb_addr, sbo, tot)) {
        ok = false;
        s_abort = 1;
        if (threadIdx.x == 0) atomicCAS(err, 0, 1);  // the other CTAs stop at their next wait
        break;
      }
      const int t32 = t128 * 4 + warp;
      if (t32 < w.rows_pad / 32) epi(t32 * 32 + lane, kslice, tot);
    }
    // drain an unused prologue (a CTA without items never issued one)
    tc::cp_wait<0>();
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
  prefetch(a.layers[0].qkv, a.ks_qkv);
  barrier();

  for (int l = 0; l < a.L && ok; l++) {
    const PassLayer& W = a.layers[l];
    // ---- QKV: RMSNorm(x) -> q|k|v sums (+ bias once) ----
    rms_stats(a.x, T, h, a.eps, s_inv);
    __syncthreads();
    gemv_phase(
        W.qkv, a.ks_qkv,
        [&](int col0, int ncol, uint32_t sbo) {
          stage_b<NT>(xb, sbo, T, col0, ncol, [&](int t, int c) {
            return from_fix(ldcg_ll(a.x + (size_t)t * h + c)) * s_inv[t] * bf16f(W.in_norm[c]);
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

    // ---- attention (the block's K/V appended to the cache); zero the gate/up accumulators ----
    for (int it = blockIdx.x; it < a.heads * a.slots; it += gridDim.x) {
      __syncthreads();
      attention_item(a, l, it / a.slots, it % a.slots, reinterpret_cast<float*>(xb));
    }
    zero_ll(a.gu, (size_t)T * 2 * I);
    prefetch(W.o, a.ks_o);
    if (!barrier()) break;

    // ---- O: combine the attention slots while staging, residual add into x ----
    gemv_phase(
        W.o, a.ks_o,
        [&](int col0, int ncol, uint32_t sbo) {
          // per (head, token) slot weights e^(m_s - m*) / L, then the weighted sum of acc_s
          const int HD = a.hd, S = a.slots;
          const int h0 = col0 / HD, nh = (ncol + HD - 1) / HD;
          float* wts = reinterpret_cast<float*>(xb + (size_t)NT * ncol * 2);  // [nh][T][S]
          for (int i = threadIdx.x; i < nh * T; i += PK_THREADS) {
            const int hi = i / T, t = i - hi * T;
            const float* base = a.att_part + (size_t)(h0 + hi) * S * T * (HD + 2) + (size_t)t * (HD + 2);
            float mx = -CUDART_INF_F;
            for (int s = 0; s < S; s++) mx = fmaxf(mx, __ldcg(base + (size_t)s * T * (HD + 2)));
            float L = 0.f;
            for (int s = 0; s < S; s++) {
              const float ms = __ldcg(base + (size_t)s * T * (HD + 2));
              L += (ms == -CUDART_INF_F) ? 0.f : __ldcg(base + (size_t)s * T * (HD + 2) + 1) * expf(ms - mx);
            }
            for (int s = 0; s < S; s++) {
              const float ms = __ldcg(base + (size_t)s * T * (HD + 2));
              wts[(size_t)i * S + s] = (ms == -CUDART_INF_F) ? 0.f : expf(ms - mx) / L;
            }
          }
          __syncthreads();
          stage_b<NT>(xb, sbo, T, col0, ncol, [&](int t, int c) {
            const int hh = c / HD, d = c - hh * HD;
            const float* base = a.att_part + (size_t)hh * S * T * (HD + 2) + (size_t)t * (HD + 2) + 2 + d;
            const float* w = wts + ((size_t)(hh - h0) * T + t) * S;
            float o = 0.f;
            for (int s = 0; s < S; s++) o = fmaf(__ldcg(base + (size_t)s * T * (HD + 2)), w[s], o);
            return o;
          });
        },
        [&](int r, int, float (&tot)[NT]) {
          if (r >= h) return;
#pragma unroll
          for (int t = 0; t < NT; t++)
            if (t < T) fix_add(a.x + (size_t)t * h + r, tot[t]);
        });
    zero_ll(a.qkv, (size_t)T * QS);
    prefetch(W.gu, a.ks_gu);
    if (!barrier()) break;

    // ---- gate/up: RMSNorm(x) -> gate/up sums ----
    rms_stats(a.x, T, h, a.eps, s_inv);
    __syncthreads();
    gemv_phase(
        W.gu, a.ks_gu,
        [&](int col0, int ncol, uint32_t sbo) {
          stage_b<NT>(xb, sbo, T, col0, ncol, [&](int t, int c) {
            return from_fix(ldcg_ll(a.x + (size_t)t * h + c)) * s_inv[t] * bf16f(W.post_norm[c]);
          });
        },
        [&](int r, int, float (&tot)[NT]) {
#pragma unroll
          for (int t = 0; t < NT; t++)
            if (t < T) fix_add(a.gu + (size_t)t * 2 * I + r, tot[t]);
        });
    prefetch(W.down, a.ks_down);
    if (!barrier()) break;

    // ---- down: SwiGLU while staging, residual add into x ----
    gemv_phase(
        W.down, a.ks_down,
        [&](int col0, int ncol, uint32_t sbo) {
          stage_b<NT>(xb, sbo, T, col0, ncol, [&](int t, int j) {
            const long long* row = a.gu + (size_t)t * 2 * I + (j / 16) * 32 + (j % 16);
            const float gt = from_fix(ldcg_ll(row)), up = from_fix(ldcg_ll(row + 16));
            return gt / (1.0f + expf(-gt)) * up;
          });
        },
        [&](int r, int, float (&tot)[NT]) {
          if (r >= h) return;
#pragma unroll
          for (int t = 0; t < NT; t++)
            if (t < T) fix_add(a.x + (size_t)t * h + r, tot[t]);
        });
    if (l + 1 < a.L) prefetch(a.layers[l + 1].qkv, a.ks_qkv);
    else prefetch(a.embed, 1);
    if (!barrier()) break;
  }

  // ---- LM head on the last n_logits rows: final RMSNorm, per-CTA argmax parts ----
  if (ok && a.n_logits > 0) {
    const int n = a.n_logits, r0 = T - n;
    for (int i = threadIdx.x; i < PK_NW * NT; i += PK_THREADS) {
      (&s_bv[0][0])[i] = -CUDART_INF_F;
      (&s_bi[0][0])[i] = 0xffffffffu;
    }
    rms_stats(a.x + (size_t)r0 * h, n, h, a.eps, s_inv);
    __syncthreads();
    gemv_phase(
        a.embed, 1,
        [&](int col0, int ncol, uint32_t sbo) {
          stage_b<NT>(xb, sbo, n, col0, ncol, [&](int t, int c) {
            return from_fix(ldcg_ll(a.x + (size_t)(r0 + t) * h + c)) * s_inv[t] * a.final_norm[c];
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

  // ---- release tensor memory ----
  tc::cp_wait<0>();
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(s_tmem), "r"(128) : "memory");
  }
  if (s_abort && threadIdx.x == 0) atomicCAS(err, 0, 1);
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------

static int pk_nt(int T) { return T <= 16 ? 16 : T <= 32 ? 32 : 48; }

bool pass_kernel_supported(const WeightFormat& body, const WeightFormat& embed, int T, int hd) {
  if (!(body == embed) || T < 1 || T > 48 || hd % 2 || hd > 128) return false;
  return (body.bits == 8 && (body.group == 32 || body.group == 64)) || (body.bits == 4 && (body.group == 16 || body.group == 32));
}

size_t pass_kernel_smem(const WeightFormat& f, int T, int hidden, int inter, int hd, int heads, int slots, int ks_down,
                        int ks_o) {
  const int NT = pk_nt(T);
  const int kb = tc_kb(f.bits, f.group), cpb = kb / (128 / f.bits);
  const size_t ring = (size_t)PK_STAGES * PK_THREADS * cpb * 16;
  // largest B operand: a K slice of down (inter / ks_down), the full hidden (QKV, gate/up, head),
  // or an O slice plus its slot weights
  const int nblk_down = inter / kb;
  const int down_cols = ((nblk_down + ks_down - 1) / ks_down) * kb;
  const int nblk_o = hidden / kb;
  const int o_cols = ((nblk_o + ks_o - 1) / ks_o) * kb;
  size_t b = (size_t)NT * std::max(hidden, std::max(down_cols, o_cols)) * 2;
  b = std::max(b, (size_t)NT * o_cols * 2 + (size_t)((o_cols + hd - 1) / hd + 1) * T * slots * 4);
  const size_t att = ((size_t)T * hd + 2 * PK_ATT_TILE * (hd + 1) + (size_t)T * (hd + 2)) * 4;
  return ring + std::max(b, att);
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
  const int NT = pk_nt(a.T);
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

// Occupancy check: the cooperative launch needs every CTA resident at once.
int pass_kernel_max_grid(const WeightFormat& f, int T, size_t smem, int num_sms) {
  const int NT = pk_nt(T);
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
  return per_sm >= 1 ? num_sms : 0;
}

}  // namespace ls
