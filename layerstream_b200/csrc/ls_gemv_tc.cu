// Tensor-core (tcgen05) GEMV of the verify path.
#include <algorithm>

#include "ls_device.cuh"
#include "ls_internal.h"

namespace ls {

// ================================================================================================
// Tensor-core GEMV (tcgen05): y[t][r] = sum_k W[r][k] * x[t][k] for up to NT tokens.
//
// A (the weights, M = 128 rows per tile) lives in tensor memory: each of the 128 threads owns one
// row, streams its packed ints through a private cp.async ring, dequantises a 64-wide K block
// ((q - 8) * scale, or q * scale for int8) to f16 in registers and stores it with tcgen05.st.
// B (the activations, N = NT tokens, K-major) is staged once per CTA in shared memory in the
// canonical no-swizzle layout. One elected thread issues tcgen05.mma (kind::f16, f32 accumulate
// into tensor memory) on a double-buffered A and signals completion with tcgen05.commit on an
// mbarrier. Every wait is bounded: on a timeout the kernel records LS_ERR_DEVICE and returns after
// releasing its tensor memory.
// ================================================================================================



constexpr int TC_THREADS = 128;
constexpr int TC_STAGES = 6;

template <int BITS, int G, int NT>
__global__ void __launch_bounds__(TC_THREADS) gemv_tc_kernel(const GemvLaunch g) {
  constexpr int KB = tc_kb(BITS, G);   // K per A block
  constexpr int NS = tc_ns(BITS, G);   // scales per row per block
  constexpr int WPC = 128 / BITS;      // weights per 16-byte chunk
  constexpr int CPB = KB / WPC;        // chunks per block
  constexpr int PARTS = tc_parts(BITS);  // int8: exact hi and lo f16 parts of every weight
  constexpr int HCOLS = KB / 2;          // TMEM columns of one part of a block (two f16 per column)
  constexpr int ACOLS = HCOLS * PARTS;   // TMEM columns of one A buffer
  constexpr int TCOLS = (2 * ACOLS + NT <= 128) ? 128 : (2 * ACOLS + NT <= 256) ? 256 : 512;
  constexpr int NW = TC_THREADS / 32;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ uint64_t bar_a[2], bar_full[2], bar_d;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ float s_inv[NT];
  __shared__ float s_bv[NW][NT];
  __shared__ uint32_t s_bi[NW][NT];

  const int ks = blockIdx.y, z = blockIdx.z;
  const int tiles32 = g.w.rows_pad / 32, tiles128 = (tiles32 + 3) / 4;
  const int m0 = z * NT;
  const int Mloc = min(NT, g.M - m0);
  const int nch = g.w.chunks(), ngr = g.w.groups();
  const int nblk = nch / CPB;
  const int kb0 = (int)((long long)ks * nblk / g.ksplit), kb1 = (int)((long long)(ks + 1) * nblk / g.ksplit);
  const int c0 = kb0 * CPB, c1 = kb1 * CPB;
  const int col0 = c0 * WPC, ncol = (c1 - c0) * WPC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // shared memory: B operand [NT/8 row groups][ncol/8 K chunks][8 rows][16 B], then the load ring
  uint8_t* xb = smem_raw;
  const uint32_t sbo = (uint32_t)(ncol / 8) * 128u;
  uint8_t* ring = smem_raw + (size_t)(NT / 8) * sbo;  // [TC_STAGES][TC_THREADS][CPB][16 B]

  pdl_trigger();
  const int first = blockIdx.x;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar_a[0], 1);
    tc::mbar_init(&bar_a[1], 1);
    tc::mbar_init(&bar_full[0], TC_THREADS);
    tc::mbar_init(&bar_full[1], TC_THREADS);
    tc::mbar_init(&bar_d, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < NW * NT; i += TC_THREADS) {
    (&s_bv[0][0])[i] = -CUDART_INF_F;
    (&s_bi[0][0])[i] = 0xffffffffu;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::su32(&s_tmem)), "r"(TCOLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  const uint32_t ring_addr = tc::su32(ring) + (uint32_t)threadIdx.x * CPB * 16;
  constexpr uint32_t kStageStride = TC_THREADS * CPB * 16;
  // The weights do not depend on the previous kernel: start streaming the first tile now.
  auto issue_prologue = [&](int t128) {
    const int t32 = t128 * 4 + warp;
    const bool valid = t32 < tiles32;
    const uint8_t* db = g.w.data + ((size_t)(valid ? t32 : 0) * nch) * 512 + lane * 16;
#pragma unroll
    for (int s = 0; s < TC_STAGES - 1; s++) {
      const int kb = kb0 + s;
      if (kb < kb1 && valid) {
#pragma unroll
        for (int q = 0; q < CPB; q++) tc::cp_async16(ring_addr + s * kStageStride + q * 16, db + (size_t)(kb * CPB + q) * 512);
      }
      tc::cp_commit();
    }
  };
  if (first < tiles128) issue_prologue(first);
  pdl_wait();

  // ---- stage the activations (x * norm weight, f16, canonical K-major layout; tokens >= M are
  // zero) and, if a norm is fused, the per-token 1/rms over the full row, applied in the epilogue ----
  const bool has_norm = g.norm_bf16 != nullptr || g.norm_f32 != nullptr;
  {
    const int n8 = ncol / 8;  // 16-byte K chunks per token
    for (int i = threadIdx.x; i < NT * n8; i += TC_THREADS) {
      const int t = i / n8, kc = i - t * n8;
      uint32_t w4[4] = {0u, 0u, 0u, 0u};
      if (t < Mloc) {
        const float* xr = g.x + (size_t)(m0 + t) * g.x_stride + col0 + kc * 8;
        const float4 a = __ldg(reinterpret_cast<const float4*>(xr));
        const float4 b = __ldg(reinterpret_cast<const float4*>(xr) + 1);
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        if (has_norm) {
#pragma unroll
          for (int e = 0; e < 8; e++) {
            const int col = col0 + kc * 8 + e;
            v[e] *= g.norm_bf16 ? bf16f(g.norm_bf16[col]) : g.norm_f32[col];
          }
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const __half2 h = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
          w4[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      *reinterpret_cast<uint4*>(xb + (size_t)(t / 8) * sbo + (size_t)kc * 128 + (t % 8) * 16) =
          make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
  }
  if (has_norm && g.inv_rms) {
    for (int t = threadIdx.x; t < Mloc; t += TC_THREADS) s_inv[t] = g.inv_rms[m0 + t];
  } else if (has_norm) {
    const int cols4 = g.w.cols >> 2;
    for (int t = warp; t < Mloc; t += NW) {
      float ss = 0.f;
#pragma unroll 4
      for (int c4 = lane; c4 < cols4; c4 += 32) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(g.x + (size_t)(m0 + t) * g.x_stride) + c4);
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
      ss = warp_sum(ss);
      if (lane == 0) s_inv[t] = 1.0f / sqrtf(ss / (float)g.w.cols + g.eps);
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  const uint32_t tmem = s_tmem;
  tc::fence_after();
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t d_col = tmem + 2 * ACOLS;
  const uint32_t idesc = tc::idesc_f16(NT);
  const uint32_t xb_addr = tc::su32(xb);

  uint32_t uses[2] = {0u, 0u};
  uint32_t tiles_done = 0;
  bool failed = false;

  for (int t128 = first; t128 < tiles128; t128 += gridDim.x) {
    const int t32 = t128 * 4 + warp;
    const bool row_valid = t32 < tiles32;
    const uint8_t* db = g.w.data + ((size_t)(row_valid ? t32 : 0) * nch) * 512 + lane * 16;
    const uint16_t* sb = g.w.scales + (size_t)(row_valid ? t32 : 0) * ngr * 32 + lane;
    // raw bf16 scales, loaded two blocks ahead and converted only when used
    auto load_scales = [&](int kb, uint16_t (&sc)[NS]) {
#pragma unroll
      for (int s = 0; s < NS; s++) {
        if constexpr (BITS == 16) {
          sc[s] = 0;  // bf16 weights carry no scales
        } else {
          const int gi = (kb * KB) / G + s;
          sc[s] = (row_valid && kb < kb1) ? sb[(size_t)gi * 32] : (uint16_t)0;
        }
      }
    };
    uint16_t sraw0[NS], sraw1[NS], sraw2[NS];
    load_scales(kb0, sraw0);
    load_scales(kb0 + 1, sraw1);
    if (t128 != first) issue_prologue(t128);
    for (int kb = kb0; kb < kb1; kb++) {
      const int it = kb - kb0;
      {
        const int kn = kb + TC_STAGES - 1;
        const int sn = (it + TC_STAGES - 1) % TC_STAGES;
        if (kn < kb1 && row_valid) {
#pragma unroll
          for (int q = 0; q < CPB; q++) tc::cp_async16(ring_addr + sn * kStageStride + q * 16, db + (size_t)(kn * CPB + q) * 512);
        }
        tc::cp_commit();
      }
      load_scales(kb + 2, sraw2);
      uint32_t scur[NS];
#pragma unroll
      for (int q = 0; q < NS; q++) scur[q] = tc::h2_splat(bf16f(sraw0[q]));
      tc::cp_wait<TC_STAGES - 1>();
      uint4 wv[CPB];
      const uint8_t* rs = ring + (size_t)(it % TC_STAGES) * kStageStride + (size_t)threadIdx.x * CPB * 16;
#pragma unroll
      for (int q = 0; q < CPB; q++) wv[q] = row_valid ? *reinterpret_cast<const uint4*>(rs + q * 16) : make_uint4(0, 0, 0, 0);

      // ---- dequantise one K block of this row into f16 pairs in K order ----
      uint32_t a[HCOLS], alo[PARTS == 2 ? HCOLS : 1];
      if constexpr (PARTS == 2) tc_dequant_block_i8<G>(wv, scur, a, alo);
      else tc_dequant_block<BITS, G>(wv, scur, a);
#pragma unroll
      for (int q = 0; q < NS; q++) {
        sraw0[q] = sraw1[q];
        sraw1[q] = sraw2[q];
      }

      // ---- A buffer reuse: the MMAs that read it two blocks ago must have completed ----
      const int b = it & 1;
      if (uses[b] > 0 && !tc::mbar_wait_fast(&bar_a[b], (uses[b] - 1) & 1, &s_abort)) failed = true;
      if (__any_sync(0xffffffffu, failed)) {  // warp-uniform before the warp-collective stores
        failed = true;
        break;
      }
      tc::fence_after();
      __syncwarp();
#pragma unroll
      for (int q = 0; q < HCOLS / 16; q++) tc::st16(tmem + lane_base + b * ACOLS + q * 16, a + q * 16);
      if constexpr (PARTS == 2) {
#pragma unroll
        for (int q = 0; q < HCOLS / 16; q++) tc::st16(tmem + lane_base + b * ACOLS + HCOLS + q * 16, alo + q * 16);
      }
      tc::wait_st();
      tc::fence_before();
      // block written: one arrival per thread; only the MMA issuer waits for all 128
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::su32(&bar_full[b])) : "memory");
      if (threadIdx.x == 0) {
        if (!tc::mbar_wait_fast(&bar_full[b], uses[b] & 1, &s_abort)) {
          failed = true;
        } else {
          tc::fence_after();
#pragma unroll
          for (int j = 0; j < KB / 16; j++) {
            const uint32_t kpos = (uint32_t)(it * KB + j * 16);  // K offset inside the staged slice
            const uint64_t bd = tc::sdesc(xb_addr + (kpos / 8) * 128u, 128u, sbo);
            tc::mma_f16_ts(d_col, tmem + b * ACOLS + j * 8, bd, idesc, (it > 0 || j > 0) ? 1u : 0u);
            if constexpr (PARTS == 2) tc::mma_f16_ts(d_col, tmem + b * ACOLS + HCOLS + j * 8, bd, idesc, 1u);
          }
          tc::commit(&bar_a[b]);
        }
      }
      __syncwarp();
      uses[b]++;
      if (__any_sync(0xffffffffu, failed)) {
        failed = true;
        break;
      }
    }
    tc::cp_wait<0>();
    if (failed) break;

    // ---- accumulators of this tile ----
    if (threadIdx.x == 0) tc::commit(&bar_d);
    if (!tc::mbar_wait_fast(&bar_d, tiles_done & 1, &s_abort)) failed = true;
    if (__any_sync(0xffffffffu, failed)) {
      failed = true;
      break;
    }
    tiles_done++;
    tc::fence_after();
    float tot[NT];
#pragma unroll
    for (int q = 0; q < NT / 16; q++) {
      uint32_t v[16];
      tc::ld16(d_col + lane_base + q * 16, v);
      tc::wait_ld();
#pragma unroll
      for (int e = 0; e < 16; e++) tot[q * 16 + e] = __uint_as_float(v[e]);
    }
    tc::fence_before();
    if (has_norm) {
#pragma unroll
      for (int t = 0; t < NT; t++)
        if (t < Mloc) tot[t] *= s_inv[t];
    }
    if (!row_valid) continue;
    const int tile = t32;

    // ---- split-K: the last warp to finish this 32-row tile sums the K slices in order ----
    if (g.ksplit > 1) {
      float* part = g.partial + ((size_t)(z * tiles32 + tile) * g.ksplit) * NT * 32;
#pragma unroll
      for (int t = 0; t < NT; t++)
        if (t < Mloc) part[((size_t)ks * NT + t) * 32 + lane] = tot[t];
      __threadfence();
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) {
        unsigned* tk = g.tickets + z * tiles32 + tile;
        last = atomicAdd(tk, 1u) == (unsigned)g.ksplit - 1;
        if (last) *tk = 0u;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence();
#pragma unroll
      for (int t = 0; t < NT; t++) tot[t] = 0.f;
#pragma unroll 4
      for (int k = 0; k < g.ksplit; k++) {
#pragma unroll
        for (int t = 0; t < NT; t++)
          if (t < Mloc) tot[t] += __ldcg(part + ((size_t)k * NT + t) * 32 + lane);
      }
    }

    const int r = tile * 32 + lane;
    if (g.epi == EPI_ARGMAX) {
#pragma unroll
      for (int t = 0; t < NT; t++) {
        if (t < Mloc) {
          float v = (r < g.n_valid_rows) ? tot[t] : -CUDART_INF_F;
          uint32_t idx = (uint32_t)(r + g.row_offset);
          if (g.logits && r < g.n_valid_rows) g.logits[(size_t)(m0 + t) * g.logits_stride + g.row_offset + r] = tot[t];
          warp_argmax(v, idx);
          if (lane == 0 && arg_better(v, idx, s_bv[warp][t], s_bi[warp][t])) {
            s_bv[warp][t] = v;
            s_bi[warp][t] = idx;
          }
        }
      }
    } else if (g.epi == EPI_SWIGLU) {
#pragma unroll
      for (int t = 0; t < NT; t++) {
        const float u = __shfl_down_sync(0xffffffffu, tot[t], 16);
        if (t < Mloc && lane < 16) {
          const float gt = tot[t];
          g.y[(size_t)(m0 + t) * g.y_stride + tile * 16 + lane] = gt / (1.0f + expf(-gt)) * u;
        }
      }
    } else if (r < g.w.rows) {
#pragma unroll
      for (int t = 0; t < NT; t++) {
        if (t < Mloc) {
          float* dst = g.y + (size_t)(m0 + t) * g.y_stride + r;
          if (g.epi == EPI_RESID) *dst += tot[t];
          else if (g.epi == EPI_BIAS_STORE) *dst = tot[t] + bf16f(g.bias[r]);
          else *dst = tot[t];
        }
      }
    }
  }

  // ---- release tensor memory (also on the error path) ----
  tc::cp_wait<0>();
  tc::fence_before();
  failed = __syncthreads_or(failed || s_abort);
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
  }
  if (failed) {
    if (threadIdx.x == 0 && g.err) atomicExch(g.err, 1);
    return;
  }

  if (g.epi != EPI_ARGMAX) return;
  if (threadIdx.x < Mloc) {
    const int t = threadIdx.x;
    float v = s_bv[0][t];
    uint32_t idx = s_bi[0][t];
    for (int w = 1; w < NW; w++)
      if (arg_better(s_bv[w][t], s_bi[w][t], v, idx)) {
        v = s_bv[w][t];
        idx = s_bi[w][t];
      }
    g.arg_parts[(size_t)(blockIdx.x + g.part_tile_offset) * g.M + m0 + t] = ArgPart{v, idx};
  }
  if (!g.finalize) return;
  if (!last_cta(g.arg_ticket, (unsigned)(gridDim.x * gridDim.z))) return;
  argmax_finalize_block(g.arg_parts, g.n_part_tiles ? g.n_part_tiles : gridDim.x, g.M, g.ctl);
}

// ---- host side of the tensor-core GEMV ----

static int tc_nt(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 48 ? 48 : 64; }

bool gemv_tc_supported(const QMat& w) {
  if (w.bits == 16) return (w.cols % 64) == 0;  // bf16 weights, converted to f16 operands
  if (w.bits == 8) return w.group >= 16 && w.group <= 128 && (w.cols % 64) == 0;
  return (w.group == 16 || w.group == 32 || w.group == 64 || w.group == 128) && (w.cols % tc_kb(4, w.group)) == 0;
}

static size_t gemv_tc_smem(const QMat& w, int ksplit, int NT) {
  const int kb = tc_kb(w.bits, w.group), cpb = kb / (128 / w.bits);
  const int nblk = w.chunks() / cpb;
  int maxblk = 0;
  for (int k = 0; k < ksplit; k++) maxblk = max(maxblk, (int)((long long)(k + 1) * nblk / ksplit - (long long)k * nblk / ksplit));
  return (size_t)NT * maxblk * kb * 2 + (size_t)TC_STAGES * TC_THREADS * cpb * 16;
}

int gemv_tc_nt(int M, int max_nt) { return tc_nt(std::min(M, max_nt)); }

int gemv_tc_min_ksplit(const QMat& w, int M, int max_nt) {
  const int NT = gemv_tc_nt(M, max_nt);
  for (int ks = 1; ks <= 64; ks++)
    if (gemv_tc_smem(w, ks, NT) <= 190 * 1024) return ks;
  LS_THROW(-1, "matrix too wide for the tensor-core GEMV");
}

template <int BITS, int G, int NT>
static void launch_tc_t(const GemvLaunch& g, cudaStream_t s) {
  const size_t smem = gemv_tc_smem(g.w, g.ksplit, NT);
  ensure_smem(gemv_tc_kernel<BITS, G, NT>, smem);
  const int tiles128 = (g.w.rows_pad / 32 + 3) / 4;
  const int gx = g.grid_x > 0 ? min(g.grid_x, tiles128) : tiles128;
  dim3 grid(gx, g.ksplit, (g.M + NT - 1) / NT);
  launch_pdl(gemv_tc_kernel<BITS, G, NT>, grid, dim3(TC_THREADS), smem, s, g);
}

template <int BITS, int G>
static void launch_tc_g(const GemvLaunch& g, cudaStream_t s) {
  switch (gemv_tc_nt(g.M, g.max_nt)) {
    case 16: return launch_tc_t<BITS, G, 16>(g, s);
    case 32: return launch_tc_t<BITS, G, 32>(g, s);
    case 48: return launch_tc_t<BITS, G, 48>(g, s);
    default: return launch_tc_t<BITS, G, 64>(g, s);
  }
}

// One warp per row, the same per-lane float4 order and warp sum as the GEMV norm prologue.
__global__ void inv_rms_kernel(const float* __restrict__ x, int x_stride, int M, int cols, float eps, float* inv) {
  const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= M) return;
  const int cols4 = cols >> 2;
  float ss = 0.f;
#pragma unroll 4
  for (int c4 = lane; c4 < cols4; c4 += 32) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(x + (size_t)t * x_stride) + c4);
    ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
  }
  ss = warp_sum(ss);
  if (lane == 0) inv[t] = 1.0f / sqrtf(ss / (float)cols + eps);
}

void launch_inv_rms(const float* x, int x_stride, int M, int cols, float eps, float* inv, cudaStream_t s) {
  if (M <= 0) return;
  inv_rms_kernel<<<(M + 7) / 8, 256, 0, s>>>(x, x_stride, M, cols, eps, inv);
  LS_CUDA(cudaGetLastError());
}

void launch_gemv_tc(const GemvLaunch& g, cudaStream_t s) {
  if (g.M <= 0) return;
  if (!gemv_tc_supported(g.w)) LS_THROW(-1, "format not supported by the tensor-core GEMV");
  if (g.ksplit < gemv_tc_min_ksplit(g.w, g.M, g.max_nt)) LS_THROW(-1, "tensor-core GEMV split too small for shared memory");
  if (g.ksplit > 1 && (!g.partial || !g.tickets)) LS_THROW(-1, "a split tensor-core GEMV needs partial-sum scratch");
  if (g.w.bits == 16) return launch_tc_g<16, 16>(g, s);  // (the group argument is unused for bf16)
  if (g.w.bits == 8) {
    switch (g.w.group) {
      case 16: return launch_tc_g<8, 16>(g, s);
      case 32: return launch_tc_g<8, 32>(g, s);
      case 64: return launch_tc_g<8, 64>(g, s);
      default: return launch_tc_g<8, 128>(g, s);
    }
  }
  switch (g.w.group) {
    case 16: return launch_tc_g<4, 16>(g, s);
    case 32: return launch_tc_g<4, 32>(g, s);
    case 64: return launch_tc_g<4, 64>(g, s);
    default: return launch_tc_g<4, 128>(g, s);
  }
}

}  // namespace ls
