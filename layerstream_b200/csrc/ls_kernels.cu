// CUDA kernels of the verify path, written for sm_100a.
//
//   gemv_kernel        dequant-fused skinny GEMV for M <= 16 rows per token group: int8 / int4 weights
//                      with bf16 group scales, 128-bit coalesced loads of a 32-row tiled layout,
//                      in-register unpacking, optional RMSNorm prologue, and fused epilogues
//                      (bias, residual add, SwiGLU, LM-head argmax + longest-prefix acceptance).
//                      Replaces kernels::matmul_q8 / matmul_q4 (src/kernels.rs:53-92,123-203) and the
//                      norm / bias / silu / residual / argmax steps around them (src/model.rs:240-298,
//                      src/model.rs:190-216, src/spec.rs:41-49,120-127).
//   attention_kernel   causal GQA attention of the M block rows over the f16 KV cache with RoPE applied
//                      from a host-computed table and the block's new K/V appended. Split across CTAs
//                      along the context with an online softmax and a deterministic combine.
//                      Replaces src/model.rs:249-282 and kernels::rope_inplace / softmax_inplace.
//   embed_kernel       embedding row gather + dequantisation (src/kernels.rs:95-121), bit-exact.
//   repack_kernel      file row layout -> tiled device planes (a byte move, no arithmetic).
//   quantize_kernel    quant::quantize_group / quantize_row (src/quant.rs:35-104), bit-exact.
#include <cuda_fp16.h>
#include <math_constants.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "ls_device.cuh"
#include "ls_internal.h"

namespace ls {

// ------------------------------------------------------------------------------------------------
// GEMV
// ------------------------------------------------------------------------------------------------

constexpr int GEMV_UNROLL = 8;  // 16-byte loads in flight per lane

__global__ void __launch_bounds__(GEMV_THREADS) argmax_finalize_kernel(const ArgPart* parts, int nparts, int M, Ctl* ctl) {
  pdl_wait();
  argmax_finalize_block(parts, nparts, M, ctl);
}

void launch_argmax_finalize(const ArgPart* parts, int nparts, int M, Ctl* ctl, cudaStream_t s) {
  argmax_finalize_kernel<<<1, GEMV_THREADS, 0, s>>>(parts, nparts, M, ctl);
  LS_CUDA(cudaGetLastError());
}

// One 16-byte chunk of a row times the staged activations of up to MT tokens, accumulated into
// tot[t] with the chunk's group scale(s).
template <int BITS, bool G16, int MT>
__device__ __forceinline__ void gemv_chunk(const uint4 wv, int c, int col0, int ncol, int group, const uint16_t* sb,
                                           const float* __restrict__ xs, int Mloc, float (&tot)[MT]) {
  const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
  if constexpr (BITS == 8) {
    const float s = bf16f(sb[(size_t)((c * 16) / group) * 32]);
    float wf[16];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t wx = wd[k] ^ 0x80808080u;
#pragma unroll
      for (int b = 0; b < 4; b++) wf[4 * k + b] = s8_to_f(wx, b);
    }
    const float* xc = xs + (c * 16 - col0);
#pragma unroll
    for (int t = 0; t < MT; t++) {
      if (t < Mloc) {
        const float4* xp = reinterpret_cast<const float4*>(xc + t * ncol);
        float p = 0.f;
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float4 xv = xp[q];
          p = fmaf(wf[4 * q + 0], xv.x, p);
          p = fmaf(wf[4 * q + 1], xv.y, p);
          p = fmaf(wf[4 * q + 2], xv.z, p);
          p = fmaf(wf[4 * q + 3], xv.w, p);
        }
        tot[t] = fmaf(s, p, tot[t]);
      }
    }
  } else {
    // low nibble of byte j = weight j, high nibble = weight j + group/2 (inside the group)
    float wl[16], wh[16];
#pragma unroll
    for (int k = 0; k < 4; k++) {
#pragma unroll
      for (int b = 0; b < 4; b++) {
        wl[4 * k + b] = u4_to_f(wd[k], 8 * b);
        wh[4 * k + b] = u4_to_f(wd[k], 8 * b + 4);
      }
    }
    if constexpr (G16) {
      // the chunk holds groups 2c (bytes 0..7) and 2c+1 (bytes 8..15); columns 32c .. 32c+31
      const float s0 = bf16f(sb[(size_t)(2 * c) * 32]);
      const float s1 = bf16f(sb[(size_t)(2 * c + 1) * 32]);
      const float* xc = xs + (c * 32 - col0);
#pragma unroll
      for (int t = 0; t < MT; t++) {
        if (t < Mloc) {
          const float4* xp = reinterpret_cast<const float4*>(xc + t * ncol);
          float p0 = 0.f, p1 = 0.f;
#pragma unroll
          for (int q = 0; q < 2; q++) {
            const float4 lo = xp[q], hi = xp[2 + q];
            p0 = fmaf(wl[4 * q + 0], lo.x, p0);
            p0 = fmaf(wl[4 * q + 1], lo.y, p0);
            p0 = fmaf(wl[4 * q + 2], lo.z, p0);
            p0 = fmaf(wl[4 * q + 3], lo.w, p0);
            p0 = fmaf(wh[4 * q + 0], hi.x, p0);
            p0 = fmaf(wh[4 * q + 1], hi.y, p0);
            p0 = fmaf(wh[4 * q + 2], hi.z, p0);
            p0 = fmaf(wh[4 * q + 3], hi.w, p0);
            const float4 lo1 = xp[4 + q], hi1 = xp[6 + q];
            p1 = fmaf(wl[8 + 4 * q + 0], lo1.x, p1);
            p1 = fmaf(wl[8 + 4 * q + 1], lo1.y, p1);
            p1 = fmaf(wl[8 + 4 * q + 2], lo1.z, p1);
            p1 = fmaf(wl[8 + 4 * q + 3], lo1.w, p1);
            p1 = fmaf(wh[8 + 4 * q + 0], hi1.x, p1);
            p1 = fmaf(wh[8 + 4 * q + 1], hi1.y, p1);
            p1 = fmaf(wh[8 + 4 * q + 2], hi1.z, p1);
            p1 = fmaf(wh[8 + 4 * q + 3], hi1.w, p1);
          }
          tot[t] = fmaf(s0, p0, tot[t]);
          tot[t] = fmaf(s1, p1, tot[t]);
        }
      }
    } else {
      const int half = group >> 1;
      const int g = (c * 32) / group;
      const int j0 = (c * 16) % half;
      const float s = bf16f(sb[(size_t)g * 32]);
      const float* xlo = xs + (g * group + j0 - col0);
      const float* xhi = xlo + half;
#pragma unroll
      for (int t = 0; t < MT; t++) {
        if (t < Mloc) {
          const float4* lp = reinterpret_cast<const float4*>(xlo + t * ncol);
          const float4* hp = reinterpret_cast<const float4*>(xhi + t * ncol);
          float p = 0.f;
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const float4 lo = lp[q], hi = hp[q];
            p = fmaf(wl[4 * q + 0], lo.x, p);
            p = fmaf(wl[4 * q + 1], lo.y, p);
            p = fmaf(wl[4 * q + 2], lo.z, p);
            p = fmaf(wl[4 * q + 3], lo.w, p);
            p = fmaf(wh[4 * q + 0], hi.x, p);
            p = fmaf(wh[4 * q + 1], hi.y, p);
            p = fmaf(wh[4 * q + 2], hi.z, p);
            p = fmaf(wh[4 * q + 3], hi.w, p);
          }
          tot[t] = fmaf(s, p, tot[t]);
        }
      }
    }
  }
}

// Split boundaries in chunks, aligned so that each CTA covers whole groups (int4, group >= 32).
__host__ __device__ inline void gemv_split(int nch, int bits, int group, int ksplit, int ks, int* c0, int* c1) {
  const int U = (bits == 4 && group >= 32) ? group / 32 : 1;
  const int nu = nch / U;
  *c0 = (int)((long long)ks * nu / ksplit) * U;
  *c1 = (int)((long long)(ks + 1) * nu / ksplit) * U;
}

// Each warp owns 32-row tiles (lane = row) in a grid-stride loop over the tiles; all warps of a CTA
// share the activations of one K slice (blockIdx.y) and one token group (blockIdx.z) staged in
// shared memory. K slices are summed in a fixed order by the last warp to finish a tile.
template <int BITS, bool G16, int MT>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(const GemvLaunch g) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float s_inv[MT];
  const int ks = blockIdx.y, z = blockIdx.z;
  const int tiles = g.w.rows_pad / 32;
  const int m0 = z * MT;
  const int Mloc = min(MT, g.M - m0);
  const int nch = g.w.chunks(), ngr = g.w.groups();
  int c0, c1;
  gemv_split(nch, BITS, g.w.group, g.ksplit, ks, &c0, &c1);
  constexpr int WPC = 128 / BITS;
  const int col0 = c0 * WPC, ncol = (c1 - c0) * WPC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int first_tile = blockIdx.x * GEMV_WARPS + warp;
  const int tile_stride = gridDim.x * GEMV_WARPS;

  // weights do not depend on the previous kernel: warm L2 with this warp's first tile, then wait
  pdl_trigger();
  if (lane == 0 && first_tile < tiles)
    prefetch_l2(g.w.data + ((size_t)first_tile * nch + c0) * 512, (uint32_t)(c1 - c0) * 512u);
  pdl_wait();

  // ---- stage the activations of this K slice (float4), normalised if a norm is fused ----
  float* xs = smem;  // [MT][ncol]
  const bool has_norm = g.norm_bf16 != nullptr || g.norm_f32 != nullptr;
  const int nc4 = ncol >> 2;
#pragma unroll 4
  for (int i = threadIdx.x; i < Mloc * nc4; i += GEMV_THREADS) {
    const int t = i / nc4, c4 = i - t * nc4;
    const float4 v = __ldg(reinterpret_cast<const float4*>(g.x + (size_t)(m0 + t) * g.x_stride + col0) + c4);
    reinterpret_cast<float4*>(xs + t * ncol)[c4] = v;
  }
  if (has_norm) {
    const int cols4 = g.w.cols >> 2;
    for (int t = warp; t < Mloc; t += GEMV_WARPS) {
      float ss = 0.f;
#pragma unroll 4
      for (int c4 = lane; c4 < cols4; c4 += 32) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(g.x + (size_t)(m0 + t) * g.x_stride) + c4);
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
      ss = warp_sum(ss);
      if (lane == 0) s_inv[t] = 1.0f / sqrtf(ss / (float)g.w.cols + g.eps);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < Mloc * ncol; i += GEMV_THREADS) {
      const int t = i / ncol, cc = i - t * ncol;
      const float w = g.norm_bf16 ? bf16f(g.norm_bf16[col0 + cc]) : g.norm_f32[col0 + cc];
      xs[t * ncol + cc] = xs[t * ncol + cc] * s_inv[t] * w;
    }
  }
  __syncthreads();

  // running argmax per token of this warp (LM head)
  float bv[MT];
  uint32_t bi[MT];
#pragma unroll
  for (int t = 0; t < MT; t++) {
    bv[t] = -CUDART_INF_F;
    bi[t] = 0xffffffffu;
  }

  for (int tile = first_tile; tile < tiles; tile += tile_stride) {
    float tot[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) tot[t] = 0.f;
    const uint8_t* db = g.w.data + (size_t)tile * nch * 512 + lane * 16;
    const uint16_t* sb = g.w.scales + (size_t)tile * ngr * 32 + lane;
    int c = c0;
    for (; c + GEMV_UNROLL <= c1; c += GEMV_UNROLL) {
      uint4 wv[GEMV_UNROLL];
#pragma unroll
      for (int u = 0; u < GEMV_UNROLL; u++) wv[u] = ld_stream_v4(db + (size_t)(c + u) * 512);
#pragma unroll
      for (int u = 0; u < GEMV_UNROLL; u++) gemv_chunk<BITS, G16, MT>(wv[u], c + u, col0, ncol, g.w.group, sb, xs, Mloc, tot);
    }
    for (; c < c1; c++) {
      const uint4 wv = ld_stream_v4(db + (size_t)c * 512);
      gemv_chunk<BITS, G16, MT>(wv, c, col0, ncol, g.w.group, sb, xs, Mloc, tot);
    }

    // ---- split-K: the last warp to finish this tile sums the K slices in order ----
    if (g.ksplit > 1) {
      float* part = g.partial + ((size_t)(z * tiles + tile) * g.ksplit) * MT * 32;
#pragma unroll
      for (int t = 0; t < MT; t++) part[((size_t)ks * MT + t) * 32 + lane] = tot[t];
      __threadfence();
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) {
        unsigned* tk = g.tickets + z * tiles + tile;
        last = atomicAdd(tk, 1u) == (unsigned)g.ksplit - 1;
        if (last) *tk = 0u;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence();
#pragma unroll
      for (int t = 0; t < MT; t++) tot[t] = 0.f;
      for (int k = 0; k < g.ksplit; k++) {
        float v[MT];
#pragma unroll
        for (int t = 0; t < MT; t++) v[t] = __ldcg(part + ((size_t)k * MT + t) * 32 + lane);
#pragma unroll
        for (int t = 0; t < MT; t++) tot[t] += v[t];
      }
    }

    // ---- epilogue of this tile (lane = row) ----
    const int r = tile * 32 + lane;
    if (g.epi == EPI_ARGMAX) {
#pragma unroll
      for (int t = 0; t < MT; t++) {
        if (t < Mloc) {
          float v = (r < g.n_valid_rows) ? tot[t] : -CUDART_INF_F;
          uint32_t idx = (uint32_t)(r + g.row_offset);
          if (g.logits && r < g.n_valid_rows) g.logits[(size_t)(m0 + t) * g.logits_stride + g.row_offset + r] = tot[t];
          warp_argmax(v, idx);
          if (arg_better(v, idx, bv[t], bi[t])) {
            bv[t] = v;
            bi[t] = idx;
          }
        }
      }
    } else if (g.epi == EPI_SWIGLU) {
      // rows interleaved in 16s: lanes 0..15 hold gate rows, lanes 16..31 the matching up rows
#pragma unroll
      for (int t = 0; t < MT; t++) {
        const float u = __shfl_down_sync(0xffffffffu, tot[t], 16);
        if (t < Mloc && lane < 16) {
          const float gt = tot[t];
          g.y[(size_t)(m0 + t) * g.y_stride + tile * 16 + lane] = gt / (1.0f + expf(-gt)) * u;
        }
      }
    } else if (r < g.w.rows) {
#pragma unroll
      for (int t = 0; t < MT; t++) {
        if (t < Mloc) {
          float* dst = g.y + (size_t)(m0 + t) * g.y_stride + r;
          if (g.epi == EPI_RESID) *dst += tot[t];
          else if (g.epi == EPI_BIAS_STORE) *dst = tot[t] + bf16f(g.bias[r]);
          else *dst = tot[t];
        }
      }
    }
  }

  if (g.epi != EPI_ARGMAX) return;
  // ---- LM head: one argmax part per CTA and token, then the last CTA finalises ----
  __shared__ float s_bv[GEMV_WARPS][MT];
  __shared__ uint32_t s_bi[GEMV_WARPS][MT];
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < MT; t++) {
      s_bv[warp][t] = bv[t];
      s_bi[warp][t] = bi[t];
    }
  }
  __syncthreads();
  if (threadIdx.x < Mloc) {
    const int t = threadIdx.x;
    float v = s_bv[0][t];
    uint32_t idx = s_bi[0][t];
    for (int w = 1; w < GEMV_WARPS; w++)
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

int gemv_mt(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16; }

static size_t gemv_smem(const QMat& w, int ksplit, int MT) {
  int maxcol = 0;
  for (int k = 0; k < ksplit; k++) {
    int c0, c1;
    gemv_split(w.chunks(), w.bits, w.group, ksplit, k, &c0, &c1);
    maxcol = max(maxcol, (c1 - c0) * (128 / w.bits));
  }
  return (size_t)MT * maxcol * 4;
}

int gemv_min_ksplit(const QMat& w, int M) {
  const int MT = gemv_mt(M);
  for (int ks = 1; ks <= 64; ks++)
    if (gemv_smem(w, ks, MT) <= 200 * 1024) return ks;
  LS_THROW(-1, "matrix too wide for the GEMV kernel");
}

// Grid (CTAs along the tiles) for a launch: enough CTAs to cover 2 per SM over all K slices and
// token groups, never more than one warp per tile.
int gemv_grid_x(const QMat& w, int ksplit, int M, int num_sms) {
  const int tiles = w.rows_pad / 32, nz = (M + 15) / 16;
  const int by_tiles = (tiles + GEMV_WARPS - 1) / GEMV_WARPS;
  const int want = max(1, (2 * num_sms + ksplit * nz - 1) / (ksplit * nz));
  return max(1, min(by_tiles, want));
}

template <int BITS, bool G16, int MT>
static void launch_gemv_t(const GemvLaunch& g, cudaStream_t s) {
  const size_t smem = gemv_smem(g.w, g.ksplit, MT);
  ensure_smem(gemv_kernel<BITS, G16, MT>, smem);
  const int gx = g.grid_x > 0 ? g.grid_x : (g.w.rows_pad / 32 + GEMV_WARPS - 1) / GEMV_WARPS;
  dim3 grid(gx, g.ksplit, (g.M + MT - 1) / MT);
  launch_pdl(gemv_kernel<BITS, G16, MT>, grid, dim3(GEMV_THREADS), smem, s, g);
}

template <int BITS, bool G16>
static void launch_gemv_b(const GemvLaunch& g, cudaStream_t s) {
  switch (gemv_mt(g.M)) {
    case 1: return launch_gemv_t<BITS, G16, 1>(g, s);
    case 2: return launch_gemv_t<BITS, G16, 2>(g, s);
    case 4: return launch_gemv_t<BITS, G16, 4>(g, s);
    case 8: return launch_gemv_t<BITS, G16, 8>(g, s);
    default: return launch_gemv_t<BITS, G16, 16>(g, s);
  }
}

void launch_gemv(const GemvLaunch& g, cudaStream_t s) {
  if (g.M <= 0) return;
  if (g.ksplit < gemv_min_ksplit(g.w, g.M)) LS_THROW(-1, "GEMV split too small for shared memory");
  if (g.w.bits == 8) return launch_gemv_b<8, false>(g, s);
  if (g.w.group == 16) return launch_gemv_b<4, true>(g, s);
  return launch_gemv_b<4, false>(g, s);
}

// ------------------------------------------------------------------------------------------------
// Attention
// ------------------------------------------------------------------------------------------------

constexpr int ATT_THREADS = 128;
constexpr int ATT_TILE = 64;
constexpr int ATT_MAX_SLOTS = 16;

__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }

// Cached K/V rows [p0, p0+64) below pos0 of kv head g into the f32 tiles (16-byte loads).
template <int HD>
__device__ __forceinline__ void att_load_cached(const AttnLaunch& a, const uint16_t* kcache, const uint16_t* vcache,
                                                const int32_t* pg, int g, int p0, int pos0, float* Ks, float* Vs) {
  constexpr int HP = HD + 1, V8 = HD / 8;
  for (int i = threadIdx.x; i < ATT_TILE * V8; i += ATT_THREADS) {
    const int pl = i / V8, d8 = (i - pl * V8) * 8;
    const int p = p0 + pl;
    if (p >= pos0) {  // rows of the block (written next) and rows past the context: zero
#pragma unroll
      for (int e = 0; e < 8; e++) {
        Ks[pl * HP + d8 + e] = 0.f;
        Vs[pl * HP + d8 + e] = 0.f;
      }
      continue;
    }
    const size_t base = kv_row(pg, a.page_shift, a.num_pages, g, p) * HD + d8;
    const uint4 kr = __ldg(reinterpret_cast<const uint4*>(kcache + base));
    const uint4 vr = __ldg(reinterpret_cast<const uint4*>(vcache + base));
    const __half* kh = reinterpret_cast<const __half*>(&kr);
    const __half* vh = reinterpret_cast<const __half*>(&vr);
#pragma unroll
    for (int e = 0; e < 8; e++) {
      Ks[pl * HP + d8 + e] = __half2float(kh[e]);
      Vs[pl * HP + d8 + e] = __half2float(vh[e]);
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const AttnLaunch a) {
  extern __shared__ __align__(16) float sm[];
  constexpr int HP = HD + 1;  // padded row: conflict-free column access
  constexpr int HALF = HD / 2;
  const int hh = blockIdx.x, slot = blockIdx.y, nslot = gridDim.y, sq = blockIdx.z;
  const int group = a.heads / a.kv_heads;
  const int g = hh / group;
  const int M = a.M;
  // written by the host before the pass (or, for batches launched without PDL, by an earlier kernel)
  const int pos0 = a.pos0 ? a.pos0[sq] : a.ctl->pos0;
  const int total = pos0 + M;
  const int ntiles = (total + ATT_TILE - 1) / ATT_TILE;
  const int H = a.heads * HD, KV = a.kv_heads * HD;
  const float* qkv = a.qkv + (size_t)sq * M * a.qkv_stride;
  float* out = a.out + (size_t)sq * M * H;
  uint16_t* kcache = a.k_cache;  // this layer's page pools, shared by the sequences
  uint16_t* vcache = a.v_cache;
  const int32_t* pg = a.pages + (size_t)sq * a.max_pages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* qs = sm;                       // [M][HD]
  float* Ks = qs + M * HD;              // [64][HP]
  float* Vs = Ks + ATT_TILE * HP;       // [64][HP]
  float* st = Vs + ATT_TILE * HP;       // [M][HD + 2]  (m, l, acc)
  const float scale = 1.0f / sqrtf((float)HD);

  pdl_trigger();
  // the cached part of the first tile does not depend on the previous kernel
  if (slot < ntiles) att_load_cached<HD>(a, kcache, vcache, pg, g, slot * ATT_TILE, pos0, Ks, Vs);
  for (int i = threadIdx.x; i < M * (HD + 2); i += ATT_THREADS) st[i] = (i % (HD + 2) == 0) ? -CUDART_INF_F : 0.f;
  pdl_wait();

  for (int i = threadIdx.x; i < M * HALF; i += ATT_THREADS) {
    const int t = i / HALF, d = i - t * HALF;
    const float2 cs = a.rope[(size_t)(pos0 + t) * HALF + d];
    const float* q = qkv + (size_t)t * a.qkv_stride + hh * HD;
    const float x1 = q[d], x2 = q[d + HALF];
    qs[t * HD + d] = x1 * cs.x - x2 * cs.y;
    qs[t * HD + d + HALF] = x2 * cs.x + x1 * cs.y;
  }

  const bool writer = (hh % group) == 0;
  bool first = true;
  for (int tile = slot; tile < ntiles; tile += nslot) {
    const int p0 = tile * ATT_TILE;
    if (!first) {
      __syncthreads();
      att_load_cached<HD>(a, kcache, vcache, pg, g, p0, pos0, Ks, Vs);
    }
    first = false;
    __syncthreads();
    // the block's new rows: RoPE on K, both rounded to f16 as the cache stores them
    const int nb = max(0, min(p0 + ATT_TILE, total) - max(p0, pos0));
    for (int i = threadIdx.x; i < nb * HALF; i += ATT_THREADS) {
      const int j = i / HALF, d = i - j * HALF;
      const int p = max(p0, pos0) + j, pl = p - p0, t = p - pos0;
      const float* kr = qkv + (size_t)t * a.qkv_stride + H + g * HD;
      const float* vr = qkv + (size_t)t * a.qkv_stride + H + KV + g * HD;
      const float2 cs = a.rope[(size_t)p * HALF + d];
      const float x1 = kr[d], x2 = kr[d + HALF];
      const float k1 = f16_round(x1 * cs.x - x2 * cs.y), k2 = f16_round(x2 * cs.x + x1 * cs.y);
      const float v1 = f16_round(vr[d]), v2 = f16_round(vr[d + HALF]);
      Ks[pl * HP + d] = k1;
      Ks[pl * HP + d + HALF] = k2;
      Vs[pl * HP + d] = v1;
      Vs[pl * HP + d + HALF] = v2;
      if (writer) {
        const size_t base = kv_row(pg, a.page_shift, a.num_pages, g, p) * HD;
        kcache[base + d] = __half_as_ushort(__float2half_rn(k1));
        kcache[base + d + HALF] = __half_as_ushort(__float2half_rn(k2));
        vcache[base + d] = __half_as_ushort(__float2half_rn(v1));
        vcache[base + d + HALF] = __half_as_ushort(__float2half_rn(v2));
      }
    }
    __syncthreads();
    for (int t = warp; t < M; t += ATT_THREADS / 32) {
      const int ctx = pos0 + t + 1;
      if (p0 >= ctx) continue;
      const float* q = qs + t * HD;
      float s0 = -CUDART_INF_F, s1 = -CUDART_INF_F;
      if (p0 + lane < ctx) {
        float acc = 0.f;
#pragma unroll 16
        for (int d = 0; d < HD; d++) acc = fmaf(q[d], Ks[lane * HP + d], acc);
        s0 = acc * scale;
      }
      if (p0 + 32 + lane < ctx) {
        float acc = 0.f;
#pragma unroll 16
        for (int d = 0; d < HD; d++) acc = fmaf(q[d], Ks[(lane + 32) * HP + d], acc);
        s1 = acc * scale;
      }
      const float tmax = warp_max(fmaxf(s0, s1));
      float* S = st + t * (HD + 2);
      const float m_old = S[0];
      const float m_new = fmaxf(m_old, tmax);
      const float corr = (m_old == -CUDART_INF_F) ? 0.f : expf(m_old - m_new);
      const float e0 = (s0 == -CUDART_INF_F) ? 0.f : expf(s0 - m_new);
      const float e1 = (s1 == -CUDART_INF_F) ? 0.f : expf(s1 - m_new);
      const float lsum = warp_sum(e0 + e1);
      constexpr int DPL = (HD + 31) / 32;  // value dims owned by each lane
      float acc[DPL];
#pragma unroll
      for (int j = 0; j < DPL; j++) {
        const int d = lane + 32 * j;
        acc[j] = (d < HD) ? S[2 + d] * corr : 0.f;
      }
#pragma unroll 8
      for (int pl = 0; pl < 32; pl++) {
        const float e = __shfl_sync(0xffffffffu, e0, pl);
#pragma unroll
        for (int j = 0; j < DPL; j++)
          if (lane + 32 * j < HD) acc[j] = fmaf(e, Vs[pl * HP + lane + 32 * j], acc[j]);
      }
#pragma unroll 8
      for (int pl = 0; pl < 32; pl++) {
        const float e = __shfl_sync(0xffffffffu, e1, pl);
#pragma unroll
        for (int j = 0; j < DPL; j++)
          if (lane + 32 * j < HD) acc[j] = fmaf(e, Vs[(pl + 32) * HP + lane + 32 * j], acc[j]);
      }
#pragma unroll
      for (int j = 0; j < DPL; j++)
        if (lane + 32 * j < HD) S[2 + lane + 32 * j] = acc[j];
      __syncwarp();
      if (lane == 0) {
        S[1] = S[1] * corr + lsum;
        S[0] = m_new;
      }
      __syncwarp();
    }
  }
  __syncthreads();

  if (nslot == 1) {
    for (int i = threadIdx.x; i < M * HD; i += ATT_THREADS) {
      const int t = i / HD, d = i - t * HD;
      const float* S = st + t * (HD + 2);
      out[(size_t)t * H + hh * HD + d] = S[2 + d] / S[1];
    }
    return;
  }
  // partial (m, l, acc) of this CTA for every token, then the combine in the last CTA of the head
  float* part = a.part + (((size_t)sq * a.heads + hh) * nslot + slot) * M * (HD + 2);
  for (int i = threadIdx.x; i < M * (HD + 2); i += ATT_THREADS) part[i] = st[i];
  if (!last_cta(a.tickets + (size_t)sq * a.heads + hh, (unsigned)nslot)) return;
  const float* all = a.part + ((size_t)sq * a.heads + hh) * nslot * M * (HD + 2);
  for (int i = threadIdx.x; i < M * HD; i += ATT_THREADS) {
    const int t = i / HD, d = i - t * HD;
    float ms[ATT_MAX_SLOTS], ls[ATT_MAX_SLOTS], as[ATT_MAX_SLOTS];
#pragma unroll
    for (int s = 0; s < ATT_MAX_SLOTS; s++) {
      if (s < nslot) {
        const float* P = all + ((size_t)s * M + t) * (HD + 2);
        ms[s] = __ldcg(P);
        ls[s] = __ldcg(P + 1);
        as[s] = __ldcg(P + 2 + d);
      }
    }
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int s = 0; s < ATT_MAX_SLOTS; s++)
      if (s < nslot) mx = fmaxf(mx, ms[s]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int s = 0; s < ATT_MAX_SLOTS; s++) {
      if (s < nslot && ms[s] != -CUDART_INF_F) {
        const float w = expf(ms[s] - mx);
        L += ls[s] * w;
        acc += as[s] * w;
      }
    }
    out[(size_t)t * H + hh * HD + d] = acc / L;
  }
}

template <int HD>
static void launch_attention_t(const AttnLaunch& a, size_t smem, cudaStream_t s) {
  ensure_smem(attention_kernel<HD>, smem);
  const dim3 grid(a.heads, std::min(a.max_splits, ATT_MAX_SLOTS), a.nseq);
  if (a.pdl) {
    launch_pdl(attention_kernel<HD>, grid, dim3(ATT_THREADS), smem, s, a);
  } else {
    attention_kernel<HD><<<grid, ATT_THREADS, smem, s>>>(a);
    LS_CUDA(cudaGetLastError());
  }
}

void launch_attention(const AttnLaunch& a, cudaStream_t s) {
  if (attention_tc_supported(a)) return launch_attention_tc(a, s);
  const size_t smem = ((size_t)a.M * a.hd + 2 * ATT_TILE * (a.hd + 1) + (size_t)a.M * (a.hd + 2)) * 4;
  switch (a.hd) {
    case 16: return launch_attention_t<16>(a, smem, s);
    case 32: return launch_attention_t<32>(a, smem, s);
    case 64: return launch_attention_t<64>(a, smem, s);
    case 128: return launch_attention_t<128>(a, smem, s);
    default:
      LS_THROW(-1, "head dimension " + std::to_string(a.hd) + " is not supported by the CUDA attention kernel (16, 32, 64, 128)");
  }
}

// ------------------------------------------------------------------------------------------------
// L2 eviction for timing loops: reads a buffer larger than L2, so the lines it leaves are clean
// (a write would leave dirty lines whose write-back the next, timed kernel would pay for).
// ------------------------------------------------------------------------------------------------
__global__ void l2_evict_kernel(const uint4* p, size_t n, unsigned* sink) {
  unsigned acc = 0;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 v = __ldcg(p + i);
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  acc = __reduce_xor_sync(0xffffffffu, acc);
  if ((threadIdx.x & 31) == 0 && acc == 0x9e3779b9u) sink[blockIdx.x & 255] = acc;  // keeps the loads
}

void launch_l2_evict(const void* buf, size_t bytes, unsigned* sink, cudaStream_t s) {
  l2_evict_kernel<<<1184, 512, 0, s>>>(static_cast<const uint4*>(buf), bytes / 16, sink);
  LS_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------------------------------
// Embedding gather + dequantisation (bit-exact with src/kernels.rs:95-121)
// ------------------------------------------------------------------------------------------------

// Dequantised embedding row of token tok into xr (the CTA's threads share the columns).
__device__ __forceinline__ void embed_row(const QMat& e, uint32_t tok, float* xr, int hidden) {
  const int nch = e.chunks();
  const uint8_t* row = e.data + ((size_t)(tok / 32) * nch) * 512 + (tok % 32) * 16;
  const uint16_t* sc = e.scales + (size_t)(tok / 32) * e.groups() * 32 + (tok % 32);
  if (e.bits == 16) {  // bf16 rows: 8 values per 16-byte chunk, widened exactly
    for (int c = threadIdx.x; c < hidden; c += blockDim.x)
      xr[c] = bf16f(*reinterpret_cast<const uint16_t*>(row + (size_t)(c / 8) * 512 + (c % 8) * 2));
    return;
  }
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    float q;
    int g = c / e.group;
    if (e.bits == 8) {
      const int ch = c / 16, b = c % 16;
      q = (float)(int8_t)row[(size_t)ch * 512 + b];
    } else {
      const int half = e.group / 2;
      const int j = c % e.group;
      const int byte_in_row = g * half + (j < half ? j : j - half);
      const uint8_t by = row[(size_t)(byte_in_row / 16) * 512 + byte_in_row % 16];
      q = (float)((j < half ? (by & 15) : (by >> 4)) - 8);
    }
    xr[c] = q * bf16f(sc[(size_t)g * 32]);
  }
}

__global__ void embed_kernel(const QMat e, const Ctl* ctl, float* x, int hidden, int vocab) {
  const int t = blockIdx.x;
  const uint32_t tok = ctl->tokens[t];
  float* xr = x + (size_t)t * hidden;
  if (tok >= (uint32_t)vocab) {
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) xr[c] = 0.f;
    if (threadIdx.x == 0) const_cast<Ctl*>(ctl)->err = 2;
    return;
  }
  embed_row(e, tok, xr, hidden);
}

__global__ void embed_tokens_kernel(const QMat e, const uint32_t* tokens, float* x, int hidden, int vocab, int* err) {
  const int t = blockIdx.x;
  const uint32_t tok = tokens[t];
  float* xr = x + (size_t)t * hidden;
  if (tok >= (uint32_t)vocab) {
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) xr[c] = 0.f;
    if (threadIdx.x == 0) atomicExch(err, 2);
    return;
  }
  embed_row(e, tok, xr, hidden);
}

void launch_embed_tokens(const QMat& e, const uint32_t* tokens, int T, float* x, int hidden, int vocab, int* err,
                         cudaStream_t s) {
  embed_tokens_kernel<<<T, 256, 0, s>>>(e, tokens, x, hidden, vocab, err);
  LS_CUDA(cudaGetLastError());
}

// One warp per row: the first maximum over the per-CTA parts (value, then lower index).
__global__ void batch_argmax_kernel(const ArgPart* parts, int nparts, int T, uint32_t* argmax) {
  const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= T) return;
  float v = -CUDART_INF_F;
  uint32_t idx = 0xffffffffu;
  for (int k = lane; k < nparts; k += 32) {
    const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(parts + (size_t)k * T + t));
    const float pv = __uint_as_float(raw.x);
    if (arg_better(pv, raw.y, v, idx)) {
      v = pv;
      idx = raw.y;
    }
  }
  warp_argmax(v, idx);
  if (lane == 0) argmax[t] = idx;
}

// One warp per row: the first maximum over the per-CTA parts, kept as a (value, index) part
// (tensor-parallel heads gather these across ranks).
__global__ void row_best_kernel(const ArgPart* parts, int nparts, int T, ArgPart* best) {
  const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= T) return;
  float v = -CUDART_INF_F;
  uint32_t idx = 0xffffffffu;
  for (int k = lane; k < nparts; k += 32) {
    const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(parts + (size_t)k * T + t));
    const float pv = __uint_as_float(raw.x);
    if (arg_better(pv, raw.y, v, idx)) {
      v = pv;
      idx = raw.y;
    }
  }
  warp_argmax(v, idx);
  if (lane == 0) best[t] = ArgPart{v, idx};
}

void launch_row_best(const ArgPart* parts, int nparts, int T, ArgPart* best, cudaStream_t s) {
  row_best_kernel<<<(T + 7) / 8, 256, 0, s>>>(parts, nparts, T, best);
  LS_CUDA(cudaGetLastError());
}

__global__ void add_rows_kernel(float* __restrict__ x, const float* __restrict__ y, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) x[i] += y[i];
}

void launch_add(float* x, const float* y, size_t n, cudaStream_t s) {
  add_rows_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 2368), 256, 0, s>>>(x, y, n);
  LS_CUDA(cudaGetLastError());
}

// src/spec.rs:121-125 per sequence: m = longest prefix of guesses the target agrees with, next =
// the target's token after it (correction or bonus).
__global__ void batch_accept_kernel(const uint32_t* argmax, const uint32_t* tokens, int nseq, int M, uint32_t* m_out,
                                    uint32_t* next_out) {
  const int sq = blockIdx.x * blockDim.x + threadIdx.x;
  if (sq >= nseq) return;
  const uint32_t* am = argmax + (size_t)sq * M;
  const uint32_t* tk = tokens + (size_t)sq * M;
  int m = 0;
  while (m < M - 1 && am[m] == tk[m + 1]) m++;
  m_out[sq] = (uint32_t)m;
  next_out[sq] = am[m];
}

void launch_batch_accept(const ArgPart* parts, int nparts, int T, int M, const uint32_t* tokens, uint32_t* argmax,
                         uint32_t* m_out, uint32_t* next_out, cudaStream_t s) {
  batch_argmax_kernel<<<(T + 7) / 8, 256, 0, s>>>(parts, nparts, T, argmax);
  LS_CUDA(cudaGetLastError());
  const int nseq = T / M;
  batch_accept_kernel<<<(nseq + 127) / 128, 128, 0, s>>>(argmax, tokens, nseq, M, m_out, next_out);
  LS_CUDA(cudaGetLastError());
}

void launch_embed(const QMat& e, const Ctl* ctl, float* x, int hidden, int M, cudaStream_t s) {
  embed_kernel<<<M, 256, 0, s>>>(e, ctl, x, hidden, e.rows);
  LS_CUDA(cudaGetLastError());
}

// Streaming mode: the embedding table stays in pinned host memory in the file layout; the rows of
// the block's tokens are read through the mapped pointer (one row per token crosses the link).
// One stored embedding row (host-mapped .lsq row format) dequantised into xr.
__device__ __forceinline__ void embed_raw_row(const uint8_t* table, size_t row_bytes, int bits, int group, uint32_t tok,
                                              float* xr, int hidden) {
  const uint8_t* row = table + (size_t)tok * row_bytes;
  const uint8_t* sc = row + (size_t)hidden * bits / 8;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    const int g = c / group;
    float q;
    if (bits == 8) {
      q = (float)(int8_t)row[c];
    } else {
      const int half = group / 2, j = c % group;
      const uint8_t by = row[(size_t)g * half + (j < half ? j : j - half)];
      q = (float)((j < half ? (by & 15) : (by >> 4)) - 8);
    }
    xr[c] = q * __uint_as_float((uint32_t)(sc[2 * g] | (sc[2 * g + 1] << 8)) << 16);
  }
}

__global__ void embed_raw_kernel(const uint8_t* table, size_t row_bytes, int bits, int group, const Ctl* ctl, float* x,
                                 int hidden, int vocab) {
  const int t = blockIdx.x;
  const uint32_t tok = ctl->tokens[t];
  float* xr = x + (size_t)t * hidden;
  if (tok >= (uint32_t)vocab) {
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) xr[c] = 0.f;
    if (threadIdx.x == 0) const_cast<Ctl*>(ctl)->err = 2;
    return;
  }
  embed_raw_row(table, row_bytes, bits, group, tok, xr, hidden);
}

__global__ void embed_raw_tokens_kernel(const uint8_t* table, size_t row_bytes, int bits, int group, const uint32_t* tokens,
                                        float* x, int hidden, int vocab, int* err) {
  const int t = blockIdx.x;
  const uint32_t tok = tokens[t];
  float* xr = x + (size_t)t * hidden;
  if (tok >= (uint32_t)vocab) {
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) xr[c] = 0.f;
    if (threadIdx.x == 0) atomicExch(err, 2);
    return;
  }
  embed_raw_row(table, row_bytes, bits, group, tok, xr, hidden);
}

void launch_embed_raw_tokens(const uint8_t* table, size_t row_bytes, int bits, int group, const uint32_t* tokens, float* x,
                             int hidden, int vocab, int T, int* err, cudaStream_t s) {
  embed_raw_tokens_kernel<<<T, 256, 0, s>>>(table, row_bytes, bits, group, tokens, x, hidden, vocab, err);
  LS_CUDA(cudaGetLastError());
}

void launch_embed_raw(const uint8_t* table, size_t row_bytes, int bits, int group, const Ctl* ctl, float* x, int hidden,
                      int vocab, int M, cudaStream_t s) {
  embed_raw_kernel<<<M, 256, 0, s>>>(table, row_bytes, bits, group, ctl, x, hidden, vocab);
  LS_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------------------------------
// Repack: stored rows (packed ints ‖ bf16 scales, src/weights.rs:26-31) -> tiled planes
// ------------------------------------------------------------------------------------------------

__global__ void repack_kernel(const RepackSrc src, int bits, int group, int cols, uint8_t* data, uint16_t* scales,
                              int rows_pad) {
  const int d = blockIdx.x;
  const int tile = d / 32, lr = d % 32;
  const size_t dbytes = (size_t)cols * bits / 8;
  const int ng = bits == 16 ? 0 : cols / group;  // bf16 rows carry no scales
  const size_t row_bytes = dbytes + (size_t)ng * 2;
  const int nch = cols * bits / 128;
  // find the source row
  const uint8_t* s = nullptr;
  if (src.interleave16) {
    const int seg = lr < 16 ? 0 : 1;
    const int sr = tile * 16 + (lr & 15);
    if (sr < src.seg_rows[seg]) s = src.seg[seg] + (size_t)sr * row_bytes;
  } else {
    int r = d;
    for (int k = 0; k < src.nseg; k++) {
      if (r < src.seg_rows[k]) {
        s = src.seg[k] + (size_t)r * row_bytes;
        break;
      }
      r -= src.seg_rows[k];
    }
  }
  for (int i = threadIdx.x; i < nch * 16; i += blockDim.x) {
    const int ch = i / 16, b = i % 16;
    data[((size_t)tile * nch + ch) * 512 + lr * 16 + b] = s ? s[(size_t)ch * 16 + b] : (uint8_t)0;
  }
  for (int gi = threadIdx.x; gi < ng; gi += blockDim.x) {
    uint16_t v = 0;
    if (s) v = (uint16_t)(s[dbytes + 2 * gi] | (s[dbytes + 2 * gi + 1] << 8));
    scales[((size_t)tile * ng + gi) * 32 + lr] = v;
  }
}

void launch_repack(const RepackSrc& src, int bits, int group, int cols, uint8_t* data, uint16_t* scales, int rows_pad,
                   cudaStream_t s) {
  repack_kernel<<<rows_pad, 128, 0, s>>>(src, bits, group, cols, data, scales, rows_pad);
  LS_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------------------------------
// Control block
// ------------------------------------------------------------------------------------------------

__global__ void set_ctl_kernel(Ctl* ctl, int pos0, int M, int n_logits, int mode, const uint32_t* toks, int ntok) {
  if (threadIdx.x == 0) {
    if (pos0 >= 0) ctl->pos0 = pos0;
    if (M >= 0) ctl->M = M;
    if (n_logits >= 0) ctl->n_logits = n_logits;
    if (mode >= 0) ctl->mode = mode;
    ctl->err = 0;
  }
  if (toks)
    for (int i = threadIdx.x; i < ntok; i += blockDim.x) ctl->tokens[i] = toks[i];
}

void launch_set_ctl(Ctl* ctl, int pos0, int M, int n_logits, int mode, const uint32_t* tokens_dev, cudaStream_t s) {
  set_ctl_kernel<<<1, 128, 0, s>>>(ctl, pos0, M, n_logits, mode, tokens_dev, tokens_dev ? M : 0);
  LS_CUDA(cudaGetLastError());
}

__global__ void advance_kernel(Ctl* ctl) {
  if (threadIdx.x == 0) ctl->pos0 += ctl->M;
}
void launch_advance(Ctl* ctl, cudaStream_t s) {
  advance_kernel<<<1, 32, 0, s>>>(ctl);
  LS_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------------------------------
// Quantizer: one thread per (row, group); float steps written with explicit _rn intrinsics so that
// nothing is contracted into an FMA (the Rust reference never fuses).
// ------------------------------------------------------------------------------------------------

__device__ __forceinline__ float bf16_round_dev(float v) {
  const uint32_t b = __float_as_uint(v);
  if ((b & 0x7fffffffu) > 0x7f800000u) return v;
  const uint32_t lsb = (b >> 16) & 1u;
  return __uint_as_float((b + 0x7fffu + lsb) & 0xffff0000u);
}

__device__ __forceinline__ float qround_dev(float v, float inv, float qmax) {
  float r = roundf(__fmul_rn(v, inv));
  r = r < -qmax ? -qmax : r;
  r = r > qmax ? qmax : r;
  return r;
}

__constant__ float kClips[9] = {1.0f, 0.95f, 0.9f, 0.85f, 0.8f, 0.75f, 0.7f, 0.65f, 0.6f};

__global__ void quantize_kernel(const uint16_t* src, int rows, int cols, int bits, int group, int clip, uint8_t* dst,
                                double* err_norm) {
  const long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int ng = cols / group;
  if (gi >= (long long)rows * ng) return;
  const int r = (int)(gi / ng), g = (int)(gi % ng);
  const uint16_t* w = src + (size_t)r * cols + (size_t)g * group;
  const size_t dbytes = (size_t)cols * bits / 8;
  uint8_t* out = dst + (size_t)r * (dbytes + (size_t)ng * 2);
  const float qmax = bits == 8 ? 127.0f : 7.0f;
  float amax = 0.0f;
  double norm = 0.0;
  for (int i = 0; i < group; i++) {
    const float v = bf16f(w[i]);
    amax = fmaxf(amax, fabsf(v));
    norm += (double)__fmul_rn(v, v);
  }
  float best_s = 0.0f;
  double best_e = CUDART_INF;
  if (amax != 0.0f && isfinite(amax)) {
    const int nclip = clip ? 9 : 1;
    for (int ci = 0; ci < nclip; ci++) {
      const float s = bf16_round_dev(__fdiv_rn(__fmul_rn(kClips[ci], amax), qmax));
      if (s == 0.0f) continue;
      const float inv = __fdiv_rn(1.0f, s);
      double e = 0.0;
      for (int i = 0; i < group; i++) {
        const float v = bf16f(w[i]);
        const float d = __fsub_rn(v, __fmul_rn(qround_dev(v, inv, qmax), s));
        e += (double)__fmul_rn(d, d);
      }
      if (e < best_e) {
        best_e = e;
        best_s = s;
      }
    }
  }
  double err;
  if (best_s == 0.0f) {
    err = 0.0;
    for (int i = 0; i < group; i++) {
      const float v = bf16f(w[i]);
      err += (double)__fmul_rn(v, v);
    }
  } else {
    err = best_e;
  }
  const float inv = best_s == 0.0f ? 0.0f : __fdiv_rn(1.0f, best_s);
  if (bits == 8) {
    for (int i = 0; i < group; i++) {
      const int8_t q = best_s == 0.0f ? 0 : (int8_t)qround_dev(bf16f(w[i]), inv, qmax);
      out[(size_t)g * group + i] = (uint8_t)q;
    }
  } else {
    const int half = group / 2;
    for (int j = 0; j < half; j++) {
      const int qa = best_s == 0.0f ? 0 : (int)qround_dev(bf16f(w[j]), inv, qmax);
      const int qb = best_s == 0.0f ? 0 : (int)qround_dev(bf16f(w[j + half]), inv, qmax);
      out[(size_t)g * half + j] = (uint8_t)((qa + 8) | ((qb + 8) << 4));
    }
  }
  const uint16_t sb = (uint16_t)(__float_as_uint(best_s) >> 16);
  out[dbytes + 2 * g] = (uint8_t)(sb & 0xff);
  out[dbytes + 2 * g + 1] = (uint8_t)(sb >> 8);
  if (err_norm) {
    atomicAdd(err_norm, err);
    atomicAdd(err_norm + 1, norm);
  }
}

void launch_quantize_rows(const uint16_t* src_bf16, int rows, int cols, int bits, int group, int clip, uint8_t* dst,
                          double* err_norm, cudaStream_t s) {
  const long long n = (long long)rows * (cols / group);
  const int th = 128;
  quantize_kernel<<<(unsigned)((n + th - 1) / th), th, 0, s>>>(src_bf16, rows, cols, bits, group, clip, dst, err_norm);
  LS_CUDA(cudaGetLastError());
}



}  // namespace ls
