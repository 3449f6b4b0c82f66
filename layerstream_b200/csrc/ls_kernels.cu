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

#include "ls_device.cuh"
#include "ls_internal.h"

namespace ls {

// ------------------------------------------------------------------------------------------------
// GEMV
// ------------------------------------------------------------------------------------------------

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;
constexpr int GEMV_UNROLL = 8;  // 16-byte loads in flight per lane

// Reduces the per-CTA argmax parts of every token (first-maximum rule), then applies the
// acceptance rule of src/spec.rs:121-125 (verify) or records the next token (forward).
// Run by one whole CTA of at most GEMV_THREADS threads.
__device__ void argmax_finalize_block(const ArgPart* parts, int nparts, int M, Ctl* ctl) {
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

template <int BITS, bool G16, int MT>
static void launch_gemv_t(const GemvLaunch& g, cudaStream_t s) {
  const size_t smem = gemv_smem(g.w, g.ksplit, MT);
  static int configured[64] = {0};  // per device: the attribute is a per-device setting
  int dev = 0;
  LS_CUDA(cudaGetDevice(&dev));
  if (smem > 48 * 1024 && configured[dev & 63] < (int)smem) {
    LS_CUDA(cudaFuncSetAttribute(gemv_kernel<BITS, G16, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured[dev & 63] = (int)smem;
  }
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

__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const AttnLaunch a) {
  extern __shared__ __align__(16) float sm[];
  constexpr int HP = HD + 1;  // padded row: conflict-free column access
  constexpr int HALF = HD / 2;
  const int hh = blockIdx.x, slot = blockIdx.y, nslot = gridDim.y;
  const int group = a.heads / a.kv_heads;
  const int g = hh / group;
  const int M = a.M;
  const int pos0 = a.ctl->pos0;
  const int total = pos0 + M;
  const int ntiles = (total + ATT_TILE - 1) / ATT_TILE;
  const int H = a.heads * HD, KV = a.kv_heads * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* qs = sm;                       // [M][HD]
  float* Ks = qs + M * HD;              // [64][HP]
  float* Vs = Ks + ATT_TILE * HP;       // [64][HP]
  float* st = Vs + ATT_TILE * HP;       // [M][HD + 2]  (m, l, acc)
  const float scale = 1.0f / sqrtf((float)HD);

  for (int i = threadIdx.x; i < M * HALF; i += ATT_THREADS) {
    const int t = i / HALF, d = i - t * HALF;
    const float2 cs = a.rope[(size_t)(pos0 + t) * HALF + d];
    const float* q = a.qkv + (size_t)t * a.qkv_stride + hh * HD;
    const float x1 = q[d], x2 = q[d + HALF];
    qs[t * HD + d] = x1 * cs.x - x2 * cs.y;
    qs[t * HD + d + HALF] = x2 * cs.x + x1 * cs.y;
  }
  for (int i = threadIdx.x; i < M * (HD + 2); i += ATT_THREADS) st[i] = (i % (HD + 2) == 0) ? -CUDART_INF_F : 0.f;
  __syncthreads();

  const bool writer = (hh % group) == 0;
  for (int tile = slot; tile < ntiles; tile += nslot) {
    const int p0 = tile * ATT_TILE;
    for (int i = threadIdx.x; i < ATT_TILE * HALF; i += ATT_THREADS) {
      const int pl = i / HALF, d = i - pl * HALF;
      const int p = p0 + pl;
      float k1 = 0.f, k2 = 0.f, v1 = 0.f, v2 = 0.f;
      if (p < pos0) {
        const size_t base = ((size_t)g * a.max_ctx + p) * HD;
        k1 = __half2float(__ushort_as_half(a.k_cache[base + d]));
        k2 = __half2float(__ushort_as_half(a.k_cache[base + d + HALF]));
        v1 = __half2float(__ushort_as_half(a.v_cache[base + d]));
        v2 = __half2float(__ushort_as_half(a.v_cache[base + d + HALF]));
      } else if (p < total) {
        const int t = p - pos0;
        const float* kr = a.qkv + (size_t)t * a.qkv_stride + H + g * HD;
        const float* vr = a.qkv + (size_t)t * a.qkv_stride + H + KV + g * HD;
        const float2 cs = a.rope[(size_t)p * HALF + d];
        const float x1 = kr[d], x2 = kr[d + HALF];
        k1 = f16_round(x1 * cs.x - x2 * cs.y);
        k2 = f16_round(x2 * cs.x + x1 * cs.y);
        v1 = f16_round(vr[d]);
        v2 = f16_round(vr[d + HALF]);
        if (writer) {
          const size_t base = ((size_t)g * a.max_ctx + p) * HD;
          a.k_cache[base + d] = __half_as_ushort(__float2half_rn(k1));
          a.k_cache[base + d + HALF] = __half_as_ushort(__float2half_rn(k2));
          a.v_cache[base + d] = __half_as_ushort(__float2half_rn(v1));
          a.v_cache[base + d + HALF] = __half_as_ushort(__float2half_rn(v2));
        }
      }
      Ks[pl * HP + d] = k1;
      Ks[pl * HP + d + HALF] = k2;
      Vs[pl * HP + d] = v1;
      Vs[pl * HP + d + HALF] = v2;
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
    __syncthreads();
  }

  // partial (m, l, acc) of this CTA for every token, then the combine in the last CTA of the head
  float* part = a.part + ((size_t)hh * nslot + slot) * M * (HD + 2);
  for (int i = threadIdx.x; i < M * (HD + 2); i += ATT_THREADS) part[i] = st[i];
  if (!last_cta(a.tickets + hh, (unsigned)nslot)) return;
  const float* all = a.part + (size_t)hh * nslot * M * (HD + 2);
  for (int i = threadIdx.x; i < M * HD; i += ATT_THREADS) {
    const int t = i / HD, d = i - t * HD;
    float mx = -CUDART_INF_F;
    for (int s = 0; s < nslot; s++) mx = fmaxf(mx, __ldcg(all + ((size_t)s * M + t) * (HD + 2)));
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < nslot; s++) {
      const float* P = all + ((size_t)s * M + t) * (HD + 2);
      const float ms = __ldcg(P);
      if (ms == -CUDART_INF_F) continue;
      const float w = expf(ms - mx);
      L += __ldcg(P + 1) * w;
      acc += __ldcg(P + 2 + d) * w;
    }
    a.out[(size_t)t * H + hh * HD + d] = acc / L;
  }
}

template <int HD>
static void launch_attention_t(const AttnLaunch& a, size_t smem, cudaStream_t s) {
  static size_t configured[64] = {0};
  int dev = 0;
  LS_CUDA(cudaGetDevice(&dev));
  if (smem > 48 * 1024 && smem > configured[dev & 63]) {
    LS_CUDA(cudaFuncSetAttribute(attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured[dev & 63] = smem;
  }
  attention_kernel<HD><<<dim3(a.heads, a.max_splits), ATT_THREADS, smem, s>>>(a);
  LS_CUDA(cudaGetLastError());
}

void launch_attention(const AttnLaunch& a, cudaStream_t s) {
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
// Embedding gather + dequantisation (bit-exact with src/kernels.rs:95-121)
// ------------------------------------------------------------------------------------------------

__global__ void embed_kernel(const QMat e, const Ctl* ctl, float* x, int hidden, int vocab) {
  const int t = blockIdx.x;
  const uint32_t tok = ctl->tokens[t];
  float* xr = x + (size_t)t * hidden;
  if (tok >= (uint32_t)vocab) {
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) xr[c] = 0.f;
    if (threadIdx.x == 0) const_cast<Ctl*>(ctl)->err = 2;
    return;
  }
  const int nch = e.chunks();
  const uint8_t* row = e.data + ((size_t)(tok / 32) * nch) * 512 + (tok % 32) * 16;
  const uint16_t* sc = e.scales + (size_t)(tok / 32) * e.groups() * 32 + (tok % 32);
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

void launch_embed(const QMat& e, const Ctl* ctl, float* x, int hidden, int M, cudaStream_t s) {
  embed_kernel<<<M, 256, 0, s>>>(e, ctl, x, hidden, e.rows);
  LS_CUDA(cudaGetLastError());
}

// Streaming mode: the embedding table stays in pinned host memory in the file layout; the rows of
// the block's tokens are read through the mapped pointer (one row per token crosses the link).
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
  const size_t row_bytes = dbytes + (size_t)cols / group * 2;
  const int nch = cols * bits / 128, ng = cols / group;
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
// Bounded wait on an mbarrier phase. Returns false (and raises the CTA's abort flag) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  for (uint32_t i = 0; i < (1u << 24); i++) {
    if (mbar_try(b, parity)) return true;
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
__device__ __forceinline__ uint32_t h2_splat(float s) {
  const __half h = __float2half_rn(s);
  const uint16_t u = __half_as_ushort(h);
  return (uint32_t)u | ((uint32_t)u << 16);
}

}  // namespace tc

constexpr int TC_THREADS = 128;
constexpr int TC_STAGES = 4;

// K elements per A block: one group for int4 groups of 128, else 64.
__host__ __device__ constexpr int tc_kb(int bits, int group) { return (bits == 4 && group > 64) ? group : 64; }
// Group scales one row needs per A block.
__host__ __device__ constexpr int tc_ns(int bits, int group) {
  return tc_kb(bits, group) >= group ? tc_kb(bits, group) / group : 1;
}

template <int BITS, int G, int NT>
__global__ void __launch_bounds__(TC_THREADS) gemv_tc_kernel(const GemvLaunch g) {
  constexpr int KB = tc_kb(BITS, G);   // K per A block
  constexpr int NS = tc_ns(BITS, G);   // scales per row per block
  constexpr int WPC = 128 / BITS;      // weights per 16-byte chunk
  constexpr int CPB = KB / WPC;        // chunks per block
  constexpr int ACOLS = KB / 2;        // TMEM columns of one A buffer (two f16 per column)
  constexpr int TCOLS = (2 * ACOLS + NT <= 128) ? 128 : 256;
  constexpr int NW = TC_THREADS / 32;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ uint64_t bar_a[2], bar_d;
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
  if (threadIdx.x < 4 && first < tiles128) {
    const int t32 = first * 4 + threadIdx.x;
    if (t32 < tiles32) prefetch_l2(g.w.data + ((size_t)t32 * nch + c0) * 512, (uint32_t)(c1 - c0) * 512u);
  }
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar_a[0], 1);
    tc::mbar_init(&bar_a[1], 1);
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
  pdl_wait();

  // ---- stage the activations as f16 in the canonical K-major layout (tokens >= M are zero) ----
  const bool has_norm = g.norm_bf16 != nullptr || g.norm_f32 != nullptr;
  if (has_norm) {
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
    __syncthreads();
  }
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
            const float wn = g.norm_bf16 ? bf16f(g.norm_bf16[col]) : g.norm_f32[col];
            v[e] = v[e] * s_inv[t] * wn;
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
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  const uint32_t tmem = s_tmem;
  tc::fence_after();
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t d_col = tmem + 2 * ACOLS;
  const uint32_t idesc = tc::idesc_f16(NT);
  const uint32_t xb_addr = tc::su32(xb);
  const uint32_t ring_addr = tc::su32(ring) + (uint32_t)threadIdx.x * CPB * 16;
  constexpr uint32_t kStageStride = TC_THREADS * CPB * 16;
  const uint32_t sub8 = BITS == 8 ? 0x64806480u : 0x64086408u;  // 1152 | 1032 as f16x2

  uint32_t uses[2] = {0u, 0u};
  uint32_t tiles_done = 0;
  bool failed = false;

  for (int t128 = first; t128 < tiles128; t128 += gridDim.x) {
    const int t32 = t128 * 4 + warp;
    const bool row_valid = t32 < tiles32;
    const uint8_t* db = g.w.data + ((size_t)(row_valid ? t32 : 0) * nch) * 512 + lane * 16;
    const uint16_t* sb = g.w.scales + (size_t)(row_valid ? t32 : 0) * ngr * 32 + lane;
    auto load_scales = [&](int kb, uint32_t (&sc)[NS]) {
#pragma unroll
      for (int s = 0; s < NS; s++) {
        const int gi = (kb * KB) / G + s;
        sc[s] = tc::h2_splat(row_valid && kb < kb1 ? bf16f(sb[(size_t)gi * 32]) : 0.f);
      }
    };
    uint32_t scur[NS], snext[NS];
    load_scales(kb0, scur);
#pragma unroll
    for (int s = 0; s < TC_STAGES - 1; s++) {
      const int kb = kb0 + s;
      if (kb < kb1 && row_valid) {
#pragma unroll
        for (int q = 0; q < CPB; q++) tc::cp_async16(ring_addr + s * kStageStride + q * 16, db + (size_t)(kb * CPB + q) * 512);
      }
      tc::cp_commit();
    }
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
      load_scales(kb + 1, snext);
      tc::cp_wait<TC_STAGES - 1>();
      uint4 wv[CPB];
      const uint8_t* rs = ring + (size_t)(it % TC_STAGES) * kStageStride + (size_t)threadIdx.x * CPB * 16;
#pragma unroll
      for (int q = 0; q < CPB; q++) wv[q] = row_valid ? *reinterpret_cast<const uint4*>(rs + q * 16) : make_uint4(0, 0, 0, 0);

      // ---- dequantise one K block of this row into f16 pairs in K order ----
      uint32_t a[ACOLS];
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
            a[base + 4 + j / 2] = tc::h2_sub_mul(((p0 >> 4) & 0x000F000Fu) | 0x64006400u, sub8, sc);
            a[base + 4 + j / 2 + 1] = tc::h2_sub_mul(((p1 >> 4) & 0x000F000Fu) | 0x64006400u, sub8, sc);
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
            a[hi] = tc::h2_sub_mul(((p0 >> 4) & 0x000F000Fu) | 0x64006400u, sub8, sc);
            a[hi + 1] = tc::h2_sub_mul(((p1 >> 4) & 0x000F000Fu) | 0x64006400u, sub8, sc);
          }
        }
      }
#pragma unroll
      for (int s = 0; s < NS; s++) scur[s] = snext[s];

      // ---- A buffer reuse: the MMAs that read it two blocks ago must have completed ----
      const int b = it & 1;
      bool fail = false;
      if (uses[b] > 0) fail = !tc::mbar_wait(&bar_a[b], (uses[b] - 1) & 1, &s_abort);
      if (!fail) {
        tc::fence_after();
#pragma unroll
        for (int q = 0; q < ACOLS / 16; q++) tc::st16(tmem + lane_base + b * ACOLS + q * 16, a + q * 16);
        tc::wait_st();
      }
      tc::fence_before();
      if (__syncthreads_or(fail)) {
        failed = true;
        break;
      }
      if (threadIdx.x == 0) {
        tc::fence_after();
#pragma unroll
        for (int j = 0; j < KB / 16; j++) {
          const uint32_t kpos = (uint32_t)(it * KB + j * 16);  // K offset inside the staged slice
          const uint64_t bd = tc::sdesc(xb_addr + (kpos / 8) * 128u, 128u, sbo);
          tc::mma_f16_ts(d_col, tmem + b * ACOLS + j * 8, bd, idesc, (it > 0 || j > 0) ? 1u : 0u);
        }
        tc::commit(&bar_a[b]);
      }
      uses[b]++;
    }
    tc::cp_wait<0>();
    if (failed) break;

    // ---- accumulators of this tile ----
    if (threadIdx.x == 0) tc::commit(&bar_d);
    const bool dfail = !tc::mbar_wait(&bar_d, tiles_done & 1, &s_abort);
    if (__syncthreads_or(dfail)) {
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
  __syncthreads();
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

int gemv_tc_min_ksplit(const QMat& w, int M) {
  const int NT = tc_nt(M);
  for (int ks = 1; ks <= 64; ks++)
    if (gemv_tc_smem(w, ks, NT) <= 190 * 1024) return ks;
  LS_THROW(-1, "matrix too wide for the tensor-core GEMV");
}

template <int BITS, int G, int NT>
static void launch_tc_t(const GemvLaunch& g, cudaStream_t s) {
  const size_t smem = gemv_tc_smem(g.w, g.ksplit, NT);
  static size_t configured[64] = {0};
  int dev = 0;
  LS_CUDA(cudaGetDevice(&dev));
  if (smem > 48 * 1024 && configured[dev & 63] < smem) {
    LS_CUDA(cudaFuncSetAttribute(gemv_tc_kernel<BITS, G, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured[dev & 63] = smem;
  }
  const int tiles128 = (g.w.rows_pad / 32 + 3) / 4;
  const int gx = g.grid_x > 0 ? min(g.grid_x, tiles128) : tiles128;
  dim3 grid(gx, g.ksplit, (g.M + NT - 1) / NT);
  launch_pdl(gemv_tc_kernel<BITS, G, NT>, grid, dim3(TC_THREADS), smem, s, g);
}

template <int BITS, int G>
static void launch_tc_g(const GemvLaunch& g, cudaStream_t s) {
  switch (tc_nt(g.M)) {
    case 16: return launch_tc_t<BITS, G, 16>(g, s);
    case 32: return launch_tc_t<BITS, G, 32>(g, s);
    case 48: return launch_tc_t<BITS, G, 48>(g, s);
    default: return launch_tc_t<BITS, G, 64>(g, s);
  }
}

void launch_gemv_tc(const GemvLaunch& g, cudaStream_t s) {
  if (g.M <= 0) return;
  if (!gemv_tc_supported(g.w)) LS_THROW(-1, "format not supported by the tensor-core GEMV");
  if (g.ksplit < gemv_tc_min_ksplit(g.w, g.M)) LS_THROW(-1, "tensor-core GEMV split too small for shared memory");
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
