// Tensor-core (tcgen05) GQA attention of the verify block over the f16 KV cache.
//
// One CTA per (context split, kv head, block of 128 query rows, sequence). The query rows are the
// G = heads / kv_heads q heads that read the kv head times the M rows of the block, so every K/V
// byte crosses HBM once per kv head (not once per q head). The CTA walks its 128-position chunks:
//
//   S[128 x 128]  = Q[128 x hd] . K^T      tcgen05.mma, A = Q and B = K in shared memory
//                                          (K-major core matrices), D in tensor memory
//   softmax       each query row sits in one tensor-memory lane; the two warps of its lane
//                 quadrant take 64 positions each (tcgen05.ld), exchange the row max through
//                 shared memory, and store P = 2^(u - max) as f16 into their own columns
//                 (tcgen05.st); u = q . k * log2(e) / sqrt(hd), running max / sums in f32
//   O[128 x hd]  += P . V                  tcgen05.mma, A = P in tensor memory, B = V^T (the chunk
//                                          transposed in shared memory into K-major core matrices)
//
// O is kept in registers (each warp of a quadrant holds half of the head dimension), rescaled by
// the running-max correction after every chunk. Query rows are spread over the four lane
// quadrants (row r at lane (r % 4) * 32 + r / 4) so that blocks of a few dozen rows keep all eight
// warps busy. K/V chunks stream through a two-buffer cp.async ring; the block's own new rows (RoPE
// on K, both rounded to f16 as the cache stores them) are computed from qkv in place of cache
// reads and written to the cache by the CTA that owns their chunk. Splits of one (sequence, kv
// head, row block) leave (m, l, O) partials, merged by attention_merge_kernel, one CTA per query
// row, so that the partials (16 KB per split and kv head at M = 9) are read by many SMs instead of
// one; batches of up to AT_LAST_MERGE splits merge in their last CTA, in split order. Every mbarrier wait is bounded: on a timeout the
// kernel records the error and returns after releasing tensor memory.
//
// Scores are exact f16 x f16 products accumulated in f32 (then scaled in f32); q and P are rounded
// to f16 for the tensor core, which keeps the output within the north-star logit tolerance of the
// reference's f32 attention (softmax over q . k / sqrt(hd), then the weighted sum of v).
#include <algorithm>

#include "ls_device.cuh"
#include "ls_internal.h"

namespace ls {

constexpr int AT_THREADS = 256;  // two warps per tensor-memory lane quadrant
constexpr int AT_CH = 128;       // positions per chunk: N of the score MMA, K of the value MMA
constexpr int AT_MAX_SPLITS = 160;  // > 148: a single sequence's two kv heads fill every SM twice
constexpr int AT_LAST_MERGE = 8;    // batches: splits merged by the last CTA; above, by attention_merge_kernel
// tensor-memory columns: scores [0, 128), P as f16 pairs [128, 192), output [192, 192 + hd)
constexpr int AT_COL_P = 128, AT_COL_O = 192;
__host__ __device__ constexpr int at_tmem_cols(int hd) { return AT_COL_O + hd <= 256 ? 256 : 512; }

template <int HD>
struct AtSmem {
  static constexpr int kQ = 128 * HD * 2;   // Q rows, K-major core matrices
  static constexpr int kK = AT_CH * HD * 2; // one K chunk, K-major core matrices
  static constexpr int kV = AT_CH * HD * 2; // one V chunk as the cache stores it ([pos][hd])
  static constexpr int kVT = HD * AT_CH * 2; // V^T of a chunk, K-major core matrices
  static constexpr int kTotal = kQ + 2 * kK + 2 * kV + kVT;
};

// Byte offset of element (row, col) in a K-major no-swizzle tile: 8-row x 16-byte core matrices,
// K chunks 128 bytes apart, 8-row groups sbo apart.
__device__ __forceinline__ uint32_t km_off(int row, int col, uint32_t sbo) {
  return (uint32_t)(row >> 3) * sbo + (uint32_t)(col >> 3) * 128u + (uint32_t)(row & 7) * 16u + (uint32_t)(col & 7) * 2u;
}

__device__ __forceinline__ float f16r(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Dims [d0, d0 + 8) of a RoPE-rotated row (rotate-half pairs (d, d + hd/2)); cs = the position's
// (cos, sin) row of hd/2 entries.
template <int HD>
__device__ __forceinline__ void rope8(const float* x, const float2* cs, int d0, float (&out)[8]) {
  constexpr int HALF = HD / 2;
  const bool lo = d0 < HALF;
  const int dp = lo ? d0 : d0 - HALF;
  const float4* pa = reinterpret_cast<const float4*>(x + d0);
  const float4* pb = reinterpret_cast<const float4*>(x + (lo ? d0 + HALF : d0 - HALF));
  const float4 a0 = pa[0], a1 = pa[1], b0 = pb[0], b1 = pb[1];
  const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
  for (int e = 0; e < 8; e++) {
    const float2 c = cs[dp + e];
    out[e] = lo ? av[e] * c.x - bv[e] * c.y : av[e] * c.x + bv[e] * c.y;
  }
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Tensor-memory lane of query row r of a block: rows spread over the four lane quadrants, so the
// warps of every quadrant have rows even for blocks of a few dozen rows.
__device__ __forceinline__ int at_lane(int r) { return (r & 3) * 32 + (r >> 2); }
__device__ __forceinline__ int at_row(int lane) { return (lane & 31) * 4 + (lane >> 5); }

template <int HD>
__global__ void __launch_bounds__(AT_THREADS, HD == 64 ? 2 : 1) attention_tc_kernel(const AttnLaunch a, int nsplit, int nrb, int merge_kernel) {
  using SM = AtSmem<HD>;
  constexpr int HALF = HD / 2, C8 = HD / 8, HO = HD / 2;  // HO: output columns of each half
  constexpr uint32_t SBO_HD = C8 * 128u;                  // 8-row group stride of [rows][hd] tiles
  constexpr uint32_t SBO_CH = (AT_CH / 8) * 128u;         // 8-row group stride of V^T [hd][chunk]
  constexpr int TCOLS = at_tmem_cols(HD);
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar_s, bar_o;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ float s_red[2][128];  // per half: the chunk's raw row max; at the end the row sums
  uint8_t* sq = smem;
  uint8_t* sk = sq + SM::kQ;
  uint8_t* sv = sk + 2 * SM::kK;
  uint8_t* svt = sv + 2 * SM::kV;

  const int split = blockIdx.x, g = blockIdx.y / nrb, rb = blockIdx.y - (blockIdx.y / nrb) * nrb, seq = blockIdx.z;
  const int G = a.heads / a.kv_heads, M = a.M, R = G * M;
  const int r0 = rb * 128, nrows = min(128, R - r0);
  const int H = a.heads * HD, KV = a.kv_heads * HD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, hf = warp >> 2;  // lane quadrant, half of the chunk / of the output
  const int L = quad * 32 + lane;              // this thread's tensor-memory lane
  const int rl = at_row(L);                    // its query row in the block
  const bool row_ok = rl < nrows;
  const bool quad_active = quad < nrows;       // warp-uniform: the quadrant holds a valid row
  // written by the host before the pass (or, for batches launched without PDL, by an earlier kernel)
  // profiling timeline (a.trace): 0 start, 1 after the first chunk's loads are issued and the
  // previous kernel has finished, 2 Q staged; per chunk of the first two (k = 0, 1): 3 + 4k loads
  // landed, 4 + 4k scores ready, 5 + 4k P stored, 6 + 4k O added; 11 partials written
  auto mark = [&](int k) {
    if (a.trace && tid == 0)
      a.trace[((size_t)blockIdx.x + gridDim.x * ((size_t)blockIdx.y + gridDim.y * blockIdx.z)) * AT_TRACE_SLOTS + k] =
          (unsigned)clock();
  };
  mark(0);
  const int pos0 = a.pos0 ? a.pos0[seq] : a.ctl->pos0;
  const int total = pos0 + M;
  const int nch = (total + AT_CH - 1) / AT_CH;
  const int c0 = (int)((long long)split * nch / nsplit), c1 = (int)((long long)(split + 1) * nch / nsplit);
  const float* qkv = a.qkv + (size_t)seq * M * a.qkv_stride;
  uint16_t* kcache = a.k_cache;  // this layer's page pools, shared by the sequences
  uint16_t* vcache = a.v_cache;
  const int32_t* pg = a.pages + (size_t)seq * a.max_pages;
  // scores in the log2 domain: u = q . k * (log2(e) / sqrt(hd)), softmax weights 2^(u - max)
  const float c1s = 1.4426950408889634f / sqrtf((float)HD);

  pdl_trigger();
  if (tid == 0) {
    tc::mbar_init(&bar_s, 1);
    tc::mbar_init(&bar_o, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::su32(&s_tmem)), "r"(TCOLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // Cached rows (positions < pos0) of chunk c into buffer b: K as core matrices, V as stored; one
  // cp.async per 16-byte piece (row pl, column chunk cc). K: each warp fills tiles of 8 rows x 4
  // column chunks (lane = row % 8 + 8 x chunk % 4), so a quarter warp writes the 8 distinct 16-byte
  // slots of a core matrix (no shared-memory bank conflicts) and reads 64 contiguous bytes of each
  // row; V: consecutive pieces of one row per 8 lanes. The page-table entries of all the thread's
  // pieces are read first, in one round trip.
  constexpr int LPER = AT_CH * C8 / AT_THREADS;  // pieces of K (and of V) per thread: hd 64: 4, hd 128: 8
  auto load_chunk = [&](int c, int b) {
    const int p0 = c * AT_CH;
    const int ncached = max(0, min(AT_CH, pos0 - p0));
    const uint32_t kb = tc::su32(sk + b * SM::kK), vb = tc::su32(sv + b * SM::kV);
    const int pmask = (1 << a.page_shift) - 1;
    int kpl[LPER], kcc[LPER], kent[LPER], vent[LPER];
#pragma unroll
    for (int k = 0; k < LPER; k++) {
      const int t = warp + 8 * k, rg = t % (AT_CH / 8), cq = t / (AT_CH / 8);
      kpl[k] = rg * 8 + (lane & 7);
      kcc[k] = cq * 4 + (lane >> 3);
      const int vpl = (tid + AT_THREADS * k) / C8;
      kent[k] = kpl[k] < ncached ? pg[(p0 + kpl[k]) >> a.page_shift] : 0;
      vent[k] = vpl < ncached ? pg[(p0 + vpl) >> a.page_shift] : 0;
    }
#pragma unroll
    for (int k = 0; k < LPER; k++) {
      if (kpl[k] < ncached) {
        const int p = p0 + kpl[k];
        const size_t row = ((((size_t)g * a.num_pages + kent[k]) << a.page_shift) + (size_t)(p & pmask)) * HD + kcc[k] * 8;
        tc::cp_async16(kb + km_off(kpl[k], kcc[k] * 8, SBO_HD), kcache + row);
      }
      const int i = tid + AT_THREADS * k, vpl = i / C8, vcc = i - vpl * C8;
      if (vpl < ncached) {
        const int p = p0 + vpl;
        const size_t row = ((((size_t)g * a.num_pages + vent[k]) << a.page_shift) + (size_t)(p & pmask)) * HD + vcc * 8;
        tc::cp_async16(vb + (uint32_t)i * 16u, vcache + row);
      }
    }
    tc::cp_commit();
  };
  // the block's new rows of chunk c (RoPE on K, f16 rounding, written to the cache by the CTA that
  // owns the chunk in row block 0) and zero rows past the context
  auto fill_chunk = [&](int c, int b) {
    const int p0 = c * AT_CH;
    uint8_t* kt = sk + b * SM::kK;
    uint8_t* vt = sv + b * SM::kV;
    const int pnew = max(p0, pos0), pend = min(p0 + AT_CH, total);
    for (int i = tid; i < max(0, pend - pnew) * C8; i += AT_THREADS) {
      const int j = i / C8, cc = i - j * C8;
      const int p = pnew + j, pl = p - p0, t = p - pos0;
      const float* kr = qkv + (size_t)t * a.qkv_stride + H + g * HD;
      float kv8[8];
      rope8<HD>(kr, a.rope + (size_t)p * HALF, cc * 8, kv8);
      const float4 v0 = reinterpret_cast<const float4*>(kr + KV + cc * 8)[0];
      const float4 v1 = reinterpret_cast<const float4*>(kr + KV + cc * 8)[1];
      const uint4 kh = make_uint4(pack_h2(kv8[0], kv8[1]), pack_h2(kv8[2], kv8[3]), pack_h2(kv8[4], kv8[5]),
                                  pack_h2(kv8[6], kv8[7]));
      const uint4 vh = make_uint4(pack_h2(v0.x, v0.y), pack_h2(v0.z, v0.w), pack_h2(v1.x, v1.y), pack_h2(v1.z, v1.w));
      *reinterpret_cast<uint4*>(kt + km_off(pl, cc * 8, SBO_HD)) = kh;
      *reinterpret_cast<uint4*>(vt + (pl * HD + cc * 8) * 2) = vh;
      if (rb == 0) {
        const size_t row = kv_row(pg, a.page_shift, a.num_pages, g, p) * HD + cc * 8;
        *reinterpret_cast<uint4*>(kcache + row) = kh;
        *reinterpret_cast<uint4*>(vcache + row) = vh;
      }
    }
    const int pz = max(p0, total);
    for (int i = tid; i < max(0, p0 + AT_CH - pz) * C8; i += AT_THREADS) {
      const int pl = pz - p0 + i / C8, cc = i % C8;
      *reinterpret_cast<uint4*>(kt + km_off(pl, cc * 8, SBO_HD)) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(vt + (pl * HD + cc * 8) * 2) = make_uint4(0, 0, 0, 0);
    }
  };

  if (c0 < c1) load_chunk(c0, 0);  // the cache rows below pos0 do not depend on the previous kernel
  pdl_wait();
  mark(1);

  // Q rows of this block (row r = q head j of the group x token t, r = j * M + t) at their lanes,
  // RoPE at pos0 + t; lanes without a row are zero. The rows (f32, before RoPE) and, when they fit,
  // the RoPE rows of the block's positions are first copied into shared memory that the chunk loop
  // has not used yet (the second V buffer and the V^T tile: 128 rows x hd floats; the second K
  // buffer), every piece in flight at once: one round trip instead of one per piece.
  {
    float* qst = reinterpret_cast<float*>(sv + SM::kV);    // [nrows][HD]
    float2* rst = reinterpret_cast<float2*>(sk + SM::kK);  // [M][HALF]
    const bool rope_smem = (size_t)M * HD * 4 <= (size_t)SM::kK;
    for (int i = tid; i < nrows * (HD / 4); i += AT_THREADS) {
      const int rr = i / (HD / 4), c4 = i - rr * (HD / 4);
      const int r = r0 + rr, j = r / M, t = r - j * M;
      tc::cp_async16(tc::su32(qst + (size_t)rr * HD + c4 * 4), qkv + (size_t)t * a.qkv_stride + (g * G + j) * HD + c4 * 4);
    }
    if (rope_smem)
      for (int i = tid; i < M * (HALF / 2); i += AT_THREADS) {
        const int t = i / (HALF / 2), c2 = i - t * (HALF / 2);
        tc::cp_async16(tc::su32(rst + (size_t)t * HALF + c2 * 2), a.rope + (size_t)(pos0 + t) * HALF + c2 * 2);
      }
    tc::cp_commit();
    tc::cp_wait<0>();  // (also the first chunk's rows, which the loop needs next)
    __syncthreads();
    // (the K tiles' mapping: a quarter warp writes the 8 rows of one core matrix, no bank conflicts)
#pragma unroll 1
    for (int k = 0; k < LPER; k++) {
      const int tq = warp + 8 * k, ln = (tq % 16) * 8 + (lane & 7), cc = (tq / 16) * 4 + (lane >> 3);
      const int rr = at_row(ln);
      uint4 qh = make_uint4(0, 0, 0, 0);
      if (rr < nrows) {
        const int t = (r0 + rr) % M;
        float q8[8];
        rope8<HD>(qst + (size_t)rr * HD, rope_smem ? rst + (size_t)t * HALF : a.rope + (size_t)(pos0 + t) * HALF, cc * 8, q8);
        qh = make_uint4(pack_h2(q8[0], q8[1]), pack_h2(q8[2], q8[3]), pack_h2(q8[4], q8[5]), pack_h2(q8[6], q8[7]));
      }
      *reinterpret_cast<uint4*>(sq + km_off(ln, cc * 8, SBO_HD)) = qh;
    }
  }

  __syncthreads();
  tc::fence_after();
  mark(2);
  const uint32_t tmem = s_tmem;
  const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
  int lim = -1;  // last position this row may attend to
  if (row_ok) {
    const int r = r0 + rl, j = r / M;
    lim = pos0 + (r - j * M);
  }
  const uint32_t q_addr = tc::su32(sq), vt_addr = tc::su32(svt);
  float o[HO];
#pragma unroll
  for (int d = 0; d < HO; d++) o[d] = 0.f;
  float m_run = -CUDART_INF_F, l_half = 0.f;
  bool failed = false;

  for (int c = c0; c < c1; c++) {
    const int it = c - c0, b = it & 1, p0 = c * AT_CH;
    if (c + 1 < c1) load_chunk(c + 1, b ^ 1);
    else tc::cp_commit();
    tc::cp_wait<1>();
    fill_chunk(c, b);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (it < 2) mark(3 + 4 * it);

    // ---- scores ----
    if (tid == 0) {
      tc::fence_after();
      const uint32_t k_addr = tc::su32(sk + b * SM::kK);
#pragma unroll
      for (int j = 0; j < HD / 16; j++)
        tc::mma_f16_ss(tmem, tc::sdesc(q_addr + j * 256u, 128u, SBO_HD), tc::sdesc(k_addr + j * 256u, 128u, SBO_HD),
                       tc::idesc_f16(AT_CH), j > 0 ? 1u : 0u);
      tc::commit(&bar_s);
    }
    // ---- V^T of the chunk (value MMA operand), overlapping the score MMA ----
    {
      const uint8_t* vsrc = sv + b * SM::kV;
      for (int task = tid; task < HALF * (AT_CH / 8); task += AT_THREADS) {
        const int dp = task % HALF, ig = task / HALF;
        const uint8_t* src = vsrc + (size_t)(ig * 8) * HD * 2 + dp * 4;
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; e++) w[e] = *reinterpret_cast<const uint32_t*>(src + e * HD * 2);
        const uint4 lo = make_uint4(__byte_perm(w[0], w[1], 0x5410), __byte_perm(w[2], w[3], 0x5410),
                                    __byte_perm(w[4], w[5], 0x5410), __byte_perm(w[6], w[7], 0x5410));
        const uint4 hi = make_uint4(__byte_perm(w[0], w[1], 0x7632), __byte_perm(w[2], w[3], 0x7632),
                                    __byte_perm(w[4], w[5], 0x7632), __byte_perm(w[6], w[7], 0x7632));
        *reinterpret_cast<uint4*>(svt + km_off(2 * dp, ig * 8, SBO_CH)) = lo;
        *reinterpret_cast<uint4*>(svt + km_off(2 * dp + 1, ig * 8, SBO_CH)) = hi;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (__syncthreads_or(!tc::mbar_wait_fast(&bar_s, it & 1, &s_abort))) {
      failed = true;
      break;
    }
    tc::fence_after();
    if (it < 2) mark(4 + 4 * it);

    // ---- softmax: each half of the warps takes 64 positions of every row ----
    const int pb = p0 + hf * 64;       // first position of this half
    const bool full = pb + 63 <= lim;  // every position of this half is visible to the row
    if (quad_active) {
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int q = 0; q < 2; q++) {
        uint32_t va[16], vb[16];
        tc::ld16(t_lane + hf * 64 + q * 32, va);
        tc::ld16(t_lane + hf * 64 + q * 32 + 16, vb);
        tc::wait_ld();
        if (full) {
#pragma unroll
          for (int e = 0; e < 16; e++) mx = fmaxf(mx, fmaxf(__uint_as_float(va[e]), __uint_as_float(vb[e])));
        } else {
#pragma unroll
          for (int e = 0; e < 16; e++) {
            if (pb + q * 32 + e <= lim) mx = fmaxf(mx, __uint_as_float(va[e]));
            if (pb + q * 32 + 16 + e <= lim) mx = fmaxf(mx, __uint_as_float(vb[e]));
          }
        }
      }
      s_red[hf][L] = mx;
    }
    __syncthreads();
    float corr = 1.f;
    if (quad_active) {
      const float m_new = fmaxf(m_run, fmaxf(s_red[0][L], s_red[1][L]) * c1s);
      const float mb = (m_new == -CUDART_INF_F) ? 0.f : m_new;
      corr = (m_run == -CUDART_INF_F) ? 1.f : ex2(m_run - m_new);
      float lsum = 0.f;
#pragma unroll
      for (int q = 0; q < 2; q++) {
        uint32_t va[16], vb[16], pk[16];
        tc::ld16(t_lane + hf * 64 + q * 32, va);
        tc::ld16(t_lane + hf * 64 + q * 32 + 16, vb);
        tc::wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e++) {
          const int pa = pb + q * 32 + 2 * e;
          const float s0 = (e < 8) ? __uint_as_float(va[2 * e]) : __uint_as_float(vb[2 * e - 16]);
          const float s1 = (e < 8) ? __uint_as_float(va[2 * e + 1]) : __uint_as_float(vb[2 * e - 15]);
          float e0 = ex2(fmaf(s0, c1s, -mb)), e1 = ex2(fmaf(s1, c1s, -mb));
          if (!full) {
            e0 = (pa <= lim) ? e0 : 0.f;
            e1 = (pa + 1 <= lim) ? e1 : 0.f;
          }
          lsum += e0 + e1;
          pk[e] = pack_h2(e0, e1);
        }
        tc::st16(t_lane + AT_COL_P + hf * 32 + q * 16, pk);  // P of positions [32q, 32q + 32) of the half
      }
      tc::wait_st();
      if (m_new != -CUDART_INF_F) {
        l_half = l_half * corr + lsum;
        m_run = m_new;
      } else {
        corr = 1.f;
      }
    }
    tc::fence_before();
    __syncthreads();

    if (it < 2) mark(5 + 4 * it);
    // ---- O += P . V ----
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int j = 0; j < AT_CH / 16; j++)
        tc::mma_f16_ts(tmem + AT_COL_O, tmem + AT_COL_P + j * 8, tc::sdesc(vt_addr + j * 256u, 128u, SBO_CH),
                       tc::idesc_f16(HD), j > 0 ? 1u : 0u);
      tc::commit(&bar_o);
    }
    if (__syncthreads_or(!tc::mbar_wait_fast(&bar_o, it & 1, &s_abort))) {
      failed = true;
      break;
    }
    tc::fence_after();
    if (quad_active) {
#pragma unroll
      for (int q = 0; q < HO / 16; q++) {
        uint32_t v[16];
        tc::ld16(t_lane + AT_COL_O + hf * HO + q * 16, v);
        tc::wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e++) o[q * 16 + e] = o[q * 16 + e] * corr + __uint_as_float(v[e]);
      }
    }
    tc::fence_before();
    if (it < 2) mark(6 + 4 * it);
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
    if (tid == 0 && a.err) atomicExch(a.err, 1);
    return;
  }
  // row sum = both halves' sums (same running max)
  s_red[hf][L] = l_half;
  __syncthreads();
  const float l_run = s_red[0][L] + s_red[1][L];

  int t = 0, h = 0;
  if (row_ok) {
    const int r = r0 + rl, j = r / M;
    t = r - j * M;
    h = g * G + j;
  }
  if (nsplit == 1) {
    if (row_ok) {
      const float inv = 1.0f / l_run;
      if (a.out_h) {  // f16 in the bt layout, the next GEMM's operand
#pragma unroll
        for (int d8 = 0; d8 < HO / 8; d8++)
          *reinterpret_cast<uint4*>(a.out_h + bt_off(seq * M + t, h * HD + hf * HO + d8 * 8, H, a.out_h_n)) =
              make_uint4(pack_h2(o[8 * d8] * inv, o[8 * d8 + 1] * inv), pack_h2(o[8 * d8 + 2] * inv, o[8 * d8 + 3] * inv),
                         pack_h2(o[8 * d8 + 4] * inv, o[8 * d8 + 5] * inv), pack_h2(o[8 * d8 + 6] * inv, o[8 * d8 + 7] * inv));
      } else {
        float4* out = reinterpret_cast<float4*>(a.out + ((size_t)seq * M + t) * H + (size_t)h * HD + hf * HO);
#pragma unroll
        for (int d4 = 0; d4 < HO / 4; d4++)
          out[d4] = make_float4(o[4 * d4] * inv, o[4 * d4 + 1] * inv, o[4 * d4 + 2] * inv, o[4 * d4 + 3] * inv);
      }
    }
    return;
  }
  // partials: O as [sequence][kv head][split][row][hd] (16-byte aligned rows), then (m, l) as
  // [sequence][kv head][split][row][2] (m in the log2 domain); the last split of this row block
  // merges them
  const size_t unit = (size_t)seq * a.kv_heads + g;
  float* po = a.part + unit * nsplit * (size_t)R * HD;
  float* pml = a.part + (size_t)a.nseq * a.kv_heads * nsplit * (size_t)R * HD + unit * nsplit * (size_t)R * 2;
  if (row_ok) {
    float4* pp = reinterpret_cast<float4*>(po + ((size_t)split * R + r0 + rl) * HD + hf * HO);
#pragma unroll
    for (int d4 = 0; d4 < HO / 4; d4++) pp[d4] = make_float4(o[4 * d4], o[4 * d4 + 1], o[4 * d4 + 2], o[4 * d4 + 3]);
    if (hf == 0) reinterpret_cast<float2*>(pml)[(size_t)split * R + r0 + rl] = make_float2(m_run, l_run);
  }
  if (a.trace) {
    __syncthreads();
    mark(11);
  }
  if (merge_kernel || !last_cta(a.tickets + unit * nrb + rb, (unsigned)nsplit)) return;
  // weight of every split for every row (shared memory is free: all MMAs have completed)
  // (the weights of a row are computed by the two threads of its lane, each for half the splits:
  // the max and the sum are combined through shared memory in a fixed order)
  float* s_w = reinterpret_cast<float*>(smem);  // [AT_LAST_MERGE][128]
  const float2* ml = reinterpret_cast<const float2*>(pml) + r0 + rl;
  const int sh0 = hf * ((nsplit + 1) / 2), sh1 = hf ? nsplit : (nsplit + 1) / 2;
  float mm = -CUDART_INF_F;
  if (row_ok)
    for (int s = sh0; s < sh1; s++) mm = fmaxf(mm, __ldcg(ml + (size_t)s * R).x);
  s_red[hf][L] = mm;
  __syncthreads();
  mm = fmaxf(s_red[0][L], s_red[1][L]);
  float Lsum = 0.f;
  if (row_ok)
    for (int s = sh0; s < sh1; s++) {
      const float2 v = __ldcg(ml + (size_t)s * R);
      const float w = (v.x == -CUDART_INF_F) ? 0.f : ex2(v.x - mm);
      s_w[s * 128 + rl] = w;
      Lsum += v.y * w;
    }
  __syncthreads();
  s_red[hf][L] = Lsum;
  __syncthreads();
  if (row_ok) {
    const float inv = 1.0f / (s_red[0][L] + s_red[1][L]);
    for (int s = sh0; s < sh1; s++) s_w[s * 128 + rl] *= inv;
  }
  __syncthreads();
  constexpr int D4 = HD / 4;
  for (int i = tid; i < nrows * D4; i += AT_THREADS) {
    const int rr = i / D4, d4 = i - rr * D4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int s = 0; s < nsplit; s++) {
      const float w = s_w[s * 128 + rr];
      const float4 v = __ldcg(reinterpret_cast<const float4*>(po + ((size_t)s * R + r0 + rr) * HD) + d4);
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
    }
    const int r = r0 + rr, j = r / M, tt = r - j * M;
    if (a.out_h)
      *reinterpret_cast<uint2*>(a.out_h + bt_off(seq * M + tt, (g * G + j) * HD + 4 * d4, H, a.out_h_n)) =
          make_uint2(pack_h2(acc.x, acc.y), pack_h2(acc.z, acc.w));
    else
      reinterpret_cast<float4*>(a.out + ((size_t)seq * M + tt) * H + (size_t)(g * G + j) * HD)[d4] = acc;
  }
}

// Merge of the context splits of one query row (row = blockIdx.x of the (sequence, kv head) unit
// blockIdx.z, blockIdx.y): o = sum_s w_s O_s / sum_s w_s l_s with w_s = 2^(m_s - max m). Every
// load is issued up front (one L2 round trip): thread (split group sg, float4 column d4) holds
// O_s for s = sg, sg + NG, ... and (m, l) of splits tid, tid + 128; it sums its splits in order and
// the groups are added in order, so the result does not depend on timing.
template <int HD>
__global__ void __launch_bounds__(128) attention_merge_kernel(const AttnLaunch a, int nsplit) {
  constexpr int D4 = HD / 4, NG = 128 / D4, PER = (AT_MAX_SPLITS + NG - 1) / NG, BATCH = PER < 20 ? PER : 20;
  constexpr int MLPER = (AT_MAX_SPLITS + 127) / 128;
  __shared__ float s_w[AT_MAX_SPLITS];
  __shared__ float s_r[2][4];
  __shared__ float4 s_acc[NG][D4];
  pdl_trigger();
  const int G = a.heads / a.kv_heads, M = a.M, R = G * M;
  const int row = blockIdx.x, g = blockIdx.y, seq = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d4 = tid % D4, sg = tid / D4;
  pdl_wait();  // the attention kernel's partials
  const size_t unit = (size_t)seq * a.kv_heads + g;
  const float4* src = reinterpret_cast<const float4*>(a.part + unit * nsplit * (size_t)R * HD + (size_t)row * HD) + d4;
  const float2* pml =
      reinterpret_cast<const float2*>(a.part + (size_t)a.nseq * a.kv_heads * nsplit * (size_t)R * HD) + unit * nsplit * (size_t)R + row;
  float2 ml[MLPER];
#pragma unroll
  for (int q = 0; q < MLPER; q++) {
    const int s = tid + 128 * q;
    ml[q] = s < nsplit ? __ldcg(pml + (size_t)s * R) : make_float2(-CUDART_INF_F, 0.f);
  }
  float4 v[BATCH];
#pragma unroll
  for (int j = 0; j < BATCH; j++) {
    const int s = sg + NG * j;
    v[j] = s < nsplit ? __ldcg(src + (size_t)s * R * D4) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mm = -CUDART_INF_F;
#pragma unroll
  for (int q = 0; q < MLPER; q++) mm = fmaxf(mm, ml[q].x);
  mm = warp_max(mm);
  if (lane == 0) s_r[0][warp] = mm;
  __syncthreads();
  mm = fmaxf(fmaxf(s_r[0][0], s_r[0][1]), fmaxf(s_r[0][2], s_r[0][3]));
  float ls = 0.f;
#pragma unroll
  for (int q = 0; q < MLPER; q++) {
    const int s = tid + 128 * q;
    if (s < nsplit) {
      const float w = (ml[q].x == -CUDART_INF_F) ? 0.f : ex2(ml[q].x - mm);
      s_w[s] = w;
      ls += ml[q].y * w;
    }
  }
  ls = warp_sum(ls);
  if (lane == 0) s_r[1][warp] = ls;
  __syncthreads();
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < BATCH; j++) {
    const int s = sg + NG * j;
    if (s < nsplit) {
      const float w = s_w[s];
      acc.x += w * v[j].x;
      acc.y += w * v[j].y;
      acc.z += w * v[j].z;
      acc.w += w * v[j].w;
    }
  }
  for (int j = BATCH; j < PER; j++) {  // (head_dim 128: the splits beyond the first batch)
    const int s = sg + NG * j;
    if (s < nsplit) {
      const float w = s_w[s];
      const float4 u = __ldcg(src + (size_t)s * R * D4);
      acc.x += w * u.x;
      acc.y += w * u.y;
      acc.z += w * u.z;
      acc.w += w * u.w;
    }
  }
  s_acc[sg][d4] = acc;
  __syncthreads();
  if (tid < D4) {
    const float inv = 1.0f / (((s_r[1][0] + s_r[1][1]) + s_r[1][2]) + s_r[1][3]);
    float4 t = s_acc[0][tid];
#pragma unroll
    for (int q = 1; q < NG; q++) {
      t.x += s_acc[q][tid].x;
      t.y += s_acc[q][tid].y;
      t.z += s_acc[q][tid].z;
      t.w += s_acc[q][tid].w;
    }
    t = make_float4(t.x * inv, t.y * inv, t.z * inv, t.w * inv);
    const int j = row / M, tt = row - j * M, H = a.heads * HD;
    if (a.out_h)
      *reinterpret_cast<uint2*>(a.out_h + bt_off(seq * M + tt, (g * G + j) * HD + 4 * tid, H, a.out_h_n)) =
          make_uint2(pack_h2(t.x, t.y), pack_h2(t.z, t.w));
    else
      reinterpret_cast<float4*>(a.out + ((size_t)seq * M + tt) * H + (size_t)(g * G + j) * HD)[tid] = t;
  }
}

static int num_sms_cached() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    LS_CUDA(cudaGetDevice(&dev));
    LS_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

template <int HD>
static void launch_att_tc_t(const AttnLaunch& a, cudaStream_t s) {
  const int G = a.heads / a.kv_heads, R = G * a.M, nrb = (R + 127) / 128;
  const int units = a.kv_heads * nrb * a.nseq;
  const int want = (2 * num_sms_cached() + units - 1) / units;
  // chunks of the longest context this launch can see: every split gets at least one
  const int most = a.max_total > 0 ? a.max_total : a.max_ctx;
  const int nch = (most + AT_CH - 1) / AT_CH;
  int nsplit = std::max(1, std::min({want, nch, AT_MAX_SPLITS}));
  // as many splits as the caller's partial buffer holds (O rows and (m, l) of every split)
  if (a.part_floats == 0)
    nsplit = std::max(1, std::min(nsplit, a.max_splits));
  else
    while (nsplit > 1 && (size_t)a.nseq * a.kv_heads * nsplit * R * (HD + 2) > a.part_floats) nsplit--;
  // the splits' merge: a kernel of its own (one CTA per query row) for one sequence whenever there
  // are splits (measured: 16 against 19-20 us at 4-8 splits with the last-CTA merge), and for batches
  // above AT_LAST_MERGE splits (their many small units merge cheaply in their last CTA)
  const int merge_kernel = nsplit > (a.nseq == 1 ? 1 : AT_LAST_MERGE) ? 1 : 0;
  const size_t smem = AtSmem<HD>::kTotal;
  ensure_smem(attention_tc_kernel<HD>, smem);
  const dim3 grid(nsplit, a.kv_heads * nrb, a.nseq);
  if (a.pdl) {
    launch_pdl(attention_tc_kernel<HD>, grid, dim3(AT_THREADS), smem, s, a, nsplit, nrb, merge_kernel);
  } else {
    attention_tc_kernel<HD><<<grid, AT_THREADS, smem, s>>>(a, nsplit, nrb, merge_kernel);
    LS_CUDA(cudaGetLastError());
  }
  if (merge_kernel) launch_pdl(attention_merge_kernel<HD>, dim3(R, a.kv_heads, a.nseq), dim3(128), 0, s, a, nsplit);
}

bool attention_tc_supported(const AttnLaunch& a) {
  static int forced = -1;
  if (forced < 0) {
    const char* e = getenv("LS_ATT");
    forced = (e && std::string(e) == "simt") ? 1 : 0;
  }
  return forced == 0 && (a.hd == 64 || a.hd == 128) && a.kv_heads > 0 && a.heads % a.kv_heads == 0 && a.M >= 1 &&
         a.M <= 128;
}

void launch_attention_tc(const AttnLaunch& a, cudaStream_t s) {
  if (a.hd == 64) return launch_att_tc_t<64>(a, s);
  return launch_att_tc_t<128>(a, s);
}

}  // namespace ls
