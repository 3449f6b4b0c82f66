// Tensor-parallel reduction of the row-parallel projections (O, down) through peer memory over
// NVLink: every rank's partial rows y_r stay in its own HBM; one kernel per reduction reads the
// peers' rows directly (P2P loads through the IPC-mapped buffers) and adds the sum into the
// residual stream, x[i] += y_0[i] + y_1[i] + ... + y_{W-1}[i] (ranks in order, so every rank
// computes the same sums). It replaces an NCCL all-reduce plus an add kernel with one launch whose
// cost is one cross-GPU flag round and the peers' bytes over NVLink. The fused form also applies
// the RMSNorm that follows every residual add and writes the next GEMM's f16 operand, so the
// reduction costs no launch of its own.
//
// Protocol, per call (epoch = this rank's count of reductions + 1, the same on every rank because
// every rank makes the same calls in the same order):
//   ready   the first CTA to arrive writes epoch into slot [rank] of every peer's flag array
//           (system-scope release; the partials, written by the previous kernel, are complete);
//           every CTA's thread 0 waits until every peer's slot in its own array reaches epoch
//   sum     the peers' values are loaded uncached (ld.global.cv)
//   close   the last CTA (ticket) resets the arrival counter and advances the epoch counter
// The partials are double-buffered by the caller (reduction e writes buffer e mod 2), which makes a
// second "done" round unnecessary: a rank writes buffer e mod 2 again only for reduction e + 2,
// after its reduction e + 1 saw every peer's ready(e + 1), which each peer sends only after its
// reduction e (the last read of that buffer) has completed.
// Every wait is bounded in time (P2PReduce::limit_ns); on a timeout the kernel records error 5
// and returns, the other waits then stop at once, and the host (which reduces the error word over
// the ranks before reading it) fails the pass on every rank. No multicast, no TMA: plain loads and
// stores.
#include "ls_device.cuh"
#include "ls_internal.h"
#include "layerstream.h"

namespace ls {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits until flags[p] >= epoch for every peer p (not `rank`); false on a timeout (after limit_ns
// nanoseconds of the GPU's global timer) or an error recorded elsewhere.
__device__ bool wait_peers(const unsigned* flags, int world, int rank, unsigned epoch, int* err, unsigned long long limit_ns) {
  const unsigned long long t0 = global_ns();
  for (int p = 0; p < world; p++) {
    if (p == rank) continue;
    while (ld_acquire_sys(flags + p) < epoch) {
      if (*(volatile int*)err) return false;
      if (global_ns() - t0 > limit_ns) {
        atomicExch(err, 5);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// ready: called by every CTA once this rank's partials are complete; true when every peer's are.
__device__ bool arrive_and_wait(const P2PReduce& r, unsigned epoch) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    if (atomicAdd(r.arrive, 1u) == 0) {
      __threadfence_system();
      for (int p = 0; p < r.world; p++)
        if (p != r.rank) st_release_sys(r.peer_flags[p] + r.rank, epoch);
    }
    s_ok = wait_peers(r.flags, r.world, r.rank, epoch, r.err, r.limit_ns) ? 1 : 0;
  }
  __syncthreads();
  return s_ok != 0;
}

// close: the last CTA resets the arrival counter and advances the epoch (every CTA read the epoch
// before taking its ticket).
__device__ void depart(const P2PReduce& r, unsigned epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(r.ticket, 1u) == gridDim.x - 1) {
      *r.ticket = 0;
      *r.arrive = 0;
      *(volatile unsigned*)r.seq = epoch;
    }
  }
}

// the sum over the ranks, in rank order, of the float4 at index i of every rank's partials (+ off)
__device__ __forceinline__ float4 rank_sum4(const P2PReduce& r, size_t off, size_t i) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int p = 0; p < r.world; p++) {
    const float4* y = reinterpret_cast<const float4*>(r.peer_y[p] + off);
    const float4 v = (p == r.rank) ? y[i] : __ldcv(y + i);
    if (p == 0) {
      acc = v;
    } else {
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
  }
  return acc;
}

__global__ void __launch_bounds__(256) p2p_reduce_add_kernel(float* __restrict__ x, P2PReduce r, size_t off, size_t n) {
  const unsigned epoch = *(volatile unsigned*)r.seq + 1;
  if (arrive_and_wait(r, epoch)) {
    const size_t n4 = n / 4, stride = (size_t)gridDim.x * blockDim.x;
    float4* x4 = reinterpret_cast<float4*>(x);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
      const float4 acc = rank_sum4(r, off, i);
      float4 o = x4[i];
      o.x += acc.x;
      o.y += acc.y;
      o.z += acc.z;
      o.w += acc.w;
      x4[i] = o;
    }
    for (size_t i = 4 * n4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      float acc = 0.f;
      for (int p = 0; p < r.world; p++) {
        const float v = (p == r.rank) ? r.peer_y[p][off + i] : __ldcv(r.peer_y[p] + off + i);
        acc = p == 0 ? v : acc + v;
      }
      x[i] += acc;
    }
  }
  depart(r, epoch);
}

// The reduction fused with the RMSNorm and f16 packing of the next GEMM's operand (bt layout, as
// bt_prep_kernel writes it; rows M .. rows-1 are zero): x[t] += sum of the ranks' partials of row t,
// then out[t] = f16(x[t] * inv_rms(x[t]) * w). Launched with programmatic dependent launch: the
// partials are the previous kernel's output. The squares are summed in the same order as
// bt_prep_kernel (128 threads, float4 steps), so the result equals reduce-then-prep bit for bit.
constexpr int PREP_ITEMS = 4;  // float4s of a row per thread and step: K = 2048 in one step

__global__ void __launch_bounds__(128) p2p_reduce_prep_kernel(float* __restrict__ x, P2PReduce r, size_t off, int M, int K, int N,
                                                              int rows, const uint16_t* __restrict__ nb, const float* __restrict__ nf,
                                                              float eps, uint16_t* __restrict__ out) {
  __shared__ float s_red[4];
  __shared__ float s_inv;
  pdl_trigger();
  pdl_wait();  // the partials are the previous kernel's output
  const unsigned epoch = *(volatile unsigned*)r.seq + 1;
  const bool ok = arrive_and_wait(r, epoch);
  const bool norm = nb != nullptr || nf != nullptr;
  for (int t = blockIdx.x; t < rows; t += gridDim.x) {
    const bool live = t < M;
    float* xr = x + (size_t)t * K;
    float ss = 0.f;
    if (live) {
      // PREP_ITEMS float4s per thread at a time, every rank's loads of them issued before any sum
      // (a remote load costs about a microsecond; issued one after another they would add up)
      const int n4 = K / 4;
      const float4* yrow = nullptr;
      for (int base = 0; base < n4; base += PREP_ITEMS * 128) {
        float4 v[PREP_ITEMS], acc[PREP_ITEMS];
#pragma unroll
        for (int j = 0; j < PREP_ITEMS; j++) {
          const int c4 = base + j * 128 + (int)threadIdx.x;
          if (c4 < n4) v[j] = reinterpret_cast<const float4*>(xr)[c4];
        }
        if (ok) {
#pragma unroll 2
          for (int p = 0; p < r.world; p++) {
            yrow = reinterpret_cast<const float4*>(r.peer_y[p] + off) + (size_t)t * n4;
            float4 y[PREP_ITEMS];
#pragma unroll
            for (int j = 0; j < PREP_ITEMS; j++) {
              const int c4 = base + j * 128 + (int)threadIdx.x;
              if (c4 < n4) y[j] = (p == r.rank) ? yrow[c4] : __ldcv(yrow + c4);
            }
#pragma unroll
            for (int j = 0; j < PREP_ITEMS; j++) {
              if (p == 0) {
                acc[j] = y[j];
              } else {
                acc[j].x += y[j].x;
                acc[j].y += y[j].y;
                acc[j].z += y[j].z;
                acc[j].w += y[j].w;
              }
            }
          }
#pragma unroll
          for (int j = 0; j < PREP_ITEMS; j++) {
            const int c4 = base + j * 128 + (int)threadIdx.x;
            if (c4 < n4) {
              v[j].x += acc[j].x;
              v[j].y += acc[j].y;
              v[j].z += acc[j].z;
              v[j].w += acc[j].w;
              reinterpret_cast<float4*>(xr)[c4] = v[j];
            }
          }
        }
#pragma unroll
        for (int j = 0; j < PREP_ITEMS; j++) {
          const int c4 = base + j * 128 + (int)threadIdx.x;
          if (c4 < n4) ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
        }
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
    __syncthreads();  // also makes every thread's x writes of this row visible to the CTA
    if (threadIdx.x == 0) {
      float tot = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); w++) tot += s_red[w];
      s_inv = 1.0f / sqrtf(tot / (float)K + eps);
    }
    __syncthreads();
    const float inv = (live && norm) ? s_inv : 1.f;
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
      uint4 o = make_uint4(0, 0, 0, 0);
      if (live) {
        const float4 a = reinterpret_cast<const float4*>(xr + c * 8)[0];
        const float4 b = reinterpret_cast<const float4*>(xr + c * 8)[1];
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
    __syncthreads();  // s_red and s_inv are reused by the next row
  }
  depart(r, epoch);
}

void check_reduce(const float* x, const P2PReduce& r, size_t off) {
  if (r.world < 2 || r.world > kMaxTpWorld) LS_THROW(LS_ERR_ARG, "peer reduction: 2..8 ranks");
  // the kernels read and write float4s: every buffer must start on a 16-byte boundary
  auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  bool bad = misaligned(x) || (off % 4) != 0;
  for (int p = 0; p < r.world; p++) bad = bad || !r.peer_y[p] || misaligned(r.peer_y[p]) || !r.peer_flags[p];
  if (bad) LS_THROW(LS_ERR_ARG, "peer reduction: x and every rank's partials must be 16-byte aligned");
  if (!r.flags || !r.seq || !r.ticket || !r.arrive || !r.err) LS_THROW(LS_ERR_ARG, "peer reduction: missing control words");
}

}  // namespace

void launch_p2p_reduce_add(float* x, const P2PReduce& r, size_t off, size_t n, int num_sms, cudaStream_t s) {
  check_reduce(x, r, off);
  const int blocks = (int)std::max<size_t>(1, std::min<size_t>((size_t)num_sms, (n / 4 + 255) / 256));
  p2p_reduce_add_kernel<<<blocks, 256, 0, s>>>(x, r, off, n);
  LS_CUDA(cudaGetLastError());
}

void launch_p2p_reduce_prep(float* x, const P2PReduce& r, size_t off, int M, int K, const uint16_t* norm_bf16, const float* norm_f32,
                            float eps, uint16_t* out, int num_sms, cudaStream_t s) {
  check_reduce(x, r, off);
  if (M <= 0) LS_THROW(LS_ERR_ARG, "peer reduction: no rows");
  if (K % 8) LS_THROW(LS_ERR_ARG, "the bt layout needs K to be a multiple of 8");
  int N = 16, ng = 1;
  bgemm_groups(M, &N, &ng);
  const int rows = ng * N;
  const int blocks = std::max(1, std::min(rows, 4 * num_sms));  // every CTA resident: 128 threads, no dynamic smem
  launch_pdl(p2p_reduce_prep_kernel, dim3(blocks), dim3(128), 0, s, x, r, off, M, K, N, rows, norm_bf16, norm_f32, eps, out);
}

int tp_reduce_host(const float* x, const float* ys, int world, int rank, uint64_t n, bool preset, uint32_t wait_ms, int calls,
                   float* x_out, double* ms, uint32_t K, const float* norm, float eps, uint16_t* op_out) {
  if (world < 2 || world > kMaxTpWorld || rank < 0 || rank >= world) LS_THROW(LS_ERR_ARG, "world must be 2..8 and rank in 0..world-1");
  if (calls < 1 || calls > 1000) LS_THROW(LS_ERR_ARG, "calls must be in 1..1000");
  if (n == 0) LS_THROW(LS_ERR_ARG, "n must be positive");
  if (K && (n % K || K % 8 || n / K > 8192 || !op_out))
    LS_THROW(LS_ERR_ARG, "fused prep: n = rows x K, K a multiple of 8, rows <= 8192, op_out set");
  if (!preset) calls = 1;
  const int M = K ? (int)(n / K) : 0;
  int dev = 0, sms = 0;
  LS_CUDA(cudaGetDevice(&dev));
  LS_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  std::vector<void*> owned;
  auto dmal = [&](size_t b) {
    void* p = nullptr;
    LS_CUDA(cudaMalloc(&p, std::max<size_t>(b, 16)));
    owned.push_back(p);
    return p;
  };
  struct Free {
    std::vector<void*>& o;
    ~Free() {
      cudaDeviceSynchronize();
      for (void* p : o) cudaFree(p);
    }
  } fr{owned};
  const size_t stride = (n + 3) / 4 * 4;  // each emulated rank's partials on a 16-byte boundary
  auto* dx = static_cast<float*>(dmal(n * 4));
  auto* dy = static_cast<float*>(dmal(stride * 4 * world));
  // the flag arrays: this rank's, and one per emulated peer (written by nobody)
  auto* dflags = static_cast<unsigned*>(dmal(4 * (size_t)world * world));
  auto* dctl = static_cast<unsigned*>(dmal(16));
  auto* derr = static_cast<int*>(dmal(4));
  float* dnorm = nullptr;
  uint16_t* dop = nullptr;
  if (K) {
    dnorm = static_cast<float*>(dmal((size_t)K * 4));
    dop = static_cast<uint16_t*>(dmal(bt_elems(M, (int)K) * 2));
    if (norm) LS_CUDA(cudaMemcpy(dnorm, norm, (size_t)K * 4, cudaMemcpyHostToDevice));
  }
  LS_CUDA(cudaMemcpy(dx, x, n * 4, cudaMemcpyHostToDevice));
  for (int p = 0; p < world; p++) LS_CUDA(cudaMemcpy(dy + p * stride, ys + p * n, n * 4, cudaMemcpyHostToDevice));
  LS_CUDA(cudaMemset(dflags, 0, 4 * (size_t)world * world));
  LS_CUDA(cudaMemset(dctl, 0, 16));
  LS_CUDA(cudaMemset(derr, 0, 4));
  P2PReduce r;
  r.world = world;
  r.rank = rank;
  for (int p = 0; p < world; p++) {
    r.peer_y[p] = dy + (size_t)p * stride;
    r.peer_flags[p] = dflags + (size_t)p * world;
  }
  r.flags = r.peer_flags[rank];
  r.seq = dctl;
  r.ticket = dctl + 1;
  r.arrive = dctl + 2;
  r.err = derr;
  r.limit_ns = (unsigned long long)wait_ms * 1000000ull;
  if (preset) {  // every peer already signalled every call's ready: nothing waits
    std::vector<unsigned> f((size_t)world, (unsigned)calls);
    LS_CUDA(cudaMemcpy(r.flags, f.data(), f.size() * 4, cudaMemcpyHostToDevice));
  }
  cudaStream_t s;
  LS_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  LS_CUDA(cudaEventRecord(e0, s));
  for (int i = 0; i < calls; i++) {
    if (K) launch_p2p_reduce_prep(dx, r, 0, M, (int)K, nullptr, norm ? dnorm : nullptr, eps, dop, sms, s);
    else launch_p2p_reduce_add(dx, r, 0, n, sms, s);
  }
  LS_CUDA(cudaEventRecord(e1, s));
  const cudaError_t st = cudaStreamSynchronize(s);
  float tms = 0.f;
  cudaEventElapsedTime(&tms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaStreamDestroy(s);
  if (st != cudaSuccess) LS_THROW(LS_ERR_DEVICE, std::string("peer reduction: ") + cudaGetErrorString(st));
  if (ms) *ms = tms / calls;
  int herr = 0;
  unsigned seq = 0;
  LS_CUDA(cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost));
  LS_CUDA(cudaMemcpy(&seq, dctl, 4, cudaMemcpyDeviceToHost));
  LS_CUDA(cudaMemcpy(x_out, dx, n * 4, cudaMemcpyDeviceToHost));
  if (K) {  // the operand back in row order
    int N = 16, ng = 1;
    bgemm_groups(M, &N, &ng);
    std::vector<uint16_t> bt(bt_elems(M, (int)K));
    LS_CUDA(cudaMemcpy(bt.data(), dop, bt.size() * 2, cudaMemcpyDeviceToHost));
    for (int t = 0; t < M; t++)
      for (uint32_t k = 0; k < K; k++) op_out[(size_t)t * K + k] = bt[bt_off(t, (int)k, (int)K, N)];
  }
  if (!herr && seq != (unsigned)calls) LS_THROW(LS_ERR_DEVICE, "peer reduction: the call counter did not advance");
  return herr;
}

}  // namespace ls
