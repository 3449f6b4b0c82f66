// GEMV entry point that allocates no device memory.
//
// Who needs it: hosts whose device memory is owned by another allocator (a framework that
// reserves most of HBM at start-up and hands out slices of it, or an embedded runtime with a fixed
// memory budget) cannot let a library call cudaMalloc behind their back: the call may fail for lack
// of free memory, it escapes their accounting, and cudaMalloc/cudaFree may synchronize the device
// in the middle of their pipeline. Such callers keep the stored weight rows, the activations and
// the result in buffers they own and pass plain device pointers.
//
// The split-K partial sums this GEMV needs live in a fixed array in the library's device memory
// (a file-scope __device__ array): every GPU that loads the library holds it until the process
// exits, and every call on that GPU shares it.
#include <algorithm>
#include <mutex>
#include <string>

#include "layerstream.h"
#include "ls_device.cuh"
#include "ls_internal.h"

namespace ls {

// K slices (CTAs along K) and the scratch they write: kNoAllocSlices x M x rows floats.
constexpr int kNoAllocSlices = 4;
constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB per device
constexpr uint64_t kNoAllocMaxMRows = kNoAllocScratchBytes / (kNoAllocSlices * sizeof(float));  // M x rows
constexpr int kNoAllocMaxM = 16;

// Each call writes every element it later reads (all K slices x M x rows) before reading it, so
// nothing in the array needs clearing between calls; what a call leaves behind is the next one's
// to overwrite.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Partial dot products of one K slice, weights read in the stored row format (packed ints then
// bf16 group scales, src/weights.rs:26-31; int4 byte j of a group holds w_j + 8 in the low nibble
// and w_{j+G/2} + 8 in the high one, src/quant.rs:86-104). One warp per row; each lane walks the
// slice's groups and columns, the warp sums in a fixed order.
template <int BITS>
__global__ void __launch_bounds__(256) noalloc_partial_kernel(const uint8_t* __restrict__ w, int group, int rows, int cols,
                                                               const float* __restrict__ x, int M, float* __restrict__ part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp, ks = blockIdx.y;
  if (r >= rows) return;
  const size_t data_bytes = (size_t)cols * BITS / 8;
  const size_t rb = data_bytes + (size_t)(cols / group) * 2;
  const uint8_t* row = w + (size_t)r * rb;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(row + data_bytes);  // 2-byte aligned: rb and data_bytes are even
  const int ngr = cols / group;
  const int g0 = (int)((long long)ks * ngr / kNoAllocSlices), g1 = (int)((long long)(ks + 1) * ngr / kNoAllocSlices);
  float acc[kNoAllocMaxM];
#pragma unroll
  for (int t = 0; t < kNoAllocMaxM; t++) acc[t] = 0.f;
  for (int k = g0 * group + lane; k < g1 * group; k += 32) {
    const int gi = k / group, j = k - gi * group;
    float q;
    if (BITS == 8) {
      q = (float)(int8_t)row[k];
    } else {
      const int half = group / 2;
      const uint8_t by = row[(size_t)gi * half + (j < half ? j : j - half)];
      q = (float)((j < half ? (by & 15) : (by >> 4)) - 8);
    }
    const float v = q * bf16f(sc[gi]);
#pragma unroll
    for (int t = 0; t < kNoAllocMaxM; t++)
      if (t < M) acc[t] = fmaf(v, x[(size_t)t * cols + k], acc[t]);
  }
#pragma unroll
  for (int t = 0; t < kNoAllocMaxM; t++) {
    if (t < M) {
      const float s = warp_sum(acc[t]);
      if (lane == 0) part[((size_t)ks * M + t) * rows + r] = s;
    }
  }
}

// y[t][r] = sum of the K slices in slice order (deterministic).
__global__ void noalloc_reduce_kernel(const float* __restrict__ part, int rows, int M, float* __restrict__ y) {
  const size_t n = (size_t)M * rows;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int ks = 0; ks < kNoAllocSlices; ks++) s += part[(size_t)ks * n + i];
    y[i] = s;
  }
}

// Device address of the scratch array on the current device, looked up once per device (the first
// call on each device does it, with that device current) and kept for the life of the process: a
// cudaDeviceReset would leave the kept address pointing into the old context, so the entry point is
// not for use on a device after a reset.
static float* noalloc_scratch() {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static float* ptr[kMaxDevices] = {};
  int dev = 0;
  LS_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) LS_THROW(LS_ERR_ARG, "device index out of range for the static scratch table");
  std::lock_guard<std::mutex> lock(mu);
  if (!ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) LS_THROW(LS_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    ptr[dev] = static_cast<float*>(p);
  }
  return ptr[dev];
}

void qgemv_rows_noalloc(int bits, int group, const uint8_t* rows_dev, uint64_t rows, uint64_t cols, const float* x_dev,
                        uint64_t M, float* y_dev, cudaStream_t s) {
  if (bits != 8 && bits != 4) LS_THROW(LS_ERR_ARG, "bits must be 8 or 4");
  if (group < 16 || group > 256 || (group & (group - 1)) || cols == 0 || cols % (uint64_t)group || cols > (1u << 30))
    LS_THROW(LS_ERR_ARG, "group must be a power of two in 16..256 and cols a positive multiple of it");
  if (!rows_dev || !x_dev || !y_dev) LS_THROW(LS_ERR_ARG, "device pointers must not be NULL");
  if ((reinterpret_cast<uintptr_t>(rows_dev) & 1) || (reinterpret_cast<uintptr_t>(x_dev) & 3) ||
      (reinterpret_cast<uintptr_t>(y_dev) & 3))
    LS_THROW(LS_ERR_ARG, "rows_dev must be 2-byte aligned, x_dev and y_dev 4-byte aligned");
  if (rows == 0 || rows > (1u << 30)) LS_THROW(LS_ERR_ARG, "rows must be in 1..2^30");
  if (M == 0 || M > (uint64_t)kNoAllocMaxM) LS_THROW(LS_ERR_ARG, "the allocation-free GEMV takes 1..16 token rows");
  if (M * rows > kNoAllocMaxMRows)
    LS_THROW(LS_ERR_ARG, "M x rows = " + std::to_string(M * rows) + " exceeds the allocation-free GEMV's static scratch (" +
                             std::to_string(kNoAllocMaxMRows) + " = 4 MiB / (4 K slices x 4 bytes))");
  float* part = noalloc_scratch();
  const dim3 grid((unsigned)((rows + 7) / 8), kNoAllocSlices);
  if (bits == 8)
    noalloc_partial_kernel<8><<<grid, 256, 0, s>>>(rows_dev, group, (int)rows, (int)cols, x_dev, (int)M, part);
  else
    noalloc_partial_kernel<4><<<grid, 256, 0, s>>>(rows_dev, group, (int)rows, (int)cols, x_dev, (int)M, part);
  LS_CUDA(cudaGetLastError());
  const size_t n = M * rows;
  noalloc_reduce_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 1184), 256, 0, s>>>(part, (int)rows, (int)M, y_dev);
  LS_CUDA(cudaGetLastError());
}

}  // namespace ls
