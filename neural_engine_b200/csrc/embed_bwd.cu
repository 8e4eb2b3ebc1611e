// embed_bwd.cu -- deterministic input-embedding gradient (embed_backward,
// cpu_ops.h:441-447: dE[tok[r]] += dy[r] for every token row r).
//
// The rows are grouped by token id with a stable radix sort of (id, row index)
// pairs (CUB), then one warp owns each distinct id and adds that id's rows in
// row order before updating dE once.  No floating-point atomics: the result is
// bitwise reproducible, and every data-parallel rank that scatters the same
// gathered (id, row) list obtains identical embedding gradients.
#include <cub/device/device_radix_sort.cuh>

#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"

namespace ne {
namespace {

__global__ void iota_kernel(int32_t* __restrict__ a, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) a[i] = i;
}

// One warp per sorted position; the warp at the first position of each run of
// equal ids sums the run's rows (512 columns at a time, lane-strided so every
// load is coalesced) and adds the sum to dE[id].
__global__ void __launch_bounds__(256)
embed_runs_kernel(const int32_t* __restrict__ keys, const int32_t* __restrict__ idx, int n,
                  const float* __restrict__ dy, int V, int D, float* __restrict__ dE,
                  int* __restrict__ status) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int v = keys[i];
  if (i > 0 && keys[i - 1] == v) return;
  if (v < 0 || v >= V) {
    if (lane == 0) atomicExch(status, DEV_ERR_BOUNDS);
    return;
  }
  int end = i + 1;
  while (end < n && keys[end] == v) ++end;
  float* out = dE + (size_t)v * D;
  for (int c0 = 0; c0 < D; c0 += 512) {
    float acc[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) acc[k] = 0.f;
    for (int j = i; j < end; ++j) {
      const float* row = dy + (size_t)idx[j] * D + c0;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int c = lane + 32 * k;
        if (c0 + c < D) acc[k] += row[c];
      }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int c = lane + 32 * k;
      if (c0 + c < D) out[c0 + c] += acc[k];
    }
  }
}

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

size_t cub_bytes(int n) {
  size_t b = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, b, (const int32_t*)nullptr, (int32_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, n);
  return b;
}

}  // namespace

size_t embed_bwd_scratch_bytes(int n) { return 3 * align256((size_t)n * 4) + align256(cub_bytes(n)); }

cudaError_t launch_embed_bwd(const int32_t* tok, const float* dy, int n, int V, int D, float* dE,
                             void* scratch, size_t scratch_bytes, int* status, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (scratch_bytes < embed_bwd_scratch_bytes(n)) return cudaErrorInvalidValue;
  uint8_t* p = static_cast<uint8_t*>(scratch);
  int32_t* idx_in = reinterpret_cast<int32_t*>(p);
  int32_t* keys_out = reinterpret_cast<int32_t*>(p + align256((size_t)n * 4));
  int32_t* idx_out = reinterpret_cast<int32_t*>(p + 2 * align256((size_t)n * 4));
  void* tmp = p + 3 * align256((size_t)n * 4);
  size_t tmp_bytes = cub_bytes(n);
  iota_kernel<<<(n + 255) / 256, 256, 0, st>>>(idx_in, n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, tok, keys_out, idx_in, idx_out, n, 0, 32, st);
  if (e != cudaSuccess) return e;
  return launch_k(embed_runs_kernel, dim3((n + 7) / 8), dim3(256), 0, st, keys_out, idx_out, n, dy,
                  V, D, dE, status);
}

}  // namespace ne
