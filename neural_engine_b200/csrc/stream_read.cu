// stream_read.cu -- the read-only streaming floor for the decode attention.
//
// ne_stream_read reads a device buffer once through the same data path the
// decode attention kernel uses -- a persistent grid of 8 warps per SM, the
// buffer cut into equal per-warp ranges, each warp streaming its range through
// a private 3-stage ring of 8 KB one-dimensional bulk copies (cp.async.bulk
// completing on an mbarrier) -- and does no arithmetic beyond folding one word
// per chunk into a checksum.  Its time for N bytes is the floor any kernel with
// that data path can reach for N bytes in one launch (launch, ramp and tail
// included), so the decode attention's time divided by it says how much of the
// achievable read bandwidth the attention leaves unused.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ne.h"
#include "ne_device.cuh"
#include "ne_launch.cuh"

namespace ne {
namespace {

constexpr int SR_WARPS = 8;
constexpr int SR_STAGES = 3;
constexpr int SR_CHUNK = 8192;
constexpr int SR_SMEM = SR_WARPS * SR_STAGES * SR_CHUNK + SR_WARPS * SR_STAGES * 8;

__device__ __forceinline__ void sr_bulk(uint32_t dst, const void* src, uint32_t bytes,
                                        uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// sink[0] ^= one word per chunk; sink[1] = 1 if a wait ran out (2 s).
__global__ void __launch_bounds__(SR_WARPS * 32, 1)
stream_read_kernel(const uint8_t* __restrict__ src, long long total, unsigned int* sink) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * SR_STAGES * SR_CHUNK;
  const uint32_t bars = smem_u32(smem + SR_WARPS * SR_STAGES * SR_CHUNK) + warp * SR_STAGES * 8;
  if (lane == 0) {
    for (int s = 0; s < SR_STAGES; ++s) mbar_init(bars + 8 * s, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const long long W = (long long)gridDim.x * SR_WARPS;
  const long long w = (long long)blockIdx.x * SR_WARPS + warp;
  long long L = (total + W - 1) / W;
  L = (L + SR_CHUNK - 1) / SR_CHUNK * SR_CHUNK;
  const long long begin = w * L;
  const long long end = begin + L < total ? begin + L : total;

  long long p = begin;
  int issued = 0;
  auto issue = [&](int slot) {
    const uint32_t n = (uint32_t)(end - p < SR_CHUNK ? end - p : SR_CHUNK);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
      mbar_arrive_expect_tx(bars + 8 * slot, n);
      sr_bulk(smem_u32(ring + slot * SR_CHUNK), src + p, n, bars + 8 * slot);
    }
    p += n;
    ++issued;
  };
  for (int s = 0; s < SR_STAGES && p < end; ++s) issue(s);

  unsigned int acc = 0;
  int k = 0;
  bool ok = true;
  for (long long c = begin; c < end; ++k) {
    const int slot = k % SR_STAGES;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bars + 8 * slot, (uint32_t)((k / SR_STAGES) & 1))) {
      if (globaltimer_ns() - t0 > 2000000000ull) {
        ok = false;
        break;
      }
    }
    if (!__all_sync(0xffffffffu, ok)) {
      ok = false;
      break;
    }
    const uint32_t n = (uint32_t)(end - c < SR_CHUNK ? end - c : SR_CHUNK);
    if (lane == 0) acc ^= *reinterpret_cast<const unsigned int*>(ring + slot * SR_CHUNK);
    __syncwarp();
    c += n;
    if (p < end) issue(slot);
  }
  if (!ok) {
    if (lane == 0) sink[1] = 1u;
    for (int j = k; j < issued; ++j) {   // bounded drain of this warp's copies
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bars + 8 * (j % SR_STAGES), (uint32_t)((j / SR_STAGES) & 1)))
        if (globaltimer_ns() - t0 > 100000000ull) break;
    }
  }
  if (lane == 0 && acc) atomicXor(sink, acc);
}

}  // namespace
}  // namespace ne

extern "C" NE_API ne_status ne_stream_read(const void* d_src, long long bytes, unsigned int* d_sink,
                                           void* stream) {
  if (!d_src || !d_sink || bytes <= 0 || (bytes & 15) ||
      (reinterpret_cast<uintptr_t>(d_src) & 15))
    return NE_ERR_INVALID;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(ne::stream_read_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ne::SR_SMEM) != cudaSuccess)
      return NE_ERR_CUDA;
    attr = true;
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return NE_ERR_CUDA;
  ne::stream_read_kernel<<<sms, ne::SR_WARPS * 32, ne::SR_SMEM,
                           static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(d_src), bytes, d_sink);
  return cudaGetLastError() == cudaSuccess ? NE_OK : NE_ERR_CUDA;
}
