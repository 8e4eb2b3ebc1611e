// gemm_noalloc.cu -- split-K GEMM whose scratch lives in a static device array.
//
// Some callers cannot call cudaMalloc: code running inside a host-side
// allocator hook or a memory-pool callback, plug-ins whose host process owns
// every device allocation (and forbids others), and startup paths that run
// before the caller's own allocator exists.  ne_gemm_splitk_noalloc serves
// them: it computes the same fp32 product as ne_gemm_device (epilogue 1) with
// split-K, keeping the per-split partial slabs in a fixed-size array that is
// part of the loaded library instead of in memory it would have to allocate.
//
// Properties a caller must know:
//   * The array holds NE_NOALLOC_SCRATCH_FLOATS floats (8 MiB).  Every GPU that
//     loads libne.so keeps it resident until the process exits.  A call needs
//     splits * M * N floats of it; larger requests are rejected.
//   * The array is shared by every call in the process and keeps what the last
//     call wrote.  Each call overwrites every slab element it reads and clears
//     its status word first, so no state leaks between calls; but two calls
//     whose GPU work overlaps (different streams, or different host threads on
//     one device) race on the same array and corrupt each other's result.
//   * The first call on a device looks up the device address of the array
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture.
//   * The call synchronises the given stream before it returns, so it can
//     report a kernel wait that timed out.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/ne.h"
#include "ne_device.cuh"
#include "ne_internal.h"

namespace {

constexpr size_t kScratchFloats = NE_NOALLOC_SCRATCH_FLOATS;
constexpr int kMaxDevices = 64;

// The scratch array and the status word of the bounded waits.  In host code
// these names are host-side stand-ins, not device addresses: only the pointers
// obtained from cudaGetSymbolAddress below may be handed to a kernel.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];
static __device__ __align__(256) int g_noalloc_status;

struct DeviceSymbols {
  float* scratch = nullptr;
  int* status = nullptr;
};
DeviceSymbols g_symbols[kMaxDevices];
std::mutex g_symbols_mu;

// Device addresses of the two symbols on `device` (which must be current).
ne_status device_symbols(int device, DeviceSymbols* out) {
  if (device < 0 || device >= kMaxDevices) return NE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_symbols_mu);
  DeviceSymbols& s = g_symbols[device];
  if (s.scratch == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return NE_ERR_CUDA;
    void* q = nullptr;
    if (cudaGetSymbolAddress(&q, g_noalloc_status) != cudaSuccess || q == nullptr)
      return NE_ERR_CUDA;
    s.scratch = static_cast<float*>(p);
    s.status = static_cast<int*>(q);
  }
  *out = s;
  return NE_OK;
}

// out[m*ld + n] = sum over s of slab s at (m, n), summed in split order.
__global__ void reduce_slabs_kernel(const float* __restrict__ slabs, int splits, int M, int N,
                                    float* __restrict__ out, long long ld) {
  const long long total = (long long)M * N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += slabs[(long long)s * total + i];
    const long long m = i / N, n = i % N;
    out[m * ld + n] = acc;
  }
}

}  // namespace

extern "C" NE_API ne_status ne_gemm_splitk_noalloc(const void* d_A, long long lda, int M,
                                                   const void* d_B, long long ldb, int N, int K,
                                                   int splits, float* d_out, long long ld,
                                                   void* stream) {
  if (!d_A || !d_B || !d_out || M <= 0 || N <= 0 || K <= 0 || splits <= 0 || ld < N)
    return NE_ERR_INVALID;
  if (K % 64 != 0 || (K / 64) % splits != 0) return NE_ERR_INVALID;
  if ((size_t)splits * (size_t)M * (size_t)N > kScratchFloats) return NE_ERR_INVALID;
  // the operands are read by TMA: rows of at least K elements, row pitches of
  // whole 16-byte units and 16-byte aligned bases (what the tensor maps need)
  if (lda < K || ldb < K || lda % 8 != 0 || ldb % 8 != 0) return NE_ERR_INVALID;
  const uintptr_t a_addr = reinterpret_cast<uintptr_t>(d_A);
  const uintptr_t b_addr = reinterpret_cast<uintptr_t>(d_B);
  if ((a_addr & 15u) != 0 || (b_addr & 15u) != 0 || (reinterpret_cast<uintptr_t>(d_out) & 3u) != 0)
    return NE_ERR_INVALID;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return NE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the scratch address below belongs to the current device; a stream of
  // another device would run the kernels against that device's memory
  if (s != nullptr) {
    int stream_device = -1;
    if (cudaStreamGetDevice(s, &stream_device) != cudaSuccess || stream_device != device)
      return NE_ERR_INVALID;
  }
  DeviceSymbols sym;
  ne_status st = device_symbols(device, &sym);
  if (st != NE_OK) return st;
  if (cudaMemsetAsync(sym.status, 0, sizeof(int), s) != cudaSuccess) return NE_ERR_CUDA;

  ne::GemmCall c;
  c.A = d_A; c.lda = lda; c.M = M;
  c.B = d_B; c.ldb = ldb; c.N = N;
  c.K = K;
  c.epi = ne::EPI_F32;
  c.out = sym.scratch;
  c.ld = N;
  c.split_stride = (long long)M * N;
  c.splits = splits;
  if (ne::gemm_run(c, sym.status, s) != cudaSuccess) return NE_ERR_CUDA;
  const long long total = (long long)M * N;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  reduce_slabs_kernel<<<blocks, 256, 0, s>>>(sym.scratch, splits, M, N, d_out, ld);
  if (cudaGetLastError() != cudaSuccess) return NE_ERR_CUDA;
  int h_status = 0;
  if (cudaMemcpyAsync(&h_status, sym.status, sizeof(int), cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return NE_ERR_CUDA;
  if (h_status == ne::DEV_ERR_TIMEOUT) return NE_ERR_TIMEOUT;
  if (h_status != 0) return NE_ERR_CUDA;
  return NE_OK;
}
