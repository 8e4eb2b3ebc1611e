// px.cu -- the ZeRO-1 gradient exchange over NVLink peer memory.
//
// The reference trains on one device (train.m:391-918); its data-parallel
// form here shards the optimizer state: rank r owns part r of every trainable
// tensor.  Instead of NCCL collectives, the exchange reads the other ranks'
// buffers directly: every rank maps the others' training pool, weight pool and
// activation pool (CUDA IPC handles, exchanged once), and
//   * reduce-scatter: after a layer's backward, rank r sums part r of that
//     layer's gradients over all ranks (plain loads from each peer's pool over
//     NVLink, added in rank order) into its own pool, on the comm stream while
//     the backward carries on with the layers below;
//   * all-gather: after AdamW, rank r copies every other rank's updated part
//     of the bf16 compute weights (and of the fp32 gains) into its own pool;
//   * the input-embedding gradient's (token id, dY row) pairs and the
//     gradient norm's per-rank sums of squares are gathered the same way.
// Ordering between ranks is by epoch flags in a small shared buffer per rank:
// a rank publishes "my data for step e is ready" with a system-scope release
// store, and a consumer spins (with an acquire load) until every peer's flag
// reaches e.  Every spin is bounded by wall-clock time; on expiry the kernel
// records NE_ERR_TIMEOUT in the context's status word and skips its work, so a
// rank that stopped cannot hold the others' GPUs.  No TMA, no multicast: the
// remote traffic is ordinary vector loads.
#include <cuda_runtime.h>

#include <cstdint>

#include "ne_device.cuh"
#include "ne_px.h"

namespace ne {

namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0: wait until flags[p][slot] >= the own epoch for every rank p.
// Returns false (status set) when the wall-clock limit passes first, and from
// then on at once: the first wait that ran out sets this rank's PX_ABORT
// word, so the exchange kernels queued behind it do not each wait the limit.
__device__ bool wait_peers(const PxTables& T, int slot, uint32_t epoch, int* status) {
  volatile uint32_t* abort_word = T.flags[T.rank] + PX_ABORT;
  if (*abort_word != 0u) {
    atomicExch(status, DEV_ERR_TIMEOUT);
    return false;
  }
  const uint64_t t0 = globaltimer_ns();
  for (int p = 0; p < T.world; ++p) {
    const uint32_t* f = T.flags[p] + slot;
    while ((int)(ld_acquire_sys(f) - epoch) < 0) {
      if (*abort_word != 0u || globaltimer_ns() - t0 > T.limit_ns) {
        *abort_word = 1u;
        atomicExch(status, DEV_ERR_TIMEOUT);
        return false;
      }
      __nanosleep(200);
    }
  }
  return true;
}

// Every CTA waits (thread 0) and broadcasts the outcome to its threads.
__device__ bool cta_wait_peers(const PxTables& T, int slot, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const uint32_t epoch = T.flags[T.rank][PX_EPOCH];
    ok = wait_peers(T, slot, epoch, status) ? 1 : 0;
  }
  __syncthreads();
  return ok != 0;
}

__global__ void px_epoch_kernel(uint32_t* own) { own[PX_EPOCH] += 1u; }

// Publish "this rank's data for the current epoch is ready" in `slot`.  The
// data was written by kernels that completed before this one started (stream
// order); the fence makes it visible to the other GPUs before the flag.
__global__ void px_signal_kernel(uint32_t* own, int slot) {
  __threadfence_system();
  st_release_sys(own + slot, own[PX_EPOCH]);
}

__global__ void px_signal_next_kernel(uint32_t* own, int slot) {
  __threadfence_system();
  st_release_sys(own + slot, own[PX_EPOCH] + 1u);
}

__global__ void __launch_bounds__(256) px_zero_kernel(float* base, const PxChunk* chunks,
                                                      int nchunks) {
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const PxChunk ch = chunks[c];
    float* d = base + ch.dst_off;
    const int n4 = (reinterpret_cast<uintptr_t>(d) & 15u) == 0 ? ch.len >> 2 : 0;
    for (int i = threadIdx.x; i < n4; i += blockDim.x)
      reinterpret_cast<float4*>(d)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = (n4 << 2) + threadIdx.x; i < ch.len; i += blockDim.x) d[i] = 0.f;
  }
}

// Reduce-scatter of one bucket: own[x] = sum over ranks p (in rank order) of
// grad_p[x] for every x of the chunks (this rank's parts of the bucket's
// tensors).  Chunk offsets are multiples of 4 floats; lengths too, except a
// tensor's last chunk.  WM bounds the world size at compile time; each thread
// keeps U = 16 / WM float4 positions (U x W loads over NVLink) in flight.
template <int WM>
__global__ void __launch_bounds__(256) px_reduce_kernel(PxTables T, const PxChunk* chunks,
                                                        int nchunks, int slot, int* status) {
  constexpr int U = 16 / WM;
  if (!cta_wait_peers(T, slot, status)) return;
  const int W = T.world;
  float* own = T.grad[T.rank];
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const PxChunk ch = chunks[c];
    const long long base = ch.dst_off;   // float offset from the gradient base
    const int n4 = ch.len >> 2;
    for (int i0 = threadIdx.x; i0 < n4; i0 += blockDim.x * U) {
      float4 v[U][WM];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * blockDim.x;
#pragma unroll
        for (int p = 0; p < WM; ++p)
          if (p < W && i < n4) v[u][p] = reinterpret_cast<const float4*>(T.grad[p] + base)[i];
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i >= n4) break;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int p = 0; p < WM; ++p)
          if (p < W) {
            acc.x += v[u][p].x;
            acc.y += v[u][p].y;
            acc.z += v[u][p].z;
            acc.w += v[u][p].w;
          }
        reinterpret_cast<float4*>(own + base)[i] = acc;
      }
    }
    for (int i = (n4 << 2) + threadIdx.x; i < ch.len; i += blockDim.x) {
      float acc = 0.f;
      for (int p = 0; p < W; ++p) acc += T.grad[p][base + i];
      own[base + i] = acc;
    }
  }
}

// Copies of byte ranges from rank ch.peer's buffer (src table) into this
// rank's buffer (dst), after every rank published `slot`.  16-byte vectors
// where both ends and the length allow, bytes otherwise.
__global__ void __launch_bounds__(256) px_copy_kernel(PxTables T, const char* const* src,
                                                      char* dst, const PxChunk* chunks,
                                                      int nchunks, int slot, int* status) {
  if (!cta_wait_peers(T, slot, status)) return;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const PxChunk ch = chunks[c];
    const char* s = src[ch.peer] + ch.src_off;
    char* d = dst + ch.dst_off;
    const uintptr_t ends = reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d);
    const bool vec = (ends & 15u) == 0;
    const int n16 = vec ? ch.len >> 4 : 0;
    constexpr int U = 8;   // 16-byte loads in flight per thread
    for (int i0 = threadIdx.x; i0 < n16; i0 += blockDim.x * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < n16) v[u] = reinterpret_cast<const uint4*>(s)[i];
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < n16) reinterpret_cast<uint4*>(d)[i] = v[u];
      }
    }
    for (int i = (n16 << 4) + threadIdx.x; i < ch.len; i += blockDim.x) d[i] = s[i];
  }
}

// Wait (one thread) until every rank published `slot` for the current epoch.
__global__ void px_wait_kernel(PxTables T, int slot, int* status) {
  wait_peers(T, slot, T.flags[T.rank][PX_EPOCH], status);
}

// Sharded gradient norm: publish this rank's sum of squares (norm_out[2]),
// wait for every rank's, and leave their sum (in rank order) in norm_out[2].
__global__ void px_norm_kernel(PxTables T, float* norm_out, int* status) {
  uint32_t* own = T.flags[T.rank];
  const uint32_t epoch = own[PX_EPOCH];
  const int part = PX_NORM_PART + (int)(epoch & 1u);
  own[part] = __float_as_uint(norm_out[2]);
  __threadfence_system();
  st_release_sys(own + PX_NORM, epoch);
  if (!wait_peers(T, PX_NORM, epoch, status)) return;
  float s = 0.f;
  for (int p = 0; p < T.world; ++p) s += __uint_as_float(ld_acquire_sys(T.flags[p] + part));
  norm_out[2] = s;
}

}  // namespace

cudaError_t px_epoch(uint32_t* own_flags, cudaStream_t st) {
  px_epoch_kernel<<<1, 1, 0, st>>>(own_flags);
  return cudaGetLastError();
}

cudaError_t px_signal(uint32_t* own_flags, int slot, cudaStream_t st) {
  px_signal_kernel<<<1, 1, 0, st>>>(own_flags, slot);
  return cudaGetLastError();
}

cudaError_t px_signal_next(uint32_t* own_flags, int slot, cudaStream_t st) {
  px_signal_next_kernel<<<1, 1, 0, st>>>(own_flags, slot);
  return cudaGetLastError();
}

cudaError_t px_zero(float* base, const PxChunk* chunks, int nchunks, cudaStream_t st) {
  if (nchunks <= 0) return cudaSuccess;
  px_zero_kernel<<<nchunks < 592 ? nchunks : 592, 256, 0, st>>>(base, chunks, nchunks);
  return cudaGetLastError();
}

cudaError_t px_reduce(const PxTables& T, const PxChunk* chunks, int nchunks, int slot, int grid,
                      int* status, cudaStream_t st) {
  if (nchunks <= 0) return cudaSuccess;
  if (T.world > PX_MAX_WORLD) return cudaErrorInvalidValue;
  const int g = grid < nchunks ? grid : nchunks;
  if (T.world <= 2) px_reduce_kernel<2><<<g, 256, 0, st>>>(T, chunks, nchunks, slot, status);
  else if (T.world <= 4) px_reduce_kernel<4><<<g, 256, 0, st>>>(T, chunks, nchunks, slot, status);
  else px_reduce_kernel<8><<<g, 256, 0, st>>>(T, chunks, nchunks, slot, status);
  return cudaGetLastError();
}

cudaError_t px_copy(const PxTables& T, const char* const* src, char* dst, const PxChunk* chunks,
                    int nchunks, int slot, int grid, int* status, cudaStream_t st) {
  if (nchunks <= 0) return cudaSuccess;
  px_copy_kernel<<<grid < nchunks ? grid : nchunks, 256, 0, st>>>(T, src, dst, chunks, nchunks,
                                                                  slot, status);
  return cudaGetLastError();
}

cudaError_t px_wait(const PxTables& T, int slot, int* status, cudaStream_t st) {
  px_wait_kernel<<<1, 1, 0, st>>>(T, slot, status);
  return cudaGetLastError();
}

cudaError_t px_norm(const PxTables& T, float* norm_out, int* status, cudaStream_t st) {
  px_norm_kernel<<<1, 1, 0, st>>>(T, norm_out, status);
  return cudaGetLastError();
}

}  // namespace ne
