// ne_px.h -- internal interface of the peer-memory ZeRO-1 exchange (px.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace ne {

constexpr int PX_MAX_WORLD = 8;

// Words of each rank's flag buffer.  Flags hold the epoch (exchange count) up
// to which the rank's data is ready; PX_NORM_PART[0..1] hold the rank's sum of
// squares (float bits) of the even / odd epochs.
enum PxSlot : int {
  PX_EPOCH = 0,      // this rank's exchange count (read only by itself)
  PX_EMBED = 1,      // token ids and dY rows final, and this rank's reduce-scatters done
  PX_NORM = 2,       // sum of squares published
  PX_W16 = 3,        // AdamW done: owned parts of the weights updated
  PX_NORM_PART = 4,  // two words
  PX_ABORT = 6,      // set by this rank's first wait that ran out: its later waits give up at once
  PX_ZEROED = 7,     // this rank's owned dW parts are zero for exchanges >= this value: the
                     // other ranks' fused dW products may add into them
  PX_READY0 = 8      // + bucket: the bucket's gradients final (bucket 0 = tail, 1 + layer)
};

// Kernel-side view of all ranks (passed by value).
struct PxTables {
  uint32_t* flags[PX_MAX_WORLD];   // each rank's flag words (this rank's: local)
  float* grad[PX_MAX_WORLD];       // each rank's gradient pool
  int world = 1, rank = 0;
  unsigned long long limit_ns = 0; // wall-clock limit of one wait
};

// One unit of work.  Reduce: floats [dst_off, dst_off + len) of the gradient
// pool.  Copy: len bytes from src_off of rank `peer`'s buffer to dst_off.
struct PxChunk {
  long long src_off;
  long long dst_off;
  int len;
  int peer;
};

// Part of an n-element tensor owned by `rank` of `world`: boundaries at
// multiples of 64 elements (256-byte aligned fp32, 128-byte aligned bf16),
// the last rank taking the remainder; every element is owned exactly once.
inline void px_part(long long n, int world, int rank, long long* off, long long* len) {
  auto b = [&](int p) -> long long { return p >= world ? n : (n * p / world) / 64 * 64; };
  *off = b(rank);
  *len = b(rank + 1) - b(rank);
}

cudaError_t px_epoch(uint32_t* own_flags, cudaStream_t st);
cudaError_t px_signal(uint32_t* own_flags, int slot, cudaStream_t st);
// As px_signal, publishing the current epoch + 1 (PX_ZEROED: ready for the next exchange).
cudaError_t px_signal_next(uint32_t* own_flags, int slot, cudaStream_t st);
// Zero floats [dst_off, dst_off + len) of every chunk, relative to `base`.
cudaError_t px_zero(float* base, const PxChunk* chunks, int nchunks, cudaStream_t st);
cudaError_t px_reduce(const PxTables& T, const PxChunk* chunks, int nchunks, int slot, int grid,
                      int* status, cudaStream_t st);
cudaError_t px_copy(const PxTables& T, const char* const* src, char* dst, const PxChunk* chunks,
                    int nchunks, int slot, int grid, int* status, cudaStream_t st);
cudaError_t px_norm(const PxTables& T, float* norm_out, int* status, cudaStream_t st);
cudaError_t px_wait(const PxTables& T, int slot, int* status, cudaStream_t st);

}  // namespace ne
