// gemm_tc.cuh -- persistent tcgen05/TMEM GEMM for sm_100a.
//
//   acc[m, n] = sum_k A[m, k] * B[n, k]          (both operands K-major, bf16)
//
// A is tiled 128 rows at a time along TMEM lanes, B is tiled BN rows at a time
// along TMEM columns, K in blocks of 64 (one 128-byte swizzle atom).  The
// same kernel serves both orientations the hot path needs:
//   * token-major ("normal"):  A = activations [tokens, K], B = weight [out, K]
//     (prefill / training: many tokens, epilogue owns one token row);
//   * weight-major ("swap-AB"): A = weight [out, K], B = activations [batch, K]
//     (decode: batch <= 256 fits one N tile; output written transposed).
//
// Warp roles (320 threads, one CTA per SM, persistent over work units):
//   warp 0      TMA producer: one lane streams A/B boxes into a STAGES-deep
//               shared-memory ring (mbarrier full/empty handshake).
//   warp 1      MMA issuer: allocates TMEM, one lane issues tcgen05.mma
//               (128 x BN x 16 per instruction) into one of two accumulators,
//               commits stage release and accumulator-ready barriers.
//   warps 2-9   epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4) .. +31; warps 2-5 take the even column chunks,
//               warps 6-9 the odd ones), apply the fused epilogue functor,
//               store.  Two warps per lane quarter keep enough independent
//               instructions and stores in flight for the compute-heavy
//               epilogues (SwiGLU backward) and the fp32 outputs.
// The two TMEM accumulators let the epilogue of work unit i overlap the MMAs
// of unit i+1.  Split-K: a work unit is (m_tile, n_tile, split); the epilogue
// receives the split index and writes a partial slab that the consumer
// kernel reduces in a fixed order (deterministic, no atomics).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "ne_device.cuh"

namespace ne {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_EPI_WARPS = 8;                     // two per TMEM lane quarter
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;

struct GemmShape {
  int M, N, K;          // logical sizes (A rows, B rows, reduction)
  int m_tiles, n_tiles; // ceil(M/128), ceil(N/BN)
  int splits;           // split-K factor
  int kb_per_split;     // k-blocks (of 64) per split
  int* status;          // device status word (timeouts)
  int prefetch_a;       // A does not depend on the preceding kernel: its first
                        // tiles may be loaded before the PDL dependency wait
  int group_m;          // m-tiles per raster group (0: one group of all m-tiles)
};

// Work unit u -> (m tile, n tile, split).  Units run M-fastest inside groups
// of group_m m-tiles: a wave of consecutive units covers a block of about
// group_m x (CTAs / group_m) tiles, whose A panels and B panels both stay in
// L2 while the wave reuses them, instead of sweeping all of A once per n-tile.
__device__ __forceinline__ void unit_coords(const GemmShape& sh, int u, int& mt, int& nt,
                                            int& sp) {
  const int mn = sh.m_tiles * sh.n_tiles;
  sp = u / mn;
  const int r = u - sp * mn;
  const int G = sh.group_m;
  if (G <= 0 || G >= sh.m_tiles) {
    mt = r % sh.m_tiles;
    nt = r / sh.m_tiles;
    return;
  }
  const int per_group = G * sh.n_tiles;
  const int g = r / per_group;
  const int first = g * G;
  const int gm = sh.m_tiles - first < G ? sh.m_tiles - first : G;
  const int w = r - g * per_group;
  mt = first + w % gm;
  nt = w / gm;
}

// CG = 2: a CTA pair shares each 256 x BN tile (cta_group::2); each CTA
// stages its 128 rows of A and BN/2 rows of B.
template <int BN, int CG = 1>
struct GemmCfg {
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
  static_assert(CG == 1 || (CG == 2 && BN % 32 == 0), "pair tiles split B in halves");
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = (BN / CG) * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (196 * 1024) / STAGE_BYTES > 8 ? 8 : (196 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                                   : (2 * BN <= 256) ? 256 : 512;
  static constexpr int CH = (BN % 32 == 0) ? 32 : 16;   // epilogue column chunk
  // ring + 1 KB of barriers / bookkeeping + 1 KB alignment slack
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 2048;
  // staged epilogues add one box slot per epilogue warp after the barriers
  static constexpr int SMEM_BYTES_STAGED = SMEM_BYTES + 8 * 4096;
  static_assert(SMEM_BYTES_STAGED <= 232448, "shared memory per CTA");
};

// ------------------------------------------------------------------ epilogues
// Each functor: apply(p, m, n0, v[CH], split, M, N).  m is the A-side row,
// n0 the first B-side column of the chunk; only (m < M, n < N) is stored.
// A functor that reads global memory besides the accumulator may also define
// prefetch(p, m, n0, ncols, M, N): called one work unit ahead, it hints that
// row's inputs into L2 so the epilogue's loads hit L2 instead of waiting on
// HBM latency with few bytes in flight.
template <class E, class = void>
struct EpiHasPrefetch { static constexpr bool value = false; };
template <class E>
struct EpiHasPrefetch<E, decltype(void(&E::prefetch))> { static constexpr bool value = true; };

// Vector (16-byte) accesses are used only where the row pointer allows them;
// an output whose leading dimension leaves rows unaligned takes the scalar path.
__device__ __forceinline__ bool al16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// L2 hints for `bytes` contiguous bytes starting at p (128-byte lines).
__device__ __forceinline__ void prefetch_row_l2(const void* p, int bytes) {
  const char* c = reinterpret_cast<const char*>(p);
  for (int o = 0; o < bytes; o += 128) prefetch_l2(c + o);
}

// fp32 store, transposed (swap-AB):  out[split*split_stride + n*ld + m]
struct EpiF32T {
  struct Params { float* out; long long ld; long long split_stride; };
  template <int CH>
  __device__ static void apply(const Params& p, int m, int n0, const float (&v)[CH], int split,
                               int M, int N) {
    if (m >= M) return;
    float* base = p.out + (long long)split * p.split_stride + m;
#pragma unroll
    for (int j = 0; j < CH; ++j)
      if (n0 + j < N) base[(long long)(n0 + j) * p.ld] = v[j];
  }
};

// Swap-AB LM head fused with the greedy choice (A = the tied embedding, row m
// = token id; B = the batch): instead of storing logits[n][m], every
// (token id, batch row) value becomes a 64-bit key whose order is that of the
// logit, ties broken towards the smaller id (numpy's first-index argmax), and
// the key of each batch row's best id is kept with one atomicMax per column
// per warp.  A warp's 32 rows x 32 columns are first reduced with a
// transposing butterfly (31 exchanges) so lane j ends with column j's best.
__device__ __forceinline__ unsigned long long argmax_key(float v, int m) {
  const uint32_t u = __float_as_uint(v);
  const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);   // order-preserving
  return ((unsigned long long)o << 32) | (uint32_t)~(uint32_t)m;
}
struct EpiArgmaxT {
  struct Params { unsigned long long* keys; };
  template <int CH>
  __device__ static void apply(const Params& p, int m, int n0, const float (&v)[CH], int, int M,
                               int N) {
    static_assert(CH == 32, "one column per lane");
    const int lane = threadIdx.x & 31;
    unsigned long long k[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) k[j] = m < M ? argmax_key(v[j], m) : 0ull;
#pragma unroll
    for (int o = 16, cnt = 32; o >= 1; o >>= 1, cnt >>= 1) {
      const bool up = (lane & o) != 0;   // keeps the upper half of its columns
#pragma unroll
      for (int i = 0; i < cnt / 2; ++i) {
        const unsigned long long send = up ? k[i] : k[i + cnt / 2];
        const unsigned long long keep = up ? k[i + cnt / 2] : k[i];
        const unsigned long long recv = __shfl_xor_sync(0xffffffffu, send, o);
        k[i] = keep > recv ? keep : recv;
      }
    }
    if (n0 + lane < N && k[0] != 0ull) atomicMax(p.keys + n0 + lane, k[0]);
  }
};

// Swap-AB W1/W3 projection with the SwiGLU fused (decode, K not split): the
// accumulator rows are the 16-row-interleaved W13 features -- rows
// [32c, 32c+16) hold h1 of features [16c, 16c+16), rows [32c+16, 32c+32) their
// h3 -- and its columns are batch rows.  A warp's lanes hold 32 consecutive
// rows starting at a multiple of 32, so lane i < 16 has h1 and lane i + 16 has
// h3 of feature 16c + i.  Per pair of columns, lanes < 16 finish the even
// column and lanes >= 16 the odd one, each taking the value it lacks from its
// partner (one exchange):
//   gate[n * ld + f] = bf16( silu(h1) * h3 ),  silu(x) = x * (1 / (1 + exp(-x)))
// (generate.py:93-94,190; the same expression as swiglu_split_kernel).
struct EpiSwiGLUT {
  struct Params { __nv_bfloat16* gate; long long ld; };
  template <int CH>
  __device__ static void apply(const Params& p, int m, int n0, const float (&v)[CH], int, int M,
                               int N) {
    static_assert(CH % 2 == 0, "column pairs");
    const int lane = threadIdx.x & 31;
    const bool hi = lane >= 16;
    const int f = (m >> 5) * 16 + (lane & 15);
    __nv_bfloat16* const col = p.gate + f;
#pragma unroll
    for (int j = 0; j < CH; j += 2) {
      const float give = hi ? v[j] : v[j + 1];
      const float got = __shfl_xor_sync(0xffffffffu, give, 16);
      const float h1 = hi ? got : v[j];
      const float h3 = hi ? v[j + 1] : got;
      const int n = n0 + j + (hi ? 1 : 0);
      if (m < M && n < N)
        col[(long long)n * p.ld] = __float2bfloat16_rn(h1 * (1.0f / (1.0f + expf(-h1))) * h3);
    }
  }
};

// fp32 store, row-major:  out[split*split_stride + m*ld + n]
struct EpiF32 {
  struct Params { float* out; long long ld; long long split_stride; };
  template <int CH>
  __device__ static void apply(const Params& p, int m, int n0, const float (&v)[CH], int split,
                               int M, int N) {
    if (m >= M) return;
    float* row = p.out + (long long)split * p.split_stride + (long long)m * p.ld + n0;
    if (n0 + CH <= N && al16(row)) {
#pragma unroll
      for (int j = 0; j < CH; j += 4)
        *reinterpret_cast<float4*>(row + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
      for (int j = 0; j < CH; ++j)
        if (n0 + j < N) row[j] = v[j];
    }
  }
};

// fp32 store, row-major, plus softmax statistics of the stored chunk (the
// classifier logits of the training step):
//   out[m*ld + n] = acc;   stats[m*stats_ld + n0/32] = (max_j acc, sum_j exp(acc - max))
// over the chunk's columns n0 .. n0+31 that are < N.  The cross-entropy
// kernel combines a row's chunk statistics into its log-sum-exp, so it reads
// the logits once instead of twice.
struct EpiF32Stats {
  struct Params { float* out; long long ld; float2* stats; long long stats_ld; };
  template <int CH>
  __device__ static void apply(const Params& p, int m, int n0, const float (&v)[CH], int,
                               int M, int N) {
    static_assert(CH == 32, "statistics epilogue needs 32-column chunks");
    if (m >= M || n0 >= N) return;
    float* row = p.out + (long long)m * p.ld + n0;
    float mx = -3.402823466e38f;
    if (n0 + CH <= N && al16(row)) {
#pragma unroll
      for (int j = 0; j < CH; j += 4)
        *reinterpret_cast<float4*>(row + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
#pragma unroll
      for (int j = 0; j < CH; ++j) mx = fmaxf(mx, v[j]);
    } else {
      for (int j = 0; j < CH; ++j)
        if (n0 + j < N) {
          row[j] = v[j];
          mx = fmaxf(mx, v[j]);
        }
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < CH; ++j)
      if (n0 + j < N) sum += __expf(v[j] - mx);
    p.stats[(long long)m * p.stats_ld + n0 / CH] = make_float2(mx, sum);
  }
};

// 16-bit store, row-major:  out[m*ld + n] = alpha * acc  (bf16, or fp16 if half_out)
struct EpiBF16 {
  struct Params { void* out; long long ld; float alpha; int half_out; };
  template <int CH>
  __device__ static void apply(const Params& p, int m, int n0, const float (&v)[CH], int,
                               int M, int N) {
    if (m >= M) return;
    const long long base = (long long)m * p.ld + n0;
    float w[CH];
#pragma unroll
    for (int j = 0; j < CH; ++j) w[j] = p.alpha * v[j];
    if (p.half_out) {
      __half* row = reinterpret_cast<__half*>(p.out) + base;
      if (n0 + CH <= N && al16(row)) {
#pragma unroll
        for (int j = 0; j < CH; j += 8) {
          uint4 pk;
          __half2* h = reinterpret_cast<__half2*>(&pk);
#pragma unroll
          for (int t = 0; t < 4; ++t) h[t] = __floats2half2_rn(w[j + 2 * t], w[j + 2 * t + 1]);
          *reinterpret_cast<uint4*>(row + j) = pk;
        }
      } else {
        for (int j = 0; j < CH; ++j)
          if (n0 + j < N) row[j] = __float2half_rn(w[j]);
      }
      return;
    }
    __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(p.out) + base;
    if (n0 + CH <= N && al16(row)) {
#pragma unroll
      for (int j = 0; j < CH; j += 8) {
        uint4 pk;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int t = 0; t < 4; ++t) h[t] = __floats2bfloat162_rn(w[j + 2 * t], w[j + 2 * t + 1]);
        *reinterpret_cast<uint4*>(row + j) = pk;
      }
    } else {
      for (int j = 0; j < CH; ++j)
        if (n0 + j < N) row[j] = __float2bfloat16_rn(w[j]);
    }
  }
};

// fp32 add, row-major:  out[m*ld + n] = in[m*ld + n] + alpha * acc
struct EpiAdd {
  struct Params { float* out; const float* in; long long ld; float alpha; };
  __device__ static void prefetch(const Params& p, int m, int n0, int ncols, int M, int N) {
    if (m >= M || n0 >= N) return;
    prefetch_row_l2(p.in + (long long)m * p.ld + n0, 4 * min(ncols, N - n0));
  }
  template <int CH>
  __device__ static void apply(const Params& p, int m, int n0, const float (&v)[CH], int,
                               int M, int N) {
    if (m >= M) return;
    float* orow = p.out + (long long)m * p.ld + n0;
    const float* irow = p.in + (long long)m * p.ld + n0;
    if (n0 + CH <= N && al16(orow) && al16(irow)) {
      float4 r[CH / 4];   // every load issued before the first store
#pragma unroll
      for (int j = 0; j < CH; j += 4) r[j / 4] = *reinterpret_cast<const float4*>(irow + j);
#pragma unroll
      for (int j = 0; j < CH; j += 4) {
        float4 q = r[j / 4];
        q.x += p.alpha * v[j]; q.y += p.alpha * v[j + 1];
        q.z += p.alpha * v[j + 2]; q.w += p.alpha * v[j + 3];
        *reinterpret_cast<float4*>(orow + j) = q;
      }
    } else {
      for (int j = 0; j < CH; ++j)
        if (n0 + j < N) orow[j] = irow[j] + p.alpha * v[j];
    }
  }
};

// fp32 residual update, row-major:  x[m*ld + n] += alpha * acc
// (atomic: red.global.add, for split-K accumulation into gradient buffers)
struct EpiResid {
  struct Params { float* x; long long ld; float alpha; int atomic; };
  __device__ static void prefetch(const Params& p, int m, int n0, int ncols, int M, int N) {
    if (p.atomic || m >= M || n0 >= N) return;
    prefetch_row_l2(p.x + (long long)m * p.ld + n0, 4 * min(ncols, N - n0));
  }
  template <int CH>
  __device__ static void apply(const Params& p, int m, int n0, const float (&v)[CH], int,
                               int M, int N) {
    if (m >= M) return;
    float* row = p.x + (long long)m * p.ld + n0;
    if (p.atomic) {
#pragma unroll
      for (int j = 0; j < CH; ++j)
        if (n0 + j < N) atomicAdd(row + j, p.alpha * v[j]);
      return;
    }
    if (n0 + CH <= N && al16(row)) {
      float4 rr[CH / 4];   // every load issued before the first store
#pragma unroll
      for (int j = 0; j < CH; j += 4) rr[j / 4] = *reinterpret_cast<const float4*>(row + j);
#pragma unroll
      for (int j = 0; j < CH; j += 4) {
        float4 r = rr[j / 4];
        if (p.alpha == 1.0f) {
          r.x += v[j]; r.y += v[j + 1]; r.z += v[j + 2]; r.w += v[j + 3];
        } else {
          r.x += p.alpha * v[j]; r.y += p.alpha * v[j + 1];
          r.z += p.alpha * v[j + 2]; r.w += p.alpha * v[j + 3];
        }
        *reinterpret_cast<float4*>(row + j) = r;
      }
    } else {
      for (int j = 0; j < CH; ++j)
        if (n0 + j < N) row[j] += (p.alpha == 1.0f) ? v[j] : p.alpha * v[j];
    }
  }
};


// ------------------------------------------------------------------ staged epilogues
// A staged functor (kStage 1: store, 2: element-wise add into the output)
// turns one accumulator chunk of its row into kCols output values; the kernel
// writes the warp's 32 rows into a swizzled shared-memory box and one lane
// sends the box with a TMA tensor store (or reduce-add), so global memory
// sees whole 128-byte lines written asynchronously instead of 32 scattered
// row segments per store instruction.  The output tensor map (tmC) describes
// the destination; boxes are clipped to its extent by the hardware.
template <class E, class = void>
struct EpiStage { static constexpr int value = 0; };
template <class E>
struct EpiStage<E, decltype(void(E::kStage))> { static constexpr int value = E::kStage; };

constexpr int GEMM_STAGE_SLOT = 4096;   // shared-memory box(es) per epilogue warp
constexpr int GEMM_STAGE_BOX2 = 2048;   // offset of an optional second box in the slot

template <class E, class = void>
struct EpiTransposed { static constexpr bool value = false; };
template <class E>
struct EpiTransposed<E, decltype(void(E::kTransposed))> { static constexpr bool value = true; };

// A functor with kCols2 also fills a second box (tmD), e.g. an activation
// saved for the backward pass.
template <class E, class = void>
struct EpiHasBox2 { static constexpr bool value = false; };
template <class E>
struct EpiHasBox2<E, decltype(void(E::kCols2))> { static constexpr bool value = true; };

// A functor with a `Pre` type reads global memory for each chunk: preload()
// issues the loads of a chunk into registers one chunk ahead of its stage(),
// so their latency overlaps the current chunk's TMEM read, arithmetic and
// store instead of stalling every chunk.
template <class E, class = void>
struct EpiPre { static constexpr bool value = false; struct type {}; };
template <class E>
struct EpiPre<E, decltype(void(sizeof(typename E::Pre)))> {
  static constexpr bool value = true;
  using type = typename E::Pre;
};

// Write this lane's row (N 16-bit or 32-bit values, 32, 64 or 128 bytes) of a
// 32-row box at `box`, in the layout of the TMA swizzle that matches the row
// size (the 16-byte chunk index XORed with address bits 7.. of the row start):
// conflict-free, 8 lanes cover all banks.
template <class T, int N>
__device__ __forceinline__ void stage_row(uint32_t box, int lane, const T (&o)[N]) {
  constexpr int ROWB = N * (int)sizeof(T);
  static_assert(ROWB == 32 || ROWB == 64 || ROWB == 128, "box rows of 32, 64 or 128 bytes");
  const uint32_t row = box + lane * ROWB;
#pragma unroll
  for (int q = 0; q < ROWB / 16; ++q) {
    const int phys = ROWB == 128 ? (q ^ (lane & 7))
                     : ROWB == 64 ? (q ^ ((lane >> 1) & 3))
                                  : (q ^ ((lane >> 2) & 1));
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (sizeof(T) == 4) {
        w[k] = __float_as_uint(o[4 * q + k]);
      } else {
        w[k] = (uint32_t)o[8 * q + 2 * k] | ((uint32_t)o[8 * q + 2 * k + 1] << 16);
      }
    }
    st_shared_v4(row + phys * 16, w[0], w[1], w[2], w[3]);
  }
}

// Weight-major ("swap-AB") GEMMs: the accumulator row is an output feature
// and its columns are batch rows, so the chunk is written transposed into the
// box (box row = batch row, box column = feature) and added element-wise into
// out [N (batch), M (features)] fp32 with alpha: split-K units add into the same
// output, so no partial slabs are written or re-read.
struct EpiF32TS {
  static constexpr int kStage = 2;
  static constexpr int kCols = 32;
  static constexpr int kTransposed = 1;
  using Out = float;
  struct Params { float alpha; };
  template <int CH>
  __device__ static void stage(const Params& p, int, int, const float (&v)[CH], Out (&o)[kCols],
                               int, int) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) o[j] = p.alpha * v[j];
  }
};

// fp32 row-major store (tmC: fp32 [M, N]).
struct EpiF32S {
  static constexpr int kStage = 1;
  static constexpr int kCols = 32;
  using Out = float;
  struct Params { int unused; };
  __device__ static int out_col(const Params&, int n0) { return n0; }
  template <int CH>
  __device__ static void stage(const Params&, int, int, const float (&v)[CH], Out (&o)[kCols],
                               int, int) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) o[j] = v[j];
  }
};

// 16-bit row-major store of alpha*acc (bf16, or fp16 if half_out).
struct EpiBF16S {
  static constexpr int kStage = 1;
  static constexpr int kCols = 32;
  using Out = uint16_t;
  struct Params { float alpha; int half_out; };
  __device__ static int out_col(const Params&, int n0) { return n0; }
  template <int CH>
  __device__ static void stage(const Params& p, int, int, const float (&v)[CH], Out (&o)[kCols],
                               int, int) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) {
      const float x = p.alpha * v[j];
      o[j] = p.half_out ? __half_as_ushort(__float2half_rn(x))
                        : __bfloat16_as_ushort(__float2bfloat16_rn(x));
    }
  }
};

// fp32 accumulation into the owner of each element (the dW products of the
// peer-memory ZeRO-1 exchange): element m*ld + n of the output goes to the rank
// whose part holds it, local or over NVLink.  Staged (kStage 3): the warp's
// 32 x 32 box is read back from shared memory one row per instruction, so a
// warp's 32 adds cover one contiguous 128-byte row segment, as element-wise
// fp32 reductions (red.add: atomic at the destination, so every rank and
// every split-K unit may add into the same element; system scope for another
// GPU's memory).  Parts start at multiples of 64 elements and ld is a
// multiple of 64, so a 32-column chunk of a row has one owner.
struct EpiResidPeer {
  static constexpr int kStage = 3;
  static constexpr int kCols = 32;
  using Out = float;
  struct Params {
    float* dst[8];
    long long bound[9];
    long long ld;
    const unsigned* abort;   // nonzero: the exchange gave up; no more adds into other ranks
    float alpha;
    int world, rank;
  };
  __device__ static int out_col(const Params&, int n0) { return n0; }
  template <int CH>
  __device__ static void stage(const Params& p, int, int, const float (&v)[CH], Out (&o)[kCols],
                               int, int) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) o[j] = p.alpha * v[j];
  }
  // rows y .. y+31, columns n0 .. n0+31 from the box (stage_row layout: row r
  // at r*128 bytes, its 16-byte chunk q at (q ^ (r & 7)) * 16)
  __device__ static void flush(const Params& p, uint32_t box, int lane, int y, int n0, int M,
                               int N) {
    const bool stopped = p.abort && *reinterpret_cast<const volatile unsigned*>(p.abort) != 0u;
    const bool col_ok = n0 + lane < N;
    const uint32_t col = ((lane & 3) << 2);
    // owner of row y's chunk, then advanced row by row (parts are contiguous)
    long long e = (long long)y * p.ld + n0;
    int o = 0;
    while (o + 1 < p.world && e >= p.bound[o + 1]) ++o;
#pragma unroll 4
    for (int r = 0; r < 32; ++r, e += p.ld) {
      if (y + r >= M) break;
      while (o + 1 < p.world && e >= p.bound[o + 1]) ++o;
      float w;
      asm volatile("ld.shared.f32 %0, [%1];"
                   : "=f"(w)
                   : "r"(box + r * 128 + ((((lane >> 2) ^ (r & 7)) << 4) | col)));
      if (!col_ok) continue;
      float* d = p.dst[o] + e + lane;
      if (o != p.rank) {
        if (!stopped)
          asm volatile("red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(d), "f"(w) : "memory");
      } else {
        asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(d), "f"(w) : "memory");
      }
    }
  }
};

// fp32 accumulation  out[m][n] += alpha * acc  through the TMA add (atomic per
// element in L2, so split-K units may add into the same tile).
struct EpiResidS {
  static constexpr int kStage = 2;
  static constexpr int kCols = 32;
  using Out = float;
  struct Params { float alpha; };
  __device__ static int out_col(const Params&, int n0) { return n0; }
  template <int CH>
  __device__ static void stage(const Params& p, int, int, const float (&v)[CH], Out (&o)[kCols],
                               int, int) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) o[j] = p.alpha * v[j];
  }
};

// Classifier logits (fp32 store) plus the chunk's softmax statistics, as EpiF32Stats.
struct EpiF32StatsS {
  static constexpr int kStage = 1;
  static constexpr int kCols = 32;
  using Out = float;
  struct Params { float2* stats; long long stats_ld; };
  __device__ static int out_col(const Params&, int n0) { return n0; }
  template <int CH>
  __device__ static void stage(const Params& p, int m, int n0, const float (&v)[CH],
                               Out (&o)[kCols], int M, int N) {
    float mx = -3.402823466e38f;
#pragma unroll
    for (int j = 0; j < kCols; ++j) {
      o[j] = v[j];
      if (n0 + j < N) mx = fmaxf(mx, v[j]);
    }
    if (m >= M || n0 >= N) return;
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kCols; ++j)
      if (n0 + j < N) sum += __expf(v[j] - mx);
    p.stats[(long long)m * p.stats_ld + n0 / kCols] = make_float2(mx, sum);
  }
};

// SwiGLU on the W1/W3 16-row-interleaved projection (ffnFused,
// mil_dynamic.h:238-306): columns [32c, 32c+16) of the accumulator hold h1 of
// features [16c, 16c+16), [32c+16, 32c+32) their h3.
//   gate[m, 16c + j] = bf16( silu(h1_j) * h3_j )          (box 1: 16 columns)
//   h13[m, 32c .. 32c+32) = bf16(acc)  (optional box 2, saved for the backward)
struct EpiSwiGLUS {
  static constexpr int kStage = 1;
  static constexpr int kCols = 16;
  using Out = uint16_t;
  static constexpr int kCols2 = 32;
  using Out2 = uint16_t;
  struct Params { int save_h13; };
  __device__ static int out_col(const Params&, int n0) { return n0 >> 1; }
  __device__ static int out_col2(const Params&, int n0) { return n0; }
  __device__ static bool has_box2(const Params& p) { return p.save_h13 != 0; }
  template <int CH>
  __device__ static void stage(const Params& p, int, int, const float (&v)[CH], Out (&o)[kCols],
                               Out2 (&o2)[kCols2], int, int) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float h1 = v[j], h3 = v[16 + j];
      o[j] = __bfloat16_as_ushort(__float2bfloat16_rn(__fdividef(h1, 1.0f + __expf(-h1)) * h3));
    }
    if (p.save_h13) {
#pragma unroll
      for (int j = 0; j < 32; ++j) o2[j] = __bfloat16_as_ushort(__float2bfloat16_rn(v[j]));
    }
  }
};

// SwiGLU backward (ffnBwdFull, mil_dynamic.h:320-409): acc = d_gate[m, f] for
// 32 consecutive features f0 .. f0+31; with h1, h3 from the saved interleaved
// projection h13 [m, 2F] (bf16, EpiSwiGLUS's second box):
//   dh1 = alpha*dg * h3 * s * (1 + h1 * (1 - s)),  s = sigmoid(h1)
//   dh3 = alpha*dg * h1 * s
// written bf16 into dh13 [m, 2F] columns [2*f0, 2*f0 + 64): two 16-feature
// blocks of (dh1 | dh3), the W1/W3 16-row-interleaved order.
struct EpiSwiGLUBwdS {
  static constexpr int kStage = 1;
  static constexpr int kCols = 64;
  using Out = uint16_t;
  struct Params { const __nv_bfloat16* h13; long long F; float alpha; };
  __device__ static int out_col(const Params&, int n0) { return 2 * n0; }
  __device__ static void prefetch(const Params& p, int m, int n0, int ncols, int M, int N) {
    if (m >= M || n0 >= N) return;
    prefetch_row_l2(p.h13 + (long long)m * 2 * p.F + 2 * n0, 4 * min(ncols, N - n0));
  }
  // 128 contiguous bytes of the chunk's row: (h1 x16 | h3 x16) for each of its
  // two 16-feature blocks, loaded one chunk ahead
  struct Pre { uint4 r[8]; };
  __device__ static void preload(const Params& p, int m, int n0, int M, int N, Pre& pr) {
    if (m < M && n0 < N) {
      const uint4* src = reinterpret_cast<const uint4*>(p.h13 + (long long)m * 2 * p.F + 2 * n0);
#pragma unroll
      for (int q = 0; q < 8; ++q) pr.r[q] = src[q];
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) pr.r[q] = make_uint4(0, 0, 0, 0);
    }
  }
  template <int CH>
  __device__ static void stage(const Params& p, int m, int n0, const float (&v)[CH],
                               Out (&o)[kCols], int M, int N, const Pre& pr) {
    static_assert(CH == 32, "SwiGLU backward epilogue needs 32-column chunks");
    const uint4 (&r)[8] = pr.r;
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&r[4 * b + q]);
        const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&r[4 * b + 2 + q]);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 x1 = __bfloat1622float2(ha[t]);
          const float2 x3 = __bfloat1622float2(hb[t]);
          const int f = 16 * b + 8 * q + 2 * t;      // feature offset in the chunk
          const float g0 = p.alpha * v[f], g1 = p.alpha * v[f + 1];
          const float s0 = __fdividef(1.0f, 1.0f + __expf(-x1.x));
          const float s1 = __fdividef(1.0f, 1.0f + __expf(-x1.y));
          const int slot = 32 * b + 8 * q + 2 * t;   // dh1 slot; dh3 is 16 further
          o[slot] = __bfloat16_as_ushort(__float2bfloat16_rn(g0 * x3.x * s0 * (1.0f + x1.x * (1.0f - s0))));
          o[slot + 1] = __bfloat16_as_ushort(__float2bfloat16_rn(g1 * x3.y * s1 * (1.0f + x1.y * (1.0f - s1))));
          o[slot + 16] = __bfloat16_as_ushort(__float2bfloat16_rn(g0 * x1.x * s0));
          o[slot + 17] = __bfloat16_as_ushort(__float2bfloat16_rn(g1 * x1.y * s1));
        }
      }
  }
};

// ------------------------------------------------------------------ kernel
// A_MN / B_MN: the operand is stored MN-major in global memory ([K rows][MN
// contiguous]); its tile is then loaded as 64-wide MN boxes of 64 K-rows (8 KB
// each, placed 8 KB apart) and described to the MMA as MN-major.
template <int BN, class Epi, int AB_FMT, int A_MN = 0, int B_MN = 0, int CG = 1>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
               const GemmShape sh, const typename Epi::Params ep) {
  using C = GemmCfg<BN, CG>;
  constexpr bool PAIR = CG == 2;
  constexpr int TILE_M = GEMM_BM * CG;          // rows of A per work unit (both CTAs)
  static_assert(!PAIR || !EpiTransposed<Epi>::value, "pair tiles: row-major epilogues only");
  // 0: direct stores, 1: TMA store, 2: TMA add, 3: the warp adds the box itself (Epi::flush)
  constexpr int STG = EpiStage<Epi>::value;
  static_assert(!B_MN || BN % 64 == 0, "MN-major B needs whole 64-wide boxes");
  constexpr uint32_t MN_BOX = 64 * GEMM_BK * 2;   // one 64 (MN) x 64 (K) box
  constexpr int STAGES = C::STAGES;
  constexpr int CH = C::CH;
  constexpr uint32_t IDESC = umma_idesc_f16(TILE_M, BN, AB_FMT, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled tiles
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t tiles = base;                                   // STAGES x (A | B)
  const uint32_t bars = base + STAGES * C::STAGE_BYTES;          // barriers
  const uint32_t full_bar = bars;                                // [STAGES]
  const uint32_t empty_bar = bars + 8 * STAGES;                  // [STAGES]
  const uint32_t tfull_bar = bars + 16 * STAGES;                 // [2]
  const uint32_t tempty_bar = bars + 16 * STAGES + 16;           // [2]
  const uint32_t drain_bar = bars + 16 * STAGES + 32;            // [1]
  uint8_t* const gbars = gbase + STAGES * C::STAGE_BYTES;
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(gbars + 16 * STAGES + 40);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(gbars + 16 * STAGES + 44);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int units = sh.m_tiles * sh.n_tiles * sh.splits;
  // pair mode: both CTAs of a cluster walk the same units (one per cluster)
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const int u_first = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int u_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(empty_bar + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar + 8 * a, 1);
      // pair mode: one arrival per epilogue warp of both CTAs (on the even CTA's)
      mbar_init(tempty_bar + 8 * a, PAIR ? 2 * GEMM_EPI_WARPS : 32 * GEMM_EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (STG == 1 || STG == 2) tma_prefetch_desc(&tmC);
    if constexpr (EpiHasBox2<Epi>::value) tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();   // the peer's barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      // A is streamed (evict first) unless a raster group reuses its panels
      const uint64_t pol_a = sh.group_m > 0 ? policy_evict_normal() : policy_evict_first();
      const uint64_t pol_b = policy_evict_last();
      // pair mode: every load of both CTAs completes on the even CTA's full
      // barrier, which the even CTA arms for the bytes of both
      auto tma_ld = [&](uint32_t dst, const CUtensorMap* tm, uint32_t bar, int c0, int c1,
                        uint64_t pol) {
        if constexpr (PAIR) tma_load_2d_pair(dst, tm, mapa_shared(bar, 0), c0, c1, pol);
        else tma_load_2d(dst, tm, bar, c0, c1, pol);
      };
      auto load_a = [&](uint32_t dst, uint32_t bar, int k0, int m0) {
        if constexpr (A_MN) {
#pragma unroll
          for (int j = 0; j < GEMM_BM / 64; ++j)
            tma_ld(dst + j * MN_BOX, &tmA, bar, m0 + 64 * j, k0, pol_a);
        } else {
          tma_ld(dst, &tmA, bar, k0, m0, pol_a);
        }
      };
      auto load_b = [&](uint32_t dst, uint32_t bar, int k0, int n0) {
        if constexpr (B_MN) {
#pragma unroll
          for (int j = 0; j < BN / CG / 64; ++j)
            tma_ld(dst + j * MN_BOX, &tmB, bar, n0 + 64 * j, k0, pol_b);
        } else {
          tma_ld(dst, &tmB, bar, k0, n0, pol_b);
        }
      };
      const bool arms = !PAIR || crank == 0;
      const int a_row0 = (int)crank * GEMM_BM;          // this CTA's rows of the unit
      const int b_row0 = (int)crank * (BN / CG);
      // Prologue overlap: the first stages' A tiles of this CTA's first unit
      // (weights that no preceding kernel writes) are requested before the
      // programmatic-dependency wait; their B tiles follow after it.
      int pre = 0;
      if (sh.prefetch_a && u_first < units) {
        int mt, nt_unused, sp0;
        unit_coords(sh, u_first, mt, nt_unused, sp0);
        const int kb0 = sp0 * sh.kb_per_split;
        pre = sh.kb_per_split < STAGES ? sh.kb_per_split : STAGES;
        for (int kb = 0; kb < pre; ++kb) {
          if (arms) mbar_arrive_expect_tx(full_bar + 8 * kb, CG * C::STAGE_BYTES);
          load_a(tiles + kb * C::STAGE_BYTES, full_bar + 8 * kb, (kb0 + kb) * GEMM_BK,
                 mt * TILE_M + a_row0);
        }
      }
      pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool first = true;
      for (int u = u_first; u < units && ok; u += u_step) {
        int mt, nt, sp;
        unit_coords(sh, u, mt, nt, sp);
        const int kb0 = sp * sh.kb_per_split;
        for (int kb = 0; kb < sh.kb_per_split; ++kb) {
          const uint32_t sa = tiles + stage * C::STAGE_BYTES;
          if (!(first && kb < pre)) {
            if (!mbar_wait(empty_bar + 8 * stage, phase ^ 1u, sh.status, abort_flag)) {
              ok = false;
              break;
            }
            if (arms) mbar_arrive_expect_tx(full_bar + 8 * stage, CG * C::STAGE_BYTES);
            load_a(sa, full_bar + 8 * stage, (kb0 + kb) * GEMM_BK, mt * TILE_M + a_row0);
          }
          load_b(sa + C::A_BYTES, full_bar + 8 * stage, (kb0 + kb) * GEMM_BK, nt * BN + b_row0);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        first = false;
      }
      // Drain: wait (bounded) until the most recent load issued into every
      // stage has landed, so no TMA write is in flight when the CTA exits.
      // Stages below `stage` were last filled in the current lap (parity
      // `phase`), the others in the previous lap (or never: parity 1 on a
      // fresh barrier reads as complete).  In pair mode only the even CTA's
      // barriers count the loads (of both CTAs); the odd CTA relies on it and
      // on the closing cluster barrier.
      if (arms) {
        for (int s = 0; s < STAGES; ++s) {
          const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(full_bar + 8 * s, par)) {
            if (globaltimer_ns() - t0 > 100000000ull) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0 && (!PAIR || crank == 0)) {   // pair mode: the even CTA issues for both
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = u_first; u < units; u += u_step) {
        if (!mbar_wait(tempty_bar + 8 * acc, acc_phase ^ 1u, sh.status, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < sh.kb_per_split; ++kb) {
          if (!mbar_wait(full_bar + 8 * stage, phase, sh.status, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = tiles + stage * C::STAGE_BYTES;
          // K-major: advance 16 elements (32 B) inside the swizzle atom (+2 in
          // addr>>4); MN-major: advance 16 K-rows (2 x 1 KB groups, +128).
          const uint64_t adesc = A_MN ? smem_desc_mn_sw128(sa, MN_BOX) : smem_desc_k_sw128(sa);
          const uint64_t bdesc = B_MN ? smem_desc_mn_sw128(sa + C::A_BYTES, MN_BOX)
                                      : smem_desc_k_sw128(sa + C::A_BYTES);
          constexpr uint64_t A_STEP = A_MN ? 128 : 2;
          constexpr uint64_t B_STEP = B_MN ? 128 : 2;
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k)
            if constexpr (PAIR)
              umma_f16_pair(d_tmem, adesc + A_STEP * k, bdesc + B_STEP * k, IDESC, (kb | k) != 0);
            else
              umma_f16(d_tmem, adesc + A_STEP * k, bdesc + B_STEP * k, IDESC, (kb | k) != 0);
          // the stage is free again in both CTAs of a pair
          if constexpr (PAIR) umma_commit_pair(empty_bar + 8 * stage, 0x3);
          else umma_commit(empty_bar + 8 * stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if constexpr (PAIR) umma_commit_pair(tfull_bar + 8 * acc, 0x3);   // both epilogues
        else umma_commit(tfull_bar + 8 * acc);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      // Wait (bounded) for every MMA this thread issued before TMEM is freed.
      if constexpr (PAIR) umma_commit_pair(drain_bar, 0x1);
      else umma_commit(drain_bar);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain_bar, 0)) {
        if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..9)
    pdl_wait();   // outputs may still be read by the preceding kernel until it completes
    const int quarter = warp & 3;               // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    const int chunk0 = ((warp - 2) >> 2) * CH;  // first column chunk of this warp
    // staged epilogues: this warp's shared-memory box (1 KB aligned, after the barriers)
    const uint32_t sbuf = base + STAGES * C::STAGE_BYTES + 1024 + (warp - 2) * GEMM_STAGE_SLOT;
    (void)sbuf;

    int acc = 0;
    uint32_t acc_phase = 0;
    const int row0 = (int)crank * GEMM_BM;   // this CTA's rows within a unit
    for (int u = u_first; u < units; u += u_step) {
      int mt, nt, sp;
      unit_coords(sh, u, mt, nt, sp);
      if constexpr (EpiHasPrefetch<Epi>::value) {
        // this unit's rows (first unit only: the others were hinted one unit
        // ahead), then the next unit's, so they are L2-resident by the time
        // the epilogue (which, when it reads inputs, is usually the slower
        // side of the pipeline) reaches them
        if (u == u_first && chunk0 == 0)
          Epi::prefetch(ep, mt * TILE_M + row0 + row_in_tile, nt * BN, BN, sh.M, sh.N);
        const int un = u + u_step;
        if (un < units && chunk0 == 0) {
          int mn, nn, sn;
          unit_coords(sh, un, mn, nn, sn);
          Epi::prefetch(ep, mn * TILE_M + row0 + row_in_tile, nn * BN, BN, sh.M, sh.N);
        }
      }
      // warp-uniform outcome: tcgen05.ld below is a warp-collective instruction
      const bool ready = mbar_wait(tfull_bar + 8 * acc, acc_phase, sh.status, abort_flag);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const int m = mt * TILE_M + row0 + row_in_tile;
      [[maybe_unused]] typename EpiPre<Epi>::type pre_cur, pre_nxt;
      if constexpr (EpiPre<Epi>::value) Epi::preload(ep, m, nt * BN + chunk0, sh.M, sh.N, pre_cur);
#pragma unroll 1
      for (int c = chunk0; c < BN; c += 2 * CH) {
        if constexpr (EpiPre<Epi>::value) {
          if (c + 2 * CH < BN) Epi::preload(ep, m, nt * BN + c + 2 * CH, sh.M, sh.N, pre_nxt);
        }
        float v[CH];
        if constexpr (CH == 32) {
          uint32_t r[32];
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
              "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
              "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
              : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
                "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                "=r"(r[30]), "=r"(r[31])
              : "r"(t_row + c));
          asm volatile(
              "tcgen05.wait::ld.sync.aligned;"
              : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                "+r"(r[30]), "+r"(r[31])
              :
              : "memory");
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        } else {
          uint32_t r[16];
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
              "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
              : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
              : "r"(t_row + c));
          asm volatile(
              "tcgen05.wait::ld.sync.aligned;"
              : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
              :
              : "memory");
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
        }
        if constexpr (STG == 0) {
          Epi::template apply<CH>(ep, m, nt * BN + c, v, sp, sh.M, sh.N);
        } else {
          // staged: 32 rows x kCols outputs -> swizzled box -> one TMA store / add
          static_assert(CH == 32, "staged epilogues work on 32-column chunks");
          constexpr bool BOX2 = EpiHasBox2<Epi>::value;
          static_assert(32 * Epi::kCols * sizeof(typename Epi::Out) <=
                            (BOX2 ? GEMM_STAGE_BOX2 : GEMM_STAGE_SLOT), "staged box exceeds its slot");
          const int n0 = nt * BN + c;
          typename Epi::Out o[Epi::kCols];
          if (lane == 0) bulk_wait_read_all();   // the previous boxes have left the slot
          __syncwarp();
          if constexpr (BOX2) {
            typename Epi::Out2 o2[Epi::kCols2];
            Epi::template stage<CH>(ep, m, n0, v, o, o2, sh.M, sh.N);
            stage_row(sbuf + GEMM_STAGE_BOX2, lane, o2);
          } else if constexpr (EpiPre<Epi>::value) {
            Epi::template stage<CH>(ep, m, n0, v, o, sh.M, sh.N, pre_cur);
            pre_cur = pre_nxt;
          } else {
            Epi::template stage<CH>(ep, m, n0, v, o, sh.M, sh.N);
          }
          if constexpr (EpiTransposed<Epi>::value) {
            // box row j = batch row n0 + j, column lane = this thread's feature:
            // 4-byte stores, one box row per instruction (128B swizzle)
            static_assert(Epi::kCols == 32 && sizeof(typename Epi::Out) == 4, "32x32 fp32 box");
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const uint32_t a = sbuf + j * 128 + ((((lane >> 2) ^ (j & 7)) << 4) | ((lane & 3) << 2));
              asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(__float_as_uint(o[j])) : "memory");
            }
          } else {
            stage_row(sbuf, lane, o);
          }
          if constexpr (STG == 3) {
            __syncwarp();
            Epi::flush(ep, sbuf, lane, mt * TILE_M + row0 + quarter * 32, n0, sh.M, sh.N);
            __syncwarp();   // every lane has read the box before the next chunk's rows
          } else {
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              const int y = mt * TILE_M + row0 + quarter * 32;
              if constexpr (EpiTransposed<Epi>::value) {
                // output [N (batch), M (features)]: x = feature, y = batch row
                if (y < sh.M && n0 < sh.N) tma_reduce_add_2d(&tmC, sbuf, y, n0);
              } else {
                if (y < sh.M && n0 < sh.N) {
                  const int x = Epi::out_col(ep, n0);
                  if constexpr (STG == 1) tma_store_2d(&tmC, sbuf, x, y);
                  else tma_reduce_add_2d(&tmC, sbuf, x, y);
                  if constexpr (EpiHasBox2<Epi>::value) {
                    if (Epi::has_box2(ep))
                      tma_store_2d(&tmD, sbuf + GEMM_STAGE_BOX2, Epi::out_col2(ep, n0), y);
                  }
                }
              }
              bulk_commit_group();
            }
          }
        }
      }
      tc_fence_before();
      if constexpr (PAIR) {
        // one arrival per warp, on the even CTA's barrier (the MMA issuer's)
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar + 8 * acc, 0));
      } else {
        mbar_arrive(tempty_bar + 8 * acc);
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
    if constexpr (STG != 0) {
      if (lane == 0) bulk_wait_all();   // every box written before the CTA exits
    }
  }

  tc_fence_before();
  __syncthreads();
  // pair mode: neither CTA leaves (or frees its TMEM) while the other may
  // still signal its barriers or the pair's MMAs may read its tiles
  if constexpr (PAIR) cluster_sync_all();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace ne
