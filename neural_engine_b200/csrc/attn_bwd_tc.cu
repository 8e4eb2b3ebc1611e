// attn_bwd_tc.cu -- causal GQA attention backward on the tcgen05 tensor cores
// (training step, head_dim 128 or 64, bf16 operands, fp32 accumulation in TMEM).
//
// Same mathematics as attn_bwd.cu (the reference's sdpaBwd1 / sdpaBwd2,
// ane-training/training/training_dynamic/mil_dynamic.h:583-707, then the GQA
// group reduction gqa_reduce_kv_f16, cpu_ops.h:585, and the RoPE / QK-norm
// backward, cpu_ops.h:510-537): P is recomputed from the forward's log2-domain
// row log-sum-exp, dS = P (dP - D) with D = rowsum(dO * O).
//
//   dq_tc_kernel    one CTA per (128-query tile, q-head, sequence).  Per key
//                   tile up to the diagonal: S = Q K^T and dP = dO V^T into
//                   TMEM, dS (bf16) written by the softmax warps into shared
//                   memory as a K-major operand, dQ += dS K in TMEM (K read
//                   MN-major from the same shared tile).  It also computes D
//                   for its queries and publishes it for the dK/dV kernel.
//   dkdv_tc_kernel  one CTA per (128-key tile, kv-head, sequence), thread =
//                   key.  Per (q-head of the group, query tile at or after the
//                   keys): S^T = K Q^T and dP^T = V dO^T into TMEM, P^T and
//                   dS^T (bf16) into shared memory, dV += P^T dO and
//                   dK += dS^T Q in TMEM, so the group's dK / dV are summed in
//                   the accumulators (no atomics).
//   attn_rowdot_kernel  D = rowsum(dO * O) for the pipelined kernels.
//   dq_tp / dkdv_tp     the same products pipelined: the tile split into two
//                   64-wide halves run as independent streams, P / dS kept in
//                   TMEM in place over the scores as the A operand of the
//                   accumulating products, the streamed operand double-
//                   buffered (the defaults; bodies shared by dq_tp_kernel,
//                   dkdv_tp_kernel and bwd_tp_kernel, which runs both in one
//                   launch, dK/dV units first).
// Roles (320 threads): warp 0 TMA producer, warp 1 MMA issuer (one thread),
// warps 2-9 element-wise work, two per TMEM lane quarter, each of the pair
// owning 64 of the 128 score columns (and HD / 2 of the head columns).  Epilogues run the inverse RoPE and the
// QK-norm backward on each thread's row and write bf16 into the gradient of
// the fused QKV projection; the norm gains' gradients are reduced per CTA in
// shared memory and added with one atomic per column.  Every mbarrier wait is
// bounded (2 s) and records a timeout in the status word; the named barriers
// of the epilogue are reached by every element-wise warp whatever happened
// before them.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"

namespace ne {
namespace {

using bf16 = __nv_bfloat16;
constexpr int TB_THREADS = 320;
constexpr int TB_EW = 256;                        // element-wise threads (warps 2..9)
constexpr uint32_t TB_ATOM = 128 * 128;           // 128 rows x 64 bf16, 128-byte swizzle
constexpr uint32_t TB_TILE = 2 * TB_ATOM;         // 128 rows x 128 bf16 (P, dS)
constexpr uint32_t TB_HALF_ROWS = 64 * 128;       // 64 rows of one atom (MN-major K step)
// barrier area: 128 bytes of barriers / TMEM slot / abort flag, then the pair
// exchange [2 quantities][2 halves][128 rows] floats
constexpr int TB_BAR_AREA = 128 + 2 * 2 * 128 * 4;

// Sizes for head dim HD (64 or 128): the Q, dO, K and V tiles hold 128 rows
// of HD / 64 atoms; each element-wise thread of a pair owns CW = HD / 2 head
// columns of its row.
template <int HD>
struct TbCfg {
  static_assert(HD == 64 || HD == 128, "head dim 64 or 128");
  static constexpr int NA = HD / 64;
  static constexpr int CW = HD / 2;
  static constexpr uint32_t TILE = NA * TB_ATOM;
  // gain-gradient staging: 128 rows x (HD + 1) floats (padded against bank conflicts)
  static constexpr uint32_t RED_BYTES = 128 * (HD + 1) * 4;
  static_assert(RED_BYTES <= 4 * TILE, "staging fits in the operand tiles");
  // dq: Q | dO | K | V | dS, then the barrier area (+1 KB alignment slack)
  static constexpr int DQ_SMEM = 4 * TILE + TB_TILE + TB_BAR_AREA + 1024;
  // dkdv: K | V | Q | dO | P | dS | LSE, D (2 x 128 floats, 1 KB), barrier area
  static constexpr int DKV_SMEM = 4 * TILE + 2 * TB_TILE + 1024 + TB_BAR_AREA + 1024;
  // dq_tp: Q | dO | K[2] | V[2] | barrier area
  static constexpr int DQ_TP_SMEM = 6 * TILE + TB_BAR_AREA + 1024;
  // dkdv_tp: K | V | Q[2] | dO[2] | LSE, D [2][2][128] floats (2 KB), barrier area
  static constexpr int DKV_TP_SMEM = 6 * TILE + 2048 + TB_BAR_AREA + 1024;
  static constexpr int BWD_TP_SMEM = DQ_TP_SMEM > DKV_TP_SMEM ? DQ_TP_SMEM : DKV_TP_SMEM;
  static_assert(DKV_TP_SMEM <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
        "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
        "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane (completion: tmem_wait_st).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 32 bf16 values (16 packed words) of one row into a 128-byte-swizzled K-major
// atom: columns c0 .. c0+31 (c0 a multiple of 32 within the atom's 64).
__device__ __forceinline__ void st_row32(uint32_t atom, int row, int c0, const uint32_t (&w)[16]) {
  const uint32_t rbase = atom + row * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int chunk = (c0 >> 3) + q;
    st_shared_v4(rbase + ((chunk ^ (row & 7)) << 4), w[4 * q], w[4 * q + 1], w[4 * q + 2],
                 w[4 * q + 3]);
  }
}

// S-type product: D[128 x 128] = A[128 x HD] . B[128 x HD]^T, both K-major tiles.
template <int HD>
__device__ __forceinline__ void mma_kk(uint32_t d, uint32_t a, uint32_t b, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint64_t ad = smem_desc_k_sw128(a + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
    const uint64_t bd = smem_desc_k_sw128(b + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
    umma_f16(d, ad, bd, idesc, kk > 0);
  }
}
// Accumulating product: D[128 x N] (+)= A[128 x 128 (K)] . B where B is a
// K-major tile [K rows][N] read MN-major (the K dimension runs over its rows;
// N = the idesc's width, 64-column chunks one atom apart).
__device__ __forceinline__ void mma_kmn(uint32_t d, uint32_t a, uint32_t b, uint32_t idesc,
                                        bool acc) {
#pragma unroll
  for (int kk = 0; kk < 128 / 16; ++kk) {
    const uint64_t ad = smem_desc_k_sw128(a + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
    const uint64_t bd = smem_desc_mn_sw128(b + (kk >> 2) * TB_HALF_ROWS, TB_ATOM) + 128 * (kk & 3);
    umma_f16(d, ad, bd, idesc, (acc || kk > 0) ? 1u : 0u);
  }
}

// Inverse RoPE and QK-norm backward of one head row's gradient, this thread
// holding CW = HD / 2 consecutive columns c_lo .. c_lo+CW-1 (the pair's other
// thread the other half): d (in/out), x = raw pre-norm row (same columns),
// dg += d x rrms.
// `xch` is the pair's exchange area [2][128] floats, `bar_id` its barrier.
// Every thread of the pair calls this (ok or not) so the barriers match.
struct RowBwd {
  const float* gain;      // QK-norm gain (nullptr: none)
  float eps;
  const float2* rope_cs;  // [pos][HD / 2] (cos, sin)
};
// cs_smem (optional): this row's (cos, sin) pairs staged by rope_stage,
// pair i at cs_smem[i ^ swz]; otherwise they are read from the table.
template <int HD>
__device__ __forceinline__ void row_bwd(float (&d)[HD / 2], const float* raw, int pos, bool ok,
                                        int c_lo, const RowBwd& rb, float* xch, int half,
                                        int row, int bar_id, float (&dg)[HD / 2],
                                        const float2* cs_smem = nullptr, int swz = 0) {
  constexpr int CW = HD / 2;
  if (ok) {
    const float2* cs = rb.rope_cs + (size_t)pos * (HD / 2) + c_lo / 2;
#pragma unroll
    for (int i = 0; i < CW / 2; ++i) {
      const float2 c = cs_smem ? cs_smem[i ^ swz] : cs[i];
      const float d0 = d[2 * i], d1 = d[2 * i + 1];
      d[2 * i] = d0 * c.x + d1 * c.y;
      d[2 * i + 1] = d1 * c.x - d0 * c.y;
    }
  }
  if (rb.gain == nullptr) return;
  float x[CW];
  float ss = 0.f, dot = 0.f;
#pragma unroll
  for (int i = 0; i < CW; i += 4) {
    const float4 xv = ok ? *reinterpret_cast<const float4*>(raw + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    x[i] = xv.x; x[i + 1] = xv.y; x[i + 2] = xv.z; x[i + 3] = xv.w;
  }
#pragma unroll
  for (int i = 0; i < CW; ++i) {
    ss += x[i] * x[i];
    dot += d[i] * rb.gain[c_lo + i] * x[i];
  }
  xch[half * 128 + row] = ss;
  xch[256 + half * 128 + row] = dot;
  named_bar(bar_id, 64);
  ss += xch[(half ^ 1) * 128 + row];
  dot += xch[256 + (half ^ 1) * 128 + row];
  named_bar(bar_id, 64);   // the exchange area is reusable
  const float rrms = 1.0f / sqrtf(ss / (float)HD + rb.eps);
  const float c = rrms * rrms * dot / (float)HD;
#pragma unroll
  for (int i = 0; i < CW; ++i) {
    if (ok) dg[i] += d[i] * x[i] * rrms;
    d[i] = rrms * (rb.gain[c_lo + i] * d[i] - x[i] * c);
  }
}

// Sum the element-wise threads' gain-gradient rows (each thread: HD / 2
// columns of one of 128 rows) over the rows and add them to dgain[HD].  `red`
// is free shared memory of TbCfg<HD>::RED_BYTES; all 256 element-wise threads
// call it.
template <int HD>
__device__ __forceinline__ void gain_flush(const float (&dg)[HD / 2], float* red, int half,
                                           int row, int t, float* dgain) {
  constexpr int CW = HD / 2;
#pragma unroll
  for (int i = 0; i < CW; ++i) red[row * (HD + 1) + half * CW + i] = dg[i];
  named_bar(5, TB_EW);
  if (t < HD) {
    float s = 0.f;
    for (int r = 0; r < 128; ++r) s += red[r * (HD + 1) + t];
    atomicAdd(dgain + t, s);
  }
}

template <int N>
__device__ __forceinline__ void store_row_bf16(bf16* dst, const float (&d)[N]) {
#pragma unroll
  for (int i = 0; i < N; i += 8) {
    uint4 pk;
    __nv_bfloat162* hv = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
    for (int t = 0; t < 4; ++t) hv[t] = __floats2bfloat162_rn(d[i + 2 * t], d[i + 2 * t + 1]);
    *reinterpret_cast<uint4*>(dst + i) = pk;
  }
}

// Bounded wait that every lane of the warp performs; warp-uniform outcome.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int* status,
                                          volatile int* abort_flag) {
  const bool ok = mbar_wait(bar, parity, status, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

// ================================================================== dQ
template <int HD>
__global__ void __launch_bounds__(TB_THREADS, 1)
dq_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmdO,
             const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
             const bf16* __restrict__ O, const bf16* __restrict__ dO,
             const float* __restrict__ LSE, float* __restrict__ Dl, int S, int Hq, int Hkv,
             int Tmax, float scale_log2, float scale, const float* __restrict__ qkv_raw,
             RowBwd rb, bf16* __restrict__ dqkv, float* __restrict__ dqn, int* status) {
  using C = TbCfg<HD>;
  constexpr int CW = C::CW;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t sQ = base, sdO = sQ + C::TILE, sK = sdO + C::TILE, sV = sK + C::TILE;
  const uint32_t sdS = sV + C::TILE;
  const uint32_t bars = sdS + TB_TILE;
  const uint32_t q_full = bars, kv_full = bars + 8, kv_empty = bars + 16, s_full = bars + 24;
  const uint32_t ds_full = bars + 32, dq_done = bars + 40, drain = bars + 48;
  uint8_t* const gbars = gbase + (bars - base);
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(gbars + 64);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(gbars + 68);
  float* const xch = reinterpret_cast<float*>(gbars + 128);   // [2][2][128], indexed by row

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest-first order: CTAs start in linear block order and the query
  // tiles furthest down the causal triangle walk the most key tiles, so the
  // linear index runs over every (sequence, head) of the last query tile first
  const int nbh = gridDim.y * gridDim.z;
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int qt = gridDim.x - 1 - lin / nbh;
  const int h = (lin % nbh) % gridDim.y, b = (lin % nbh) / gridDim.y;
  const int kvh = h / (Hq / Hkv);
  const int q0 = qt * 128;
  const int n_keys = min(S, q0 + 128);
  const int n_kt = (n_keys + 127) / 128;
  constexpr uint32_t IDESC_S = umma_idesc_f16(128, 128, 1, 0, 0);
  constexpr uint32_t IDESC_Q = umma_idesc_f16(128, HD, 1, 0, 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(ds_full, TB_EW);
    mbar_init(dq_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmdO);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;   // S at +0, dP at +128, dQ at +256 (HD columns)

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      const uint64_t pol = policy_evict_last();
      const int qrow = b * S + q0;
      const int kvrow = (b * Hkv + kvh) * Tmax;
      mbar_arrive_expect_tx(q_full, 2 * C::TILE);
      for (int a = 0; a < C::NA; ++a) {
        tma_load_2d(sQ + a * TB_ATOM, &tmQ, q_full, h * HD + a * 64, qrow, pol);
        tma_load_2d(sdO + a * TB_ATOM, &tmdO, q_full, h * HD + a * 64, qrow, pol);
      }
      int j = 0;
      for (; j < n_kt; ++j) {
        if (j > 0 && !mbar_wait(kv_empty, (j - 1) & 1, status, abort_flag)) break;
        mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
        for (int a = 0; a < C::NA; ++a) {
          tma_load_2d(sK + a * TB_ATOM, &tmK, kv_full, a * 64, kvrow + j * 128, pol);
          tma_load_2d(sV + a * TB_ATOM, &tmV, kv_full, a * 64, kvrow + j * 128, pol);
        }
      }
      // drain (bounded): the loads issued have landed before the CTA exits
      {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
      if (j > 0) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(kv_full, (j - 1) & 1))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, status, abort_flag);
      for (int j = 0; j < n_kt && ok; ++j) {
        if (!(ok = mbar_wait(kv_full, j & 1, status, abort_flag))) break;
        tc_fence_after();
        mma_kk<HD>(tmem, sQ, sK, IDESC_S);           // S = Q K^T
        mma_kk<HD>(tmem + 128, sdO, sV, IDESC_S);    // dP = dO V^T
        umma_commit(s_full);
        if (!(ok = mbar_wait(ds_full, j & 1, status, abort_flag))) break;
        tc_fence_after();
        mma_kmn(tmem + 256, sdS, sK, IDESC_Q, j > 0);   // dQ += dS K
        umma_commit(dq_done);
        umma_commit(kv_empty);
      }
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > 100000000ull) break;
    }
  } else {
    // ------------------------------------------------ element-wise warps
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const bool qv = q < S;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int c_lo = half * 64;    // this thread's score (key) columns
    const int h_lo = half * CW;    // and head columns
    float* const pxch = xch;   // pairs own disjoint rows of the shared exchange area
    pdl_wait();   // O, dO and LSE come from earlier kernels
    // D = rowsum(dO * O) over this thread's CW columns, then the pair's sum
    float dsum = 0.f;
    if (qv) {
      const size_t off = ((size_t)(b * S + q) * Hq + h) * HD + h_lo;
#pragma unroll
      for (int i = 0; i < CW; i += 8) {
        const uint4 ov = *reinterpret_cast<const uint4*>(O + off + i);
        const uint4 gv = *reinterpret_cast<const uint4*>(dO + off + i);
        const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
        const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 of = __bfloat1622float2(o2[t]), gf = __bfloat1622float2(g2[t]);
          dsum += of.x * gf.x + of.y * gf.y;
        }
      }
    }
    pxch[half * 128 + row] = dsum;
    named_bar(1 + quarter, 64);
    const float Drow = dsum + pxch[(half ^ 1) * 128 + row];
    named_bar(1 + quarter, 64);
    if (half == 0 && qv) Dl[((size_t)b * Hq + h) * S + q] = Drow;
    const float Lrow = qv ? LSE[((size_t)b * Hq + h) * S + q] : 0.f;

    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      bool ready = true;
      if (j > 0) ready = warp_wait(dq_done, (j - 1) & 1, status, abort_flag);   // dS free
      ready = warp_wait(s_full, j & 1, status, abort_flag) && ready;
      if (!ready) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t srow = tmem + lane_off;
      const int kbase = j * 128;
      for (int c = c_lo; c < c_lo + 64; c += 32) {
        uint32_t rs[32], rp[32];
        tmem_ld32(srow + c, rs);
        tmem_ld32(srow + 128 + c, rp);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float ds2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = kbase + c + i + e;
            const float p = (qv && key <= q && key < S)
                                ? exp2f(__uint_as_float(rs[i + e]) * scale_log2 - Lrow) : 0.f;
            ds2[e] = p * (__uint_as_float(rp[i + e]) - Drow);
          }
          const __nv_bfloat162 pk = __floats2bfloat162_rn(ds2[0], ds2[1]);
          w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
        }
        st_row32(sdS + (c >> 6) * TB_ATOM, row, c & 63, w);
      }
      fence_async_smem();   // dS visible to the tensor cores
      tc_fence_before();
      mbar_arrive(ds_full);
    }
    // ---- epilogue: dQ * scale through the RoPE / q-norm backward, bf16 out
    if (ok && n_kt > 0) ok = warp_wait(dq_done, (n_kt - 1) & 1, status, abort_flag);
    float d[CW];
#pragma unroll
    for (int i = 0; i < CW; ++i) d[i] = 0.f;
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < CW; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 256 + h_lo + c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) d[c + i] = __uint_as_float(r[i]) * scale;
      }
    }
    const int qkv_dim = (Hq + 2 * Hkv) * HD;
    const size_t tok = (size_t)b * S + (qv ? q : 0);
    const bool rv = ok && qv;
    float dg[CW];
#pragma unroll
    for (int i = 0; i < CW; ++i) dg[i] = 0.f;
    row_bwd<HD>(d, qkv_raw + tok * qkv_dim + (size_t)h * HD + h_lo, q, rv, h_lo, rb, pxch, half,
                row, 1 + quarter, dg);
    if (rv) store_row_bf16(dqkv + tok * qkv_dim + (size_t)h * HD + h_lo, d);
    if (rb.gain != nullptr) {
      // every MMA and load of this CTA has completed (dq_done of the last
      // tile, or nothing was issued): reuse the operand tiles as staging
      gain_flush<HD>(dg, reinterpret_cast<float*>(gbase), half, row, threadIdx.x - 64, dqn);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ================================================================== dK, dV
template <int HD>
__global__ void __launch_bounds__(TB_THREADS, 1)
dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmdO,
               const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
               const float* __restrict__ LSE, const float* __restrict__ Dl, int S, int Hq,
               int Hkv, int Tmax, float scale_log2, float scale,
               const float* __restrict__ qkv_raw, RowBwd rb, bf16* __restrict__ dqkv,
               float* __restrict__ dkn, int* status) {
  using C = TbCfg<HD>;
  constexpr int CW = C::CW;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t sK = base, sV = sK + C::TILE, sQ = sV + C::TILE, sdO = sQ + C::TILE;
  const uint32_t sP = sdO + C::TILE, sdS = sP + TB_TILE;
  float* const sL = reinterpret_cast<float*>(gbase + 4 * C::TILE + 2 * TB_TILE);   // [128]
  float* const sD = sL + 128;                                        // [128]
  const uint32_t bars = sdS + TB_TILE + 1024;
  const uint32_t kv_full = bars, qd_full = bars + 8, qd_empty = bars + 16, s_full = bars + 24;
  const uint32_t ps_full = bars + 32, mm2_done = bars + 40, drain = bars + 48;
  uint8_t* const gbars = gbase + (bars - base);
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(gbars + 64);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(gbars + 68);
  float* const xch = reinterpret_cast<float*>(gbars + 128);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest-first order: the key tiles nearest the start see the most query
  // tiles, so the linear block index runs over every (sequence, kv-head) of
  // key tile 0 first
  const int nbh = gridDim.y * gridDim.z;
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int kt = lin / nbh;
  const int kvh = (lin % nbh) % gridDim.y, b = (lin % nbh) / gridDim.y;
  const int G = Hq / Hkv;
  const int k0 = kt * 128;
  const int n_qt_all = (S + 127) / 128;
  const int n_qt = n_qt_all - kt;          // query tiles at or after this key tile
  const int n_it = G * n_qt;
  constexpr uint32_t IDESC_S = umma_idesc_f16(128, 128, 1, 0, 0);
  constexpr uint32_t IDESC_O = umma_idesc_f16(128, HD, 1, 0, 1);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(qd_full, 32);       // the producer warp's lanes (LSE / D) + the TMA bytes
    mbar_init(qd_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(ps_full, TB_EW);
    mbar_init(mm2_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmdO);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;   // S^T +0, dP^T +128, dV +256, dK +384 (HD columns each)

  if (warp == 0) {
    // ------------------------------------------------ producer (whole warp)
    pdl_wait();
    const uint64_t pol = policy_evict_last();
    const int kvrow = (b * Hkv + kvh) * Tmax + k0;
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
      for (int a = 0; a < C::NA; ++a) {
        tma_load_2d(sK + a * TB_ATOM, &tmK, kv_full, a * 64, kvrow, pol);
        tma_load_2d(sV + a * TB_ATOM, &tmV, kv_full, a * 64, kvrow, pol);
      }
    }
    int it = 0;
    for (; it < n_it; ++it) {
      const int h = kvh * G + it / n_qt;
      const int q0 = (kt + it % n_qt) * 128;
      if (it > 0 && !warp_wait(qd_empty, (it - 1) & 1, status, abort_flag)) break;
      // the tile copies first, then the row statistics (plain loads) while
      // they are in flight; every lane arrives after its own stores
      if (lane == 0) {
        mbar_expect_tx(qd_full, 2 * C::TILE);
        const int qrow = b * S + q0;
        for (int a = 0; a < C::NA; ++a) {
          tma_load_2d(sQ + a * TB_ATOM, &tmQ, qd_full, h * HD + a * 64, qrow, pol);
          tma_load_2d(sdO + a * TB_ATOM, &tmdO, qd_full, h * HD + a * 64, qrow, pol);
        }
      }
      for (int r = lane; r < 128; r += 32) {
        const int qq = q0 + r;
        const bool v = qq < S;
        sL[r] = v ? LSE[((size_t)b * Hq + h) * S + qq] : 0.f;
        sD[r] = v ? Dl[((size_t)b * Hq + h) * S + qq] : 0.f;
      }
      mbar_arrive(qd_full);
    }
    if (lane == 0) {   // drain (bounded)
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(kv_full, 0))
        if (globaltimer_ns() - t0 > 100000000ull) break;
      if (it > 0) {
        const uint64_t t1 = globaltimer_ns();
        while (!mbar_try_wait(qd_full, (it - 1) & 1))
          if (globaltimer_ns() - t1 > 100000000ull) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(kv_full, 0, status, abort_flag);
      for (int it = 0; it < n_it && ok; ++it) {
        if (!(ok = mbar_wait(qd_full, it & 1, status, abort_flag))) break;
        tc_fence_after();
        mma_kk<HD>(tmem, sK, sQ, IDESC_S);           // S^T = K Q^T
        mma_kk<HD>(tmem + 128, sV, sdO, IDESC_S);    // dP^T = V dO^T
        umma_commit(s_full);
        if (!(ok = mbar_wait(ps_full, it & 1, status, abort_flag))) break;
        tc_fence_after();
        mma_kmn(tmem + 256, sP, sdO, IDESC_O, it > 0);    // dV += P^T dO
        mma_kmn(tmem + 384, sdS, sQ, IDESC_O, it > 0);    // dK += dS^T Q
        umma_commit(mm2_done);
        umma_commit(qd_empty);
      }
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > 100000000ull) break;
    }
  } else {
    // ------------------------------------------------ element-wise warps
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int key = k0 + row;
    const bool kv = key < S;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int c_lo = half * 64;
    float* const pxch = xch;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int q0 = (kt + it % n_qt) * 128;
      bool ready = true;
      if (it > 0) ready = warp_wait(mm2_done, (it - 1) & 1, status, abort_flag);   // P, dS free
      ready = warp_wait(s_full, it & 1, status, abort_flag) && ready;
      ready = warp_wait(qd_full, it & 1, status, abort_flag) && ready;   // LSE / D of this tile
      if (!ready) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t srow = tmem + lane_off;
      for (int c = c_lo; c < c_lo + 64; c += 32) {
        uint32_t rs[32], rp[32];
        tmem_ld32(srow + c, rs);
        tmem_ld32(srow + 128 + c, rp);
        uint32_t wp[16], wd[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float p2[2], d2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int ql = c + i + e;
            const int qq = q0 + ql;
            const float p = (kv && key <= qq && qq < S)
                                ? exp2f(__uint_as_float(rs[i + e]) * scale_log2 - sL[ql]) : 0.f;
            p2[e] = p;
            d2[e] = p * (__uint_as_float(rp[i + e]) - sD[ql]);
          }
          const __nv_bfloat162 pp = __floats2bfloat162_rn(p2[0], p2[1]);
          const __nv_bfloat162 dd = __floats2bfloat162_rn(d2[0], d2[1]);
          wp[i >> 1] = *reinterpret_cast<const uint32_t*>(&pp);
          wd[i >> 1] = *reinterpret_cast<const uint32_t*>(&dd);
        }
        st_row32(sP + (c >> 6) * TB_ATOM, row, c & 63, wp);
        st_row32(sdS + (c >> 6) * TB_ATOM, row, c & 63, wd);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(ps_full);
    }
    // ---- epilogue: dV unchanged, dK * scale through RoPE / k-norm backward
    if (ok && n_it > 0) ok = warp_wait(mm2_done, (n_it - 1) & 1, status, abort_flag);
    const int qd = Hq * HD, qkv_dim = (Hq + 2 * Hkv) * HD;
    const size_t tok = (size_t)b * S + (kv ? key : 0);
    const size_t kcol = (size_t)qd + (size_t)kvh * HD, vcol = kcol + (size_t)Hkv * HD;
    const bool rv = ok && kv;
    const int h_lo = half * CW;   // this thread's head columns
    float d[CW];
    if (ok) tc_fence_after();
    // dV
#pragma unroll
    for (int i = 0; i < CW; ++i) d[i] = 0.f;
    if (ok && n_it > 0) {
#pragma unroll
      for (int c = 0; c < CW; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 256 + h_lo + c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) d[c + i] = __uint_as_float(r[i]);
      }
    }
    if (rv) store_row_bf16(dqkv + tok * qkv_dim + vcol + h_lo, d);
    // dK
#pragma unroll
    for (int i = 0; i < CW; ++i) d[i] = 0.f;
    if (ok && n_it > 0) {
#pragma unroll
      for (int c = 0; c < CW; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 384 + h_lo + c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) d[c + i] = __uint_as_float(r[i]) * scale;
      }
    }
    float dg[CW];
#pragma unroll
    for (int i = 0; i < CW; ++i) dg[i] = 0.f;
    row_bwd<HD>(d, qkv_raw + tok * qkv_dim + kcol + h_lo, key, rv, h_lo, rb, pxch, half, row,
                1 + quarter, dg);
    if (rv) store_row_bf16(dqkv + tok * qkv_dim + kcol + h_lo, d);
    if (rb.gain != nullptr)
      gain_flush<HD>(dg, reinterpret_cast<float*>(gbase), half, row, threadIdx.x - 64, dkn);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// The RoPE (cos, sin) pairs of this warp's 32 rows (positions pos0 .. pos0+31,
// lane r = row r), HD / 4 pairs from pair c_lo / 2 on, into stg[32][HD / 4]:
// each row read by the whole warp in one coalesced pass, pair i of row r
// stored at i ^ (r & 15), so the row-per-thread reads that follow hit
// distinct banks.  Positions at or past S are not read (zeros).
template <int HD>
__device__ __forceinline__ void rope_stage(float2* stg, const float2* table, int pos0, int S,
                                           int c_lo, int lane) {
  constexpr int NP = HD / 4;
  if (lane < NP) {
    float2 v[32];   // every row's load in flight before the first store
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      const int pos = pos0 + r;
      v[r] = pos < S ? table[(size_t)pos * (HD / 2) + c_lo / 2 + lane] : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int r = 0; r < 32; ++r) stg[r * NP + (lane ^ (r & 15))] = v[r];
  }
  __syncwarp();
}

// This thread's HD / 2 values of row `row` as bf16 into a tile of 128 rows x
// HD in 128-byte-swizzled atoms of 64 columns (the layout a SWIZZLE_128B
// tensor store reads), columns h_lo .. h_lo + HD / 2 - 1.
template <int HD>
__device__ __forceinline__ void stage_row_bf16(uint32_t tile, int row, int h_lo,
                                               const float (&d)[HD / 2]) {
#pragma unroll
  for (int c = 0; c < HD / 2; c += 32) {
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const __nv_bfloat162 pk = __floats2bfloat162_rn(d[c + i], d[c + i + 1]);
      w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
    }
    const int col = h_lo + c;
    st_row32(tile + (col >> 6) * TB_ATOM, row, col & 63, w);
  }
}

// ================================================================== D = rowsum(dO * O)
// One pass over the attention output and its gradient before the pipelined
// dQ / dK-dV kernels: D[b, h, q] = sum_d dO[b, q, h, d] * O[b, q, h, d]
// (the softmax backward's row term, FlashAttention-2's preprocessing step).
// Rows (token, head) are HD contiguous bf16 in both tensors; a warp takes 8
// consecutive rows, every lane HD / 32 contiguous columns of each, all 16
// loads in flight before the sums.  HBM-bound: 4 * HD bytes read per row.
constexpr int RD_ROWS_PER_WARP = 8;
constexpr int RD_THREADS = 256;

template <int HD>
__global__ void __launch_bounds__(RD_THREADS)
attn_rowdot_kernel(const bf16* __restrict__ O, const bf16* __restrict__ dO, float* __restrict__ Dl,
                   int rows, int S, int Hq) {
  constexpr int EPL = HD / 32;
  using V = typename std::conditional<EPL == 4, uint2, uint32_t>::type;
  pdl_trigger();
  pdl_wait();   // dO comes from the preceding product
  const int lane = threadIdx.x & 31;
  const int r0 = (blockIdx.x * (RD_THREADS / 32) + (threadIdx.x >> 5)) * RD_ROWS_PER_WARP;
  V ov[RD_ROWS_PER_WARP], gv[RD_ROWS_PER_WARP];
#pragma unroll
  for (int k = 0; k < RD_ROWS_PER_WARP; ++k) {
    if (r0 + k < rows) {
      const size_t off = (size_t)(r0 + k) * HD + lane * EPL;
      ov[k] = *reinterpret_cast<const V*>(O + off);
      gv[k] = *reinterpret_cast<const V*>(dO + off);
    } else {
      ov[k] = V{};
      gv[k] = V{};
    }
  }
#pragma unroll
  for (int k = 0; k < RD_ROWS_PER_WARP; ++k) {
    const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov[k]);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv[k]);
    float d = 0.f;
#pragma unroll
    for (int t = 0; t < EPL / 2; ++t) {
      const float2 of = __bfloat1622float2(o2[t]), gf = __bfloat1622float2(g2[t]);
      d += of.x * gf.x + of.y * gf.y;
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) d += __shfl_xor_sync(0xffffffffu, d, sh);
    const int r = r0 + k;
    if (lane == k && r < rows) {
      // row r = (b * S + q) * Hq + h  ->  D[(b * Hq + h) * S + q]
      const int h = r % Hq, bq = r / Hq;
      const int q = bq % S, b = bq / S;
      Dl[((size_t)b * Hq + h) * S + q] = d;
    }
  }
}

// ================================================================== dQ (pipelined)
// dq_tc_kernel's product with the key tile split into two 64-key halves run
// as independent streams (half h: S_h = Q K_h^T at TMEM columns [64h, 64h+64),
// dP_h at [128+64h, ...); the element-wise warps owning those columns write
// bf16 dS_h in place over S_h, and dQ += dS_h K_h reads it from tensor memory
// as its A operand; dQ at 256), with K / V double-buffered so the next key
// tile loads while the current one is in use.  D comes from attn_rowdot_kernel
// (computing it here held every element-wise warp ~8 us before its first tile).
// Work unit `lin` of B x Hq x (query tiles) units, longest first; the tensor
// maps are the kernel's own parameters (passed by reference, so TMA reads them
// from parameter space).
template <int HD>
__device__ __forceinline__ void
dq_tp_body(const CUtensorMap& tmQ, const CUtensorMap& tmdO, const CUtensorMap& tmK,
           const CUtensorMap& tmV, const CUtensorMap& tmO, const float* __restrict__ LSE,
           const float* __restrict__ Dl, int S, int Hq, int Hkv, int Tmax, float scale_log2,
           float scale, const float* __restrict__ qkv_raw, RowBwd rb, bf16* __restrict__ dqkv,
           float* __restrict__ dqn, int* status, int lin, int B) {
  using C = TbCfg<HD>;
  constexpr int CW = C::CW;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  // Q | dO | K[2] | V[2] | barrier area
  const uint32_t sQ = base, sdO = sQ + C::TILE, sK0 = sdO + C::TILE, sV0 = sK0 + 2 * C::TILE;
  const uint32_t bars = base + 6 * C::TILE;
  const uint32_t q_full = bars;
  const uint32_t kv_full = bars + 8;     // [2]
  const uint32_t kv_empty = bars + 24;   // [2]
  const uint32_t s_full = bars + 40;     // [2] per half
  const uint32_t ds_full = bars + 56;    // [2] per half
  const uint32_t acc_done = bars + 72, drain = bars + 80;
  uint8_t* const gbars = gbase + (bars - base);
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(gbars + 96);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(gbars + 100);
  float* const xch = reinterpret_cast<float*>(gbars + 128);   // [2][2][128], indexed by row

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbh = Hq * B;   // longest-first (see dq_tc_kernel)
  const int qt = (S + 127) / 128 - 1 - lin / nbh;
  const int h = (lin % nbh) % Hq, b = (lin % nbh) / Hq;
  const int kvh = h / (Hq / Hkv);
  const int q0 = qt * 128;
  const int n_keys = min(S, q0 + 128);
  const int n_kt = (n_keys + 127) / 128;
  constexpr uint32_t IDESC_S = umma_idesc_f16(128, 64, 1, 0, 0);    // 128 queries x 64 keys
  constexpr uint32_t IDESC_Q = umma_idesc_f16(128, HD, 1, 0, 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(kv_full + 8 * i, 1);
      mbar_init(kv_empty + 8 * i, 1);
      mbar_init(s_full + 8 * i, 1);
      mbar_init(ds_full + 8 * i, TB_EW / 2);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmdO);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      pdl_wait();
      const uint64_t pol = policy_evict_last();
      const int qrow = b * S + q0;
      const int kvrow = (b * Hkv + kvh) * Tmax;
      mbar_arrive_expect_tx(q_full, 2 * C::TILE);
      for (int a = 0; a < C::NA; ++a) {
        tma_load_2d(sQ + a * TB_ATOM, &tmQ, q_full, h * HD + a * 64, qrow, pol);
        tma_load_2d(sdO + a * TB_ATOM, &tmdO, q_full, h * HD + a * 64, qrow, pol);
      }
      int j = 0;
      for (; j < n_kt; ++j) {
        const int buf = j & 1;
        if (j >= 2 && !mbar_wait(kv_empty + 8 * buf, ((j >> 1) - 1) & 1, status, abort_flag))
          break;
        mbar_arrive_expect_tx(kv_full + 8 * buf, 2 * C::TILE);
        for (int a = 0; a < C::NA; ++a) {
          tma_load_2d(sK0 + buf * C::TILE + a * TB_ATOM, &tmK, kv_full + 8 * buf, a * 64,
                      kvrow + j * 128, pol);
          tma_load_2d(sV0 + buf * C::TILE + a * TB_ATOM, &tmV, kv_full + 8 * buf, a * 64,
                      kvrow + j * 128, pol);
        }
      }
      // drain (bounded): the loads issued have landed before the CTA exits
      {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
      for (int i = (j > 2 ? j - 2 : 0); i < j; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(kv_full + 8 * (i & 1), (i >> 1) & 1))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      // half hh of key tile j: S_hh = Q K_hh^T, dP_hh = dO V_hh^T
      auto mma1 = [&](int j, int hh) {
        const int buf = j & 1;
        const uint32_t k = sK0 + buf * C::TILE + hh * TB_HALF_ROWS;
        const uint32_t v = sV0 + buf * C::TILE + hh * TB_HALF_ROWS;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t qd = smem_desc_k_sw128(sQ + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
          const uint64_t kd = smem_desc_k_sw128(k + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
          umma_f16(tmem + 64 * hh, qd, kd, IDESC_S, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t gd = smem_desc_k_sw128(sdO + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
          const uint64_t vd = smem_desc_k_sw128(v + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
          umma_f16(tmem + 128 + 64 * hh, gd, vd, IDESC_S, kk > 0);
        }
        umma_commit(s_full + 8 * hh);
      };
      // dQ += dS_hh K_hh (A from tensor memory, K = 64 keys)
      auto mma2 = [&](int j, int hh) {
        const uint32_t k = sK0 + (j & 1) * C::TILE + hh * TB_HALF_ROWS;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t kd = smem_desc_mn_sw128(k, TB_ATOM) + 128 * kk;
          umma_f16_ts(tmem + 256, tmem + 64 * hh + 8 * kk, kd, IDESC_Q,
                      (j > 0 || hh > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, status, abort_flag);
      if (ok && n_kt > 0 && (ok = mbar_wait(kv_full, 0, status, abort_flag))) {
        tc_fence_after();
        mma1(0, 0);
        mma1(0, 1);
      }
      for (int j = 0; j < n_kt && ok; ++j) {
        for (int hh = 0; hh < 2 && ok; ++hh) {
          if (!(ok = mbar_wait(ds_full + 8 * hh, j & 1, status, abort_flag))) break;
          tc_fence_after();
          mma2(j, hh);
          if (hh == 1) umma_commit(kv_empty + 8 * (j & 1));
          if (j + 1 < n_kt) {
            if (hh == 0) {
              if (!(ok = mbar_wait(kv_full + 8 * ((j + 1) & 1), ((j + 1) >> 1) & 1, status,
                                   abort_flag)))
                break;
              tc_fence_after();
            }
            mma1(j + 1, hh);
          }
        }
      }
      umma_commit(acc_done);
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > 100000000ull) break;
    }
  } else {
    // ------------------------------------------------ element-wise warps
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;   // key half of each tile this warp owns
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const bool qv = q < S;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int h_lo = half * CW;         // head columns of the epilogue
    float* const pxch = xch;
    pdl_wait();   // D (attn_rowdot_kernel) and LSE come from earlier kernels
    const float Drow = qv ? Dl[((size_t)b * Hq + h) * S + q] : 0.f;
    const float Lrow = qv ? LSE[((size_t)b * Hq + h) * S + q] : 0.f;

    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      if (!warp_wait(s_full + 8 * half, j & 1, status, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t srow = tmem + lane_off + 64 * half;
      const int kbase = j * 128 + 64 * half;
      const bool nomask = qv && j < qt;   // key tiles before the diagonal: keys < q0 <= q
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        uint32_t rs[32], rp[32];
        tmem_ld32(srow + c, rs);
        tmem_ld32(srow + 128 + c, rp);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float ds2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float p = ex2_fast(fmaf(__uint_as_float(rs[i + e]), scale_log2, -Lrow));
            if (!nomask) {
              const int key = kbase + c + i + e;
              if (!(qv && key <= q && key < S)) p = 0.f;
            }
            ds2[e] = p * (__uint_as_float(rp[i + e]) - Drow);
          }
          const __nv_bfloat162 pk = __floats2bfloat162_rn(ds2[0], ds2[1]);
          w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
        }
        tmem_st16(srow + (c >> 1), w);   // in place over scores this warp has read
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_full + 8 * half);
    }
    // ---- epilogue: dQ * scale through the RoPE / q-norm backward, bf16 out
    if (ok && n_kt > 0) ok = warp_wait(acc_done, 0, status, abort_flag);
    float d[CW];
#pragma unroll
    for (int i = 0; i < CW; ++i) d[i] = 0.f;
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < CW; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 256 + h_lo + c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) d[c + i] = __uint_as_float(r[i]) * scale;
      }
    }
    const int qkv_dim = (Hq + 2 * Hkv) * HD;
    const size_t tok = (size_t)b * S + (qv ? q : 0);
    const bool rv = ok && qv;
    // every MMA has completed: the operand tiles are free.  RoPE rows of this
    // warp's 32 queries in the Q / dO tiles, the dQ tile in the last V tile
    float2* const rstg = reinterpret_cast<float2*>(gbase) + (warp - 2) * 32 * (HD / 4);
    const uint32_t st_q = sV0 + C::TILE;
    rope_stage<HD>(rstg, rb.rope_cs, q0 + quarter * 32, S, h_lo, lane);
    float dg[CW];
#pragma unroll
    for (int i = 0; i < CW; ++i) dg[i] = 0.f;
    row_bwd<HD>(d, qkv_raw + tok * qkv_dim + (size_t)h * HD + h_lo, q, rv, h_lo, rb, pxch, half,
                row, 1 + quarter, dg, rstg + lane * (HD / 4), lane & 15);
    stage_row_bf16<HD>(st_q, row, h_lo, d);
    fence_async_smem();
    named_bar(6, TB_EW);   // the tile staged; the RoPE rows read
    if (warp == 2 && lane == 0 && ok) {
      // one tensor store per 64 columns (rows at or past S are clipped)
      for (int a = 0; a < C::NA; ++a) tma_store_3d(&tmO, st_q + a * TB_ATOM, h * HD + a * 64, q0, b);
      bulk_commit_group();
      bulk_wait_all();
    }
    if (rb.gain != nullptr)
      gain_flush<HD>(dg, reinterpret_cast<float*>(gbase), half, row, threadIdx.x - 64, dqn);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ================================================================== dK, dV (pipelined)
// The same product as dkdv_tc_kernel with the query tile split into two
// 64-query halves that run as independent streams, P^T and dS^T kept in
// tensor memory, and Q / dO double-buffered:
//   * TMEM: half h's S^T at columns [64h, 64h+64) and dP^T at [128+64h, ...);
//     the element-wise warps of half h (the pair member owning those
//     columns) overwrite them in place with bf16 P^T / dS^T (32 columns
//     each), which the dV += P^T dO and dK += dS^T Q products read as their A
//     operand straight from tensor memory; dV at 256, dK at 384.
//   * The MMA thread issues half A's dV/dK products and the next tile's S^T /
//     dP^T for half A while half B's warps are still in their element-wise
//     pass, and the other way round, so the tensor cores and the element-wise
//     warps overlap; the next Q / dO tile is loaded while the current one is
//     in use.
// Work unit `lin` of B x Hkv x (key tiles) units, longest (key tile 0) first.
template <int HD>
__device__ __forceinline__ void
dkdv_tp_body(const CUtensorMap& tmQ, const CUtensorMap& tmdO, const CUtensorMap& tmK,
             const CUtensorMap& tmV, const CUtensorMap& tmO, const float* __restrict__ LSE,
             const float* __restrict__ Dl, int S, int Hq, int Hkv, int Tmax, float scale_log2,
             float scale, const float* __restrict__ qkv_raw, RowBwd rb, bf16* __restrict__ dqkv,
             float* __restrict__ dkn, int* status, int lin, int B) {
  using C = TbCfg<HD>;
  constexpr int CW = C::CW;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  // K | V | Q[2] | dO[2] | LSE, D [2 buffers][2][128] floats | barrier area
  const uint32_t sK = base, sV = sK + C::TILE;
  const uint32_t sQ0 = sV + C::TILE, sdO0 = sQ0 + 2 * C::TILE;
  float* const sLD = reinterpret_cast<float*>(gbase + 6 * C::TILE);   // [2][2][128]
  const uint32_t bars = base + 6 * C::TILE + 2048;
  const uint32_t kv_full = bars;
  const uint32_t qd_full = bars + 8;     // [2]
  const uint32_t qd_empty = bars + 24;   // [2]
  const uint32_t s_full = bars + 40;     // [2] per half
  const uint32_t ps_full = bars + 56;    // [2] per half
  const uint32_t acc_done = bars + 72, drain = bars + 80;
  uint8_t* const gbars = gbase + (bars - base);
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(gbars + 96);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(gbars + 100);
  float* const xch = reinterpret_cast<float*>(gbars + 128);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest-first order (key tile 0 sees every query tile)
  const int nbh = Hkv * B;
  const int kt = lin / nbh;
  const int kvh = (lin % nbh) % Hkv, b = (lin % nbh) / Hkv;
  const int G = Hq / Hkv;
  const int k0 = kt * 128;
  const int n_qt_all = (S + 127) / 128;
  const int n_qt = n_qt_all - kt;          // query tiles at or after this key tile
  const int n_it = G * n_qt;
  constexpr uint32_t IDESC_S = umma_idesc_f16(128, 64, 1, 0, 0);    // 128 keys x 64 queries
  constexpr uint32_t IDESC_O = umma_idesc_f16(128, HD, 1, 0, 1);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(qd_full + 8 * i, 32);   // the producer warp's lanes (LSE / D) + the TMA bytes
      mbar_init(qd_empty + 8 * i, 1);
      mbar_init(s_full + 8 * i, 1);
      mbar_init(ps_full + 8 * i, TB_EW / 2);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmdO);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ producer (whole warp)
    pdl_wait();
    const uint64_t pol = policy_evict_last();
    const int kvrow = (b * Hkv + kvh) * Tmax + k0;
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
      for (int a = 0; a < C::NA; ++a) {
        tma_load_2d(sK + a * TB_ATOM, &tmK, kv_full, a * 64, kvrow, pol);
        tma_load_2d(sV + a * TB_ATOM, &tmV, kv_full, a * 64, kvrow, pol);
      }
    }
    int it = 0;
    for (; it < n_it; ++it) {
      const int buf = it & 1;
      const int h = kvh * G + it / n_qt;
      const int q0 = (kt + it % n_qt) * 128;
      if (it >= 2 && !warp_wait(qd_empty + 8 * buf, ((it >> 1) - 1) & 1, status, abort_flag))
        break;
      if (lane == 0) {
        mbar_expect_tx(qd_full + 8 * buf, 2 * C::TILE);
        const int qrow = b * S + q0;
        for (int a = 0; a < C::NA; ++a) {
          tma_load_2d(sQ0 + buf * C::TILE + a * TB_ATOM, &tmQ, qd_full + 8 * buf, h * HD + a * 64,
                      qrow, pol);
          tma_load_2d(sdO0 + buf * C::TILE + a * TB_ATOM, &tmdO, qd_full + 8 * buf,
                      h * HD + a * 64, qrow, pol);
        }
      }
      float* const L = sLD + buf * 256;
      for (int r = lane; r < 128; r += 32) {
        const int qq = q0 + r;
        const bool v = qq < S;
        L[r] = v ? LSE[((size_t)b * Hq + h) * S + qq] : 0.f;
        L[128 + r] = v ? Dl[((size_t)b * Hq + h) * S + qq] : 0.f;
      }
      mbar_arrive(qd_full + 8 * buf);
    }
    if (lane == 0) {   // drain (bounded): every load issued has landed
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(kv_full, 0))
        if (globaltimer_ns() - t0 > 100000000ull) break;
      for (int j = (it > 2 ? it - 2 : 0); j < it; ++j) {
        const uint64_t t1 = globaltimer_ns();
        while (!mbar_try_wait(qd_full + 8 * (j & 1), (j >> 1) & 1))
          if (globaltimer_ns() - t1 > 100000000ull) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      // half hh of iteration it: S^T = K Q_hh^T and dP^T = V dO_hh^T
      auto mma1 = [&](int it, int hh) {
        const int buf = it & 1;
        const uint32_t q = sQ0 + buf * C::TILE + hh * TB_HALF_ROWS;
        const uint32_t g = sdO0 + buf * C::TILE + hh * TB_HALF_ROWS;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t kd = smem_desc_k_sw128(sK + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
          const uint64_t qdsc = smem_desc_k_sw128(q + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
          umma_f16(tmem + 64 * hh, kd, qdsc, IDESC_S, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t vd = smem_desc_k_sw128(sV + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
          const uint64_t gd = smem_desc_k_sw128(g + (kk >> 2) * TB_ATOM) + 2 * (kk & 3);
          umma_f16(tmem + 128 + 64 * hh, vd, gd, IDESC_S, kk > 0);
        }
        umma_commit(s_full + 8 * hh);
      };
      // dV += P^T_hh dO_hh, dK += dS^T_hh Q_hh (A from tensor memory, K = 64 queries)
      auto mma2 = [&](int it, int hh) {
        const int buf = it & 1;
        const uint32_t q = sQ0 + buf * C::TILE + hh * TB_HALF_ROWS;
        const uint32_t g = sdO0 + buf * C::TILE + hh * TB_HALF_ROWS;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t gd = smem_desc_mn_sw128(g, TB_ATOM) + 128 * kk;
          umma_f16_ts(tmem + 256, tmem + 64 * hh + 8 * kk, gd, IDESC_O,
                      (it > 0 || hh > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t qdsc = smem_desc_mn_sw128(q, TB_ATOM) + 128 * kk;
          umma_f16_ts(tmem + 384, tmem + 128 + 64 * hh + 8 * kk, qdsc, IDESC_O,
                      (it > 0 || hh > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(kv_full, 0, status, abort_flag);
      if (ok && n_it > 0 && (ok = mbar_wait(qd_full, 0, status, abort_flag))) {
        tc_fence_after();
        mma1(0, 0);
        mma1(0, 1);
      }
      for (int it = 0; it < n_it && ok; ++it) {
        for (int hh = 0; hh < 2 && ok; ++hh) {
          if (!(ok = mbar_wait(ps_full + 8 * hh, it & 1, status, abort_flag))) break;
          tc_fence_after();
          mma2(it, hh);
          if (hh == 1) umma_commit(qd_empty + 8 * (it & 1));   // both halves read Q / dO
          if (it + 1 < n_it) {
            if (hh == 0) {
              const int nb = (it + 1) & 1;
              if (!(ok = mbar_wait(qd_full + 8 * nb, ((it + 1) >> 1) & 1, status, abort_flag)))
                break;
              tc_fence_after();
            }
            mma1(it + 1, hh);
          }
        }
      }
      umma_commit(acc_done);
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > 100000000ull) break;
    }
  } else {
    // ------------------------------------------------ element-wise warps
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;        // query half of the tile this warp owns
    const int row = quarter * 32 + lane;
    const int key = k0 + row;
    const bool kv = key < S;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float* const pxch = xch;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int buf = it & 1;
      const int q0 = (kt + it % n_qt) * 128;
      bool ready = warp_wait(s_full + 8 * half, it & 1, status, abort_flag);
      ready = warp_wait(qd_full + 8 * buf, (it >> 1) & 1, status, abort_flag) && ready;
      if (!ready) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* L = sLD + buf * 256 + 64 * half;
      const float* Dv = L + 128;
      const uint32_t srow = tmem + lane_off + 64 * half;
      // queries of an off-diagonal, complete tile all follow every key of
      // this tile: no causal or length mask there
      const bool nomask = kv && (it % n_qt) != 0 && q0 + 128 <= S;
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        uint32_t rs[32], rp[32];
        tmem_ld32(srow + c, rs);
        tmem_ld32(srow + 128 + c, rp);
        uint32_t wp[16], wd[16];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 lv = *reinterpret_cast<const float4*>(L + c + i);
          const float4 dv = *reinterpret_cast<const float4*>(Dv + c + i);
          const float la[4] = {lv.x, lv.y, lv.z, lv.w}, da[4] = {dv.x, dv.y, dv.z, dv.w};
          float p4[4], d4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float p = ex2_fast(fmaf(__uint_as_float(rs[i + e]), scale_log2, -la[e]));
            if (!nomask) {
              const int qq = q0 + 64 * half + c + i + e;
              if (!(kv && key <= qq && qq < S)) p = 0.f;
            }
            p4[e] = p;
            d4[e] = p * (__uint_as_float(rp[i + e]) - da[e]);
          }
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const __nv_bfloat162 pp = __floats2bfloat162_rn(p4[e], p4[e + 1]);
            const __nv_bfloat162 dd = __floats2bfloat162_rn(d4[e], d4[e + 1]);
            wp[(i + e) >> 1] = *reinterpret_cast<const uint32_t*>(&pp);
            wd[(i + e) >> 1] = *reinterpret_cast<const uint32_t*>(&dd);
          }
        }
        // in place: the packed words of columns c..c+31 land in columns
        // c/2 .. c/2+15, all of which this warp has already read
        tmem_st16(srow + (c >> 1), wp);
        tmem_st16(srow + 128 + (c >> 1), wd);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ps_full + 8 * half);
    }
    // ---- epilogue: dV unchanged, dK * scale through RoPE / k-norm backward
    if (ok && n_it > 0) ok = warp_wait(acc_done, 0, status, abort_flag);
    const int qd = Hq * HD, qkv_dim = (Hq + 2 * Hkv) * HD;
    const size_t tok = (size_t)b * S + (kv ? key : 0);
    const size_t kcol = (size_t)qd + (size_t)kvh * HD, vcol = kcol + (size_t)Hkv * HD;
    const bool rv = ok && kv;
    const int h_lo = half * CW;   // this thread's head columns
    // every MMA has completed: the operand tiles are free.  RoPE rows of this
    // warp's 32 keys in the K / V tiles, the dV and dK tiles in the dO tiles
    float2* const rstg = reinterpret_cast<float2*>(gbase) + (warp - 2) * 32 * (HD / 4);
    const uint32_t st_v = sdO0, st_k = sdO0 + C::TILE;
    rope_stage<HD>(rstg, rb.rope_cs, k0 + quarter * 32, S, h_lo, lane);
    float d[CW];
    if (ok) tc_fence_after();
#pragma unroll
    for (int i = 0; i < CW; ++i) d[i] = 0.f;
    if (ok && n_it > 0) {
#pragma unroll
      for (int c = 0; c < CW; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 256 + h_lo + c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) d[c + i] = __uint_as_float(r[i]);
      }
    }
    stage_row_bf16<HD>(st_v, row, h_lo, d);
#pragma unroll
    for (int i = 0; i < CW; ++i) d[i] = 0.f;
    if (ok && n_it > 0) {
#pragma unroll
      for (int c = 0; c < CW; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 384 + h_lo + c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) d[c + i] = __uint_as_float(r[i]) * scale;
      }
    }
    float dg[CW];
#pragma unroll
    for (int i = 0; i < CW; ++i) dg[i] = 0.f;
    row_bwd<HD>(d, qkv_raw + tok * qkv_dim + kcol + h_lo, key, rv, h_lo, rb, pxch, half, row,
                1 + quarter, dg, rstg + lane * (HD / 4), lane & 15);
    stage_row_bf16<HD>(st_k, row, h_lo, d);
    fence_async_smem();
    named_bar(6, TB_EW);   // both tiles staged; the RoPE rows read
    if (warp == 2 && lane == 0 && ok) {
      // one tensor store per 64 columns of each (rows at or past S are clipped)
      for (int a = 0; a < C::NA; ++a) {
        tma_store_3d(&tmO, st_v + a * TB_ATOM, (int)vcol + a * 64, k0, b);
        tma_store_3d(&tmO, st_k + a * TB_ATOM, (int)kcol + a * 64, k0, b);
      }
      bulk_commit_group();
      bulk_wait_all();
    }
    if (rb.gain != nullptr)
      gain_flush<HD>(dg, reinterpret_cast<float*>(gbase), half, row, threadIdx.x - 64, dkn);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

template <int HD>
__global__ void __launch_bounds__(TB_THREADS, 1)
dq_tp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmdO,
             const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
             const __grid_constant__ CUtensorMap tmO, const float* __restrict__ LSE,
             const float* __restrict__ Dl, int S, int Hq, int Hkv, int Tmax, float scale_log2,
             float scale, const float* __restrict__ qkv_raw, RowBwd rb, bf16* __restrict__ dqkv,
             float* __restrict__ dqn, int* status) {
  dq_tp_body<HD>(tmQ, tmdO, tmK, tmV, tmO, LSE, Dl, S, Hq, Hkv, Tmax, scale_log2, scale, qkv_raw,
                 rb, dqkv, dqn, status,
                 blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), gridDim.z);
}

template <int HD>
__global__ void __launch_bounds__(TB_THREADS, 1)
dkdv_tp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmdO,
               const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
               const __grid_constant__ CUtensorMap tmO, const float* __restrict__ LSE,
               const float* __restrict__ Dl, int S, int Hq, int Hkv, int Tmax, float scale_log2,
               float scale, const float* __restrict__ qkv_raw, RowBwd rb,
               bf16* __restrict__ dqkv, float* __restrict__ dkn, int* status) {
  dkdv_tp_body<HD>(tmQ, tmdO, tmK, tmV, tmO, LSE, Dl, S, Hq, Hkv, Tmax, scale_log2, scale,
                   qkv_raw, rb, dqkv, dkn, status,
                   blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), gridDim.z);
}

// dK/dV and dQ in one launch (both read D from the pre-pass and nothing the
// other writes): CTAs [0, n_kv) take the dK/dV units, the rest the dQ units,
// so the longest units (dK/dV of key tile 0) start first and the two kernels'
// partial last waves share the SMs instead of following one another.
template <int HD>
__global__ void __launch_bounds__(TB_THREADS, 1)
bwd_tp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmdO,
              const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
              const __grid_constant__ CUtensorMap tmO, const float* __restrict__ LSE,
              const float* __restrict__ Dl, int S, int Hq, int Hkv, int Tmax, float scale_log2,
              float scale, const float* __restrict__ qkv_raw, RowBwd rbq, RowBwd rbk,
              bf16* __restrict__ dqkv, float* __restrict__ dqn, float* __restrict__ dkn,
              int* status, int B) {
  const int n_kv = ((S + 127) / 128) * Hkv * B;
  if ((int)blockIdx.x < n_kv)
    dkdv_tp_body<HD>(tmQ, tmdO, tmK, tmV, tmO, LSE, Dl, S, Hq, Hkv, Tmax, scale_log2, scale,
                     qkv_raw, rbk, dqkv, dkn, status, (int)blockIdx.x, B);
  else
    dq_tp_body<HD>(tmQ, tmdO, tmK, tmV, tmO, LSE, Dl, S, Hq, Hkv, Tmax, scale_log2, scale,
                   qkv_raw, rbq, dqkv, dqn, status, (int)blockIdx.x - n_kv, B);
}

// ------------------------------------------------------------------ host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 [rows, cols] row-major, 128-byte-swizzled boxes of 64 columns x 128 rows.
bool tmap_tile(CUtensorMap* tm, const void* ptr, long long rows, long long cols) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// bf16 [B][S][cols] (row-major, cols contiguous) as a 3D map with
// 128-byte-swizzled boxes of 64 columns x 128 rows x 1 sequence: tensor
// stores of a 128-row tile stop at the sequence's end.
bool tmap_rows3d(CUtensorMap* tm, const void* ptr, long long B, long long S, long long cols) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)(S * cols * 2)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace

bool attn_bwd_tc_supported(int hd) { return hd == 128 || hd == 64; }

namespace {

// dK / dV kernel (NE_DKDV_TP): the pipelined one with P^T / dS^T in tensor
// memory (default), or "0" the one with P^T / dS^T in shared memory.
bool dkdv_pipelined() {
  static const bool on = [] {
    const char* e = std::getenv("NE_DKDV_TP");
    return !(e && e[0] == '0');
  }();
  return on;
}
// The tcgen05 dQ kernel (NE_DQ_TP): pipelined with dS in tensor memory
// (default), or "0" the serial one with dS in shared memory.
bool dq_pipelined() {
  static const bool on = [] {
    const char* e = std::getenv("NE_DQ_TP");
    return !(e && e[0] == '0');
  }();
  return on;
}

// The pipelined dQ and dK/dV kernels in one launch (NE_ATTN_BWD_MERGE, "0"
// keeps two launches).
bool bwd_merged() {
  static const bool on = [] {
    const char* e = std::getenv("NE_ATTN_BWD_MERGE");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int HD>
cudaError_t launch_bwd_tc_hd(const CUtensorMap& tq, const CUtensorMap& tdo, const CUtensorMap& tk,
                             const CUtensorMap& tv, const CUtensorMap& to, const __nv_bfloat16* Q,
                             const __nv_bfloat16* K, const __nv_bfloat16* V,
                             const __nv_bfloat16* O, const __nv_bfloat16* dO, const float* LSE,
                             float* Dl, int B, int S, int Hq, int Hkv, int Tmax,
                             const float* qkv_raw, const float* qn, const float* kn, float qk_eps,
                             const float2* rope_cs, __nv_bfloat16* dqkv, float* dqn, float* dkn,
                             int* status, cudaStream_t st, bool tc_dq) {
  using C = TbCfg<HD>;
  static bool attr = false;   // one flag per instantiation
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(dq_tc_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::DQ_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(dkdv_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::DKV_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(dkdv_tp_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::DKV_TP_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(dq_tp_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::DQ_TP_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd_tp_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::BWD_TP_SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const float scale = 1.0f / sqrtf((float)HD);
  const float scale_log2 = scale * 1.4426950408889634f;
  const int n_t = (S + 127) / 128;
  // dQ first: the mma.sync and serial tcgen05 kernels also publish D, which
  // dK / dV read; the pipelined one reads D from its own pre-pass
  cudaError_t e;
  if (!tc_dq) {
    e = launch_attn_dq_mma(Q, K, V, O, dO, LSE, Dl, B, S, Hq, Hkv, HD, Tmax, qkv_raw, qn, qk_eps,
                           rope_cs, dqkv, dqn, st);
  } else if (dq_pipelined()) {
    const int rows = B * S * Hq;
    const int per_block = RD_ROWS_PER_WARP * (RD_THREADS / 32);
    e = launch_k(attn_rowdot_kernel<HD>, dim3((rows + per_block - 1) / per_block),
                 dim3(RD_THREADS), 0, st, O, dO, Dl, rows, S, Hq);
    if (e != cudaSuccess) return e;
    if (dkdv_pipelined() && bwd_merged())
      return launch_k(bwd_tp_kernel<HD>, dim3(n_t * (Hkv + Hq) * B), dim3(TB_THREADS),
                      (size_t)C::BWD_TP_SMEM, st, tq, tdo, tk, tv, to, LSE, (const float*)Dl, S,
                      Hq, Hkv, Tmax, scale_log2, scale, qkv_raw, RowBwd{qn, qk_eps, rope_cs},
                      RowBwd{kn, qk_eps, rope_cs}, dqkv, dqn, dkn, status, B);
    e = launch_k(dq_tp_kernel<HD>, dim3(n_t, Hq, B), dim3(TB_THREADS), (size_t)C::DQ_TP_SMEM, st,
                 tq, tdo, tk, tv, to, LSE, (const float*)Dl, S, Hq, Hkv, Tmax, scale_log2, scale,
                 qkv_raw, RowBwd{qn, qk_eps, rope_cs}, dqkv, dqn, status);
  } else {
    e = launch_k(dq_tc_kernel<HD>, dim3(n_t, Hq, B), dim3(TB_THREADS), (size_t)C::DQ_SMEM, st, tq,
                 tdo, tk, tv, O, dO, LSE, Dl, S, Hq, Hkv, Tmax, scale_log2, scale, qkv_raw,
                 RowBwd{qn, qk_eps, rope_cs}, dqkv, dqn, status);
  }
  if (e != cudaSuccess) return e;
  if (dkdv_pipelined())
    return launch_k(dkdv_tp_kernel<HD>, dim3(n_t, Hkv, B), dim3(TB_THREADS),
                    (size_t)C::DKV_TP_SMEM, st, tq, tdo, tk, tv, to, LSE, (const float*)Dl, S, Hq, Hkv,
                    Tmax, scale_log2, scale, qkv_raw, RowBwd{kn, qk_eps, rope_cs}, dqkv, dkn,
                    status);
  return launch_k(dkdv_tc_kernel<HD>, dim3(n_t, Hkv, B), dim3(TB_THREADS), (size_t)C::DKV_SMEM,
                  st, tq, tdo, tk, tv, LSE, (const float*)Dl, S, Hq, Hkv, Tmax, scale_log2, scale,
                  qkv_raw, RowBwd{kn, qk_eps, rope_cs}, dqkv, dkn, status);
}

}  // namespace

cudaError_t launch_attn_bwd_tc(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                               const __nv_bfloat16* V, const __nv_bfloat16* O,
                               const __nv_bfloat16* dO, const float* LSE, float* Dl, int B, int S,
                               int Hq, int Hkv, int hd, int Tmax, const float* qkv_raw,
                               const float* qn, const float* kn, float qk_eps,
                               const float2* rope_cs, __nv_bfloat16* dqkv, float* dqn, float* dkn,
                               int* status, cudaStream_t st, bool tc_dq) {
  if ((hd != 128 && hd != 64) || Hq % Hkv || S <= 0 || rope_cs == nullptr)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
       reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(O) |
       reinterpret_cast<uintptr_t>(dO) | reinterpret_cast<uintptr_t>(dqkv) |
       reinterpret_cast<uintptr_t>(qkv_raw)) & 15)
    return cudaErrorInvalidValue;
  CUtensorMap tq, tdo, tk, tv, to;
  if (!tmap_tile(&tq, Q, (long long)B * S, (long long)Hq * hd) ||
      !tmap_tile(&tdo, dO, (long long)B * S, (long long)Hq * hd) ||
      !tmap_tile(&tk, K, (long long)B * Hkv * Tmax, hd) ||
      !tmap_tile(&tv, V, (long long)B * Hkv * Tmax, hd) ||
      !tmap_rows3d(&to, dqkv, B, S, (long long)(Hq + 2 * Hkv) * hd))
    return cudaErrorInvalidValue;
  if (hd == 128)
    return launch_bwd_tc_hd<128>(tq, tdo, tk, tv, to, Q, K, V, O, dO, LSE, Dl, B, S, Hq, Hkv, Tmax,
                                 qkv_raw, qn, kn, qk_eps, rope_cs, dqkv, dqn, dkn, status, st,
                                 tc_dq);
  return launch_bwd_tc_hd<64>(tq, tdo, tk, tv, to, Q, K, V, O, dO, LSE, Dl, B, S, Hq, Hkv, Tmax,
                              qkv_raw, qn, kn, qk_eps, rope_cs, dqkv, dqn, dkn, status, st,
                              tc_dq);
}

}  // namespace ne
