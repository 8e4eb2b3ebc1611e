// attn_fwd_tc.cu -- causal GQA attention forward on the tcgen05 tensor cores
// (training step and the token loop's prompt pass; head_dim 128 or 64).
//
// Math of the reference's sdpaFwd kernel (ane-training/training/
// training_dynamic/mil_dynamic.h:184-198: softmax(Q K^T / sqrt(hd) + causal
// mask) V with GQA head sharing) evaluated flash-style: one CTA owns 128
// query rows of one (sequence, q-head) and walks 128-key tiles up to the
// diagonal with an online softmax; it also writes the row log-sum-exp (log2
// domain) that the backward recomputes P from.
//
// Roles (320 threads):
//   warp 0     TMA producer: Q once, then K and V tiles into a 2-deep ring.
//   warp 1     MMA issuer: S_j = Q K_j^T into one of two TMEM score buffers
//              (128 x 128 fp32), and O += P_j V_j into the TMEM output
//              accumulator (128 x 128 fp32); S_{j+1} is issued before waiting
//              for P_j so the score MMAs overlap the softmax, and P is double
//              buffered so the softmax of tile j+1 overlaps the P.V product of
//              tile j (it waits for that product only to rescale O).
//   warps 2-9  softmax: two warps per TMEM lane quarter, thread = query row,
//              each warp of the pair owning 64 of the tile's 128 key columns
//              (and 64 of the 128 output columns); per tile: row max of the
//              scaled, masked scores (first pass over TMEM, the pair's halves
//              combined through shared memory), then p = exp2(s - m) written
//              bf16 into shared memory as the K-major A operand of the P.V
//              product (128-byte swizzle), row sums, and the running output
//              rescaled in TMEM by exp2(m_old - m_new).  At the end O / l
//              leaves as bf16, and m + log2(l) as the LSE.
// Operand layouts: Q, K and P K-major (64-element 128-byte swizzle atoms), V
// read MN-major (64 x 64 boxes) so V[keys][hd] needs no transpose.  Every
// mbarrier wait is bounded (2 s) and records a timeout in the status word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"

namespace ne {
namespace {

constexpr int TA_BQ = 128;          // query rows per CTA (UMMA M)
constexpr int TA_BK = 128;          // keys per tile (UMMA N of the score product)
constexpr int TA_THREADS = 320;
constexpr int TA_SOFTMAX = 256;     // softmax threads (warps 2..9)
constexpr uint32_t TA_P_BYTES = TA_BQ * TA_BK * 2;      // 32 KB: 2 atoms of 64 keys
constexpr uint32_t TA_ATOM = 128 * 128;                 // 128 rows x 64 16-bit elements
constexpr uint32_t TA_MN_BOX = 64 * 64 * 2;             // one 64 (hd) x 64 (keys) V box

// Sizes for head dim HD (64 or 128): Q, K and V tiles hold HD / 64 atoms
// (or boxes) per 128 rows.
template <int HD>
struct TaCfg {
  static_assert(HD == 64 || HD == 128, "head dim 64 or 128");
  static constexpr int NA = HD / 64;                          // 64-element column blocks
  static constexpr uint32_t Q_BYTES = TA_BQ * HD * 2;
  static constexpr uint32_t K_BYTES = TA_BK * HD * 2;
  static constexpr uint32_t V_BYTES = TA_BK * HD * 2;         // 2 key blocks x NA hd boxes
  static constexpr int OC = HD / 2;                           // output columns per softmax warp
  // Q | K[2] | V[2] | P[2] | barriers + row-max exchange (2 x 128 floats), plus
  // 1 KB alignment slack (227 KB, the per-CTA maximum, at HD 128)
  static constexpr int SMEM = Q_BYTES + 2 * K_BYTES + 2 * V_BYTES + 2 * TA_P_BYTES + 2048 + 1024;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};
static_assert(1312 + 32 <= 2048, "barrier / exchange area");

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

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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

// T = __nv_bfloat16 (training: Q, K, V and P bf16) or __half (the token
// loop's prefill over the fp16 KV cache: Q, K, V and P fp16); the output is
// bf16 either way.  HD = head dim (64: Stories110M, 128: Qwen3).
template <typename T, int HD>
__global__ void __launch_bounds__(TA_THREADS, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                   int S, int Hq, int Hkv, int Tmax,
                   float qscale_log2, __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                   int* status) {
  using C = TaCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t sQ = base;
  const uint32_t sK = sQ + C::Q_BYTES;                    // [2]
  const uint32_t sV = sK + 2 * C::K_BYTES;                // [2]
  const uint32_t sP = sV + 2 * C::V_BYTES;                // [2]
  const uint32_t bars = sP + 2 * TA_P_BYTES;
  const uint32_t q_full = bars;
  const uint32_t kv_full = bars + 8;      // [2]
  const uint32_t kv_empty = bars + 24;    // [2]
  const uint32_t s_full = bars + 40;      // [2]
  const uint32_t s_free = bars + 56;      // [2]
  const uint32_t p_full = bars + 72;      // [2]
  const uint32_t drain = bars + 88;
  const uint32_t o_done = bars + 96;      // [2]
  uint8_t* const gbars = gbase + (bars - base);
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(gbars + 128);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(gbars + 132);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest-first order: CTAs are issued in linear block order, and the query
  // tiles furthest down the causal triangle walk the most key tiles, so the
  // linear index runs over every (sequence, head) of the last query tile first
  const int nbh = gridDim.y * gridDim.z;
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int qt = gridDim.x - 1 - lin / nbh;
  const int h = (lin % nbh) % gridDim.y, b = (lin % nbh) / gridDim.y;
  const int kvh = h / (Hq / Hkv);
  const int q0 = qt * TA_BQ;
  const int n_keys = min(S, q0 + TA_BQ);                // causal: keys < q0 + 128
  const int n_kt = (n_keys + TA_BK - 1) / TA_BK;
  constexpr bool kF16 = std::is_same<T, __half>::value;
  constexpr int FMT = kF16 ? 0 : 1;      // instruction-descriptor A/B format: 0 f16, 1 bf16
  constexpr uint32_t IDESC_S = umma_idesc_f16(TA_BQ, TA_BK, FMT, 0, 0);
  constexpr uint32_t IDESC_O = umma_idesc_f16(TA_BQ, HD, FMT, 0, 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(kv_full + 8 * i, 1);
      mbar_init(kv_empty + 8 * i, 1);
      mbar_init(s_full + 8 * i, 1);
      mbar_init(s_free + 8 * i, TA_SOFTMAX);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(p_full + 8 * i, TA_SOFTMAX);
      mbar_init(o_done + 8 * i, 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
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
  const uint32_t tmem = *tmem_slot;          // S0 at +0, S1 at +128, O at +256 (HD columns)

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      pdl_wait();
      const uint64_t pol = policy_evict_last();
      const int qrow = b * S + q0;
      const int kvrow = (b * Hkv + kvh) * Tmax;
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      for (int a = 0; a < C::NA; ++a)
        tma_load_2d(sQ + a * TA_ATOM, &tmQ, q_full, h * HD + a * 64, qrow, pol);
      for (int j = 0; j < n_kt; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(kv_empty + 8 * st, ((j >> 1) - 1) & 1, status, abort_flag)) break;
        mbar_arrive_expect_tx(kv_full + 8 * st, C::K_BYTES + C::V_BYTES);
        const int k0 = kvrow + j * TA_BK;
        for (int a = 0; a < C::NA; ++a)
          tma_load_2d(sK + st * C::K_BYTES + a * TA_ATOM, &tmK, kv_full + 8 * st, a * 64, k0, pol);
        for (int kb = 0; kb < 2; ++kb)
          for (int c = 0; c < C::NA; ++c)
            tma_load_2d(sV + st * C::V_BYTES + kb * C::NA * TA_MN_BOX + c * TA_MN_BOX, &tmV,
                        kv_full + 8 * st, c * 64, k0 + kb * 64, pol);
      }
      // drain (bounded): every load issued has landed before the CTA exits
      {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
      for (int j = (n_kt > 2 ? n_kt - 2 : 0); j < n_kt; ++j) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(kv_full + 8 * (j & 1), (j >> 1) & 1))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(kv_full + 8 * st, (j >> 1) & 1, status, abort_flag)) return false;
        if (j >= 2 && !mbar_wait(s_free + 8 * st, ((j >> 1) - 1) & 1, status, abort_flag))
          return false;
        tc_fence_after();
        const uint32_t kbase = sK + st * C::K_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t ad = smem_desc_k_sw128(sQ + (kk >> 2) * TA_ATOM) + 2 * (kk & 3);
          const uint64_t bd = smem_desc_k_sw128(kbase + (kk >> 2) * TA_ATOM) + 2 * (kk & 3);
          umma_f16(tmem + st * TA_BK, ad, bd, IDESC_S, kk > 0);
        }
        umma_commit(s_full + 8 * st);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, status, abort_flag);
      if (ok && n_kt > 0) ok = issue_s(0);
      for (int j = 0; j < n_kt && ok; ++j) {
        if (j + 1 < n_kt && !(ok = issue_s(j + 1))) break;
        if (!(ok = mbar_wait(p_full + 8 * (j & 1), (j >> 1) & 1, status, abort_flag))) break;
        tc_fence_after();
        const uint32_t vbase = sV + (j & 1) * C::V_BYTES;
        const uint32_t pbase = sP + (j & 1) * TA_P_BYTES;
#pragma unroll
        for (int kk = 0; kk < TA_BK / 16; ++kk) {
          const uint64_t ad = smem_desc_k_sw128(pbase + (kk >> 2) * TA_ATOM) + 2 * (kk & 3);
          const uint64_t bd =
              smem_desc_mn_sw128(vbase + (kk >> 2) * C::NA * TA_MN_BOX, TA_MN_BOX) + 128 * (kk & 3);
          umma_f16(tmem + 256, ad, bd, IDESC_O, (j | kk) != 0);
        }
        umma_commit(o_done + 8 * (j & 1));
        umma_commit(kv_empty + 8 * (j & 1));
      }
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > 100000000ull) break;
    }
  } else {
    // ------------------------------------------------ softmax / output (warps 2..9)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;             // which 64 columns of S / O
    const int row = quarter * 32 + lane;          // query row within the tile = TMEM lane
    const int qpos = q0 + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float* const xmax = reinterpret_cast<float*>(gbars + 256);   // [2][128] row-max halves
    const int c_lo = half * 64;
    float m = -1e30f, l = 0.f;
    bool ok = true;
    int* const xok = reinterpret_cast<int*>(gbars + 1280);         // [2][4] per-warp outcome
    int* const xok2 = reinterpret_cast<int*>(gbars + 1312);        // [2][4] after the rescale wait
    for (int j = 0; j < n_kt; ++j) {
      const int st = j & 1;
      // scores of tile j ready, and the P buffer of this tile free (the P.V
      // product of tile j - 2 done).  Both warps of the pair reach the exchange
      // barriers whatever the outcome, and leave together.
      bool ready = true;
      if (j >= 2) ready = mbar_wait(o_done + 8 * st, ((j >> 1) - 1) & 1, status, abort_flag);
      ready = mbar_wait(s_full + 8 * st, (j >> 1) & 1, status, abort_flag) && ready;
      ready = __all_sync(0xffffffffu, ready);
      tc_fence_after();
      const uint32_t srow = tmem + lane_off + st * TA_BK;
      const int kbase = j * TA_BK;
      // pass 1: this warp's 64 scores (kept in registers for pass 2), their
      // row max, then the max over both halves
      // Tiles left of the diagonal tile hold only keys < q0 <= every row's
      // position (and < S): no mask there (warp-uniform).  The maximum is taken
      // over the raw scores and scaled once (qscale > 0, so exactly the maximum
      // of the scaled scores).
      const bool full = j < qt;
      uint32_t sr[2][32];
      float mx = m;
      if (ready) {
        float mraw = -3.0e38f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tmem_ld32(srow + c_lo + 32 * h, sr[h]);
          if (full) {
            // four independent chains (the compiler keeps fmaxf's order)
            float m4[4] = {mraw, -3.0e38f, -3.0e38f, -3.0e38f};
#pragma unroll
            for (int i = 0; i < 32; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(sr[h][i]));
            mraw = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int key = kbase + c_lo + 32 * h + i;
              if (key <= qpos && key < S) mraw = fmaxf(mraw, __uint_as_float(sr[h][i]));
            }
          }
        }
        mx = fmaxf(mx, mraw > -3.0e38f ? mraw * qscale_log2 : -1e30f);
      }
      xmax[half * 128 + row] = mx;
      if (lane == 0) xok[half * 4 + quarter] = ready ? 1 : 0;
      // the two warps of this lane quarter (64 threads) exchange their halves
      asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
      mx = fmaxf(mx, xmax[(half ^ 1) * 128 + row]);
      bool both = ready && xok[(half ^ 1) * 4 + quarter] != 0;
      // Lazy rescaling: the running max m moves (and O, l are rescaled) only
      // when the tile's max exceeds it by more than 2^8; otherwise p = exp2(s - m)
      // stays below 256, well inside bf16 and fp32, and the TMEM round trip of
      // O is skipped.  The decision is per row, but tcgen05.ld / st are
      // warp-collective, so a warp rescales its rows of O when any of them
      // moves (corr = 1 for the others); both warps of the pair hold the same
      // rows, m and mx, so both wait (or neither) for the previous P.V product.
      const bool move_row = both && mx > m + 8.0f;
      const bool move = __any_sync(0xffffffffu, move_row);
      bool rs_ok = true;
      if (move && j > 0)
        rs_ok = mbar_wait(o_done + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1, status, abort_flag);
      rs_ok = __all_sync(0xffffffffu, rs_ok);
      if (lane == 0) xok2[half * 4 + quarter] = rs_ok ? 1 : 0;
      asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");   // xmax / xok reusable
      both = both && rs_ok && xok2[(half ^ 1) * 4 + quarter] != 0;
      if (!both) {
        ok = false;
        break;
      }
      // the scores are in registers: the tensor cores may reuse this S buffer
      tc_fence_before();
      mbar_arrive(s_free + 8 * st);
      const float corr = move_row ? exp2f(m - mx) : 1.0f;
      if (move_row) m = mx;
      // pass 2: p = exp2(s - m) -> P (T, swizzled K-major rows), row sum
      float sum = 0.f, sum2 = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = c_lo + 32 * h;
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int key = kbase + c + i;
          float p0 = ex2_fast(fmaf(__uint_as_float(sr[h][i]), qscale_log2, -m));
          float p1 = ex2_fast(fmaf(__uint_as_float(sr[h][i + 1]), qscale_log2, -m));
          if (!full) {
            if (!(key <= qpos && key < S)) p0 = 0.f;
            if (!(key + 1 <= qpos && key + 1 < S)) p1 = 0.f;
          }
          sum += p0;
          sum2 += p1;
          if constexpr (kF16) {
            const __half2 pk = __floats2half2_rn(p0, p1);
            w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
          } else {
            const __nv_bfloat162 pk = __floats2bfloat162_rn(p0, p1);
            w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
          }
        }
        // 32 keys = 4 chunks of 8 (16 bytes) in atom c / 64, chunk index (c % 64) / 8 + q
        const uint32_t atom = sP + st * TA_P_BYTES + (c >> 6) * TA_ATOM + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = ((c & 63) >> 3) + q;
          st_shared_v4(atom + ((chunk ^ (row & 7)) << 4), w[4 * q], w[4 * q + 1], w[4 * q + 2],
                       w[4 * q + 3]);
        }
      }
      l = l * corr + (sum + sum2);   // this half's share of the row sum
      // running output *= corr (the accumulator holds tiles < j); this warp's
      // HD / 2 columns
      if (j > 0 && move) {
        const uint32_t orow = tmem + lane_off + 256;
        for (int c = half * C::OC; c < half * C::OC + C::OC; c += 32) {
          uint32_t r[32];
          tmem_ld32(orow + c, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st32(orow + c, r);
        }
      }
      fence_async_smem();        // P visible to the tensor cores
      tc_fence_before();
      mbar_arrive(p_full + 8 * st);
    }
    // ---- output: O / l (bf16) and the row LSE (log2 domain).  Every MMA has
    // completed once the last P.V product is done, so the first K buffer
    // holds the bf16 output tile (swizzled atoms) for one tensor store per 64
    // columns; rows at or past S are clipped by the store.
    bool staged = false;
    if (ok && n_kt > 0) {
      const bool od =
          mbar_wait(o_done + 8 * ((n_kt - 1) & 1), ((n_kt - 1) >> 1) & 1, status, abort_flag);
      // full row sum = both halves (same running max)
      xmax[half * 128 + row] = l;
      asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
      const float lrow = l + xmax[(half ^ 1) * 128 + row];
      if (__all_sync(0xffffffffu, od)) {
        tc_fence_after();
        pdl_wait();
        const uint32_t orow = tmem + lane_off + 256;
        const float inv = 1.0f / lrow;
        for (int c = half * C::OC; c < half * C::OC + C::OC; c += 32) {
          uint32_t r[32];
          tmem_ld32(orow + c, r);
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const __nv_bfloat162 pk = __floats2bfloat162_rn(__uint_as_float(r[i]) * inv,
                                                            __uint_as_float(r[i + 1]) * inv);
            w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
          }
          const uint32_t atom = sK + (c >> 6) * TA_ATOM + row * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = ((c & 63) >> 3) + q;
            st_shared_v4(atom + ((chunk ^ (row & 7)) << 4), w[4 * q], w[4 * q + 1],
                         w[4 * q + 2], w[4 * q + 3]);
          }
        }
        staged = true;
        if (half == 0 && qpos < S && lse) lse[((size_t)b * Hq + h) * S + qpos] = m + log2f(lrow);
      }
    }
    // every softmax warp reaches this barrier, whatever happened before
    if (lane == 0) xok[half * 4 + quarter] = staged ? 1 : 0;
    fence_async_smem();
    asm volatile("bar.sync 5, %0;" ::"r"(TA_SOFTMAX) : "memory");
    if (warp == 2 && lane == 0) {
      bool all = true;
      for (int i = 0; i < 8; ++i) all = all && xok[i] != 0;
      if (all) {
        for (int a = 0; a < C::NA; ++a) tma_store_3d(&tmO, sK + a * TA_ATOM, h * HD + a * 64, q0, b);
        bulk_commit_group();
        bulk_wait_all();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ two query tiles
// A second form for GQA groups of even size: one CTA owns the same 128 query
// rows of two q-heads that share a kv-head (tiles A and B), so every K / V
// tile it loads serves both.  Each element-wise thread owns a whole score row
// (no exchange between warps), P overwrites its scores in tensor memory as
// bf16 / fp16 (the A operand of O += P V read from TMEM), and the MMA thread
// alternates between the tiles: while tile A's warps run the softmax of key
// tile j, the tensor cores run tile B's products, and the other way round.
//   TMEM: S_A [0, 128), S_B [128, 256), O_A at 256, O_B at 256 + HD.
//   warps 2-5: tile A (one per TMEM lane quarter), warps 6-9: tile B.
template <int HD>
struct Ta2Cfg {
  static constexpr int NA = HD / 64;
  static constexpr uint32_t Q_BYTES = 128 * HD * 2;         // one query tile
  static constexpr uint32_t K_BYTES = 128 * HD * 2;
  static constexpr uint32_t KV_BYTES = 2 * K_BYTES;         // K then V of one stage
  static constexpr int NS = HD == 128 ? 2 : 3;              // K / V stages
  static constexpr int SMEM = 2 * Q_BYTES + NS * KV_BYTES + 1024 + 1024;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

template <typename T, int HD>
__global__ void __launch_bounds__(TA_THREADS, 1)
attn_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    int S, int Hq, int Hkv, int Tmax, float qscale_log2, float* __restrict__ lse,
                    int* status) {
  using C = Ta2Cfg<HD>;
  constexpr int NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t sQ = base;                                 // [2] tiles A, B
  const uint32_t sKV = sQ + 2 * C::Q_BYTES;                 // [NS] stages: K | V
  const uint32_t bars = sKV + NS * C::KV_BYTES;
  const uint32_t q_full = bars;
  const uint32_t kv_full = bars + 8;      // [NS]
  const uint32_t kv_empty = bars + 32;    // [NS]
  const uint32_t s_full = bars + 56;      // [2] per tile
  const uint32_t p_full = bars + 72;      // [2] per tile
  const uint32_t o_last = bars + 88;      // [2] per tile: its last P.V product done
  const uint32_t drain = bars + 104;
  uint8_t* const gbars = gbase + (bars - base);
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(gbars + 112);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(gbars + 116);
  int* const xok = reinterpret_cast<int*>(gbars + 128);     // [8] per softmax warp

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest-first order over (query tile, head pair, sequence)
  const int nbh = gridDim.y * gridDim.z;
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int qt = gridDim.x - 1 - lin / nbh;
  const int hp = (lin % nbh) % gridDim.y, b = (lin % nbh) / gridDim.y;
  const int hA = 2 * hp;
  const int kvh = hA / (Hq / Hkv);                          // shared by hA and hA + 1
  const int q0 = qt * TA_BQ;
  const int n_keys = min(S, q0 + TA_BQ);
  const int n_kt = (n_keys + TA_BK - 1) / TA_BK;
  constexpr bool kF16 = std::is_same<T, __half>::value;
  constexpr int FMT = kF16 ? 0 : 1;
  constexpr uint32_t IDESC_S = umma_idesc_f16(TA_BQ, TA_BK, FMT, 0, 0);
  constexpr uint32_t IDESC_O = umma_idesc_f16(TA_BQ, HD, FMT, 0, 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(kv_full + 8 * i, 1);
      mbar_init(kv_empty + 8 * i, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full + 8 * t, 1);
      mbar_init(p_full + 8 * t, 128);
      mbar_init(o_last + 8 * t, 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
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
      mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int a = 0; a < C::NA; ++a)
          tma_load_2d(sQ + t * C::Q_BYTES + a * TA_ATOM, &tmQ, q_full, (hA + t) * HD + a * 64,
                      qrow, pol);
      int j = 0;
      for (; j < n_kt; ++j) {
        const int st = j % NS;
        if (j >= NS && !mbar_wait(kv_empty + 8 * st, ((j / NS) - 1) & 1, status, abort_flag))
          break;
        mbar_arrive_expect_tx(kv_full + 8 * st, C::KV_BYTES);
        const uint32_t sk = sKV + st * C::KV_BYTES, sv = sk + C::K_BYTES;
        const int k0 = kvrow + j * TA_BK;
        for (int a = 0; a < C::NA; ++a)
          tma_load_2d(sk + a * TA_ATOM, &tmK, kv_full + 8 * st, a * 64, k0, pol);
        for (int kb = 0; kb < 2; ++kb)
          for (int c = 0; c < C::NA; ++c)
            tma_load_2d(sv + kb * C::NA * TA_MN_BOX + c * TA_MN_BOX, &tmV, kv_full + 8 * st,
                        c * 64, k0 + kb * 64, pol);
      }
      // drain (bounded): every load issued has landed before the CTA exits
      {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
      for (int i = (j > NS ? j - NS : 0); i < j; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(kv_full + 8 * (i % NS), (i / NS) & 1))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      auto issue_s = [&](int t, int j) {   // S_t = Q_t K_j^T
        const uint32_t kbase = sKV + (j % NS) * C::KV_BYTES;
        const uint32_t qbase = sQ + t * C::Q_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t ad = smem_desc_k_sw128(qbase + (kk >> 2) * TA_ATOM) + 2 * (kk & 3);
          const uint64_t bd = smem_desc_k_sw128(kbase + (kk >> 2) * TA_ATOM) + 2 * (kk & 3);
          umma_f16(tmem + 128 * t, ad, bd, IDESC_S, kk > 0);
        }
        umma_commit(s_full + 8 * t);
      };
      auto issue_pv = [&](int t, int j) {   // O_t += P_t V_j (P_t from TMEM)
        const uint32_t vbase = sKV + (j % NS) * C::KV_BYTES + C::K_BYTES;
#pragma unroll
        for (int kk = 0; kk < TA_BK / 16; ++kk) {
          const uint64_t bd =
              smem_desc_mn_sw128(vbase + (kk >> 2) * C::NA * TA_MN_BOX, TA_MN_BOX) + 128 * (kk & 3);
          umma_f16_ts(tmem + 256 + HD * t, tmem + 128 * t + 8 * kk, bd, IDESC_O, (j | kk) != 0);
        }
      };
      bool ok = mbar_wait(q_full, 0, status, abort_flag) && mbar_wait(kv_full, 0, status, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      for (int j = 0; j < n_kt && ok; ++j) {
        for (int t = 0; t < 2 && ok; ++t) {
          if (!(ok = mbar_wait(p_full + 8 * t, j & 1, status, abort_flag))) break;
          tc_fence_after();
          issue_pv(t, j);
          if (t == 1) umma_commit(kv_empty + 8 * (j % NS));   // K_j / V_j read by both tiles
          if (j + 1 < n_kt) {
            if (t == 0) {
              const int nst = (j + 1) % NS;
              if (!(ok = mbar_wait(kv_full + 8 * nst, ((j + 1) / NS) & 1, status, abort_flag)))
                break;
              tc_fence_after();
            }
            issue_s(t, j + 1);
          } else {
            umma_commit(o_last + 8 * t);
          }
        }
      }
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0))
        if (globaltimer_ns() - t0 > 100000000ull) break;
    }
  } else {
    // ------------------------------------------------ softmax / output (warps 2..9)
    const int t = (warp - 2) >> 2;                 // tile A or B
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;           // query row within the tile = TMEM lane
    const int qpos = q0 + row;
    const int h = hA + t;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t srow = tmem + lane_off + 128 * t;
    const uint32_t orow = tmem + lane_off + 256 + HD * t;
    float m = -1e30f, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      const bool ready =
          __all_sync(0xffffffffu, mbar_wait(s_full + 8 * t, j & 1, status, abort_flag));
      if (!ready) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool full = j < qt;                   // left of the diagonal: no mask
      const int kbase = j * TA_BK;
      // pass 1: the row maximum of the raw scores (scaled once; qscale > 0)
      float m4[4] = {-3.0e38f, -3.0e38f, -3.0e38f, -3.0e38f};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(srow + 32 * c, r);
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(r[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = kbase + 32 * c + i;
            if (key <= qpos && key < S) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(r[i]));
          }
        }
      }
      const float mraw = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      const float mx = fmaxf(m, mraw > -3.0e38f ? mraw * qscale_log2 : -1e30f);
      // lazy rescale (see attn_fwd_tc_kernel), decided per warp: O_t's last
      // product is complete (S_t of this tile was issued after it)
      const bool move_row = mx > m + 8.0f;
      const bool move = __any_sync(0xffffffffu, move_row);
      const float corr = move_row ? ex2_fast(m - mx) : 1.0f;
      if (move_row) m = mx;
      if (move && j > 0) {
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          uint32_t r[32];
          tmem_ld32(orow + c, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st32(orow + c, r);
        }
      }
      // pass 2: p = exp2(s - m), 16-bit, over the scores in place (chunk c's
      // packed words go to columns 16c .. 16c+15, all read already)
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(srow + 32 * c, r);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float p0 = ex2_fast(fmaf(__uint_as_float(r[i]), qscale_log2, -m));
          float p1 = ex2_fast(fmaf(__uint_as_float(r[i + 1]), qscale_log2, -m));
          if (!full) {
            const int key = kbase + 32 * c + i;
            if (!(key <= qpos && key < S)) p0 = 0.f;
            if (!(key + 1 <= qpos && key + 1 < S)) p1 = 0.f;
          }
          sum0 += p0;
          sum1 += p1;
          if constexpr (kF16) {
            const __half2 pk = __floats2half2_rn(p0, p1);
            w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
          } else {
            const __nv_bfloat162 pk = __floats2bfloat162_rn(p0, p1);
            w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
          }
        }
        tmem_st16(srow + 16 * c, w);
      }
      l = l * corr + (sum0 + sum1);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full + 8 * t);
    }
    // ---- output: O / l into this tile's (now free) Q buffer, one tensor
    // store per 64 columns (rows at or past S are clipped); the row LSE
    bool staged = false;
    if (ok && __all_sync(0xffffffffu, mbar_wait(o_last + 8 * t, 0, status, abort_flag))) {
      tc_fence_after();
      pdl_wait();
      const float inv = 1.0f / l;
      const uint32_t stile = sQ + t * C::Q_BYTES;
#pragma unroll
      for (int c = 0; c < HD; c += 32) {
        uint32_t r[32];
        tmem_ld32(orow + c, r);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const __nv_bfloat162 pk = __floats2bfloat162_rn(__uint_as_float(r[i]) * inv,
                                                          __uint_as_float(r[i + 1]) * inv);
          w[i >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
        }
        const uint32_t atom = stile + (c >> 6) * TA_ATOM + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = ((c & 63) >> 3) + q;
          st_shared_v4(atom + ((chunk ^ (row & 7)) << 4), w[4 * q], w[4 * q + 1], w[4 * q + 2],
                       w[4 * q + 3]);
        }
      }
      staged = true;
      if (qpos < S && lse) lse[((size_t)b * Hq + h) * S + qpos] = m + log2f(l);
    }
    if (lane == 0) xok[warp - 2] = staged ? 1 : 0;
    fence_async_smem();
    asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");   // this tile's four warps
    if (warp == 2 + 4 * t && lane == 0) {
      bool all = true;
      for (int i = 0; i < 4; ++i) all = all && xok[4 * t + i] != 0;
      if (all) {
        for (int a = 0; a < C::NA; ++a)
          tma_store_3d(&tmO, sQ + t * C::Q_BYTES + a * TA_ATOM, h * HD + a * 64, q0, b);
        bulk_commit_group();
        bulk_wait_all();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 16-bit [rows, cols] row-major (bf16 or fp16), 128-byte-swizzled boxes of 64
// columns x box_rows.
bool tmap_16(CUtensorMap* tm, const void* ptr, long long rows, long long cols, int box_rows,
             CUtensorMapDataType dt) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(tm, dt, 2, const_cast<void*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// bf16 [B][S][cols] as a 3D map with 128-byte-swizzled boxes of 64 columns
// x 128 rows x 1 sequence (tensor stores of a 128-row tile stop at S).
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

namespace {

// GQA groups of even size take the two-tile kernel (NE_ATTN_FWD2=0: the
// one-tile kernel for every group size).
bool fwd_two_tiles() {
  static const bool on = [] {
    const char* e = std::getenv("NE_ATTN_FWD2");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename T, int HD>
cudaError_t launch_tc(const T* Q, const T* K, const T* V, int B, int S, int Hq, int Hkv, int hd,
                      int Tmax, __nv_bfloat16* out, float* lse, int* status, cudaStream_t st) {
  if (hd != HD || Hq % Hkv) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
       reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(out)) & 15)
    return cudaErrorInvalidValue;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq, tk, tv, to;
  if (!tmap_16(&tq, Q, (long long)B * S, (long long)Hq * hd, TA_BQ, dt) ||
      !tmap_16(&tk, K, (long long)B * Hkv * Tmax, hd, TA_BK, dt) ||
      !tmap_16(&tv, V, (long long)B * Hkv * Tmax, hd, 64, dt) ||
      !tmap_rows3d(&to, out, B, S, (long long)Hq * hd))
    return cudaErrorInvalidValue;
  static bool attr = false;   // one flag per instantiation
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_tc_kernel<T, HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         TaCfg<HD>::SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attn_fwd_tc2_kernel<T, HD>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, Ta2Cfg<HD>::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const float qscale_log2 = (1.0f / sqrtf((float)hd)) * 1.4426950408889634f;
  if ((Hq / Hkv) % 2 == 0 && fwd_two_tiles())
    return launch_k(attn_fwd_tc2_kernel<T, HD>, dim3((S + TA_BQ - 1) / TA_BQ, Hq / 2, B),
                    dim3(TA_THREADS), (size_t)Ta2Cfg<HD>::SMEM, st, tq, tk, tv, to, S, Hq, Hkv,
                    Tmax, qscale_log2, lse, status);
  return launch_k(attn_fwd_tc_kernel<T, HD>, dim3((S + TA_BQ - 1) / TA_BQ, Hq, B),
                  dim3(TA_THREADS), (size_t)TaCfg<HD>::SMEM, st, tq, tk, tv, to, S, Hq, Hkv, Tmax,
                  qscale_log2, out, lse, status);
}

template <typename T>
cudaError_t launch_tc_hd(const T* Q, const T* K, const T* V, int B, int S, int Hq, int Hkv,
                         int hd, int Tmax, __nv_bfloat16* out, float* lse, int* status,
                         cudaStream_t st) {
  if (hd == 128) return launch_tc<T, 128>(Q, K, V, B, S, Hq, Hkv, hd, Tmax, out, lse, status, st);
  if (hd == 64) return launch_tc<T, 64>(Q, K, V, B, S, Hq, Hkv, hd, Tmax, out, lse, status, st);
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_attn_fwd_tc(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                               const __nv_bfloat16* V, int B, int S, int Hq, int Hkv, int hd,
                               int Tmax, __nv_bfloat16* out, float* lse, int* status,
                               cudaStream_t st) {
  return launch_tc_hd(Q, K, V, B, S, Hq, Hkv, hd, Tmax, out, lse, status, st);
}

cudaError_t launch_attn_fwd_tc_f16(const __half* Q, const __half* K, const __half* V, int B,
                                   int S, int Hq, int Hkv, int hd, int Tmax,
                                   __nv_bfloat16* out, int* status, cudaStream_t st) {
  return launch_tc_hd(Q, K, V, B, S, Hq, Hkv, hd, Tmax, out, nullptr, status, st);
}

}  // namespace ne
