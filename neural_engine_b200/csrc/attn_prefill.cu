// attn_prefill.cu -- causal GQA attention over a prompt (prefill / training fwd).
//
// Math of the reference's sdpaFwd kernel (ane-training/training/training_dynamic/
// mil_dynamic.h:184-198: softmax(Q K^T / sqrt(hd) + causal mask) V, K/V
// heads shared by GQA groups, mil_dynamic.h:171-182) and of the numpy loop
// (tools/generate.py:164-181), evaluated flash-style: the S x S score matrix
// is never materialised; each CTA streams K/V tiles of 64 positions through
// shared memory with an online softmax (running max / sum per query row).
//
// Tile: 64 query rows x one q-head per CTA (4 warps x 16 rows), K/V tiles of
// 64 positions double-buffered with cp.async, fp16 m16n8k16 tensor-core MMAs
// with fp32 accumulation, P kept in registers between the two products.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"
#include "ne_mma.cuh"

namespace ne {
namespace {

constexpr int FA_BQ = 64;
constexpr int FA_BK = 64;

template <int HD, typename T>
__global__ void __launch_bounds__(128)
prefill_attn_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc, int S, int pos0, int Hq, int Hkv, int Tmax,
                    float qscale_log2, __nv_bfloat16* __restrict__ out, float* __restrict__ lse) {
  constexpr int LD = HD + 8;              // padded smem row (halves): conflict-free ldmatrix
  constexpr int KSTEPS = HD / 16;         // k-steps of Q.K^T
  constexpr int DTILES = HD / 8;          // n-tiles of the output
  extern __shared__ __align__(16) unsigned char smem_raw_fa[];
  T* smem = reinterpret_cast<T*>(smem_raw_fa);
  T* sQ = smem;                           // [FA_BQ][LD]
  T* sK = sQ + FA_BQ * LD;                // [2][FA_BK][LD]
  T* sV = sK + 2 * FA_BK * LD;            // [2][FA_BK][LD]

  pdl_trigger();
  pdl_wait();
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (Hq / Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qt * FA_BQ;              // first query row (within the sequence)
  const int n_keys = pos0 + min(S, q0 + FA_BQ);   // keys needed by this tile (causal)
  const int n_kt = (n_keys + FA_BK - 1) / FA_BK;

  const size_t kv_base = ((size_t)b * Hkv + kvh) * Tmax * HD;
  const T* kg = kc + kv_base;
  const T* vg = vc + kv_base;

  // ---- load Q tile (rows beyond S are zero-filled)
  constexpr int CPR = HD / 8;             // 16-byte chunks per row
  for (int i = threadIdx.x; i < FA_BQ * CPR; i += 128) {
    const int r = i / CPR, c = i % CPR;
    const bool ok = q0 + r < S;
    const T* src = q + (((size_t)b * S + (ok ? q0 + r : 0)) * Hq + h) * HD + c * 8;
    cp_async16(smem_u32_local(sQ + r * LD + c * 8), src, ok);
  }
  auto load_kv = [&](int kt, int buf) {
    T* dK = sK + buf * FA_BK * LD;
    T* dV = sV + buf * FA_BK * LD;
    for (int i = threadIdx.x; i < FA_BK * CPR; i += 128) {
      const int r = i / CPR, c = i % CPR;
      const int t = kt * FA_BK + r;
      const bool ok = t < n_keys;
      const size_t off = (size_t)(ok ? t : 0) * HD + c * 8;
      cp_async16(smem_u32_local(dK + r * LD + c * 8), kg + off, ok);
      cp_async16(smem_u32_local(dV + r * LD + c * 8), vg + off, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  // ---- per-warp state: rows (warp*16 + g) and (+8)
  const int g = lane >> 2, tq = lane & 3;
  float o[DTILES][4];
#pragma unroll
  for (int j = 0; j < DTILES; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {-1e30f, -1e30f}, lrow[2] = {0.f, 0.f};
  uint32_t qa[KSTEPS][4];
  const int qpos0 = pos0 + q0 + warp * 16 + g;     // absolute position of row g
  const int qpos1 = qpos0 + 8;

  for (int kt = 0; kt < n_kt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kt) load_kv(kt + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kt == 0) {
      // Q fragments (A operand, row-major 16 x HD per warp)
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 16 + (lane >> 4) * 8;
        ldsm_x4(smem_u32_local(sQ + r * LD + c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }
    const T* cK = sK + buf * FA_BK * LD;
    const T* cV = sV + buf * FA_BK * LD;

    // ---- S = Q K^T  (16 x 64 per warp: 8 n-tiles of 8 keys)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {   // pairs of key n-tiles
        uint32_t b0, b1, b2, b3;
        const int key = jp * 16 + (lane >> 4) * 8 + (lane & 7);
        const int col = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(smem_u32_local(cK + key * LD + col), b0, b1, b2, b3);
        Mma16<T>::mma(s[2 * jp], qa[ks], b0, b1);
        Mma16<T>::mma(s[2 * jp + 1], qa[ks], b2, b3);
      }
    }
    // ---- scale, causal mask, online softmax (log2 domain)
    const int kbase = kt * FA_BK;
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + j * 8 + 2 * tq + (e & 1);
        const int qp = (e < 2) ? qpos0 : qpos1;
        float v = s[j][e] * qscale_log2;
        if (key > qp || key >= n_keys) v = -1e30f;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) corr[r] = exp2f(mrow[r] - mx[r]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = (s[j][e] <= -1e29f) ? 0.f : exp2f(s[j][e] - mx[e >> 1]);
        s[j][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      lrow[r] = lrow[r] * corr[r] + rs[r];
      mrow[r] = mx[r];
    }
#pragma unroll
    for (int j = 0; j < DTILES; ++j) {
      o[j][0] *= corr[0]; o[j][1] *= corr[0];
      o[j][2] *= corr[1]; o[j][3] *= corr[1];
    }
    // ---- O += P V   (k = 64 keys in 4 steps of 16; P from registers)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = Mma16<T>::pack(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = Mma16<T>::pack(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = Mma16<T>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = Mma16<T>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < DTILES / 2; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int key = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int col = dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(smem_u32_local(cV + key * LD + col), b0, b1, b2, b3);
        Mma16<T>::mma(o[2 * dp], pa, b0, b1);
        Mma16<T>::mma(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }

  // ---- normalise and store bf16 [row][Hq*HD]
  const float inv0 = 1.f / lrow[0], inv1 = 1.f / lrow[1];
  const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;
  // log2-domain log-sum-exp of each row's scaled scores, for the backward pass:
  // P = exp2(s * scale * log2(e) - lse); layout [b][h][row]
  if (lse != nullptr && tq == 0) {
    if (r0 < S) lse[((size_t)b * Hq + h) * S + r0] = mrow[0] + log2f(lrow[0]);
    if (r1 < S) lse[((size_t)b * Hq + h) * S + r1] = mrow[1] + log2f(lrow[1]);
  }
#pragma unroll
  for (int j = 0; j < DTILES; ++j) {
    const int d = j * 8 + 2 * tq;
    if (r0 < S) {
      __nv_bfloat16* dst = out + (((size_t)b * S + r0) * Hq + h) * HD + d;
      *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(o[j][0] * inv0, o[j][1] * inv0);
    }
    if (r1 < S) {
      __nv_bfloat16* dst = out + (((size_t)b * S + r1) * Hq + h) * HD + d;
      *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(o[j][2] * inv1, o[j][3] * inv1);
    }
  }
}

template <typename T>
cudaError_t launch_fa(const T* q, const T* kc, const T* vc, int B, int S, int pos0, int Hq, int Hkv,
                      int hd, int Tmax, __nv_bfloat16* out, cudaStream_t st, float* lse) {
  if (pos0 + S > Tmax || Hq % Hkv) return cudaErrorInvalidValue;
  const float qs = (1.0f / sqrtf((float)hd)) * 1.4426950408889634f;
  const dim3 grid((S + FA_BQ - 1) / FA_BQ, Hq, B);
  if (hd == 128) {
    constexpr int LD = 128 + 8;
    const size_t smem = (size_t)(FA_BQ + 4 * FA_BK) * LD * sizeof(T);
    static bool done = false;
    if (!done) {
      cudaFuncSetAttribute(prefill_attn_kernel<128, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      done = true;
    }
    return launch_k(prefill_attn_kernel<128, T>, grid, dim3(128), smem, st, q, kc, vc, S, pos0, Hq,
                    Hkv, Tmax, qs, out, lse);
  } else if (hd == 64) {
    constexpr int LD = 64 + 8;
    const size_t smem = (size_t)(FA_BQ + 4 * FA_BK) * LD * sizeof(T);
    return launch_k(prefill_attn_kernel<64, T>, grid, dim3(128), smem, st, q, kc, vc, S, pos0, Hq,
                    Hkv, Tmax, qs, out, lse);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_prefill_attn(const __half* q, const __half* kc, const __half* vc, int B, int S,
                                int pos0, int Hq, int Hkv, int hd, int Tmax, __nv_bfloat16* out,
                                cudaStream_t st, float* lse) {
  return launch_fa<__half>(q, kc, vc, B, S, pos0, Hq, Hkv, hd, Tmax, out, st, lse);
}

cudaError_t launch_prefill_attn_bf16(const __nv_bfloat16* q, const __nv_bfloat16* kc,
                                     const __nv_bfloat16* vc, int B, int S, int pos0, int Hq,
                                     int Hkv, int hd, int Tmax, __nv_bfloat16* out, cudaStream_t st,
                                     float* lse) {
  return launch_fa<__nv_bfloat16>(q, kc, vc, B, S, pos0, Hq, Hkv, hd, Tmax, out, st, lse);
}

}  // namespace ne
