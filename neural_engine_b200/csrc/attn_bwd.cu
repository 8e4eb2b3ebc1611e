// attn_bwd.cu -- causal GQA attention backward (training step).
//
// Gradients of O = softmax(Q K^T / sqrt(hd) + causal mask) V, the reference's
// sdpaBwd1 / sdpaBwd2 kernels (ane-training/training/training_dynamic/
// mil_dynamic.h:583-707: recompute P, dV = P^T dO, dP = dO V^T,
// dS = P (dP - rowsum(P dP)), dQ = dS K / sqrt(hd), dK = dS^T Q / sqrt(hd))
// followed by the GQA head-group reduction of dK / dV (cpu_ops.h:585
// gqa_reduce_kv_f16), evaluated flash-style without materialising P:
//   dq_kernel      one CTA per (64-query tile, q-head, sequence); each warp
//                  owns 16 queries and walks the key tiles up to the diagonal.
//                  It first forms D[b,h,s] = sum_d dO * O (= rowsum(P * dP))
//                  for its queries and publishes it for dkdv_kernel.
//   dkdv_kernel    one CTA per (64-key tile, kv-head, sequence); each warp owns
//                  16 keys and walks the query tiles at or after its keys,
//                  for every q-head of the group, so dK/dV of the group are
//                  summed in registers (no atomics, deterministic)
// P is recomputed from the forward's log2-domain row log-sum-exp.  Operands
// are bf16 (fp16 would underflow dS), fp32 accumulation, m16n8k16 MMAs.
// The dQ and dK results leave through the RoPE and QK-norm backward
// (rope_backward_inplace_f16, cpu_ops.h:510-537, and the RMSNorm derivative)
// applied to the accumulator fragments, and are written as bf16 straight into
// the gradient of the fused QKV projection; dV is written there unchanged.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>

#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"
#include "ne_mma.cuh"

namespace ne {
namespace {

using bf16 = __nv_bfloat16;
constexpr int KT_KEYS = 64;   // dkdv: keys per CTA
constexpr int KT_Q = 32;      // dkdv: queries per iteration
constexpr int QT_Q = 64;      // dq: queries per CTA
constexpr int QT_KEYS = 32;   // dq: keys per iteration

// Fill `rows` x HD of a padded smem tile from global rows (zero beyond `valid`).
template <int HD>
__device__ __forceinline__ void load_rows(bf16* dst, const bf16* src, size_t row_stride, int rows,
                                          int valid) {
  constexpr int LD = HD + 8, CPR = HD / 8;
  for (int i = threadIdx.x; i < rows * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i % CPR;
    const bool ok = r < valid;
    cp_async16(smem_u32_local(dst + r * LD + c * 8), src + (size_t)(ok ? r : 0) * row_stride + c * 8,
               ok);
  }
}

// ---------------------------------------------------------------- fragment epilogue
// Gradient of one head-vector row held as m16n8k16 accumulator fragments: the
// lane's values are columns 8j + 2tq, 8j + 2tq + 1 (j < HD/8) of a row; the 4
// lanes with equal g (lane >> 2) share the row.  Applies the inverse RoPE
// rotation at `pos` and, with a gain, the QK-norm backward of the raw
// (pre-norm) row, accumulates the gain gradient into dg, and stores bf16.
struct QkBwd {
  const float* gain;      // QK-norm gain (nullptr: no QK-norm)
  float eps;
  const float2* rope_cs;  // [pos][HD/2] (cos, sin); nullptr: no rotation (V)
};

template <int HD>
__device__ __forceinline__ void head_row_grad_store(const float (&acc)[HD / 8][4], int e0,
                                                    float scale, bool ok, int pos,
                                                    const float* raw, const QkBwd& qb,
                                                    bf16* out, float (&dg)[HD / 8][2], int tq) {
  constexpr int DT = HD / 8;
  float d[DT][2];
#pragma unroll
  for (int j = 0; j < DT; ++j) {
    d[j][0] = acc[j][e0] * scale;
    d[j][1] = acc[j][e0 + 1] * scale;
  }
  if (qb.rope_cs != nullptr) {
    const float2* cs = qb.rope_cs + (size_t)(ok ? pos : 0) * (HD / 2) + tq;
#pragma unroll
    for (int j = 0; j < DT; ++j) {
      const float2 c = cs[4 * j];
      const float d0 = d[j][0], d1 = d[j][1];
      d[j][0] = d0 * c.x + d1 * c.y;
      d[j][1] = d1 * c.x - d0 * c.y;
    }
    if (qb.gain != nullptr) {
      float x[DT][2], ss = 0.f, dot = 0.f;
#pragma unroll
      for (int j = 0; j < DT; ++j) {
        const float2 xv = ok ? *reinterpret_cast<const float2*>(raw + 8 * j + 2 * tq)
                             : make_float2(0.f, 0.f);
        const float2 gv = *reinterpret_cast<const float2*>(qb.gain + 8 * j + 2 * tq);
        x[j][0] = xv.x;
        x[j][1] = xv.y;
        ss += xv.x * xv.x + xv.y * xv.y;
        dot += d[j][0] * gv.x * xv.x + d[j][1] * gv.y * xv.y;
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      const float rrms = 1.0f / sqrtf(ss / (float)HD + qb.eps);
      const float c = rrms * rrms * dot / (float)HD;
#pragma unroll
      for (int j = 0; j < DT; ++j) {
        const float2 gv = *reinterpret_cast<const float2*>(qb.gain + 8 * j + 2 * tq);
        if (ok) {
          dg[j][0] += d[j][0] * x[j][0] * rrms;
          dg[j][1] += d[j][1] * x[j][1] * rrms;
        }
        d[j][0] = rrms * (gv.x * d[j][0] - x[j][0] * c);
        d[j][1] = rrms * (gv.y * d[j][1] - x[j][1] * c);
      }
    }
  }
  if (!ok) return;
#pragma unroll
  for (int j = 0; j < DT; ++j)
    *reinterpret_cast<__nv_bfloat162*>(out + 8 * j + 2 * tq) = __floats2bfloat162_rn(d[j][0], d[j][1]);
}

// Sum the per-lane gain-gradient partials of the CTA (4 warps) and add them
// to dgain[HD] (one atomic per column per CTA).
template <int HD>
__device__ __forceinline__ void gain_grad_flush(float (&dg)[HD / 8][2], float* red,
                                                float* dgain) {
  constexpr int DT = HD / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tq = lane & 3;
#pragma unroll
  for (int j = 0; j < DT; ++j)
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float v = dg[j][k];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (lane < 4) red[warp * HD + 8 * j + 2 * tq + k] = v;
    }
  __syncthreads();
  for (int c = threadIdx.x; c < HD; c += blockDim.x)
    atomicAdd(dgain + c, red[c] + red[HD + c] + red[2 * HD + c] + red[3 * HD + c]);
}

// ---------------------------------------------------------------- dK, dV
template <int HD>
__global__ void __launch_bounds__(128)
dkdv_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K, const bf16* __restrict__ V,
            const bf16* __restrict__ dO, const float* __restrict__ LSE,
            const float* __restrict__ Dl, int S, int Hq, int Hkv, int Tmax, float scale_log2,
            float scale, const float* __restrict__ qkv_raw, QkBwd kq, bf16* __restrict__ dqkv,
            float* __restrict__ dkn) {
  constexpr int LD = HD + 8, KS = HD / 16, DT = HD / 8;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  bf16* sK = reinterpret_cast<bf16*>(smem_raw);   // [64][LD]
  bf16* sV = sK + KT_KEYS * LD;                    // [64][LD]
  bf16* sQb = sV + KT_KEYS * LD;                   // [2][32][LD]
  bf16* sdOb = sQb + 2 * KT_Q * LD;                // [2][32][LD]
  float* sLb = reinterpret_cast<float*>(sdOb + 2 * KT_Q * LD);   // [2][32]
  float* sDb = sLb + 2 * KT_Q;                                   // [2][32]
  pdl_trigger();
  pdl_wait();
  const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int k0 = kt * KT_KEYS;
  const size_t kv_base = ((size_t)b * Hkv + kvh) * Tmax * HD;
  load_rows<HD>(sK, K + kv_base + (size_t)k0 * HD, HD, KT_KEYS, S - k0);
  load_rows<HD>(sV, V + kv_base + (size_t)k0 * HD, HD, KT_KEYS, S - k0);
  // iterations: (q-head of the group, query tile at or after the keys), the
  // next one's tiles loading while the current one computes
  const int qstart = (k0 / KT_Q) * KT_Q;
  const int n_qt = (S - qstart + KT_Q - 1) / KT_Q;
  const int n_it = G * n_qt;
  auto load_it = [&](int it, int buf) {
    const int h = kvh * G + it / n_qt;
    const int q0 = qstart + (it % n_qt) * KT_Q;
    const size_t qrow = ((size_t)b * S + q0) * Hq + h;
    load_rows<HD>(sQb + buf * KT_Q * LD, Q + qrow * HD, (size_t)Hq * HD, KT_Q, S - q0);
    load_rows<HD>(sdOb + buf * KT_Q * LD, dO + qrow * HD, (size_t)Hq * HD, KT_Q, S - q0);
    if (threadIdx.x < KT_Q) {
      const int qq = q0 + threadIdx.x;
      sLb[buf * KT_Q + threadIdx.x] = qq < S ? LSE[((size_t)b * Hq + h) * S + qq] : 0.f;
      sDb[buf * KT_Q + threadIdx.x] = qq < S ? Dl[((size_t)b * Hq + h) * S + qq] : 0.f;
    }
  };
  if (n_it > 0) load_it(0, 0);
  cp_async_commit();

  float dk[DT][4], dv[DT][4];
#pragma unroll
  for (int j = 0; j < DT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[j][e] = dv[j][e] = 0.f;
  const int kw = warp * 16;                 // this warp's keys within the tile
  const int key0 = k0 + kw + g, key1 = key0 + 8;

  for (int it = 0; it < n_it; ++it) {
    {
      const int buf = it & 1;
      const int q0 = qstart + (it % n_qt) * KT_Q;
      if (it + 1 < n_it) load_it(it + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
      __syncthreads();
      const bf16* sQ = sQb + buf * KT_Q * LD;
      const bf16* sdO = sdOb + buf * KT_Q * LD;
      const float* sL = sLb + buf * KT_Q;
      const float* sD = sDb + buf * KT_Q;

      // S^T = K_w Q^T   [16 keys x 32 queries] : 4 n-tiles of 8 queries
      float st[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        ldsm_x4(smem_u32_local(sK + (kw + (lane & 15)) * LD + ks * 16 + (lane >> 4) * 8), a[0], a[1],
                a[2], a[3]);
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
          uint32_t b0, b1, b2, b3;
          const int qr = jp * 16 + (lane >> 4) * 8 + (lane & 7);
          ldsm_x4(smem_u32_local(sQ + qr * LD + ks * 16 + ((lane >> 3) & 1) * 8), b0, b1, b2, b3);
          mma16816_bf16(st[2 * jp], a, b0, b1);
          mma16816_bf16(st[2 * jp + 1], a, b2, b3);
        }
      }
      // P^T (causal: key <= query)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int ql = j * 8 + 2 * tq + (e & 1);
          const int qq = q0 + ql;
          const int key = (e < 2) ? key0 : key1;
          st[j][e] = (key <= qq && qq < S && key < S) ? exp2f(st[j][e] * scale_log2 - sL[ql]) : 0.f;
        }
      // dV += P^T dO
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_bf162(st[2 * kk][0], st[2 * kk][1]);
        pa[1] = pack_bf162(st[2 * kk][2], st[2 * kk][3]);
        pa[2] = pack_bf162(st[2 * kk + 1][0], st[2 * kk + 1][1]);
        pa[3] = pack_bf162(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
        for (int dp = 0; dp < DT / 2; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int qr = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
          ldsm_x4_t(smem_u32_local(sdO + qr * LD + dp * 16 + (lane >> 4) * 8), b0, b1, b2, b3);
          mma16816_bf16(dv[2 * dp], pa, b0, b1);
          mma16816_bf16(dv[2 * dp + 1], pa, b2, b3);
        }
      }
      // dP^T = V_w dO^T
      float dpt[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) dpt[j][0] = dpt[j][1] = dpt[j][2] = dpt[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        ldsm_x4(smem_u32_local(sV + (kw + (lane & 15)) * LD + ks * 16 + (lane >> 4) * 8), a[0], a[1],
                a[2], a[3]);
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
          uint32_t b0, b1, b2, b3;
          const int qr = jp * 16 + (lane >> 4) * 8 + (lane & 7);
          ldsm_x4(smem_u32_local(sdO + qr * LD + ks * 16 + ((lane >> 3) & 1) * 8), b0, b1, b2, b3);
          mma16816_bf16(dpt[2 * jp], a, b0, b1);
          mma16816_bf16(dpt[2 * jp + 1], a, b2, b3);
        }
      }
      // dS^T = P^T (dP^T - D)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int ql = j * 8 + 2 * tq + (e & 1);
          dpt[j][e] = st[j][e] * (dpt[j][e] - sD[ql]);
        }
      // dK += dS^T Q
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_bf162(dpt[2 * kk][0], dpt[2 * kk][1]);
        pa[1] = pack_bf162(dpt[2 * kk][2], dpt[2 * kk][3]);
        pa[2] = pack_bf162(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
        pa[3] = pack_bf162(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
        for (int dp = 0; dp < DT / 2; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int qr = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
          ldsm_x4_t(smem_u32_local(sQ + qr * LD + dp * 16 + (lane >> 4) * 8), b0, b1, b2, b3);
          mma16816_bf16(dk[2 * dp], pa, b0, b1);
          mma16816_bf16(dk[2 * dp + 1], pa, b2, b3);
        }
      }
      __syncthreads();   // this buffer is refilled by the next iteration's prefetch
    }
  }
  // dK through the RoPE / k-norm backward, dV unchanged, both bf16 into the
  // K and V columns of the QKV-projection gradient [B*S][qkv_dim]
  const int qd = Hq * HD, qkv_dim = (Hq + 2 * Hkv) * HD;
  const size_t t0 = (size_t)b * S + key0, t1 = (size_t)b * S + key1;
  const size_t kcol = (size_t)qd + kvh * HD, vcol = kcol + (size_t)Hkv * HD;
  float dg[DT][2];
#pragma unroll
  for (int j = 0; j < DT; ++j) dg[j][0] = dg[j][1] = 0.f;
  head_row_grad_store<HD>(dk, 0, scale, key0 < S, key0, qkv_raw + t0 * qkv_dim + kcol, kq,
                          dqkv + t0 * qkv_dim + kcol, dg, tq);
  head_row_grad_store<HD>(dk, 2, scale, key1 < S, key1, qkv_raw + t1 * qkv_dim + kcol, kq,
                          dqkv + t1 * qkv_dim + kcol, dg, tq);
  const QkBwd plain{nullptr, 0.f, nullptr};
  head_row_grad_store<HD>(dv, 0, 1.0f, key0 < S, key0, nullptr, plain, dqkv + t0 * qkv_dim + vcol,
                          dg, tq);
  head_row_grad_store<HD>(dv, 2, 1.0f, key1 < S, key1, nullptr, plain, dqkv + t1 * qkv_dim + vcol,
                          dg, tq);
  if (kq.gain != nullptr) {
    __syncthreads();   // the tiles are no longer read: reuse them for the reduction
    gain_grad_flush<HD>(dg, reinterpret_cast<float*>(smem_raw), dkn);
  }
}

// ---------------------------------------------------------------- dQ
template <int HD>
__global__ void __launch_bounds__(128)
dq_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K, const bf16* __restrict__ V,
          const bf16* __restrict__ O, const bf16* __restrict__ dO, const float* __restrict__ LSE,
          float* __restrict__ Dl, int S, int Hq, int Hkv, int Tmax, float scale_log2, float scale,
          const float* __restrict__ qkv_raw, QkBwd qq_, bf16* __restrict__ dqkv,
          float* __restrict__ dqn) {
  constexpr int LD = HD + 8, KS = HD / 16, DT = HD / 8;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);   // [64][LD]
  bf16* sdO = sQ + QT_Q * LD;                      // [64][LD]
  bf16* sKb = sdO + QT_Q * LD;                     // [2][32][LD]
  bf16* sVb = sKb + 2 * QT_KEYS * LD;              // [2][32][LD]
  bf16* sO = sVb + 2 * QT_KEYS * LD;               // [64][LD]
  float* sDv = reinterpret_cast<float*>(sO + QT_Q * LD);   // [64]
  pdl_trigger();
  pdl_wait();
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (Hq / Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int q0 = qt * QT_Q;
  const size_t qrow = ((size_t)b * S + q0) * Hq + h;
  load_rows<HD>(sQ, Q + qrow * HD, (size_t)Hq * HD, QT_Q, S - q0);
  load_rows<HD>(sdO, dO + qrow * HD, (size_t)Hq * HD, QT_Q, S - q0);
  load_rows<HD>(sO, O + qrow * HD, (size_t)Hq * HD, QT_Q, S - q0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  // D = rowsum(dO * O) of this tile's queries: two threads per row
  {
    const int r = threadIdx.x >> 1, hf = threadIdx.x & 1;
    float acc = 0.f;
#pragma unroll 8
    for (int c = hf * (HD / 2); c < (hf + 1) * (HD / 2); c += 2) {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sdO + r * LD + c));
      const float2 o = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sO + r * LD + c));
      acc += a.x * o.x + a.y * o.y;
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (hf == 0) {
      sDv[r] = acc;
      if (q0 + r < S) Dl[((size_t)b * Hq + h) * S + q0 + r] = acc;
    }
  }
  __syncthreads();
  uint32_t qa[KS][4], oa[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const int r = warp * 16 + (lane & 15), c = ks * 16 + (lane >> 4) * 8;
    ldsm_x4(smem_u32_local(sQ + r * LD + c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
    ldsm_x4(smem_u32_local(sdO + r * LD + c), oa[ks][0], oa[ks][1], oa[ks][2], oa[ks][3]);
  }
  const int qa0 = q0 + warp * 16 + g, qa1 = qa0 + 8;
  const float L0 = qa0 < S ? LSE[((size_t)b * Hq + h) * S + qa0] : 0.f;
  const float L1 = qa1 < S ? LSE[((size_t)b * Hq + h) * S + qa1] : 0.f;
  const float D0 = sDv[warp * 16 + g];
  const float D1 = sDv[warp * 16 + g + 8];
  float dq[DT][4];
#pragma unroll
  for (int j = 0; j < DT; ++j) dq[j][0] = dq[j][1] = dq[j][2] = dq[j][3] = 0.f;
  const size_t kv_base = ((size_t)b * Hkv + kvh) * Tmax * HD;
  const int kend = min(S, q0 + QT_Q);
  const int n_kt = (kend + QT_KEYS - 1) / QT_KEYS;
  auto load_kt = [&](int i, int buf) {
    const int k0 = i * QT_KEYS;
    load_rows<HD>(sKb + buf * QT_KEYS * LD, K + kv_base + (size_t)k0 * HD, HD, QT_KEYS, S - k0);
    load_rows<HD>(sVb + buf * QT_KEYS * LD, V + kv_base + (size_t)k0 * HD, HD, QT_KEYS, S - k0);
  };
  if (n_kt > 0) load_kt(0, 0);
  cp_async_commit();
  for (int i = 0; i < n_kt; ++i) {
    const int k0 = i * QT_KEYS, buf = i & 1;
    if (i + 1 < n_kt) load_kt(i + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const bf16* sK = sKb + buf * QT_KEYS * LD;
    const bf16* sV = sVb + buf * QT_KEYS * LD;
    float s[4][4], dp[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[j][e] = dp[j][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 2; ++jp) {
        uint32_t b0, b1, b2, b3;
        const int kr = jp * 16 + (lane >> 4) * 8 + (lane & 7);
        const int col = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(smem_u32_local(sK + kr * LD + col), b0, b1, b2, b3);
        mma16816_bf16(s[2 * jp], qa[ks], b0, b1);
        mma16816_bf16(s[2 * jp + 1], qa[ks], b2, b3);
        ldsm_x4(smem_u32_local(sV + kr * LD + col), b0, b1, b2, b3);
        mma16816_bf16(dp[2 * jp], oa[ks], b0, b1);
        mma16816_bf16(dp[2 * jp + 1], oa[ks], b2, b3);
      }
    }
    // dS = P (dP - D)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + j * 8 + 2 * tq + (e & 1);
        const int qq = (e < 2) ? qa0 : qa1;
        const float L = (e < 2) ? L0 : L1, Dd = (e < 2) ? D0 : D1;
        const float p = (key <= qq && key < S && qq < S) ? exp2f(s[j][e] * scale_log2 - L) : 0.f;
        s[j][e] = p * (dp[j][e] - Dd);
      }
    // dQ += dS K
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf162(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf162(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf162(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf162(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dpi = 0; dpi < DT / 2; ++dpi) {
        uint32_t b0, b1, b2, b3;
        const int kr = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        ldsm_x4_t(smem_u32_local(sK + kr * LD + dpi * 16 + (lane >> 4) * 8), b0, b1, b2, b3);
        mma16816_bf16(dq[2 * dpi], pa, b0, b1);
        mma16816_bf16(dq[2 * dpi + 1], pa, b2, b3);
      }
    }
    __syncthreads();   // this buffer is refilled by the next iteration's prefetch
  }
  // dQ through the RoPE / q-norm backward, bf16 into the Q columns of the
  // QKV-projection gradient [B*S][qkv_dim]
  const int qkv_dim = (Hq + 2 * Hkv) * HD;
  const size_t t0 = (size_t)b * S + qa0, t1 = (size_t)b * S + qa1;
  float dg[DT][2];
#pragma unroll
  for (int j = 0; j < DT; ++j) dg[j][0] = dg[j][1] = 0.f;
  head_row_grad_store<HD>(dq, 0, scale, qa0 < S, qa0, qkv_raw + t0 * qkv_dim + (size_t)h * HD,
                          qq_, dqkv + t0 * qkv_dim + (size_t)h * HD, dg, tq);
  head_row_grad_store<HD>(dq, 2, scale, qa1 < S, qa1, qkv_raw + t1 * qkv_dim + (size_t)h * HD,
                          qq_, dqkv + t1 * qkv_dim + (size_t)h * HD, dg, tq);
  if (qq_.gain != nullptr) {
    __syncthreads();
    gain_grad_flush<HD>(dg, reinterpret_cast<float*>(smem_raw), dqn);
  }
}

template <int HD>
cudaError_t launch_bwd_t(const bf16* Q, const bf16* K, const bf16* V, const bf16* O, const bf16* dO,
                         const float* LSE, float* Dl, int B, int S, int Hq, int Hkv, int Tmax,
                         const float* qkv_raw, const float* qn, const float* kn, float qk_eps,
                         const float2* rope_cs, bf16* dqkv, float* dqn, float* dkn,
                         cudaStream_t st) {
  constexpr int LD = HD + 8;
  const float scale = 1.0f / sqrtf((float)HD);
  const float scale_log2 = scale * 1.4426950408889634f;
  const size_t smem1 = (size_t)(2 * KT_KEYS + 4 * KT_Q) * LD * sizeof(bf16) + 4 * KT_Q * sizeof(float);
  const size_t smem2 = (size_t)(3 * QT_Q + 4 * QT_KEYS) * LD * sizeof(bf16) + QT_Q * sizeof(float);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(dkdv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
    cudaFuncSetAttribute(dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
    attr = true;
  }
  // dQ first: it also publishes D, which dK / dV read
  cudaError_t e = launch_k(dq_kernel<HD>, dim3((S + QT_Q - 1) / QT_Q, Hq, B), dim3(128), smem2, st,
                           Q, K, V, O, dO, LSE, Dl, S, Hq, Hkv, Tmax, scale_log2, scale, qkv_raw,
                           QkBwd{qn, qk_eps, rope_cs}, dqkv, dqn);
  if (e != cudaSuccess) return e;
  return launch_k(dkdv_kernel<HD>, dim3((S + KT_KEYS - 1) / KT_KEYS, Hkv, B), dim3(128), smem1, st,
                  Q, K, V, dO, LSE, (const float*)Dl, S, Hq, Hkv, Tmax, scale_log2, scale, qkv_raw,
                  QkBwd{kn, qk_eps, rope_cs}, dqkv, dkn);
}

}  // namespace

namespace {

template <int HD>
cudaError_t launch_dq_mma_hd(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                             const __nv_bfloat16* V, const __nv_bfloat16* O,
                             const __nv_bfloat16* dO, const float* LSE, float* Dl, int B, int S,
                             int Hq, int Hkv, int Tmax, const float* qkv_raw, const float* qn,
                             float qk_eps, const float2* rope_cs, __nv_bfloat16* dqkv,
                             float* dqn, cudaStream_t st) {
  constexpr int LD = HD + 8;
  const float scale = 1.0f / sqrtf((float)HD);
  const float scale_log2 = scale * 1.4426950408889634f;
  const size_t smem2 = (size_t)(3 * QT_Q + 4 * QT_KEYS) * LD * sizeof(bf16) + QT_Q * sizeof(float);
  static bool attr = false;   // one flag per instantiation
  if (!attr) {
    cudaFuncSetAttribute(dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
    attr = true;
  }
  return launch_k(dq_kernel<HD>, dim3((S + QT_Q - 1) / QT_Q, Hq, B), dim3(128), smem2, st, Q, K,
                  V, O, dO, LSE, Dl, S, Hq, Hkv, Tmax, scale_log2, scale, qkv_raw,
                  QkBwd{qn, qk_eps, rope_cs}, dqkv, dqn);
}

}  // namespace

cudaError_t launch_attn_dq_mma(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                               const __nv_bfloat16* V, const __nv_bfloat16* O,
                               const __nv_bfloat16* dO, const float* LSE, float* Dl, int B, int S,
                               int Hq, int Hkv, int hd, int Tmax, const float* qkv_raw,
                               const float* qn, float qk_eps, const float2* rope_cs,
                               __nv_bfloat16* dqkv, float* dqn, cudaStream_t st) {
  if (hd == 128)
    return launch_dq_mma_hd<128>(Q, K, V, O, dO, LSE, Dl, B, S, Hq, Hkv, Tmax, qkv_raw, qn,
                                 qk_eps, rope_cs, dqkv, dqn, st);
  if (hd == 64)
    return launch_dq_mma_hd<64>(Q, K, V, O, dO, LSE, Dl, B, S, Hq, Hkv, Tmax, qkv_raw, qn, qk_eps,
                                rope_cs, dqkv, dqn, st);
  return cudaErrorInvalidValue;
}

cudaError_t launch_attn_bwd(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                            const __nv_bfloat16* V, const __nv_bfloat16* O,
                            const __nv_bfloat16* dO, const float* LSE, float* Dl, int B, int S,
                            int Hq, int Hkv, int hd, int Tmax, const float* qkv_raw,
                            const float* qn, const float* kn, float qk_eps, const float2* rope_cs,
                            __nv_bfloat16* dqkv, float* dqn, float* dkn, int* status,
                            cudaStream_t st) {
  // Kernel choice for head_dim 128 and 64 (NE_ATTN_BWD_TC): "0" the mma.sync pair,
  // "1" the tcgen05 pair, "dkdv" mma.sync dQ + tcgen05 dK/dV; unset: by
  // sequence length (TC_BOTH_MIN_S and longer take the tcgen05 pair).
  static const int mode = [] {
    const char* e = std::getenv("NE_ATTN_BWD_TC");
    if (!e) return -1;
    if (e[0] == '0') return 0;
    if (e[0] == 'd') return 2;
    return 1;
  }();
  // from 256 positions (two 128-key tiles) the pipelined tcgen05 dQ with its D
  // pre-pass, merged with dK/dV, measured at least as fast as the mma.sync dQ
  constexpr int TC_BOTH_MIN_S = 256;
  if ((hd == 128 || (hd == 64 && attn_tc64())) && rope_cs != nullptr && mode != 0) {
    const bool tc_dq = mode == 1 || (mode == -1 && S >= TC_BOTH_MIN_S);
    return launch_attn_bwd_tc(Q, K, V, O, dO, LSE, Dl, B, S, Hq, Hkv, hd, Tmax, qkv_raw, qn, kn,
                              qk_eps, rope_cs, dqkv, dqn, dkn, status, st, tc_dq);
  }
  if (hd == 128)
    return launch_bwd_t<128>(Q, K, V, O, dO, LSE, Dl, B, S, Hq, Hkv, Tmax, qkv_raw, qn, kn, qk_eps,
                             rope_cs, dqkv, dqn, dkn, st);
  if (hd == 64)
    return launch_bwd_t<64>(Q, K, V, O, dO, LSE, Dl, B, S, Hq, Hkv, Tmax, qkv_raw, qn, kn, qk_eps,
                            rope_cs, dqkv, dqn, dkn, st);
  return cudaErrorInvalidValue;
}

}  // namespace ne
