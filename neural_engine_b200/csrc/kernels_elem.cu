// kernels_elem.cu -- HBM-bound kernels of the token loop and forward pass.
//
// Row layout everywhere is token-major: activations are [rows, features]
// with the feature axis contiguous (the reference keeps channel-first
// [DIM, SEQ] IOSurfaces, ane-training/training/training_dynamic/io.h:6-62;
// token-major is the natural layout for TMA-fed GEMMs and coalesced rows).
//
//   embed_rmsnorm     x = E[tok] (fp32), xn = bf16(rmsnorm(x) * g)
//                     (cpu_ops.h:433-439 embed_lookup + cpu_ops.h:20-60)
//   resid_rmsnorm     x += alpha * sum_s P[s]  (split-K partials, fixed order),
//                     xn = bf16(rmsnorm(x) * g)   (io.h:25-37 residual + rmsnorm)
//   qkv_post          sum split partials of the fused QKV projection, optional
//                     per-head QK RMSNorm, interleaved-pair RoPE
//                     (tools/generate.py:97-110), write q and append K/V (fp16)
//                     to the cache (generate.py:159-162)
//   swiglu_split      gate = silu(h1) * h3 from split partials of the W1/W3
//                     row-interleaved projection (generate.py:188-190)
//   argmax_rows       greedy next token, first index of the maximum
//                     (generate.py:200, numpy argmax tie rule)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"

namespace ne {

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ float block_sum(float v, float* red /*[32]*/) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

// rmsnorm of one row held as fp32 in shared memory `xs` (length D), written as
// bf16 to `out`.  rms = sqrt(mean(x^2) + eps); y = (x / rms) * g  (generate.py:81-84)
__device__ __forceinline__ void rmsnorm_row_store(const float* xs, const float* g, int D,
                                                  float eps, __nv_bfloat16* out, float* red) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) ss += xs[i] * xs[i];
  ss = block_sum(ss, red);
  const float rms = sqrtf(ss / (float)D + eps);
  for (int i = threadIdx.x * 2; i < D; i += blockDim.x * 2) {
    const float a = (xs[i] / rms) * g[i];
    const float b = (xs[i + 1] / rms) * g[i + 1];
    *reinterpret_cast<__nv_bfloat162*>(out + i) = __floats2bfloat162_rn(a, b);
  }
}

// ---------------------------------------------------------------- embed + norm
// One block per row.  tok: [rows]; table bf16 [V, D] (or fp32 if table_f32).
__global__ void embed_rmsnorm_kernel(const int32_t* __restrict__ tok, const void* __restrict__ table,
                                     int table_f32, int V, int D, const float* __restrict__ g,
                                     float eps, float* __restrict__ x, __nv_bfloat16* __restrict__ xn,
                                     int* status) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];
  float* xs = sm;
  float* red = sm + D;
  const int r = blockIdx.x;
  int t = tok[r];
  if (t < 0 || t >= V) {
    if (threadIdx.x == 0) atomicExch(status, DEV_ERR_BOUNDS);
    t = 0;
  }
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v;
    if (table_f32) v = reinterpret_cast<const float*>(table)[(size_t)t * D + i];
    else v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(table)[(size_t)t * D + i]);
    xs[i] = v;
    x[(size_t)r * D + i] = v;
  }
  __syncthreads();
  rmsnorm_row_store(xs, g, D, eps, xn + (size_t)r * D, red);
}

// ---------------------------------------------------------------- residual + norm
// x[r] += alpha * sum_{s<nsplit} P[s][r] (nsplit may be 0), then xn = rmsnorm.
__global__ void resid_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ P,
                                     int nsplit, long long split_stride, float alpha, int D,
                                     const float* __restrict__ g, float eps,
                                     __nv_bfloat16* __restrict__ xn, float* __restrict__ copy) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];
  float* xs = sm;
  float* red = sm + D;
  const int r = blockIdx.x;
  float* xr = x + (size_t)r * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = xr[i];
    if (nsplit > 0) {
      float acc = 0.f;
      for (int s = 0; s < nsplit; ++s) acc += P[(size_t)s * split_stride + (size_t)r * D + i];
      v += (alpha == 1.0f) ? acc : alpha * acc;
      xr[i] = v;
    }
    xs[i] = v;
    if (copy) copy[(size_t)r * D + i] = v;
  }
  __syncthreads();
  rmsnorm_row_store(xs, g, D, eps, xn + (size_t)r * D, red);
}

// Norm only (nsplit == 0), one warp per row: each lane holds V4 float4 of the
// row (lane-contiguous, so every load instruction is coalesced), the sum of
// squares is a warp reduction, no block barrier.  Same arithmetic as
// rmsnorm_row_store.
template <int V4>
__global__ void __launch_bounds__(256)
rmsnorm_rows_kernel(const float* __restrict__ x, int rows, const float* __restrict__ g,
                    float eps, __nv_bfloat16* __restrict__ xn, float* __restrict__ copy) {
  pdl_trigger();
  pdl_wait();
  constexpr int D = V4 * 128;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)r * D);
  float4 v[V4];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < V4; ++k) {
    v[k] = xr[lane + 32 * k];
    ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
  }
  if (copy) {
    float4* cr = reinterpret_cast<float4*>(copy + (size_t)r * D);
#pragma unroll
    for (int k = 0; k < V4; ++k) cr[lane + 32 * k] = v[k];
  }
  ss = warp_sum(ss);
  const float rms = sqrtf(ss / (float)D + eps);
  const float4* g4 = reinterpret_cast<const float4*>(g);
  uint2* out = reinterpret_cast<uint2*>(xn + (size_t)r * D);
#pragma unroll
  for (int k = 0; k < V4; ++k) {
    const float4 gg = g4[lane + 32 * k];
    uint2 pk;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
    h[0] = __floats2bfloat162_rn((v[k].x / rms) * gg.x, (v[k].y / rms) * gg.y);
    h[1] = __floats2bfloat162_rn((v[k].z / rms) * gg.z, (v[k].w / rms) * gg.w);
    out[lane + 32 * k] = pk;
  }
}

// ---------------------------------------------------------------- QKV post
// One warp per (row, head-vector).  Head vectors per row: Hq + 2*Hkv (q, k, v).
// qkv row layout (the fused projection's output): [q (Hq*hd) | k (Hkv*hd) | v (Hkv*hd)].
// Row r belongs to sequence b = r / S_rows at position pos0 + r % S_rows.
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// PER consecutive values -> one vector store (PER * sizeof(T) bytes, aligned
// because rows and heads are multiples of PER elements).
template <typename T, int PER>
__device__ __forceinline__ void store_vec(T* dst, const float (&v)[PER]) {
  if constexpr (PER == 4 && sizeof(T) == 2) {
    T t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) t[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(t);
  } else if constexpr (PER == 4 && sizeof(T) == 4) {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) dst[i] = from_f32<T>(v[i]);
  }
}

// One warp per (row, group of HPW heads): the group's loads are all issued
// before any of them is used, so each warp keeps HPW x 512 bytes in flight.
template <int HD, typename QT, typename KT, int HPW>
__global__ void qkv_post_kernel(const float* __restrict__ qkv, int nsplit, long long split_stride,
                                int rows, int S_rows, const int* __restrict__ d_pos, int pos0,
                                int Hq, int Hkv, const float* __restrict__ qn,
                                const float* __restrict__ kn, float qk_eps,
                                const float2* __restrict__ rope_cs, QT* __restrict__ q_out,
                                KT* __restrict__ kc, KT* __restrict__ vc, int Tmax,
                                int* status, int zero_src) {
  pdl_trigger();
  pdl_wait();
  constexpr int PER = HD / 32;  // elements per lane (2 or 4), consecutive
  const int warps_per_block = blockDim.x >> 5;
  const int gw = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int nh = Hq + 2 * Hkv;
  const int groups = nh / HPW;
  if (gw >= rows * groups) return;
  const int r = gw / groups, h0 = (gw % groups) * HPW;
  const int lane = threadIdx.x & 31;
  const int b = r / S_rows;
  const int pos = (d_pos ? *d_pos : pos0) + r % S_rows;
  if (pos < 0 || pos >= Tmax) {
    if (lane == 0) atomicExch(status, DEV_ERR_BOUNDS);
    return;
  }
  const int qkv_dim = nh * HD;
  const float* src = qkv + (size_t)r * qkv_dim + h0 * HD + lane * PER;
  float v[HPW][PER];
#pragma unroll
  for (int j = 0; j < HPW; ++j)
#pragma unroll
    for (int i = 0; i < PER; ++i) v[j][i] = 0.f;
  for (int s = 0; s < (nsplit > 0 ? nsplit : 1); ++s) {
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      const float* p = src + (size_t)s * split_stride + j * HD;
      if constexpr (PER == 4) {   // 16-byte aligned: rows and heads are multiples of 4 floats
        const float4 t = __ldcs(reinterpret_cast<const float4*>(p));
        v[j][0] += t.x; v[j][1] += t.y; v[j][2] += t.z; v[j][3] += t.w;
      } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) v[j][i] += p[i];
      }
    }
  }
  if (zero_src) {
    // the source is an accumulator the next projection adds into: leave it zeroed
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      float* z = const_cast<float*>(src) + j * HD;
      if constexpr (PER == 4) {
        *reinterpret_cast<float4*>(z) = make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) z[i] = 0.f;
      }
    }
  }
  // RoPE table row of this position: interleaved pairs (2i, 2i+1), PER/2 per lane
  float2 cs[PER / 2];
#pragma unroll
  for (int i = 0; i < PER / 2; ++i) cs[i] = rope_cs[(size_t)pos * (HD / 2) + lane * (PER / 2) + i];
#pragma unroll
  for (int j = 0; j < HPW; ++j) {
    const int h = h0 + j;
    const bool is_q = h < Hq, is_k = !is_q && h < Hq + Hkv;
    if ((is_q || is_k) && qn != nullptr) {
      const float* gain = is_q ? qn : kn;
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) ss += v[j][i] * v[j][i];
      ss = warp_sum(ss);
      const float rms = sqrtf(ss / (float)HD + qk_eps);
#pragma unroll
      for (int i = 0; i < PER; ++i) v[j][i] = (v[j][i] / rms) * gain[lane * PER + i];
    }
    if (is_q || is_k) {
#pragma unroll
      for (int i = 0; i < PER / 2; ++i) {
        const float v0 = v[j][2 * i], v1 = v[j][2 * i + 1];
        v[j][2 * i] = v0 * cs[i].x - v1 * cs[i].y;
        v[j][2 * i + 1] = v0 * cs[i].y + v1 * cs[i].x;
      }
    }
    if (is_q) {
      QT* dst = q_out + ((size_t)r * Hq + h) * HD + lane * PER;
      store_vec<QT, PER>(dst, v[j]);
    } else {
      const int kvh = is_k ? (h - Hq) : (h - Hq - Hkv);
      KT* cache = is_k ? kc : vc;
      KT* dst = cache + (((size_t)b * Hkv + kvh) * Tmax + pos) * HD + lane * PER;
      store_vec<KT, PER>(dst, v[j]);
    }
  }
}

// ---------------------------------------------------------------- SwiGLU (split partials)
// P: [nsplit][rows][2F] fp32 with W1/W3 interleaved in 16-row blocks.
__global__ void swiglu_split_kernel(float* __restrict__ P, int nsplit, long long split_stride,
                                    int rows, int F, __nv_bfloat16* __restrict__ gate,
                                    int zero_src) {
  pdl_trigger();
  pdl_wait();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)rows * F) return;
  const int r = (int)(idx / F), j = (int)(idx % F);
  const long long c1 = (long long)r * 2 * F + (j >> 4) * 32 + (j & 15);
  float h1 = 0.f, h3 = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    h1 += P[(size_t)s * split_stride + c1];
    h3 += P[(size_t)s * split_stride + c1 + 16];
  }
  if (zero_src) {   // accumulator of the next W1/W3 projection
    P[c1] = 0.f;
    P[c1 + 16] = 0.f;
  }
  // generate.py:93-94,190:  silu(h1) * h3,  silu(x) = x * (1 / (1 + exp(-x)))
  gate[idx] = __float2bfloat16_rn(h1 * (1.0f / (1.0f + expf(-h1))) * h3);
}

// ---------------------------------------------------------------- argmax
// One block per row; first index of the maximum (numpy argmax).  Writes the
// token into next_tok[r] and, when out_tokens is given, into
// out_tokens[(d_state[1]) * rows + r] (d_state = [pos, step]).
__global__ void argmax_rows_kernel(const float* __restrict__ logits, int V, int32_t* next_tok,
                                   int32_t* out_tokens, const int* d_state) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int r = blockIdx.x;
  const float* row = logits + (size_t)r * V;
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = row[i];
    if (v > best) { best = v; bi = i; }   // per-thread indices increase: strict > keeps first
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sv[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = (l < nw) ? sv[l] : -FLT_MAX;
    bi = (l < nw) ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (l == 0) {
      if (bi == 0x7fffffff) bi = 0;   // all NaN row: deterministic fallback
      next_tok[r] = bi;
      if (out_tokens) out_tokens[(size_t)d_state[1] * gridDim.x + r] = bi;
    }
  }
}

// Advance the on-device decode state [pos, step] by one token.
__global__ void advance_state_kernel(int* d_state) {
  pdl_trigger();
  pdl_wait();
  d_state[0] += 1;
  d_state[1] += 1;
}

// ================================================================ launchers
cudaError_t launch_embed_rmsnorm(const int32_t* tok, const void* table, int table_f32, int V, int D,
                                 const float* g, float eps, float* x, __nv_bfloat16* xn, int rows,
                                 int* status, cudaStream_t st) {
  const int threads = D >= 1024 ? 256 : 128;
  const size_t smem = (size_t)(D + 32) * sizeof(float);
  return launch_k(embed_rmsnorm_kernel, dim3(rows), dim3(threads), smem, st, tok, table,
                  table_f32, V, D, g, eps, x, xn, status);
}

cudaError_t launch_resid_rmsnorm(float* x, const float* P, int nsplit, long long split_stride,
                                 float alpha, int D, const float* g, float eps, __nv_bfloat16* xn,
                                 int rows, cudaStream_t st, float* copy) {
  if (nsplit == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(copy) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(g) & 15) == 0 && (reinterpret_cast<uintptr_t>(xn) & 7) == 0) {
    const dim3 grid((rows + 7) / 8);
    switch (D) {
      case 512: return launch_k(rmsnorm_rows_kernel<4>, grid, dim3(256), 0, st, x, rows, g, eps, xn,
                          copy);
      case 768: return launch_k(rmsnorm_rows_kernel<6>, grid, dim3(256), 0, st, x, rows, g, eps, xn,
                          copy);
      case 1024: return launch_k(rmsnorm_rows_kernel<8>, grid, dim3(256), 0, st, x, rows, g, eps, xn,
                          copy);
      case 2048: return launch_k(rmsnorm_rows_kernel<16>, grid, dim3(256), 0, st, x, rows, g, eps, xn,
                          copy);
      default: break;
    }
  }
  const int threads = D >= 1024 ? 256 : 128;
  const size_t smem = (size_t)(D + 32) * sizeof(float);
  return launch_k(resid_rmsnorm_kernel, dim3(rows), dim3(threads), smem, st, x, P, nsplit,
                  split_stride, alpha, D, g, eps, xn, copy);
}

cudaError_t launch_qkv_post(const float* qkv, int nsplit, long long split_stride, int rows,
                            int S_rows, const int* d_pos, int pos0, int Hq, int Hkv, int hd,
                            const float* qn, const float* kn, float qk_eps, const float2* rope_cs,
                            void* q_out, int q_type, void* kc, void* vc, int Tmax, int* status,
                            cudaStream_t st, int kv_bf16, int zero_src) {
  const int nh = Hq + 2 * Hkv;
  // four heads per warp where they divide the row (measured, Qwen3: one head
  // per warp cost 1 ms more per S 256 training step and 0.05 ms per B 256
  // decode step; eight per warp no better for training, 0.05 ms worse for decode)
  const bool by4 = nh % 4 == 0;
  const int warps = rows * (by4 ? nh / 4 : nh);
  const int threads = 256;
  const int blocks = (warps + 7) / 8;
#define NE_QKV(HD_, QT_, KT_)                                                                    \
  return by4 ? launch_k(qkv_post_kernel<HD_, QT_, KT_, 4>, dim3(blocks), dim3(threads), 0, st,   \
                        qkv, nsplit, split_stride, rows, S_rows, d_pos, pos0, Hq, Hkv, qn, kn,   \
                        qk_eps, rope_cs, reinterpret_cast<QT_*>(q_out),                          \
                        reinterpret_cast<KT_*>(kc), reinterpret_cast<KT_*>(vc), Tmax, status,    \
                        zero_src)                                                                \
             : launch_k(qkv_post_kernel<HD_, QT_, KT_, 1>, dim3(blocks), dim3(threads), 0, st,   \
                        qkv, nsplit, split_stride, rows, S_rows, d_pos, pos0, Hq, Hkv, qn, kn,   \
                        qk_eps, rope_cs, reinterpret_cast<QT_*>(q_out),                          \
                        reinterpret_cast<KT_*>(kc), reinterpret_cast<KT_*>(vc), Tmax, status,    \
                        zero_src)
  if (hd == 128) {
    if (kv_bf16) NE_QKV(128, __nv_bfloat16, __nv_bfloat16);
    if (q_type == 1) NE_QKV(128, __half, __half);
    NE_QKV(128, float, __half);
  } else if (hd == 64) {
    if (kv_bf16) NE_QKV(64, __nv_bfloat16, __nv_bfloat16);
    if (q_type == 1) NE_QKV(64, __half, __half);
    NE_QKV(64, float, __half);
  }
#undef NE_QKV
  return cudaErrorInvalidValue;
}

cudaError_t launch_swiglu_split(float* P, int nsplit, long long split_stride, int rows, int F,
                                __nv_bfloat16* gate, cudaStream_t st, int zero_src) {
  const long long n = (long long)rows * F;
  return launch_k(swiglu_split_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, P,
                  nsplit, split_stride, rows, F, gate, zero_src);
}

__global__ void argmax_keys_kernel(unsigned long long* keys, int rows, int32_t* next_tok,
                                   int32_t* out_tokens, int* d_state) {
  pdl_trigger();
  pdl_wait();
  const int step = d_state[1];
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const int32_t id = (int32_t)~(uint32_t)(keys[r] & 0xffffffffull);
    next_tok[r] = id;
    if (out_tokens) out_tokens[(size_t)step * rows + r] = id;
    keys[r] = 0ull;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    d_state[0] += 1;
    d_state[1] += 1;
  }
}

cudaError_t launch_argmax_keys(unsigned long long* keys, int rows, int32_t* next_tok,
                               int32_t* out_tokens, int* d_state, cudaStream_t st) {
  return launch_k(argmax_keys_kernel, dim3(1), dim3(256), 0, st, keys, rows, next_tok, out_tokens,
                  d_state);
}

cudaError_t launch_argmax(const float* logits, int rows, int V, int32_t* next_tok,
                          int32_t* out_tokens, int* d_state, int adv_state, cudaStream_t st) {
  cudaError_t e = launch_k(argmax_rows_kernel, dim3(rows), dim3(1024), 0, st, logits, V, next_tok,
                           out_tokens, (const int*)d_state);
  if (e == cudaSuccess && adv_state) e = launch_k(advance_state_kernel, dim3(1), dim3(1), 0, st, d_state);
  return e;
}

}  // namespace ne
