// kernels_train.cu -- elementwise / reduction kernels of the training step.
//
//   rmsnorm_bwd       dx = rrms * (w*dy - x * rrms^2 * sum(dy*w*x) / D) (+ residual),
//                     dw += dy * x * rrms.  The reference's CPU routine
//                     (ane-training/training/training_dynamic/cpu_ops.h:108-261)
//                     multiplies its whole result by w (exact only for unit
//                     gains); this kernel is the exact derivative of
//                     rmsnorm (generate.py:81-84), the oracle's definition.
//   ce_rows           per token: loss = -log(softmax(logits)[target] + 1e-10),
//                     dlogits = (softmax - onehot) * scale  (cpu_ops.h:348-382)
//   (the RoPE / QK-norm backward runs inside the attention backward, attn_bwd.cu)
//   adamw             decoupled AdamW with bias correction (cpu_ops.h:266-303)
//                     on fp32 masters, writing the bf16 compute copy
//   sumsq             sum of squares for the global gradient norm (train.m:805-826)
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"

namespace ne {
namespace {

using bf16 = __nv_bfloat16;
using bf162 = __nv_bfloat162;

__device__ __forceinline__ float block_sum256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

// ------------------------------------------------------------ RMSNorm backward
// One warp per row (no block barriers in the row reductions); 8 warps per
// block walk RB_ROWS rows each and reduce their dw partials once per block.
// All of a row's loads (x, dy, the residual) are issued before its reductions.
// Measured (Qwen3 S 256 step, one box, in this order): 2 rows per warp
// 24.03 ms, 1 row 24.34 ms, 4 rows 24.53 ms (within the drift of later runs).
constexpr int RB_ROWS = 2;
template <int PER>
__global__ void __launch_bounds__(256)
rmsnorm_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                   const float* __restrict__ w, float eps, int M, int D,
                   const float* __restrict__ residual, float* __restrict__ dx,
                   bf16* __restrict__ dx16, float* __restrict__ dw) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sdw[];   // [8][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float4 dwp[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) dwp[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 wv[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = (k * 32 + lane) * 4;
    wv[k] = i < D ? *reinterpret_cast<const float4*>(w + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const int r0 = (blockIdx.x * 8 + warp) * RB_ROWS;
  for (int rr = 0; rr < RB_ROWS; ++rr) {
    const int r = r0 + rr;
    if (r >= M) break;
    float4 xv[PER], gv[PER], rv[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = (k * 32 + lane) * 4;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      xv[k] = i < D ? *reinterpret_cast<const float4*>(x + (size_t)r * D + i) : z;
      gv[k] = i < D ? *reinterpret_cast<const float4*>(dy + (size_t)r * D + i) : z;
      rv[k] = (residual && i < D) ? *reinterpret_cast<const float4*>(residual + (size_t)r * D + i) : z;
    }
    float ss = 0.f, dot = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      ss += xv[k].x * xv[k].x + xv[k].y * xv[k].y + xv[k].z * xv[k].z + xv[k].w * xv[k].w;
      dot += gv[k].x * wv[k].x * xv[k].x + gv[k].y * wv[k].y * xv[k].y +
             gv[k].z * wv[k].z * xv[k].z + gv[k].w * wv[k].w * xv[k].w;
    }
    ss = warp_sum(ss);
    dot = warp_sum(dot);
    const float rrms = 1.0f / sqrtf(ss / (float)D + eps);
    const float c = rrms * rrms * dot / (float)D;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = (k * 32 + lane) * 4;
      if (i >= D) continue;
      float4 o;
      o.x = rrms * (wv[k].x * gv[k].x - xv[k].x * c) + rv[k].x;
      o.y = rrms * (wv[k].y * gv[k].y - xv[k].y * c) + rv[k].y;
      o.z = rrms * (wv[k].z * gv[k].z - xv[k].z * c) + rv[k].z;
      o.w = rrms * (wv[k].w * gv[k].w - xv[k].w * c) + rv[k].w;
      dwp[k].x += gv[k].x * xv[k].x * rrms;
      dwp[k].y += gv[k].y * xv[k].y * rrms;
      dwp[k].z += gv[k].z * xv[k].z * rrms;
      dwp[k].w += gv[k].w * xv[k].w * rrms;
      *reinterpret_cast<float4*>(dx + (size_t)r * D + i) = o;
      if (dx16) {
        uint2 pk;
        bf162* h = reinterpret_cast<bf162*>(&pk);
        h[0] = __floats2bfloat162_rn(o.x, o.y);
        h[1] = __floats2bfloat162_rn(o.z, o.w);
        *reinterpret_cast<uint2*>(dx16 + (size_t)r * D + i) = pk;
      }
    }
  }
  if (dw) {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = (k * 32 + lane) * 4;
      if (i < D) *reinterpret_cast<float4*>(sdw + warp * D + i) = dwp[k];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int w8 = 0; w8 < 8; ++w8) t += sdw[w8 * D + i];
      atomicAdd(dw + i, t);
    }
  }
}

// ------------------------------------------------------------ cross-entropy
// cpu_ops.h:348-382.  One block (512 threads) per row of logits [rows, V]
// (fp32).  The row's softmax statistics come from the classifier GEMM's
// epilogue as (max, sum exp) per 32-column chunk; they are combined into the
// row's (m, s), then the logits are read once to write
//   dlogits (bf16) = (softmax - onehot(target)) * scale
// and the row's loss -log(p_target + 1e-10).
__device__ __forceinline__ void ms_combine(float& m, float& s, float om, float os) {
  const float nm = fmaxf(m, om);
  s = (m == -FLT_MAX ? 0.f : s * __expf(m - nm)) + (om == -FLT_MAX ? 0.f : os * __expf(om - nm));
  m = nm;
}

constexpr int CE_THREADS = 512;
__global__ void __launch_bounds__(CE_THREADS)
ce_rows_kernel(const float* __restrict__ logits, int ld, const float2* __restrict__ stats,
               int stats_ld, const int32_t* __restrict__ tgt, const int32_t* __restrict__ remap,
               int V, float scale, float* __restrict__ loss, bf16* __restrict__ dlogits,
               int* status) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red_m[32], red_s[32];
  const int r = blockIdx.x;
  const float* row = logits + (size_t)r * ld;
  const float2* st = stats + (size_t)r * stats_ld;
  const int nck = (V + 31) / 32;
  float m = -FLT_MAX, s = 0.f;
  for (int i = threadIdx.x; i < nck; i += CE_THREADS) {
    const float2 c = st[i];
    ms_combine(m, s, c.x, c.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    ms_combine(m, s, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { red_m[w] = m; red_s[w] = s; }
  __syncthreads();
  if (w == 0) {
    m = l < CE_THREADS / 32 ? red_m[l] : -FLT_MAX;
    s = l < CE_THREADS / 32 ? red_s[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      ms_combine(m, s, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o));
    if (l == 0) { red_m[0] = m; red_s[0] = s; }
  }
  __syncthreads();
  m = red_m[0];
  s = red_s[0];
  int t = tgt[r];
  if (remap) t = (t >= 0) ? remap[t] : -1;   // full vocabulary id -> classifier column
  if (t < 0 || t >= V) {
    if (threadIdx.x == 0) atomicExch(status, DEV_ERR_BOUNDS);
    t = 0;
  }
  const float inv = 1.0f / s;
  if (threadIdx.x == 0) {
    const float pt = expf(row[t] - m) * inv;
    loss[r] = -logf(pt + 1e-10f);
  }
  bf16* drow = dlogits + (size_t)r * ld;
  if ((V & 3) == 0 && (ld & 3) == 0) {
    const float4* row4 = reinterpret_cast<const float4*>(row);
#pragma unroll 4
    for (int i = threadIdx.x; i < (V >> 2); i += CE_THREADS) {
      const float4 x = row4[i];
      float p0 = __expf(x.x - m) * inv, p1 = __expf(x.y - m) * inv;
      float p2 = __expf(x.z - m) * inv, p3 = __expf(x.w - m) * inv;
      const int d = t - 4 * i;
      if (d == 0) p0 -= 1.0f;
      if (d == 1) p1 -= 1.0f;
      if (d == 2) p2 -= 1.0f;
      if (d == 3) p3 -= 1.0f;
      uint2 pk;
      bf162* h = reinterpret_cast<bf162*>(&pk);
      h[0] = __floats2bfloat162_rn(p0 * scale, p1 * scale);
      h[1] = __floats2bfloat162_rn(p2 * scale, p3 * scale);
      *reinterpret_cast<uint2*>(drow + 4 * i) = pk;
    }
  } else {
    for (int i = threadIdx.x; i < V; i += CE_THREADS) {
      float p = __expf(row[i] - m) * inv;
      if (i == t) p -= 1.0f;
      drow[i] = __float2bfloat16_rn(p * scale);
    }
  }
}

// ------------------------------------------------------------ AdamW
// cpu_ops.h:266-303, element by element in the same order:
//   m = b1*m + (1-b1)*g;  v = b2*v + (1-b2)*g*g
//   upd = (m / bc1) / (sqrt(v / bc2) + eps) + wd * w;  w -= lr * upd
// g is the accumulated gradient times gscale (unscale and clip factors).
struct AdamElt {
  float lr, b1, b2, ob1, ob2, eps, inv_bc1, inv_bc2, gscale, wd;
  __device__ __forceinline__ void step(float& w, float g, float& m, float& v) const {
    const float gi = g * gscale;
    float mi = m * b1;
    mi = gi * ob1 + mi;
    float vi = v * b2;
    vi = (gi * gi) * ob2 + vi;
    const float mh = mi * inv_bc1;
    const float vh = sqrtf(vi * inv_bc2) + eps;
    float upd = mh / vh;
    upd = w * wd + upd;
    w = upd * (-lr) + w;
    m = mi;
    v = vi;
  }
};

// ------------------------------------------------------------ chunked multi-tensor forms
// Every trainable tensor is cut into chunks of OPT_CHUNK elements and one
// 256-thread block owns one chunk, so all blocks stream the same number of
// bytes whatever the tensor sizes (the gains are 128..1024 elements, the
// tied embedding 1.5e8).  Chunks whose four pointers are 16-byte aligned use
// float4 loads and stores.
__device__ __forceinline__ double block_sum256_d(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.0;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;   // valid in thread 0
}

// Sum of squares of every gradient (train.m:805-826).  Each block writes its
// chunk's partial sum; the block that finishes last (ticket) adds the partials
// in chunk order (deterministic), and writes
//   norm_out[0] = sqrt(sum) * grad_scale              (pre-clip global norm)
//   norm_out[1] = grad_scale * min(1, clip / norm)    (factor AdamW applies)
__global__ void __launch_bounds__(256)
sumsq_chunks_kernel(const AdamSeg* __restrict__ segs, const OptChunk* __restrict__ chunks,
                    int nchunks, float* __restrict__ partial, unsigned* __restrict__ ticket,
                    float grad_scale, float grad_clip, float* __restrict__ norm_out,
                    int partial_only) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  __shared__ double redd[32];
  __shared__ int last;
  const OptChunk c = chunks[blockIdx.x];
  const AdamSeg sg = segs[c.seg];
  const int n = c.norm ? c.n : 0;   // chunks outside this rank's share add nothing
  const float* g = sg.g + c.off;
  float acc = 0.f;
  if (c.vec) {
    const float4* g4 = reinterpret_cast<const float4*>(g);
#pragma unroll 4
    for (int i = threadIdx.x; i < (n >> 2); i += 256) {
      const float4 x = g4[i];
      acc += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
    for (int i = (n & ~3) + threadIdx.x; i < n; i += 256) acc += g[i] * g[i];
  } else {
    for (int i = threadIdx.x; i < n; i += 256) acc += g[i] * g[i];
  }
  acc = block_sum256(acc, red);
  if (threadIdx.x == 0) {
    partial[blockIdx.x] = acc;
    __threadfence();
    last = (atomicAdd(ticket, 1u) == (unsigned)nchunks - 1u);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  double s = 0.0;
  for (int i = threadIdx.x; i < nchunks; i += 256) s += (double)__ldcg(partial + i);
  s = block_sum256_d(s, redd);
  if (threadIdx.x == 0) {
    norm_out[2] = (float)s;
    if (!partial_only) {
      const float norm = (float)(sqrt(s) * (double)grad_scale);
      float scale = grad_scale;
      if (grad_clip > 0.f && norm > grad_clip) scale *= grad_clip / norm;
      norm_out[0] = norm;
      norm_out[1] = scale;
    }
  }
}

// Norm and clip factor from the rank-summed sum of squares in norm_out[2].
__global__ void norm_finish_kernel(float* norm_out, float grad_scale, float grad_clip) {
  pdl_trigger();
  pdl_wait();
  const float norm = sqrtf(norm_out[2]) * grad_scale;
  float scale = grad_scale;
  if (grad_clip > 0.f && norm > grad_clip) scale *= grad_clip / norm;
  norm_out[0] = norm;
  norm_out[1] = scale;
}

// AdamW over every chunk; the gradient factor is norm_out[1] (written by
// sumsq_chunks_kernel earlier on the same stream).
__global__ void __launch_bounds__(256)
adamw_chunks_kernel(const AdamSeg* __restrict__ segs, const OptChunk* __restrict__ chunks,
                    float lr, float b1, float b2, float eps, float inv_bc1, float inv_bc2,
                    const float* __restrict__ norm_out) {
  pdl_trigger();
  pdl_wait();
  const OptChunk c = chunks[blockIdx.x];
  const AdamSeg sg = segs[c.seg];
  const int n = c.n;
  const AdamElt a{lr, b1, b2, 1.0f - b1, 1.0f - b2, eps, inv_bc1, inv_bc2, norm_out[1], sg.wd};
  float* w = sg.w + c.off;
  const float* g = sg.g + c.off;
  float* m = sg.m + c.off;
  float* v = sg.v + c.off;
  bf16* w16 = sg.w16 ? sg.w16 + c.off : nullptr;
  int i0 = 0;
  if (c.vec) {
    float4* w4 = reinterpret_cast<float4*>(w);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
#pragma unroll 2
    for (int i = threadIdx.x; i < (n >> 2); i += 256) {
      float4 wv = w4[i], mv = m4[i], vv = v4[i];
      const float4 gv = g4[i];
      a.step(wv.x, gv.x, mv.x, vv.x);
      a.step(wv.y, gv.y, mv.y, vv.y);
      a.step(wv.z, gv.z, mv.z, vv.z);
      a.step(wv.w, gv.w, mv.w, vv.w);
      w4[i] = wv;
      m4[i] = mv;
      v4[i] = vv;
      if (w16) {
        uint2 pk;
        bf162* h = reinterpret_cast<bf162*>(&pk);
        h[0] = __floats2bfloat162_rn(wv.x, wv.y);
        h[1] = __floats2bfloat162_rn(wv.z, wv.w);
        *reinterpret_cast<uint2*>(w16 + 4 * i) = pk;
      }
    }
    i0 = n & ~3;
  }
  for (int i = i0 + threadIdx.x; i < n; i += 256) {
    float wi = w[i], mi = m[i], vi = v[i];
    a.step(wi, g[i], mi, vi);
    w[i] = wi;
    m[i] = mi;
    v[i] = vi;
    if (w16) w16[i] = __float2bfloat16_rn(wi);
  }
}

// fp32 -> bf16 elementwise copy
__global__ void f32_to_bf16_kernel(const float* __restrict__ a, bf16* __restrict__ b, long long n) {
  pdl_trigger();
  pdl_wait();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    b[i] = __float2bfloat16_rn(a[i]);
}

int grid_for(long long n, int threads) {
  long long g = (n + threads - 1) / threads;
  const long long cap = (long long)device_num_sms() * 8;
  return (int)(g < cap ? (g < 1 ? 1 : g) : cap);
}

}  // namespace

cudaError_t launch_rmsnorm_bwd(const float* dy, const float* x, const float* w, float eps, int M,
                               int D, const float* residual, float* dx, __nv_bfloat16* dx16,
                               float* dw, cudaStream_t st) {
  if (D > 1024 || D % 4) return cudaErrorInvalidValue;
  const dim3 grid((M + 8 * RB_ROWS - 1) / (8 * RB_ROWS));
  const size_t smem = (size_t)8 * D * sizeof(float);
  if (D <= 512)
    return launch_k(rmsnorm_bwd_kernel<4>, grid, dim3(256), smem, st, dy, x, w, eps, M, D, residual,
                    dx, dx16, dw);
  return launch_k(rmsnorm_bwd_kernel<8>, grid, dim3(256), smem, st, dy, x, w, eps, M, D, residual,
                  dx, dx16, dw);
}

cudaError_t launch_ce_rows(const float* logits, int ld, const float2* stats, int stats_ld,
                           const int32_t* tgt, const int32_t* remap, int rows, int V, float scale,
                           float* loss, __nv_bfloat16* dlogits, int* status, cudaStream_t st) {
  return launch_k(ce_rows_kernel, dim3(rows), dim3(CE_THREADS), 0, st, logits, ld, stats,
                  stats_ld, tgt, remap, V, scale, loss, dlogits, status);
}

// ------------------------------------------------------------ vocabulary compaction
// (vocab_compact_embed / vocab_scatter_grads, cpu_ops.h:416-431)
namespace {
__global__ void gather_rows_kernel(const bf16* __restrict__ src, const int32_t* __restrict__ idx,
                                   int n, int D, bf16* __restrict__ dst) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= n) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(src + (size_t)idx[r] * D);
  uint4* d4 = reinterpret_cast<uint4*>(dst + (size_t)r * D);
  for (int i = threadIdx.x; i < D / 8; i += blockDim.x) d4[i] = s4[i];
}
// dst[idx[r]] += src[r]; src[r] = 0 (each destination row appears once)
__global__ void scatter_add_rows_kernel(float* __restrict__ src, const int32_t* __restrict__ idx,
                                        int n, int D, float* __restrict__ dst) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= n) return;
  float* s = src + (size_t)r * D;
  float* d = dst + (size_t)idx[r] * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    d[i] += s[i];
    s[i] = 0.f;
  }
}
}  // namespace

cudaError_t launch_gather_rows(const __nv_bfloat16* src, const int32_t* idx, int n, int D,
                               __nv_bfloat16* dst, cudaStream_t st) {
  if (D % 8) return cudaErrorInvalidValue;
  return launch_k(gather_rows_kernel, dim3(n), dim3(128), 0, st, src, idx, n, D, dst);
}

cudaError_t launch_scatter_add_rows(float* src, const int32_t* idx, int n, int D, float* dst,
                                    cudaStream_t st) {
  return launch_k(scatter_add_rows_kernel, dim3(n), dim3(256), 0, st, src, idx, n, D, dst);
}



cudaError_t launch_sumsq_chunks(const AdamSeg* segs, const OptChunk* chunks, int nchunks,
                                float* partial, unsigned* ticket, float grad_scale,
                                float grad_clip, float* norm_out, cudaStream_t st,
                                int partial_only) {
  cudaError_t e = cudaMemsetAsync(ticket, 0, sizeof(unsigned), st);
  if (e != cudaSuccess) return e;
  return launch_k(sumsq_chunks_kernel, dim3(nchunks), dim3(256), 0, st, segs, chunks, nchunks,
                  partial, ticket, grad_scale, grad_clip, norm_out, partial_only);
}

cudaError_t launch_norm_finish(float* norm_out, float grad_scale, float grad_clip, cudaStream_t st) {
  return launch_k(norm_finish_kernel, dim3(1), dim3(1), 0, st, norm_out, grad_scale, grad_clip);
}

cudaError_t launch_adamw_chunks(const AdamSeg* segs, const OptChunk* chunks, int nchunks,
                                float lr, float b1, float b2, float eps, float inv_bc1,
                                float inv_bc2, const float* norm_out, cudaStream_t st) {
  return launch_k(adamw_chunks_kernel, dim3(nchunks), dim3(256), 0, st, segs, chunks, lr, b1, b2,
                  eps, inv_bc1, inv_bc2, norm_out);
}

// ------------------------------------------------------------ value ranges
// out[0] = min, out[1] = max of a[0..n) (the step line's x[...] / dy[...]
// ranges, train.m:771-776); out must hold (+inf, -inf) before the launch.
namespace {
__device__ __forceinline__ void atomic_min_f(float* a, float v) {
  if (v >= 0.f) atomicMin(reinterpret_cast<int*>(a), __float_as_int(v));
  else atomicMax(reinterpret_cast<unsigned*>(a), __float_as_uint(v));
}
__device__ __forceinline__ void atomic_max_f(float* a, float v) {
  if (v >= 0.f) atomicMax(reinterpret_cast<int*>(a), __float_as_int(v));
  else atomicMin(reinterpret_cast<unsigned*>(a), __float_as_uint(v));
}
__global__ void __launch_bounds__(256) minmax_kernel(const float* __restrict__ a, long long n,
                                                     float* out) {
  pdl_trigger();
  pdl_wait();
  float lo = INFINITY, hi = -INFINITY;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float v = a[i];
    lo = fminf(lo, v);
    hi = fmaxf(hi, v);
  }
  for (int o = 16; o; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  __shared__ float slo[8], shi[8];
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    slo[w] = lo;
    shi[w] = hi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) {
      lo = fminf(lo, slo[i]);
      hi = fmaxf(hi, shi[i]);
    }
    atomic_min_f(out, lo);
    atomic_max_f(out + 1, hi);
  }
}
__global__ void minmax_init_kernel(float* out) {
  out[0] = INFINITY;
  out[1] = -INFINITY;
}
}  // namespace

cudaError_t launch_minmax(const float* a, long long n, float* out, cudaStream_t st) {
  minmax_init_kernel<<<1, 1, 0, st>>>(out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_k(minmax_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, a, n, out);
}

cudaError_t launch_f32_to_bf16(const float* a, __nv_bfloat16* b, long long n, cudaStream_t st) {
  return launch_k(f32_to_bf16_kernel, dim3(grid_for(n, 256)), dim3(256), 0, st, a, b, n);
}

}  // namespace ne
