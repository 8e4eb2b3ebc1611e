// attn_decode.cu -- split-KV GQA attention of one new query per sequence.
//
// Arithmetic of the reference's token loop (tools/generate.py:164-181): for
// every q-head, scores = q . K[t] / sqrt(hd) over the cached positions
// t <= pos, softmax, weighted sum of V[t]; q-head h reads kv-head h / group.
// The fp16 KV cache is [sequence][kv_head][position][head_dim], so the K (and
// V) rows one (sequence, kv-head) needs are one contiguous stream.
//
// Organisation (the kernel is HBM-bound: one pass over the cache):
//   * A work item is (sequence, kv-head, split): a contiguous position range
//     serving the group's q-heads together (both Qwen3 q-heads of a kv-head
//     share every K/V byte read).
//   * Each warp owns a private 3-stage shared-memory ring and streams its
//     items' K and V rows into it with 1-D TMA bulk copies
//     (cp.async.bulk ... mbarrier::complete_tx), issued by lane 0 ahead of the
//     consumer, so the bytes in flight do not depend on registers.
//   * Chunk = 32/group positions.  Lane l owns head dims [l*hd/32, +hd/32);
//     each lane forms 32 partial dot products (positions x heads) and a
//     31-shuffle butterfly reduce-scatter leaves lane l with the full score of
//     (position l/group, head l%group).  Online softmax per head in the log2
//     domain (q is pre-scaled by log2(e)/sqrt(hd)); the chunk's weights go
//     through shared memory to the P.V accumulation, where each lane again
//     owns its head dims.
//   * Persistent grid (one CTA of 8 warps per SM); warp w takes items
//     w, w + W, ...; split partials (m, l, unnormalised O) are merged by
//     attn_combine_kernel.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ne_device.cuh"
#include "ne_internal.h"

namespace ne {
namespace {

constexpr int DA_MAX_WARPS = 8;

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int HD, int GROUP>
struct DaCfg {
  static constexpr int CHP = 32 / GROUP;                 // positions per chunk
  static constexpr int DPL = HD / 32;                    // head dims per lane
  static constexpr int ROW = HD * 2;                     // bytes per cache row
  static constexpr int CHUNK = CHP * ROW;                // bytes of K (or V) per chunk
  static constexpr int STAGES_RAW = 24576 / (2 * CHUNK);
  static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW);
  static constexpr int WARP_BYTES = STAGES * 2 * CHUNK;
  // as many warps (each with its own ring) as fit in ~196 KB, at most 8
  static constexpr int WARPS_RAW = 200704 / WARP_BYTES;
  static constexpr int WARPS = WARPS_RAW > DA_MAX_WARPS ? DA_MAX_WARPS : WARPS_RAW;
  static constexpr int SMEM = WARPS * WARP_BYTES + WARPS * 32 * 4 + WARPS * STAGES * 8 + 16;
};

struct ItemGeo {
  int b, kvh, split, t0, n;
};

__device__ __forceinline__ ItemGeo item_geo(int item, int n_splits, int Hkv, int T, int chunk_len) {
  ItemGeo g;
  const int pair = item / n_splits;
  g.split = item % n_splits;
  g.b = pair / Hkv;
  g.kvh = pair % Hkv;
  g.t0 = g.split * chunk_len;
  const int t1 = min(T, g.t0 + chunk_len);
  g.n = t1 > g.t0 ? t1 - g.t0 : 0;
  return g;
}

template <int HD, int GROUP>
__global__ void __launch_bounds__(DaCfg<HD, GROUP>::WARPS * 32, 1)
decode_attn_bulk_kernel(const float* __restrict__ q, const __half* __restrict__ kc,
                        const __half* __restrict__ vc, int Tmax, const int* __restrict__ d_pos,
                        int B, int Hq, int Hkv, int n_splits, float qscale,
                        float* __restrict__ part_o, float* __restrict__ part_ml,
                        __nv_bfloat16* __restrict__ out, int* status) {
  using C = DaCfg<HD, GROUP>;
  constexpr int CHP = C::CHP, DPL = C::DPL, STAGES = C::STAGES, DA_WARPS = C::WARPS;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * C::WARP_BYTES;
  float* sE = reinterpret_cast<float*>(smem + DA_WARPS * C::WARP_BYTES) + warp * 32;
  const uint32_t bars =
      smem_u32(smem + DA_WARPS * C::WARP_BYTES + DA_WARPS * 32 * 4) + warp * STAGES * 8;
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(smem + DA_WARPS * C::WARP_BYTES + DA_WARPS * 32 * 4 +
                                      DA_WARPS * STAGES * 8);
  if (threadIdx.x == 0) *abort_flag = 0;
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(bars + 8 * s, 1);
    fence_barrier_init();
  }
  __syncthreads();

  const int T = *d_pos + 1;
  int chunk_len = (T + n_splits - 1) / n_splits;
  chunk_len = (chunk_len + CHP - 1) / CHP * CHP;
  const int items = B * Hkv * n_splits;
  const int W = gridDim.x * DA_WARPS;
  const int wg = blockIdx.x * DA_WARPS + warp;

  // ---- producer cursor (lane 0 issues; all lanes track it identically)
  int p_item = wg, p_chunk = 0;
  auto skip_empty = [&]() {
    while (p_item < items) {
      const ItemGeo g = item_geo(p_item, n_splits, Hkv, T, chunk_len);
      if (p_chunk * CHP < g.n) return;
      p_item += W;
      p_chunk = 0;
    }
  };
  auto issue = [&](int slot) {
    // issue the chunk under the producer cursor into ring slot `slot`, advance
    const ItemGeo g = item_geo(p_item, n_splits, Hkv, T, chunk_len);
    const int tt = g.t0 + p_chunk * CHP;
    const int rows = min(CHP, g.n - p_chunk * CHP);
    if (lane == 0) {
      const size_t off = (((size_t)g.b * Hkv + g.kvh) * Tmax + tt) * HD;
      const uint32_t bytes = (uint32_t)rows * C::ROW;
      const uint32_t dst = smem_u32(ring + slot * 2 * C::CHUNK);
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bars + 8 * slot, 2 * bytes);
      bulk_g2s(dst, kc + off, bytes, bars + 8 * slot);
      bulk_g2s(dst + C::CHUNK, vc + off, bytes, bars + 8 * slot);
    }
    ++p_chunk;
    skip_empty();
  };
  skip_empty();
  int issued = 0;
  for (int s = 0; s < STAGES && p_item < items; ++s) {
    issue(s);
    ++issued;
  }

  int gc = 0;  // chunks consumed by this warp
  bool ok = true;
  for (int it = wg; it < items && ok; it += W) {
    const ItemGeo g = item_geo(it, n_splits, Hkv, T, chunk_len);
    float qf[GROUP][DPL];
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      const float* qp = q + ((size_t)g.b * Hq + g.kvh * GROUP + h) * HD + lane * DPL;
#pragma unroll
      for (int d = 0; d < DPL; ++d) qf[h][d] = qp[d] * qscale;
    }
    float m[GROUP], l[GROUP], acc[GROUP][DPL];
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      m[h] = -1e30f;
      l[h] = 0.f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[h][d] = 0.f;
    }
    const int nch = (g.n + CHP - 1) / CHP;
    for (int c = 0; c < nch; ++c) {
      const int slot = gc % STAGES;
      // every lane waits (each needs the barrier's acquire); the outcome is
      // made warp-uniform so no lane reaches a shuffle the others skip
      const bool landed = mbar_wait(bars + 8 * slot, (uint32_t)((gc / STAGES) & 1), status, abort_flag);
      if (!__all_sync(0xffffffffu, landed)) {
        ok = false;
        break;
      }
      const int nvalid = min(CHP, g.n - c * CHP);
      const uint8_t* sK = ring + slot * 2 * C::CHUNK + lane * DPL * 2;
      const uint8_t* sV = sK + C::CHUNK;
      // partial dot products over this lane's dims: index p*GROUP + h
      float v[32];
#pragma unroll
      for (int p = 0; p < CHP; ++p) {
        float kf[DPL];
        if constexpr (DPL == 4) {
          const uint2 raw = *reinterpret_cast<const uint2*>(sK + p * C::ROW);
          const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
          const float2 b2 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
          kf[0] = a.x; kf[1] = a.y; kf[2] = b2.x; kf[3] = b2.y;
        } else {
          const uint32_t raw = *reinterpret_cast<const uint32_t*>(sK + p * C::ROW);
          const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw));
          kf[0] = a.x; kf[1] = a.y;
        }
#pragma unroll
        for (int h = 0; h < GROUP; ++h) {
          float sdot = 0.f;
#pragma unroll
          for (int d = 0; d < DPL; ++d) sdot += qf[h][d] * kf[d];
          v[p * GROUP + h] = sdot;
        }
      }
      // butterfly reduce-scatter: lane l ends with the full sum of index l
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int j = 0; j < off; ++j) {
          const float send = upper ? v[j] : v[j + off];
          const float keep = upper ? v[j + off] : v[j];
          v[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      const int myh = lane % GROUP;
      const bool valid = (lane / GROUP) < nvalid;
      const float s = valid ? v[0] : -1e30f;
      float mc = s;
#pragma unroll
      for (int off = GROUP; off < 32; off <<= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
      float corr[GROUP], mnew[GROUP];
#pragma unroll
      for (int h = 0; h < GROUP; ++h) {
        const float mh = __shfl_sync(0xffffffffu, mc, h);
        mnew[h] = fmaxf(m[h], mh);
        corr[h] = exp2f(m[h] - mnew[h]);
      }
      float mine = mnew[0];
#pragma unroll
      for (int h = 1; h < GROUP; ++h)
        if (myh == h) mine = mnew[h];
      const float e = valid ? exp2f(s - mine) : 0.f;
      float se = e;
#pragma unroll
      for (int off = GROUP; off < 32; off <<= 1) se += __shfl_xor_sync(0xffffffffu, se, off);
#pragma unroll
      for (int h = 0; h < GROUP; ++h) {
        l[h] = l[h] * corr[h] + __shfl_sync(0xffffffffu, se, h);
        m[h] = mnew[h];
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[h][d] *= corr[h];
      }
      sE[lane] = e;
      __syncwarp();
      for (int p = 0; p < nvalid; ++p) {
        float vf[DPL];
        if constexpr (DPL == 4) {
          const uint2 raw = *reinterpret_cast<const uint2*>(sV + p * C::ROW);
          const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
          const float2 b2 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
          vf[0] = a.x; vf[1] = a.y; vf[2] = b2.x; vf[3] = b2.y;
        } else {
          const uint32_t raw = *reinterpret_cast<const uint32_t*>(sV + p * C::ROW);
          const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw));
          vf[0] = a.x; vf[1] = a.y;
        }
#pragma unroll
        for (int h = 0; h < GROUP; ++h) {
          const float w = sE[p * GROUP + h];
#pragma unroll
          for (int d = 0; d < DPL; ++d) acc[h][d] += w * vf[d];
        }
      }
      __syncwarp();
      ++gc;
      if (p_item < items) {
        issue(slot);
        ++issued;
      }
    }
    if (!ok) break;
    // ---- item result
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      const int qh = g.kvh * GROUP + h;
      if (n_splits == 1) {
        const float inv = 1.f / l[h];
        __nv_bfloat16* dst = out + ((size_t)g.b * Hq + qh) * HD + lane * DPL;
#pragma unroll
        for (int d = 0; d < DPL; d += 2)
          *reinterpret_cast<__nv_bfloat162*>(dst + d) =
              __floats2bfloat162_rn(acc[h][d] * inv, acc[h][d + 1] * inv);
      } else {
        const size_t pi = ((size_t)g.b * Hq + qh) * n_splits + g.split;
        float* dst = part_o + pi * HD + lane * DPL;
#pragma unroll
        for (int d = 0; d < DPL; ++d) dst[d] = acc[h][d];
        if (lane == 0) {
          part_ml[2 * pi] = m[h];
          part_ml[2 * pi + 1] = l[h];
        }
      }
    }
  }
  // Drain (bounded): copies issued but not consumed (only after an abort).
  for (int k = gc; k < issued; ++k) {
    const int slot = k % STAGES;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bars + 8 * slot, (uint32_t)((k / STAGES) & 1))) {
      if (globaltimer_ns() - t0 > 100000000ull) break;
    }
  }
}

// Grid (Hq, B), HD threads: merge the split partials of one head.
template <int HD>
__global__ void attn_combine_kernel(const float* __restrict__ part_o,
                                    const float* __restrict__ part_ml, int n_splits,
                                    __nv_bfloat16* __restrict__ out, int Hq) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const size_t base = ((size_t)b * Hq + h) * n_splits;
  float M = -1e30f;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, part_ml[2 * (base + s)]);
  float L = 0.f, O = 0.f;
  for (int s = 0; s < n_splits; ++s) {
    const float w = exp2f(part_ml[2 * (base + s)] - M);
    L += part_ml[2 * (base + s) + 1] * w;
    O += part_o[(base + s) * HD + d] * w;
  }
  out[((size_t)b * Hq + h) * HD + d] = __float2bfloat16_rn(O / L);
}

template <int HD, int G>
cudaError_t launch_bulk(const float* q, const __half* kc, const __half* vc, int B, int Hq, int Hkv,
                        int Tmax, const int* d_pos, int n_splits, float qscale, float* part_o,
                        float* part_ml, __nv_bfloat16* out, int* status, cudaStream_t st) {
  using C = DaCfg<HD, G>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(decode_attn_bulk_kernel<HD, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int items = B * Hkv * n_splits;
  int grid = (items + C::WARPS - 1) / C::WARPS;
  const int sms = device_num_sms();
  if (grid > sms) grid = sms;
  decode_attn_bulk_kernel<HD, G><<<grid, C::WARPS * 32, C::SMEM, st>>>(
      q, kc, vc, Tmax, d_pos, B, Hq, Hkv, n_splits, qscale, part_o, part_ml, out, status);
  return cudaGetLastError();
}

}  // namespace

int decode_attn_splits(int B, int Hkv, int Tmax, int num_sms) {
  const int pairs = B * Hkv;
  const int target = 8 * DA_MAX_WARPS * num_sms;   // about 8 items per warp
  int s = (target + pairs - 1) / pairs;
  const int max_s = (Tmax + 63) / 64;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  return s;
}

cudaError_t launch_decode_attn(const float* q, const __half* kc, const __half* vc, int B, int Hq,
                               int Hkv, int hd, int Tmax, const int* d_pos, int n_splits,
                               float* part_o, float* part_ml, __nv_bfloat16* out, int* status,
                               cudaStream_t st) {
  const float qscale = (1.0f / sqrtf((float)hd)) * 1.4426950408889634f;
  const int group = Hq / Hkv;
  cudaError_t e;
  if (hd == 128 && group == 2)
    e = launch_bulk<128, 2>(q, kc, vc, B, Hq, Hkv, Tmax, d_pos, n_splits, qscale, part_o, part_ml, out, status, st);
  else if (hd == 128 && group == 1)
    e = launch_bulk<128, 1>(q, kc, vc, B, Hq, Hkv, Tmax, d_pos, n_splits, qscale, part_o, part_ml, out, status, st);
  else if (hd == 64 && group == 1)
    e = launch_bulk<64, 1>(q, kc, vc, B, Hq, Hkv, Tmax, d_pos, n_splits, qscale, part_o, part_ml, out, status, st);
  else if (hd == 64 && group == 2)
    e = launch_bulk<64, 2>(q, kc, vc, B, Hq, Hkv, Tmax, d_pos, n_splits, qscale, part_o, part_ml, out, status, st);
  else
    return cudaErrorInvalidValue;
  if (e != cudaSuccess || n_splits == 1) return e;
  const dim3 g2(Hq, B);
  if (hd == 128) attn_combine_kernel<128><<<g2, 128, 0, st>>>(part_o, part_ml, n_splits, out, Hq);
  else attn_combine_kernel<64><<<g2, 64, 0, st>>>(part_o, part_ml, n_splits, out, Hq);
  return cudaGetLastError();
}

}  // namespace ne
