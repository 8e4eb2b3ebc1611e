// attn_decode.cu -- split-KV GQA attention of one new query per sequence.
//
// Arithmetic of the reference's token loop (tools/generate.py:164-181): for
// every q-head, scores = q . K[t] / sqrt(hd) over the cached positions
// t <= pos, softmax, weighted sum of V[t]; q-head h reads kv-head h / group.
// The fp16 KV cache is [sequence][kv_head][position][head_dim], so the K (and
// V) rows one (sequence, kv-head) pair needs are one contiguous stream.
//
// Organisation (the kernel is HBM-bound: one pass over the cache):
//   * Even partition.  The P = B * Hkv pairs, each with T = pos + 1 cached
//     positions, are laid end to end (P * T positions) and cut into W equal
//     ranges, one per warp (W = warps of the persistent grid), rounded to
//     whole chunks.  A range covers the tail of one pair, whole pairs and the
//     head of another; each piece is a segment with its own online softmax,
//     and every warp streams the same number of bytes.
//   * Each warp owns a private shared-memory ring and streams K and V rows
//     into it with 1-D TMA bulk copies (cp.async.bulk ...
//     mbarrier::complete_tx) issued by lane 0 ahead of the consumer, so the
//     bytes in flight do not depend on registers.
//   * Chunk = 32/group positions.  Lane l owns head dims [l*hd/32, +hd/32);
//     each lane forms 32 partial dot products (positions x heads) and a
//     31-shuffle butterfly reduce-scatter leaves lane l with the full score of
//     (position l/group, head l%group).  Online softmax per head in the log2
//     domain (q is pre-scaled by log2(e)/sqrt(hd)); the chunk's weights go
//     through shared memory to the P.V accumulation.
//   * A pair covered by one segment is normalised and written directly.
//     Otherwise every segment writes (m, l, unnormalised O) per q-head and
//     takes a ticket on the pair's counter; the warp that takes the last
//     ticket merges the pair's segments (log-sum-exp rescaling), writes the
//     output and resets the counter -- no second kernel, no waiting.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"

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

// Range length per warp: ceil(P*T / W) rounded up to whole chunks.
__device__ __forceinline__ long long range_len(long long total, int W, int chp) {
  long long L = (total + W - 1) / W;
  return (L + chp - 1) / chp * chp;
}

template <int HD, int GROUP>
__global__ void __launch_bounds__(DaCfg<HD, GROUP>::WARPS * 32, 1)
decode_attn_kernel(const float* __restrict__ q, const __half* __restrict__ kc,
                   const __half* __restrict__ vc, int Tmax, const int* __restrict__ d_pos, int P,
                   int Hq, int Hkv, float qscale, float* __restrict__ part_o,
                   float* __restrict__ part_ml, int* __restrict__ pair_cnt,
                   __nv_bfloat16* __restrict__ out, int* status) {
  using C = DaCfg<HD, GROUP>;
  constexpr int CHP = C::CHP, DPL = C::DPL, STAGES = C::STAGES, NW = C::WARPS;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * C::WARP_BYTES;
  float* sE = reinterpret_cast<float*>(smem + NW * C::WARP_BYTES) + warp * 32;
  const uint32_t bars = smem_u32(smem + NW * C::WARP_BYTES + NW * 32 * 4) + warp * STAGES * 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(
      smem + NW * C::WARP_BYTES + NW * 32 * 4 + NW * STAGES * 8);
  if (threadIdx.x == 0) *abort_flag = 0;
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(bars + 8 * s, 1);
    fence_barrier_init();
  }
  pdl_trigger();
  __syncthreads();
  pdl_wait();   // q and the new K/V row come from the preceding kernel

  const int T = *d_pos + 1;
  const int W = gridDim.x * NW;
  const int w = blockIdx.x * NW + warp;
  const long long total = (long long)P * T;
  const long long L = range_len(total, W, CHP);
  const long long w_begin = (long long)w * L;
  const long long w_end = w_begin + L < total ? w_begin + L : total;
  const int seg_per_warp = (int)((L + T - 1) / T) + 1;
  const int first_pair = (int)(w_begin / T);

  // ---- producer (lane 0 issues; all lanes track the cursor identically)
  long long p_pos = w_begin;
  auto issue = [&](int slot) {
    const int pair = (int)(p_pos / T);
    const int tin = (int)(p_pos % T);
    long long rows = CHP;
    if (w_end - p_pos < rows) rows = w_end - p_pos;
    if (T - tin < rows) rows = T - tin;
    if (lane == 0) {
      const size_t off = ((size_t)pair * Tmax + tin) * HD;   // pair = b*Hkv + kvh
      const uint32_t bytes = (uint32_t)rows * C::ROW;
      const uint32_t dst = smem_u32(ring + slot * 2 * C::CHUNK);
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bars + 8 * slot, 2 * bytes);
      bulk_g2s(dst, kc + off, bytes, bars + 8 * slot);
      bulk_g2s(dst + C::CHUNK, vc + off, bytes, bars + 8 * slot);
    }
    p_pos += rows;
  };
  int issued = 0;
  for (int s = 0; s < STAGES && p_pos < w_end; ++s) {
    issue(s);
    ++issued;
  }

  int gc = 0;  // chunks consumed by this warp
  bool ok = true;
  long long c_pos = w_begin;
  while (c_pos < w_end && ok) {
    const int pair = (int)(c_pos / T);
    const long long seg_end = ((long long)(pair + 1) * T < w_end) ? (long long)(pair + 1) * T : w_end;
    const int b = pair / Hkv, kvh = pair % Hkv;
    float qf[GROUP][DPL];
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      const float* qp = q + ((size_t)b * Hq + kvh * GROUP + h) * HD + lane * DPL;
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
    while (c_pos < seg_end) {
      const int slot = gc % STAGES;
      // every lane waits (each needs the barrier's acquire); the outcome is
      // made warp-uniform so no lane reaches a shuffle the others skip
      const bool landed =
          mbar_wait(bars + 8 * slot, (uint32_t)((gc / STAGES) & 1), status, abort_flag);
      if (!__all_sync(0xffffffffu, landed)) {
        ok = false;
        break;
      }
      const int nvalid = (int)((seg_end - c_pos) < CHP ? (seg_end - c_pos) : CHP);
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
      const bool valid = (lane / GROUP) < nvalid;   // rows past nvalid are stale smem
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
          const float wgt = sE[p * GROUP + h];
#pragma unroll
          for (int d = 0; d < DPL; ++d) acc[h][d] += wgt * vf[d];
        }
      }
      __syncwarp();
      c_pos += nvalid;
      ++gc;
      if (p_pos < w_end) {
        issue(slot);
        ++issued;
      }
    }
    if (!ok) break;
    // segments of this pair: warps w0 .. w1 (the same cut as every warp makes)
    const int w0 = (int)(((long long)pair * T) / L);
    const int w1 = (int)(((long long)(pair + 1) * T - 1) / L);
    if (w0 == w1) {
      // the whole pair is this segment: normalise and write the output
#pragma unroll
      for (int h = 0; h < GROUP; ++h) {
        __nv_bfloat16* o = out + ((size_t)b * Hq + kvh * GROUP + h) * HD + lane * DPL;
        const float inv = 1.0f / l[h];
#pragma unroll
        for (int d = 0; d < DPL; ++d) o[d] = __float2bfloat16_rn(acc[h][d] * inv);
      }
      continue;
    }
    // ---- segment partial: slot (w, pair - first_pair)
    const size_t si = (size_t)w * seg_per_warp + (pair - first_pair);
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      float* dst = part_o + (si * GROUP + h) * HD + lane * DPL;
#pragma unroll
      for (int d = 0; d < DPL; ++d) dst[d] = acc[h][d];
      if (lane == 0) {
        part_ml[(si * GROUP + h) * 2] = m[h];
        part_ml[(si * GROUP + h) * 2 + 1] = l[h];
      }
    }
    __threadfence();   // partials visible device-wide before the ticket
    __syncwarp();
    int ticket = 0;
    if (lane == 0) ticket = atomicAdd(pair_cnt + pair, 1);
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != w1 - w0) continue;
    // last segment of the pair to finish: merge all of them
    __threadfence();
    if (lane == 0) pair_cnt[pair] = 0;   // ready for the next launch
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      float M = -1e30f;
      for (int ww = w0; ww <= w1; ++ww) {
        const size_t sj = (size_t)ww * seg_per_warp + (pair - (int)(((long long)ww * L) / T));
        M = fmaxf(M, __ldcg(part_ml + (sj * GROUP + h) * 2));
      }
      float Lsum = 0.f, O[DPL];
#pragma unroll
      for (int d = 0; d < DPL; ++d) O[d] = 0.f;
      for (int ww = w0; ww <= w1; ++ww) {
        const size_t sj = (size_t)ww * seg_per_warp + (pair - (int)(((long long)ww * L) / T));
        const float wt = exp2f(__ldcg(part_ml + (sj * GROUP + h) * 2) - M);
        Lsum += __ldcg(part_ml + (sj * GROUP + h) * 2 + 1) * wt;
        const float* src = part_o + (sj * GROUP + h) * HD + lane * DPL;
#pragma unroll
        for (int d = 0; d < DPL; ++d) O[d] += __ldcg(src + d) * wt;
      }
      __nv_bfloat16* o = out + ((size_t)b * Hq + kvh * GROUP + h) * HD + lane * DPL;
      const float inv = 1.0f / Lsum;
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[d] = __float2bfloat16_rn(O[d] * inv);
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

template <int HD, int G>
cudaError_t launch_t(const float* q, const __half* kc, const __half* vc, int B, int Hq, int Hkv,
                     int Tmax, const int* d_pos, float qscale, float* part_o, float* part_ml,
                     int* pair_cnt, __nv_bfloat16* out, int* status, cudaStream_t st) {
  using C = DaCfg<HD, G>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<HD, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  // Persistent grid of up to one CTA per SM, fewer when the cache is short:
  // every warp should stream at least ~128 positions, so few sequences (B 1:
  // 8 histories) are not cut into dozens of segments that one warp per history
  // must then merge.  Sized by the cache capacity Tmax (the graph replays the
  // launch for every position); the kernel cuts the current positions over
  // however many warps it has.
  const int P = B * Hkv;
  const long long want_warps = ((long long)P * Tmax + 127) / 128;
  const long long want_ctas = (want_warps + C::WARPS - 1) / C::WARPS;
  const int grid = (int)(want_ctas < device_num_sms() ? (want_ctas < 1 ? 1 : want_ctas)
                                                      : device_num_sms());
  return launch_k(decode_attn_kernel<HD, G>, dim3(grid), dim3(C::WARPS * 32), (size_t)C::SMEM,
                  st, q, kc, vc, Tmax, d_pos, P, Hq, Hkv, qscale, part_o, part_ml, pair_cnt, out,
                  status);
}

}  // namespace

// Segment slots the partial buffers must hold.  Warp w writes at most
// ceil(L/T) + 1 segments with L <= P*T/W + CHP, so all warps together write
// at most P + 3W of them (W = SMs x 8 warps bounds every configuration).
size_t decode_attn_partial_slots(int B, int Hkv, int num_sms) {
  const size_t W = (size_t)num_sms * DA_MAX_WARPS;
  return (size_t)B * Hkv + 3 * W + 64;
}

cudaError_t launch_decode_attn(const float* q, const __half* kc, const __half* vc, int B, int Hq,
                               int Hkv, int hd, int Tmax, const int* d_pos, float* part_o,
                               float* part_ml, int* pair_cnt, __nv_bfloat16* out, int* status,
                               cudaStream_t st) {
  const float qscale = (1.0f / sqrtf((float)hd)) * 1.4426950408889634f;
  const int group = Hq / Hkv;
  if (hd == 128 && group == 2)
    return launch_t<128, 2>(q, kc, vc, B, Hq, Hkv, Tmax, d_pos, qscale, part_o, part_ml, pair_cnt, out, status, st);
  if (hd == 128 && group == 1)
    return launch_t<128, 1>(q, kc, vc, B, Hq, Hkv, Tmax, d_pos, qscale, part_o, part_ml, pair_cnt, out, status, st);
  if (hd == 64 && group == 1)
    return launch_t<64, 1>(q, kc, vc, B, Hq, Hkv, Tmax, d_pos, qscale, part_o, part_ml, pair_cnt, out, status, st);
  if (hd == 64 && group == 2)
    return launch_t<64, 2>(q, kc, vc, B, Hq, Hkv, Tmax, d_pos, qscale, part_o, part_ml, pair_cnt, out, status, st);
  return cudaErrorInvalidValue;
}

}  // namespace ne
