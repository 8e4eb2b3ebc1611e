// gemm.cu -- host side of the tcgen05 GEMM: TMA descriptors, tiling, dispatch.
#include <algorithm>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gemm_tc.cuh"
#include "ne_internal.h"
#include "ne_launch.cuh"

namespace ne {

namespace {

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

// 2-D K-major operand [rows, K] (leading dim ld elements), 128B-swizzled box
// of 64 x box_rows.
bool make_tmap(CUtensorMap* tm, const void* ptr, int rows, int K, long long ld, int box_rows,
               int fp16) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)GEMM_BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D MN-major operand: global [K rows, MN] (MN contiguous, leading dim ld),
// boxes of 64 (MN) x 64 (K rows), 128B-swizzled.
bool make_tmap_mn(CUtensorMap* tm, const void* ptr, int mn, int K, long long ld) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)mn, (cuuint64_t)K};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)GEMM_BK};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output of a staged epilogue: [rows, cols] row-major with leading dim ld
// elements, boxes of box_cols x 32 rows whose 32-, 64- or 128-byte rows use
// the matching swizzle (the kernel writes the box in that layout).
bool make_tmap_out(CUtensorMap* tm, void* ptr, int rows, int cols, long long ld,
                   CUtensorMapDataType dt, int elem_bytes, int box_cols) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const int row_bytes = box_cols * elem_bytes;
  if (row_bytes != 32 && row_bytes != 64 && row_bytes != 128) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * elem_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, dt, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   row_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                   : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                     : CU_TENSOR_MAP_SWIZZLE_32B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// A staged epilogue needs a 16-byte aligned output base and row pitch.
bool stage_ok(const void* out, long long ld, int elem_bytes) {
  return out && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && (ld * elem_bytes) % 16 == 0;
}

template <int BN, class Epi, int FMT, int AMN, int BMN, int CG = 1>
cudaError_t launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                     const CUtensorMap& td, const GemmShape& sh, const typename Epi::Params& p,
                     int grid, cudaStream_t st) {
  using C = GemmCfg<BN, CG>;
  constexpr int smem = EpiStage<Epi>::value ? C::SMEM_BYTES_STAGED : C::SMEM_BYTES;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, Epi, FMT, AMN, BMN, CG>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  if constexpr (CG == 2)
    return launch_k_cluster(gemm_tc_kernel<BN, Epi, FMT, AMN, BMN, CG>, dim3(grid),
                            dim3(GEMM_THREADS), (size_t)smem, st, 2u, ta, tb, tc, td, sh, p);
  return launch_k(gemm_tc_kernel<BN, Epi, FMT, AMN, BMN, CG>, dim3(grid), dim3(GEMM_THREADS),
                  (size_t)smem, st, ta, tb, tc, td, sh, p);
}

// Epilogue dispatch.  K-major x K-major serves every epilogue; the MN-major
// variants (training backward) instantiate only the epilogues they use.
template <int BN, int FMT, int AMN, int BMN, int CG = 1>
cudaError_t launch_epi(const GemmCall& c, const CUtensorMap& ta, const CUtensorMap& tb,
                       const GemmShape& sh, int grid, cudaStream_t st) {
  constexpr bool kk = (AMN == 0 && BMN == 0);
  constexpr bool tr_ok = CG == 1;   // transposed (swap-AB) epilogues: single-CTA tiles only
  constexpr bool kmn = (AMN == 0 && BMN == 1);
  constexpr bool ch32 = GemmCfg<BN>::CH == 32;
  CUtensorMap tc, td;
  std::memset(&tc, 0, sizeof(tc));   // direct-store epilogues ignore them
  std::memset(&td, 0, sizeof(td));
  switch (c.epi) {
    case EPI_F32T:
      if constexpr (kk && tr_ok) {
        EpiF32T::Params p{(float*)c.out, c.ld, c.split_stride};
        return launch_t<BN, EpiF32T, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    case EPI_F32T_ADD:
      if constexpr (kk && ch32 && tr_ok) {
        // out [N (batch) rows, M (features) columns], leading dim ld
        if (!stage_ok(c.out, c.ld, 4) ||
            !make_tmap_out(&tc, c.out, c.N, c.M, c.ld, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32))
          return cudaErrorInvalidValue;
        EpiF32TS::Params p{c.alpha};
        return launch_t<BN, EpiF32TS, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    case EPI_ARGMAX_T:
      if constexpr (kk && tr_ok && ch32) {
        EpiArgmaxT::Params p{(unsigned long long*)c.aux1};
        return launch_t<BN, EpiArgmaxT, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    case EPI_SWIGLU_T:
      if constexpr (kk && tr_ok && ch32) {
        EpiSwiGLUT::Params p{(__nv_bfloat16*)c.out, c.ld};
        return launch_t<BN, EpiSwiGLUT, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    case EPI_F32: {
      if constexpr (ch32) {
        if (sh.splits == 1 && stage_ok(c.out, c.ld, 4) &&
            make_tmap_out(&tc, c.out, c.M, c.N, c.ld, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32)) {
          EpiF32S::Params p{0};
          return launch_t<BN, EpiF32S, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
        }
      }
      EpiF32::Params p{(float*)c.out, c.ld, c.split_stride};
      return launch_t<BN, EpiF32, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
    }
    case EPI_BF16:
      if constexpr (kk || kmn) {
        if constexpr (ch32) {
          if (stage_ok(c.out, c.ld, 2) &&
              make_tmap_out(&tc, c.out, c.M, c.N, c.ld,
                            c.half_out ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 32)) {
            EpiBF16S::Params p{c.alpha, c.half_out};
            return launch_t<BN, EpiBF16S, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
          }
        }
        if constexpr (kk) {
          EpiBF16::Params p{c.out, c.ld, c.alpha, c.half_out};
          return launch_t<BN, EpiBF16, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
        }
      }
      break;
    case EPI_RESID: {
      if constexpr (ch32) {
        if (stage_ok(c.out, c.ld, 4) &&
            make_tmap_out(&tc, c.out, c.M, c.N, c.ld, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32)) {
          EpiResidS::Params p{c.alpha};
          return launch_t<BN, EpiResidS, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
        }
      }
      if constexpr (kk) {
        EpiResid::Params p{(float*)c.out, c.ld, c.alpha, c.atomic};
        return launch_t<BN, EpiResid, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    }
    case EPI_RESID_PEER: {
      if constexpr (AMN == 1 && BMN == 1 && ch32) {   // the dW products of the training backward
        const GemmPeerOut& po = *c.peer;
        EpiResidPeer::Params p;
        for (int r = 0; r < GEMM_PEER_MAX; ++r) p.dst[r] = r < po.world ? po.dst[r] : nullptr;
        for (int r = 0; r <= GEMM_PEER_MAX; ++r) p.bound[r] = r <= po.world ? po.bound[r] : 0;
        p.ld = c.ld;
        p.abort = po.abort;
        p.alpha = c.alpha;
        p.world = po.world;
        p.rank = po.rank;
        return launch_t<BN, EpiResidPeer, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    }
    case EPI_SWIGLU:
      if constexpr (kk && ch32) {
        // gate [M, N/2] bf16; optional h13 [M, N] bf16 (the raw projection)
        if (!make_tmap_out(&tc, c.out, c.M, c.N / 2, c.ld, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 16))
          return cudaErrorInvalidValue;
        if (c.aux1 && !make_tmap_out(&td, c.aux1, c.M, c.N, c.N, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                     2, 32))
          return cudaErrorInvalidValue;
        EpiSwiGLUS::Params p{c.aux1 != nullptr};
        return launch_t<BN, EpiSwiGLUS, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    case EPI_ADD:
      if constexpr (kk) {
        EpiAdd::Params p{(float*)c.out, (const float*)c.aux3, c.ld, c.alpha};
        return launch_t<BN, EpiAdd, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    case EPI_SWIGLU_BWD:
      if constexpr ((kk || kmn) && ch32) {
        // dh13 [M, 2F] bf16: the chunk of 32 features fills 64 columns
        if (!make_tmap_out(&tc, c.out, c.M, (int)(2 * c.aux_ld), 2 * c.aux_ld,
                           CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64))
          return cudaErrorInvalidValue;
        EpiSwiGLUBwdS::Params p{(const __nv_bfloat16*)c.aux3, c.aux_ld, c.alpha};
        return launch_t<BN, EpiSwiGLUBwdS, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    case EPI_F32_STATS:
      if constexpr (kk && ch32) {
        if (stage_ok(c.out, c.ld, 4) &&
            make_tmap_out(&tc, c.out, c.M, c.N, c.ld, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32)) {
          EpiF32StatsS::Params p{(float2*)c.aux1, c.aux_ld};
          return launch_t<BN, EpiF32StatsS, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
        }
        EpiF32Stats::Params p{(float*)c.out, c.ld, (float2*)c.aux1, c.aux_ld};
        return launch_t<BN, EpiF32Stats, FMT, AMN, BMN, CG>(ta, tb, tc, td, sh, p, grid, st);
      }
      break;
    default:
      break;
  }
  return cudaErrorInvalidValue;
}

int pick_bn(const GemmCall& c) {
  if (c.bn) return c.bn;
  if (c.N <= 16)
    return (c.epi == EPI_SWIGLU || c.epi == EPI_F32T_ADD || c.epi == EPI_ARGMAX_T ||
            c.epi == EPI_SWIGLU_T) ? 32 : 16;
  if (c.N <= 32) return 32;
  if (c.N <= 64) return 64;
  if (c.N <= 128) return 128;
  return 256;
}

}  // namespace

int device_num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// CTA pairs (cta_group::2, 256 x 256 tiles over two SMs) for the large
// token-major products; NE_GEMM_PAIR=0 keeps single-CTA tiles everywhere.
bool gemm_pair_tiles(const GemmCall& c) {
  static const bool pair_on = [] {
    const char* e = getenv("NE_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return pair_on && pick_bn(c) == 256 && (c.max_ctas <= 0 || c.max_ctas >= 2) && c.M >= 512 &&
         c.epi != EPI_F32T && c.epi != EPI_F32T_ADD && c.epi != EPI_ARGMAX_T &&
         c.epi != EPI_SWIGLU_T;
}

int gemm_pick_splits(const GemmCall& c, int num_sms) {
  if (c.splits > 0) return c.splits;
  if (c.epi == EPI_F32T_ADD) {
    // partial sums meet in L2 through the TMA add: split until the work
    // units fill the SMs, keeping at least two 64-deep k-blocks per unit
    static const int min_kb = [] {
      const char* e = getenv("NE_SPLITK_MIN_KB");   // tuning: k-blocks per split, at least
      const int v = e ? atoi(e) : 2;
      return v < 1 ? 1 : v;
    }();
    const int bn = pick_bn(c);
    const int tiles = ((c.M + GEMM_BM - 1) / GEMM_BM) * ((c.N + bn - 1) / bn);
    const int kb = c.K / GEMM_BK;
    int best = 1;
    for (int d = 1; d <= kb / min_kb; ++d) {
      if (kb % d) continue;
      if (tiles * d > num_sms) break;
      best = d;
    }
    return best;
  }
  if (c.epi != EPI_F32T && c.epi != EPI_F32) return 1;
  const int bn = pick_bn(c);
  const int tiles = ((c.M + GEMM_BM - 1) / GEMM_BM) * ((c.N + bn - 1) / bn);
  const int kb = c.K / GEMM_BK;
  // Split until the work units fill the SMs, but for wide N (large decode
  // batches) stop at half the SMs: each extra split adds a partial slab of
  // N x M fp32 that the consumer reads back (fitted to measured decode
  // shapes: N <= 128 favours ~148 units, N = 256 ~64-96).
  const int cap = c.N <= 128 ? num_sms : num_sms / 2;
  int best = 1;
  for (int d = 1; d <= kb; ++d) {
    if (kb % d) continue;
    if (kb / d < 1) break;
    if (tiles * d > cap) break;
    best = d;
  }
  return best;
}

cudaError_t gemm_run(const GemmCall& c, int* status, cudaStream_t st) {
  if (c.M <= 0 || c.N <= 0 || c.K <= 0 || c.K % GEMM_BK != 0) return cudaErrorInvalidValue;
  if ((c.lda * 2) % 16 != 0 || (c.ldb * 2) % 16 != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(c.A) & 15) || (reinterpret_cast<uintptr_t>(c.B) & 15))
    return cudaErrorInvalidValue;
  if (c.ab_fp16) return cudaErrorInvalidValue;   // bf16 operands only in this build
  if (c.a_mn && !c.b_mn) return cudaErrorInvalidValue;
  // the SwiGLU epilogues write TMA boxes: 16-byte aligned rows
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (c.epi == EPI_SWIGLU && (!a16(c.out) || c.ld % 8 || c.N % 32 || (c.aux1 && !a16(c.aux1))))
    return cudaErrorInvalidValue;
  if (c.epi == EPI_SWIGLU_BWD && (!a16(c.out) || !a16(c.aux3) || c.aux_ld % 8))
    return cudaErrorInvalidValue;
  if (c.epi == EPI_ARGMAX_T && (!c.aux1 || (reinterpret_cast<uintptr_t>(c.aux1) & 7u)))
    return cudaErrorInvalidValue;
  // the fused SwiGLU pairs rows 32c + i and 32c + 16 + i of one unsplit tile
  if (c.epi == EPI_SWIGLU_T && (c.M % 32 != 0 || !c.out || c.splits > 1)) return cudaErrorInvalidValue;
  if (c.epi == EPI_F32_STATS && (!c.aux1 || (reinterpret_cast<uintptr_t>(c.aux1) & 7u) ||
                                 c.aux_ld < (c.N + 31) / 32))
    return cudaErrorInvalidValue;
  if (c.epi == EPI_RESID_PEER &&
      (!c.peer || c.peer->world < 1 || c.peer->world > GEMM_PEER_MAX || c.ld % 64 != 0 ||
       c.peer->bound[c.peer->world] != (long long)c.M * c.ld))
    return cudaErrorInvalidValue;
  const int num_sms = device_num_sms();
  int bn = pick_bn(c);
  if (c.b_mn && bn < 64) bn = 64;
  const int splits = gemm_pick_splits(c, num_sms);
  const int kb = c.K / GEMM_BK;
  if (kb % splits != 0) return cudaErrorInvalidValue;
  if (splits > 1 && c.epi != EPI_F32T && c.epi != EPI_F32 && c.epi != EPI_F32T_ADD &&
      !(c.epi == EPI_RESID && c.atomic) && c.epi != EPI_RESID_PEER)
    return cudaErrorInvalidValue;

  const bool pair = gemm_pair_tiles(c) && bn == 256 && num_sms >= 2;
  const int tile_m = pair ? 2 * GEMM_BM : GEMM_BM;

  CUtensorMap ta, tb;
  const bool ok_a = c.a_mn ? make_tmap_mn(&ta, c.A, c.M, c.K, c.lda)
                           : make_tmap(&ta, c.A, c.M, c.K, c.lda, GEMM_BM, 0);
  // pair mode: each CTA loads half of B's rows per stage
  const bool ok_b = c.b_mn ? make_tmap_mn(&tb, c.B, c.N, c.K, c.ldb)
                           : make_tmap(&tb, c.B, c.N, c.K, c.ldb, pair ? bn / 2 : bn, 0);
  if (!ok_a || !ok_b) return cudaErrorInvalidValue;

  GemmShape sh;
  sh.M = c.M;
  sh.N = c.N;
  sh.K = c.K;
  sh.m_tiles = (c.M + tile_m - 1) / tile_m;
  sh.n_tiles = (c.N + bn - 1) / bn;
  sh.splits = splits;
  sh.kb_per_split = kb / splits;
  sh.status = status;
  sh.prefetch_a = c.prefetch_a;
  // Raster groups when A outgrows a share of L2: M-fastest order re-reads all
  // of A for every wave of n-tiles once A no longer stays resident, so the
  // units run in groups of m-tiles whose A panels total ~48 MB (the wave's B
  // panels take the rest of the 126 MB L2).  NE_GEMM_GROUP_MB overrides
  // (0 disables).
  {
    static const long long budget = [] {
      const char* e = std::getenv("NE_GEMM_GROUP_MB");
      return (e ? std::atoll(e) : 48LL) << 20;
    }();
    const long long a_panel = (long long)tile_m * c.K * 2;
    sh.group_m = 0;
    if (budget > 0 && sh.n_tiles > 1 && a_panel * sh.m_tiles > budget)
      sh.group_m = (int)std::max<long long>(1, budget / a_panel);
  }
  const long long units = (long long)sh.m_tiles * sh.n_tiles * splits;
  if (pair) {
    const int cap2 = (c.max_ctas > 0 ? c.max_ctas : num_sms) / 2;
    const long long clusters = units < cap2 ? units : cap2;
    const int grid2 = (int)(2 * clusters);
    if (!c.a_mn && !c.b_mn) return launch_epi<256, 1, 0, 0, 2>(c, ta, tb, sh, grid2, st);
    if (!c.a_mn) return launch_epi<256, 1, 0, 1, 2>(c, ta, tb, sh, grid2, st);
    return launch_epi<256, 1, 1, 1, 2>(c, ta, tb, sh, grid2, st);
  }
  const int cap = c.max_ctas > 0 ? c.max_ctas : num_sms;
  const int grid = (int)(units < cap ? units : cap);

  if (!c.a_mn && !c.b_mn) {
    switch (bn) {
      case 16: return launch_epi<16, 1, 0, 0>(c, ta, tb, sh, grid, st);
      case 32: return launch_epi<32, 1, 0, 0>(c, ta, tb, sh, grid, st);
      case 64: return launch_epi<64, 1, 0, 0>(c, ta, tb, sh, grid, st);
      case 128: return launch_epi<128, 1, 0, 0>(c, ta, tb, sh, grid, st);
      case 256: return launch_epi<256, 1, 0, 0>(c, ta, tb, sh, grid, st);
      default: return cudaErrorInvalidValue;
    }
  }
  if (!c.a_mn) {
    switch (bn) {
      case 64: return launch_epi<64, 1, 0, 1>(c, ta, tb, sh, grid, st);
      case 128: return launch_epi<128, 1, 0, 1>(c, ta, tb, sh, grid, st);
      case 256: return launch_epi<256, 1, 0, 1>(c, ta, tb, sh, grid, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (bn) {
    case 64: return launch_epi<64, 1, 1, 1>(c, ta, tb, sh, grid, st);
    case 128: return launch_epi<128, 1, 1, 1>(c, ta, tb, sh, grid, st);
    case 256: return launch_epi<256, 1, 1, 1>(c, ta, tb, sh, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ne
