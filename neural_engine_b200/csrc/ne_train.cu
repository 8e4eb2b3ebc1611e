// ne_train.cu -- the training step behind the C ABI (forward, backward, AdamW).
//
// Device counterpart of the reference's step loop (ane-training/training/
// training_dynamic/train.m:391-917): per-layer forward with saved activations
// (train.m:413-488), classifier + cross-entropy (:493-506), backward in
// reverse layer order (:508-757), then gradient unscale / global-norm clip /
// AdamW (:782-897).  Every dense contraction runs on the tcgen05 GEMM; the
// backward's transposed operands are read MN-major straight from the saved
// token-major activations, so nothing is transposed in memory.
//
// Buffers (M = B*S tokens): fp32 masters, gradients, Adam m and v for every
// trainable tensor in the device layout (Wqkv rows Wq|Wk|Wv, W13 rows
// interleaved in 16-row blocks); per-layer saved activations
//   X[l] fp32 [M,D] (layer input), XN[l] bf16, QKVR[l] fp32 [M,qkv],
//   Q/K/V[l] bf16 (post QK-norm + RoPE), O[l] bf16, LSE[l] fp32 [B,Hq,S],
//   X2[l] fp32, X2N[l] bf16, H13[l] bf16 [M,2F] (raw W1/W3 projection), GATE[l] bf16 [M,F]
// and backward scratch.  The tied embedding's gradient collects the LM-head
// part (dense GEMM) and the gather's scatter-add.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/ne.h"
#include "ne_ckpt.h"
#include "ne_comm.h"
#include "ne_ctx.h"
#include "ne_internal.h"
#include "ne_fault.h"

namespace ne {

// One trainable tensor: fp32 master w (device), its gradient / Adam state,
// optional bf16 compute copy, element count and weight decay.
struct Seg {
  float* w;
  float* g;
  float* m;
  float* v;
  __nv_bfloat16* w16;
  long long n;
  float wd;
};

struct TrainLayerP {
  int seg0;                      // index of this layer's first segment in TrainState::segs
  float *wqkv, *wo, *w13, *w2;   // fp32 masters (device layout)
  float *gqkv, *go, *g13, *g2;   // gradients
  float *g_att, *g_ffn, *g_qn, *g_kn;
};

struct TrainActs {
  float *X, *QKVR, *LSE, *X2;
  __nv_bfloat16 *XN, *Q, *K, *V, *O, *X2N, *H13, *GATE;
};

struct TrainState {
  int B = 0, S = 0, M = 0, Mc = 0;
  float* pool = nullptr;                 // masters + grads + m + v (fp32)
  size_t pool_floats = 0;
  void* act_pool = nullptr;              // saved activations + scratch
  size_t act_bytes = 0;
  std::vector<Seg> segs;
  AdamSeg* d_segs = nullptr;             // device copy of the segment table
  float d_segs_wd = -2.f;                // weight decay the device table holds
  OptChunk* d_chunks = nullptr;          // optimizer work list (chunks of OPT_CHUNK elements)
  int nchunks = 0;
  float* opt_partial = nullptr;          // [nchunks] per-chunk sums of squares
  unsigned* opt_ticket = nullptr;        // last-block ticket of the norm kernel
  float* norm_out = nullptr;             // [0] pre-clip norm, [1] gradient factor, [2] sum of squares
  bool state_gathered = true;            // sharded mode: masters / moments whole on every rank
  float* grad_pool = nullptr;            // start of the gradients inside `pool`
  size_t grad_floats = 0;
  size_t layer_grad_floats = 0;          // one layer's gradients (contiguous, layer order)
  size_t tail_grad_off = 0;              // rms_final + embedding gradients follow the layers
  std::vector<TrainLayerP> P;
  float *embed_w = nullptr, *embed_g = nullptr, *rmsf_g = nullptr;
  std::vector<TrainActs> A;
  float* XL = nullptr;                   // final residual [M, D]
  __nv_bfloat16* XNF = nullptr;          // final normed [M, D]
  // backward scratch
  float *dY = nullptr, *dXF = nullptr, *dX2 = nullptr, *Dl = nullptr, *logits = nullptr,
        *loss_rows = nullptr;
  __nv_bfloat16 *dY16 = nullptr, *dX216 = nullptr, *DH13 = nullptr, *dO = nullptr,
                *DQKV = nullptr, *dlogits = nullptr;
  float2* ce_stats = nullptr;            // [Mc, ceil(V/32)] classifier softmax statistics
  // vocabulary compaction (the reference's classifier over the tokens present
  // in the data): CV classifier rows, padded to CVp (a multiple of 64)
  int CV = 0, CVp = 0;
  int32_t* d_c2f = nullptr;              // [CV] compact -> full id
  int32_t* d_f2c = nullptr;              // [V] full -> compact id (-1: absent)
  __nv_bfloat16* Ec = nullptr;           // [CVp, D] gathered classifier rows (bf16)
  float* dEc = nullptr;                  // [CVp, D] their gradient (scattered into embed_g)
  void* embed_scratch = nullptr;         // sort buffers of the embedding backward
  size_t embed_scratch_bytes = 0;
  // the micro-step after the token split, captured once as a CUDA graph
  // captured micro-steps: [0] without the gradient exchange, [1] with it,
  // [2] with it and the dW products added into their owners (fused exchange)
  cudaGraphExec_t step_graphs[3] = {nullptr, nullptr, nullptr};
  const void* step_graph_rope[3] = {nullptr, nullptr, nullptr};   // RoPE table each was captured with
  long long steps_run = 0;                // micro-steps so far (the first runs eagerly)
  int32_t *ids = nullptr, *tgt = nullptr, *tok = nullptr;
  double* red = nullptr;                 // [2] sum of squares / loss sum
  int micro_steps = 0;                   // fwd_bwd calls since the last optimizer step
  std::vector<cudaEvent_t> phase_ev;     // ne_train_fwd_bwd_timed: one event per phase boundary
  // page-locked staging of the host-buffer calls: the tokens of one batch,
  // then the loss (the copies run from / into it, never from caller memory)
  uint8_t* h_stage = nullptr;
  size_t h_stage_tok = 0;                // bytes of the token part
  float* range_out = nullptr;            // ne_train_value_ranges: [4]
};

// Drops the captured training step (it may hold NCCL calls of a communicator
// about to change, or the exchange may have been switched on or off) and the
// optimizer work list (whose chunks depend on this rank's share).
void train_drop_step_graph(ne_ctx* ctx) {
  if (!ctx || !ctx->train) return;
  TrainState* t = ctx->train;
  cudaStreamSynchronize(ctx->st);
  for (cudaGraphExec_t& g : t->step_graphs) {
    if (g) cudaGraphExecDestroy(g);
    g = nullptr;
  }
  if (t->d_chunks) cudaFree(t->d_chunks);
  if (t->opt_partial) cudaFree(t->opt_partial);
  t->d_chunks = nullptr;
  t->opt_partial = nullptr;
}

void free_train(ne_ctx* ctx) {
  if (!ctx || !ctx->train) return;
  TrainState* t = ctx->train;
  if (ctx->comm) {
    // the peer mappings and chunk lists describe these pools
    cudaStreamSynchronize(ctx->st);
    if (ctx->comm->cs) cudaStreamSynchronize(ctx->comm->cs);
    px_free(ctx);
  }
  if (t->d_segs) cudaFree(t->d_segs);
  if (t->d_chunks) cudaFree(t->d_chunks);
  if (t->embed_scratch) cudaFree(t->embed_scratch);
  for (cudaGraphExec_t g : t->step_graphs)
    if (g) cudaGraphExecDestroy(g);
  for (void* p : {(void*)t->d_c2f, (void*)t->d_f2c, (void*)t->Ec, (void*)t->dEc})
    if (p) cudaFree(p);
  if (t->opt_partial) cudaFree(t->opt_partial);
  for (cudaEvent_t e : t->phase_ev)
    if (e) cudaEventDestroy(e);
  if (t->range_out) cudaFree(t->range_out);
  if (t->h_stage) cudaFreeHost(t->h_stage);
  if (t->opt_ticket) cudaFree(t->opt_ticket);
  if (t->norm_out) cudaFree(t->norm_out);
  if (t->pool) cudaFree(t->pool);
  if (t->act_pool) cudaFree(t->act_pool);
  delete t;
  ctx->train = nullptr;
}

}  // namespace ne

using namespace ne;

namespace {

__global__ void split_tokens_kernel(const int32_t* __restrict__ tok, int B, int S,
                                    int32_t* __restrict__ ids, int32_t* __restrict__ tgt) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B * S) return;
  const int b = r / S, s = r % S;
  ids[r] = tok[(size_t)b * (S + 1) + s];
  tgt[r] = tok[(size_t)b * (S + 1) + s + 1];
}

__global__ void sum_rows_kernel(const float* __restrict__ x, int n, double* __restrict__ out) {
  double acc = 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    acc += (double)x[i];
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(out, acc);
}

__global__ void mean_from_sum_kernel(const double* s, int n, float* out) { *out = (float)(*s / n); }

__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ a, float* __restrict__ b,
                                   long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    b[i] = __bfloat162float(a[i]);
}

// dst[r, :] = interleave of (W1 row r, W3 row r) blocks: the W13 device layout.
size_t w13_row(size_t f, bool is_w3) { return (f / 16) * 32 + (is_w3 ? 16 : 0) + f % 16; }

// Wave efficiency units / (SMs * ceil(units / SMs)) of a tiling.
double wave_eff(long long units, int sms) {
  return (double)units / ((double)sms * ((units + sms - 1) / sms));
}

// Gradient GEMMs (weight-shaped output, K = tokens) accumulate through the
// epilogue's TMA add, which is atomic per element in L2, so they may split K
// freely: take the 256-wide N tile and the split (at most 4, dividing the
// k-blocks) whose work units fill the SMs best.
int dw_splits(const GemmCall& c, int sms) {
  // products with M >= 512 run as CTA pairs (256-row tiles, one slot per two SMs)
  const bool pair = gemm_pair_tiles(c);
  const int bm = pair ? 256 : 128;
  if (pair) sms /= 2;
  const long long tiles = (long long)((c.M + bm - 1) / bm) * ((c.N + 255) / 256);
  const int kb = c.K / 64;
  int best = 1;
  double best_eff = wave_eff(tiles, sms);
  for (int s = 2; s <= 4; ++s) {
    if (kb % s || kb / s < 4) continue;
    const double e = wave_eff(tiles * s, sms);
    if (e > best_eff + 0.03) {
      best = s;
      best_eff = e;
    }
  }
  return best;
}

// With data-parallel reduction on, the GEMMs leave NE_COMM_SMS SMs (default
// 0) to the NCCL kernels of the gradient buckets, which otherwise find every
// SM held by a persistent GEMM and run only between launches.
int comm_reserved_sms() {
  static const int r = [] {
    const char* e = std::getenv("NE_COMM_SMS");
    const int v = e ? std::atoi(e) : 0;
    return v < 0 ? 0 : (v > 64 ? 64 : v);
  }();
  return r;
}

// Split-K of the fused dW products (NE_PX_FUSED_SPLITS): 1 (default) adds
// each output element into its owner once; 0 lets the dW heuristic split K,
// every split then sending its own partial sums over NVLink.
int peer_dw_splits() {
  static const int v = [] {
    const char* e = std::getenv("NE_PX_FUSED_SPLITS");
    return e && e[0] == '0' ? 0 : 1;
  }();
  return v;
}

ne_status gemm(ne_ctx* ctx, GemmCall c) {
  c.splits = 1;
  if (ctx->comm && ctx->comm->world > 1 && ctx->comm->reduce && comm_reserved_sms() > 0)
    c.max_ctas = ctx->num_sms - comm_reserved_sms();
  if ((c.epi == EPI_RESID || c.epi == EPI_RESID_PEER) && c.a_mn && c.b_mn) {
    c.bn = 256;
    c.splits = c.epi == EPI_RESID_PEER && peer_dw_splits() == 1 ? 1 : dw_splits(c, ctx->num_sms);
    c.atomic = 1;
  }
  cudaError_t e = gemm_run(c, ctx->d_status, ctx->st);
  if (e != cudaSuccess) return fail(ctx, NE_ERR_CUDA, std::string("gemm: ") + cudaGetErrorString(e));
  ctx->launches++;
  return NE_OK;
}

// C = op(A . B^T) with A [M,K] / B [N,K] K-major (or MN-major when flagged).
GemmCall gc(const void* A, long long lda, int M, int a_mn, const void* B, long long ldb, int N,
            int b_mn, int K, int epi, void* out, long long ld, float alpha = 1.f) {
  GemmCall c;
  c.A = A; c.lda = lda; c.M = M; c.a_mn = a_mn;
  c.B = B; c.ldb = ldb; c.N = N; c.b_mn = b_mn;
  c.K = K; c.epi = epi; c.out = out; c.ld = ld; c.alpha = alpha;
  c.bn = 256;
  return c;
}

}  // namespace

extern "C" {

NE_API ne_status ne_train_alloc(ne_ctx* ctx, int B, int S) {
  if (!ctx || B <= 0 || S <= 0) return NE_ERR_INVALID;
  const ne_model_cfg& m = ctx->cfg;
  const long long M = (long long)B * S;
  if (M % 64 != 0) return fail(ctx, NE_ERR_UNSUPPORTED, "B*S must be a multiple of 64");
  if (m.vocab % 64 != 0) return fail(ctx, NE_ERR_UNSUPPORTED, "vocab must be a multiple of 64");
  if (ctx->layer_set_count != (unsigned)m.n_layers || !ctx->global_set)
    return fail(ctx, NE_ERR_STATE, "set the weights before ne_train_alloc");
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  if (!ctx->rope_cs || ctx->max_seq < S) {
    // RoPE table (and decode workspace) sized for S
    ne_status s = ne_kv_alloc(ctx, 1, std::max(S, ctx->max_seq));
    if (s != NE_OK) return s;
  }
  free_train(ctx);
  TrainState* t = new TrainState();
  ctx->train = t;
  t->B = B;
  t->S = S;
  t->M = (int)M;
  // classifier rows per chunk: fp32 logits + bf16 dlogits + statistics of one
  // chunk stay within 4 GB (multiples of 128 rows, at least 128)
  {
    const long long per_row = (long long)m.vocab * 6 + ((m.vocab + 31) / 32) * 8;
    long long mc = (4LL << 30) / per_row;
    mc = std::max<long long>(128, mc / 128 * 128);
    t->Mc = (int)std::min<long long>(M, mc);
  }
  const size_t D = m.dim, F = m.hidden, qd = (size_t)m.n_heads * m.head_dim,
               kvd = (size_t)m.kv_heads * m.head_dim, qkv = qd + 2 * kvd, V = m.vocab,
               hd = m.head_dim, L = m.n_layers;
  auto rnd = [](size_t n) { return (n + 63) & ~(size_t)63; };
  // ---- parameter pool: masters for matrices + embed, grads / m / v for all
  const size_t per_layer_w = rnd(qkv * D) + rnd(D * qd) + rnd(2 * F * D) + rnd(D * F);
  const size_t per_layer_all = per_layer_w + 2 * rnd(D) + 2 * rnd(hd);
  const size_t total_w = L * per_layer_w + rnd(V * D);                     // masters
  const size_t total_all = L * per_layer_all + rnd(D) + rnd(V * D);        // grads/m/v
  t->pool_floats = total_w + 3 * total_all;
  ne_status s;
  if ((s = dalloc(ctx, &t->pool, t->pool_floats)) != NE_OK) return s;
  NE_CUDA(cudaMemsetAsync(t->pool, 0, t->pool_floats * 4, ctx->st));
  float* pw = t->pool;
  float* pg = t->pool + total_w;
  t->grad_pool = pg;
  t->grad_floats = total_all;
  t->layer_grad_floats = per_layer_all;
  t->tail_grad_off = L * per_layer_all;
  float* pm = pg + total_all;
  float* pv = pm + total_all;
  size_t ow = 0, oa = 0;
  auto seg = [&](float* master, __nv_bfloat16* w16, size_t n, float wd) -> Seg {
    Seg sg;
    if (master == nullptr) {
      sg.w = pw + ow;
      ow += rnd(n);
    } else {
      sg.w = master;
    }
    sg.g = pg + oa;
    sg.m = pm + oa;
    sg.v = pv + oa;
    oa += rnd(n);
    sg.w16 = w16;
    sg.n = (long long)n;
    sg.wd = wd;
    return sg;
  };
  // weight decay: matrices and the embedding, not the gains (train.m:863-871, 896-897)
  const float WD = -1.0f;   // placeholder: the configured decay is applied at step time
  t->P.resize(L);
  for (size_t l = 0; l < L; ++l) {
    LayerW& w = ctx->L[l];
    TrainLayerP& p = t->P[l];
    p.seg0 = (int)t->segs.size();
    Seg a = seg(nullptr, w.wqkv, qkv * D, WD);
    Seg b = seg(nullptr, w.wo, D * qd, WD);
    Seg c = seg(nullptr, w.w13, 2 * F * D, WD);
    Seg d = seg(nullptr, w.w2, D * F, WD);
    Seg e = seg(w.rms_att, nullptr, D, 0.f);
    Seg f = seg(w.rms_ffn, nullptr, D, 0.f);
    p.wqkv = a.w; p.gqkv = a.g; p.wo = b.w; p.go = b.g; p.w13 = c.w; p.g13 = c.g;
    p.w2 = d.w; p.g2 = d.g; p.g_att = e.g; p.g_ffn = f.g;
    t->segs.insert(t->segs.end(), {a, b, c, d, e, f});
    if (m.qk_norm) {
      Seg q = seg(w.q_norm, nullptr, hd, 0.f);
      Seg k = seg(w.k_norm, nullptr, hd, 0.f);
      p.g_qn = q.g;
      p.g_kn = k.g;
      t->segs.insert(t->segs.end(), {q, k});
    } else {
      oa += 2 * rnd(hd);
      p.g_qn = p.g_kn = nullptr;
    }
  }
  Seg rf = seg(ctx->rms_final, nullptr, D, 0.f);
  Seg em = seg(nullptr, ctx->embed, V * D, WD);
  t->rmsf_g = rf.g;
  t->embed_w = em.w;
  t->embed_g = em.g;
  t->segs.push_back(rf);
  t->segs.push_back(em);
  // The fp32 masters start as the bf16 compute copies widened (exact when the
  // host weights were bf16-valued); ne_train_set_masters() loads full fp32
  // values instead.  Gains are their own masters.
  for (const Seg& sg : t->segs) {
    if (sg.w16 == nullptr) continue;
    const long long n = sg.n;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148 * 8);
    bf16_to_f32_kernel<<<blocks, 256, 0, ctx->st>>>(sg.w16, sg.w, n);
    NE_CUDA(cudaGetLastError());
  }
  // ---- activations
  const size_t Mx = (size_t)M;
  size_t bytes = 0;
  auto take = [&](size_t nbytes) {
    const size_t o = bytes;
    bytes += (nbytes + 255) & ~(size_t)255;
    return o;
  };
  struct Off {
    size_t X, QKVR, LSE, X2, XN, Q, K, V, O, X2N, H13, GATE;
  };
  std::vector<Off> off(L);
  for (size_t l = 0; l < L; ++l) {
    Off& o = off[l];
    o.X = take(Mx * D * 4); o.QKVR = take(Mx * qkv * 4); o.LSE = take(Mx * m.n_heads * 4);
    o.X2 = take(Mx * D * 4); o.XN = take(Mx * D * 2); o.Q = take(Mx * qd * 2);
    o.K = take(Mx * kvd * 2); o.V = take(Mx * kvd * 2); o.O = take(Mx * qd * 2);
    o.X2N = take(Mx * D * 2); o.H13 = take(Mx * 2 * F * 2);
    o.GATE = take(Mx * F * 2);
  }
  const size_t oXL = take(Mx * D * 4), oXNF = take(Mx * D * 2);
  const size_t odY = take(Mx * D * 4), odXF = take(Mx * D * 4), odX2 = take(Mx * D * 4);
  const size_t oDl = take(Mx * m.n_heads * 4), ologits = take((size_t)t->Mc * V * 4);
  const size_t oloss = take(Mx * 4), odY16 = take(Mx * D * 2), odX216 = take(Mx * D * 2);
  const size_t oDH13 = take(Mx * 2 * F * 2), odO = take(Mx * qd * 2), oDQKV = take(Mx * qkv * 2);
  const size_t odl = take((size_t)t->Mc * V * 2), oids = take(Mx * 4), otgt = take(Mx * 4);
  const size_t ostats = take((size_t)t->Mc * ((V + 31) / 32) * 8);
  const size_t otok = take((size_t)B * (S + 1) * 4), ored = take(64);
  uint8_t* base = nullptr;
  if ((s = dalloc(ctx, &base, bytes)) != NE_OK) return s;
  t->act_pool = base;
  t->act_bytes = bytes;
  t->A.resize(L);
  for (size_t l = 0; l < L; ++l) {
    TrainActs& a = t->A[l];
    const Off& o = off[l];
    a.X = (float*)(base + o.X); a.QKVR = (float*)(base + o.QKVR); a.LSE = (float*)(base + o.LSE);
    a.X2 = (float*)(base + o.X2); a.XN = (__nv_bfloat16*)(base + o.XN);
    a.Q = (__nv_bfloat16*)(base + o.Q); a.K = (__nv_bfloat16*)(base + o.K);
    a.V = (__nv_bfloat16*)(base + o.V); a.O = (__nv_bfloat16*)(base + o.O);
    a.X2N = (__nv_bfloat16*)(base + o.X2N); a.H13 = (__nv_bfloat16*)(base + o.H13);
    a.GATE = (__nv_bfloat16*)(base + o.GATE);
  }
  t->XL = (float*)(base + oXL); t->XNF = (__nv_bfloat16*)(base + oXNF);
  t->dY = (float*)(base + odY); t->dXF = (float*)(base + odXF); t->dX2 = (float*)(base + odX2);
  t->Dl = (float*)(base + oDl); t->logits = (float*)(base + ologits);
  t->loss_rows = (float*)(base + oloss); t->dY16 = (__nv_bfloat16*)(base + odY16);
  t->dX216 = (__nv_bfloat16*)(base + odX216); t->DH13 = (__nv_bfloat16*)(base + oDH13);
  t->dO = (__nv_bfloat16*)(base + odO); t->DQKV = (__nv_bfloat16*)(base + oDQKV);
  t->dlogits = (__nv_bfloat16*)(base + odl); t->ids = (int32_t*)(base + oids);
  t->ce_stats = (float2*)(base + ostats);
  t->tgt = (int32_t*)(base + otgt); t->tok = (int32_t*)(base + otok);
  t->red = (double*)(base + ored);
  // sort buffers of the local embedding backward (allocated here so that the
  // step can be captured in a graph)
  t->embed_scratch_bytes = embed_bwd_scratch_bytes(t->M);
  {
    uint8_t* p = nullptr;
    if ((s = dalloc(ctx, &p, t->embed_scratch_bytes)) != NE_OK) return s;
    t->embed_scratch = p;
  }
  t->h_stage_tok = ((size_t)B * (S + 1) * 4 + 255) & ~(size_t)255;
  if (cudaHostAlloc(reinterpret_cast<void**>(&t->h_stage), t->h_stage_tok + 256,
                    cudaHostAllocDefault) != cudaSuccess) {
    t->h_stage = nullptr;
    return fail(ctx, NE_ERR_OOM, "cudaHostAlloc: token staging");
  }
  return ne_sync(ctx);
}

// Overwrite the fp32 masters from host fp32 tensors (v4 layout), e.g. a
// checkpoint's exact values; also refreshes the bf16 compute copies.
NE_API ne_status ne_train_set_masters(ne_ctx* ctx, int layer, const float* h_wq, const float* h_wk,
                                      const float* h_wv, const float* h_wo, const float* h_w1,
                                      const float* h_w2, const float* h_w3) {
  if (!ctx || !ctx->train) return NE_ERR_STATE;
  const ne_model_cfg& m = ctx->cfg;
  TrainState* t = ctx->train;
  if (layer < -1 || layer >= m.n_layers) return NE_ERR_INVALID;
  NE_CUDA(cudaSetDevice(ctx->device));
  const size_t D = m.dim, F = m.hidden, qd = (size_t)m.n_heads * m.head_dim,
               kvd = (size_t)m.kv_heads * m.head_dim;
  if (layer == -1) {   // h_wq = embedding [V, D]
    NE_CUDA(cudaMemcpy(t->embed_w, h_wq, (size_t)m.vocab * D * 4, cudaMemcpyHostToDevice));
    NE_CUDA(cudaStreamSynchronize(ctx->st));
    return NE_OK;
  }
  TrainLayerP& p = t->P[layer];
  NE_CUDA(cudaMemcpy(p.wqkv, h_wq, qd * D * 4, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(p.wqkv + qd * D, h_wk, kvd * D * 4, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(p.wqkv + (qd + kvd) * D, h_wv, kvd * D * 4, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(p.wo, h_wo, D * qd * 4, cudaMemcpyHostToDevice));
  std::vector<float> w13(2 * F * D);
  for (size_t f = 0; f < F; ++f) {
    std::memcpy(&w13[w13_row(f, false) * D], h_w1 + f * D, D * 4);
    std::memcpy(&w13[w13_row(f, true) * D], h_w3 + f * D, D * 4);
  }
  NE_CUDA(cudaMemcpy(p.w13, w13.data(), 2 * F * D * 4, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(p.w2, h_w2, D * F * 4, cudaMemcpyHostToDevice));
  return NE_OK;
}

// Refresh every bf16 compute copy from the fp32 masters.
NE_API ne_status ne_train_sync_weights(ne_ctx* ctx) {
  if (!ctx || !ctx->train) return NE_ERR_STATE;
  if (ctx->comm && ctx->comm->cs) {   // after any weight all-gather still in flight
    ne_status s = comm_fence_out(ctx);
    if (s != NE_OK) return s;
  }
  for (const Seg& sg : ctx->train->segs)
    if (sg.w16) NE_LAUNCH(launch_f32_to_bf16(sg.w, sg.w16, sg.n, ctx->st));
  return ne_sync(ctx);
}

NE_API ne_status ne_gemm_dw_owned(ne_ctx* ctx, const void* d_A, long long lda, int M,
                                  const void* d_B, long long ldb, int N, int K, float alpha,
                                  float* const* h_dst, const long long* h_bound, int world,
                                  int rank, long long ld) {
  if (!ctx || !d_A || !d_B || !h_dst || !h_bound || M <= 0 || N <= 0 || K <= 0 || world < 1 ||
      world > GEMM_PEER_MAX || rank < 0 || rank >= world || lda < M || ldb < N)
    return NE_ERR_INVALID;
  if (K % 64 || ld % 64 || ld < N)
    return fail(ctx, NE_ERR_UNSUPPORTED, "K and ld must be multiples of 64, ld >= N");
  GemmPeerOut po;
  po.world = world;
  po.rank = rank;
  for (int q = 0; q <= world; ++q) {
    po.bound[q] = h_bound[q];
    if (h_bound[q] % 64 || (q > 0 && h_bound[q] < h_bound[q - 1]))
      return fail(ctx, NE_ERR_INVALID, "part boundaries: non-decreasing multiples of 64");
  }
  if (h_bound[0] != 0 || h_bound[world] != (long long)M * ld)
    return fail(ctx, NE_ERR_INVALID, "part boundaries must span [0, M*ld]");
  for (int q = 0; q < world; ++q) {
    if (!h_dst[q] || (reinterpret_cast<uintptr_t>(h_dst[q]) & 15u))
      return fail(ctx, NE_ERR_INVALID, "each copy: non-NULL and 16-byte aligned");
    po.dst[q] = h_dst[q];
  }
  NE_CUDA(cudaSetDevice(ctx->device));
  GemmCall c = gc(d_A, lda, M, 1, d_B, ldb, N, 1, K, EPI_RESID_PEER, h_dst[rank], ld, alpha);
  c.peer = &po;
  return gemm(ctx, c);
}

NE_API ne_status ne_train_zero_grads(ne_ctx* ctx) {
  if (!ctx || !ctx->train) return NE_ERR_STATE;
  TrainState* t = ctx->train;
  if (ctx->comm && ctx->comm->px && ctx->comm->pxs.ready && ctx->comm->pxs.fused) {
    // fused dW exchange: this rank's owned parts of the layer matrices take
    // the other ranks' dW products once it has published PX_ZEROED for their
    // next exchange; after that only the rest may be cleared here
    PxState& x = ctx->comm->pxs;
    if (x.owned_clean) {
      NE_CUDA(px_zero(t->grad_pool, x.d_chunks + x.zr_first, x.zr_count, ctx->st));
    } else {
      NE_CUDA(cudaMemsetAsync(t->grad_pool, 0, t->grad_floats * 4, ctx->st));
      NE_CUDA(px_signal_next(x.flags, PX_ZEROED, ctx->st));
      x.owned_clean = true;
    }
  } else {
    NE_CUDA(cudaMemsetAsync(t->grad_pool, 0, t->grad_floats * 4, ctx->st));
  }
  t->micro_steps = 0;
  return NE_OK;
}

// ---------------------------------------------------------------------------
// Data-parallel hooks (active once ne_comm_init made a communicator of more
// than one rank and ne_comm_set_reduce left reduction on).  Buckets follow the
// backward: the tied-embedding + final-norm gradients right after the
// classifier, then each layer's contiguous gradient slice as soon as its
// attention backward finished, all on the comm stream while the compute
// stream carries on with the layers below.
static bool comm_active(const ne_ctx* ctx) {
  return ctx->comm && ctx->comm->world > 1 && ctx->comm->reduce;
}

// ZeRO-1 (ne_comm_set_sharding): rank r owns part r of the training state.
// Over peer memory (the default) every tensor is owned in parts with
// boundaries at multiples of 64 elements (px_part), gains included.  Over NCCL
// (NE_COMM_PX=0) a matrix segment (or the embedding) whose size splits into
// world equal parts of a multiple of 4 elements is owned in parts and the
// gains stay replicated.  Rank r reduces, updates and keeps current its parts;
// the updated compute copies are all-gathered after the optimizer step.
static bool shard_mode(const ne_ctx* ctx) {   // ownership (optimizer), whatever the reduction
  return ctx->comm && ctx->comm->world > 1 && ctx->comm->shard;
}
static bool shard_active(const ne_ctx* ctx) {   // the buckets reduce-scatter
  return comm_active(ctx) && ctx->comm->shard;
}
static bool px_active(const ne_ctx* ctx) { return shard_active(ctx) && ctx->comm->px; }

// The part [*off, *off + *len) of segment sg that `rank` owns; false (the
// whole segment) when the segment is replicated.
static bool seg_owned(const ne_ctx* ctx, const Seg& sg, int rank, long long* off,
                      long long* len) {
  if (shard_mode(ctx)) {
    const int W = ctx->comm->world;
    if (ctx->comm->px) {
      px_part(sg.n, W, rank, off, len);
      return true;
    }
    if (sg.w16 != nullptr && sg.n % W == 0 && (sg.n / W) % 4 == 0) {
      *len = sg.n / W;
      *off = *len * rank;
      return true;
    }
  }
  *off = 0;
  *len = sg.n;
  return false;
}
static bool seg_sharded(const ne_ctx* ctx, const Seg& sg) {
  long long o, n;
  return seg_owned(ctx, sg, 0, &o, &n);
}
static long long shard_len(const ne_ctx* ctx, const Seg& sg) {
  long long o, n;
  seg_owned(ctx, sg, ctx->comm->rank, &o, &n);
  return n;
}
static long long shard_off(const ne_ctx* ctx, const Seg& sg) {
  long long o, n;
  seg_owned(ctx, sg, ctx->comm->rank, &o, &n);
  return o;
}

// Segments [s0, s1) of exchange bucket b: 0 = tail (final norm + embedding),
// 1 + l = layer l.
static void bucket_segs(const TrainState* t, int b, int* s0, int* s1) {
  const int tail0 = (int)t->segs.size() - 2;
  if (b == 0) {
    *s0 = tail0;
    *s1 = (int)t->segs.size();
    return;
  }
  const int l = b - 1;
  *s0 = t->P[l].seg0;
  *s1 = l + 1 < (int)t->P.size() ? t->P[l + 1].seg0 : tail0;
}

// Fused dW exchange over peer memory (NE_PX_FUSED_DW=1): the layer
// matrices' dW products are added into their owners' parts by the GEMM
// epilogue (fp32 red.add over NVLink) instead of being reduce-scattered
// after each layer.  The sum's order then varies between runs (the adds
// land in arrival order).  Off by default: at 2 ranks the step measured
// slower than the rank-ordered reduce-scatter kernels, which stay the
// default.
static bool px_fused_dw() {
  static const bool on = [] {
    const char* e = std::getenv("NE_PX_FUSED_DW");
    return e && e[0] == '1';
  }();
  return on;
}

// Map the other ranks' pools and build the chunk lists of the peer-memory
// exchange.  Collective (every rank, outside any stream capture): the IPC
// handles travel in one NCCL all-gather.
static ne_status px_setup(ne_ctx* ctx) {
  TrainState* t = ctx->train;
  Comm* c = ctx->comm;
  PxState& x = c->pxs;
  const int W = c->world, R = c->rank;
  if (W > PX_MAX_WORLD)
    return fail(ctx, NE_ERR_UNSUPPORTED, "peer-memory exchange: at most 8 ranks (NE_COMM_PX=0)");
  const int L = ctx->cfg.n_layers;
  ne_status s;
  if ((s = dalloc(ctx, &x.flags, 256)) != NE_OK) return s;
  NE_CUDA(cudaMemset(x.flags, 0, 256 * sizeof(uint32_t)));
  {
    // the gradients are zero at the first exchange (the pool starts zeroed
    // and every path that writes it runs a micro-step): open for epoch 1
    const uint32_t one = 1u;
    NE_CUDA(cudaMemcpy(x.flags + PX_ZEROED, &one, sizeof(one), cudaMemcpyHostToDevice));
  }
  // the (token id, dY row) gather buffer: [world][M] ids, then [world][M][D] rows
  const int M = t->M, D = ctx->cfg.dim;
  const size_t ids_bytes = ((size_t)W * M * 4 + 255) & ~(size_t)255;
  const size_t need = ids_bytes + (size_t)W * M * D * 4;
  if (c->gather_bytes < need) {
    if (c->gather) NE_CUDA(cudaFree(c->gather));
    c->gather = nullptr;
    c->gather_bytes = 0;
    uint8_t* g = nullptr;
    if ((s = dalloc(ctx, &g, need)) != NE_OK) return s;
    c->gather = g;
    c->gather_bytes = need;
  }
  struct Rec {
    cudaIpcMemHandle_t h[4];   // training pool, weight pool, activation pool, flags
    long long pool_floats, act_bytes;
    int M, L;
  };
  Rec mine{};
  void* bases[4] = {t->pool, ctx->wpool, t->act_pool, x.flags};
  for (int i = 0; i < 4; ++i) NE_CUDA(cudaIpcGetMemHandle(&mine.h[i], bases[i]));
  mine.pool_floats = (long long)t->pool_floats;
  mine.act_bytes = (long long)t->act_bytes;
  mine.M = M;
  mine.L = L;
  Rec* d_rec = nullptr;
  if ((s = dalloc(ctx, reinterpret_cast<uint8_t**>(&d_rec), sizeof(Rec) * (W + 1))) != NE_OK)
    return s;
  std::vector<Rec> all(W);
  NE_CUDA(cudaMemcpy(d_rec + W, &mine, sizeof(Rec), cudaMemcpyHostToDevice));
  NE_CUDA(cudaDeviceSynchronize());   // the zeroed flags too, before any rank may read them
  if ((s = comm_fence_in(ctx)) != NE_OK || (s = comm_allgather(ctx, d_rec + W, d_rec,
                                                               sizeof(Rec))) != NE_OK ||
      (s = comm_fence_out(ctx)) != NE_OK || (s = comm_sync(ctx)) != NE_OK) {
    cudaFree(d_rec);
    return s;
  }
  NE_CUDA(cudaMemcpy(all.data(), d_rec, sizeof(Rec) * W, cudaMemcpyDeviceToHost));
  cudaFree(d_rec);
  std::vector<const char*> wsrc(W), asrc(W);
  for (int p = 0; p < W; ++p) {
    const Rec& r = all[p];
    if (r.pool_floats != mine.pool_floats || r.act_bytes != mine.act_bytes || r.M != M ||
        r.L != L)
      return fail(ctx, NE_ERR_INVALID, "peer-memory exchange: ranks differ in model or batch");
    char* b[4];
    if (p == R) {
      for (int i = 0; i < 4; ++i) b[i] = static_cast<char*>(bases[i]);
    } else {
      for (int i = 0; i < 4; ++i) {
        void* q = nullptr;
        NE_CUDA(cudaIpcOpenMemHandle(&q, r.h[i], cudaIpcMemLazyEnablePeerAccess));
        x.mapped.push_back(q);
        b[i] = static_cast<char*>(q);
      }
    }
    x.T.grad[p] = reinterpret_cast<float*>(b[0]) + (t->grad_pool - t->pool);
    wsrc[p] = b[1];
    asrc[p] = b[2];
    x.T.flags[p] = reinterpret_cast<uint32_t*>(b[3]);
  }
  x.T.world = W;
  x.T.rank = R;
  x.T.limit_ns = (unsigned long long)c->timeout_ms * 1000000ull / 2;
  // chunk lists
  std::vector<PxChunk> ch;
  constexpr int RS_CHUNK = 8192;        // floats
  constexpr int CP_CHUNK = 64 << 10;    // bytes
  x.rs_first.assign(L + 1, 0);
  x.rs_count.assign(L + 1, 0);
  for (int b = 0; b <= L; ++b) {
    int s0, s1;
    bucket_segs(t, b, &s0, &s1);
    x.rs_first[b] = (int)ch.size();
    for (int k = s0; k < s1; ++k) {
      const Seg& sg = t->segs[k];
      long long off, len;
      seg_owned(ctx, sg, R, &off, &len);
      const long long g0 = (sg.g - t->grad_pool) + off;
      for (long long i = 0; i < len; i += RS_CHUNK)
        ch.push_back({0, g0 + i, (int)std::min<long long>(RS_CHUNK, len - i), R});
    }
    x.rs_count[b] = (int)ch.size() - x.rs_first[b];
  }
  // fused dW exchange: each layer matrix whose row length is a multiple of
  // 64 takes its dW product straight into the owners' parts
  // (EPI_RESID_PEER); its bucket then reduce-scatters only the gains
  x.fused = px_fused_dw();
  x.fused_seg.assign(t->segs.size(), 0);
  x.peer_out.assign(t->segs.size(), GemmPeerOut{});
  if (x.fused) {
    const long long qd = (long long)ctx->cfg.n_heads * ctx->cfg.head_dim;
    // row lengths of dWqkv [qkv, D], dWo [D, qd], dW13 [2F, D], dW2 [D, F]
    const long long lds[4] = {D, qd, D, ctx->cfg.hidden};
    for (int l = 0; l < L; ++l) {
      for (int i = 0; i < 4; ++i) {
        const int k = t->P[l].seg0 + i;
        const Seg& sg = t->segs[k];
        if (lds[i] % 64 != 0 || sg.n % lds[i] != 0) continue;
        GemmPeerOut& po = x.peer_out[k];
        po.world = W;
        po.rank = R;
        po.abort = x.flags + PX_ABORT;
        for (int p = 0; p < W; ++p) {
          po.dst[p] = x.T.grad[p] + (sg.g - t->grad_pool);
          long long off, len;
          px_part(sg.n, W, p, &off, &len);
          po.bound[p] = off;
        }
        po.bound[W] = sg.n;
        x.fused_seg[k] = 1;
      }
    }
  }
  x.rsf_first.assign(L + 1, 0);
  x.rsf_count.assign(L + 1, 0);
  for (int b = 0; b <= L; ++b) {
    int s0, s1;
    bucket_segs(t, b, &s0, &s1);
    x.rsf_first[b] = (int)ch.size();
    for (int k = s0; k < s1; ++k) {
      if (x.fused_seg[k]) continue;
      const Seg& sg = t->segs[k];
      long long off, len;
      seg_owned(ctx, sg, R, &off, &len);
      const long long g0 = (sg.g - t->grad_pool) + off;
      for (long long i = 0; i < len; i += RS_CHUNK)
        ch.push_back({0, g0 + i, (int)std::min<long long>(RS_CHUNK, len - i), R});
    }
    x.rsf_count[b] = (int)ch.size() - x.rsf_first[b];
  }
  // weight all-gather, bucket by bucket in the order the next forward needs
  // them: the tail (embedding, final norm), then layers 0 .. L-1
  x.ag_first = (int)ch.size();
  x.ag_bfirst.assign(L + 1, 0);
  x.ag_bcount.assign(L + 1, 0);
  const char* wbase = static_cast<const char*>(ctx->wpool);
  for (int b = 0; b <= L; ++b) {
    int s0, s1;
    bucket_segs(t, b, &s0, &s1);
    x.ag_bfirst[b] = (int)ch.size();
    for (int k = s0; k < s1; ++k) {
      const Seg& sg = t->segs[k];
      for (int p = 0; p < W; ++p) {
        if (p == R) continue;
        long long off, len;
        seg_owned(ctx, sg, p, &off, &len);
        const long long o = sg.w16 ? reinterpret_cast<const char*>(sg.w16 + off) - wbase
                                   : reinterpret_cast<const char*>(sg.w + off) - wbase;
        const long long bytes = len * (sg.w16 ? 2 : 4);
        for (long long i = 0; i < bytes; i += CP_CHUNK)
          ch.push_back({o + i, o + i, (int)std::min<long long>(CP_CHUNK, bytes - i), p});
      }
    }
    x.ag_bcount[b] = (int)ch.size() - x.ag_bfirst[b];
  }
  x.ag_count = (int)ch.size() - x.ag_first;
  x.ag_ev.assign(L + 1, nullptr);
  for (cudaEvent_t& e : x.ag_ev) NE_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  // captured micro-steps from before the exchange existed do not wait for its
  // all-gathers: capture them again
  for (cudaGraphExec_t& g : t->step_graphs) {
    if (g) cudaGraphExecDestroy(g);
    g = nullptr;
  }
  x.em_first = (int)ch.size();
  const char* abase = static_cast<const char*>(t->act_pool);
  const long long ids_off = reinterpret_cast<const char*>(t->ids) - abase;
  const long long dy_off = reinterpret_cast<const char*>(t->dY) - abase;
  for (int p = 0; p < W; ++p) {
    ch.push_back({ids_off, (long long)p * M * 4, M * 4, p});
    const long long rows = (long long)M * D * 4;
    for (long long i = 0; i < rows; i += CP_CHUNK)
      ch.push_back({dy_off + i, (long long)ids_bytes + (long long)p * rows + i,
                    (int)std::min<long long>(CP_CHUNK, rows - i), p});
  }
  x.em_count = (int)ch.size() - x.em_first;
  // zeroing lists: this rank's owned parts of the fused segments (cleared
  // right after its optimizer step, before PX_ZEROED), and the complement in
  // the gradient pool (cleared once every rank finished reading it)
  {
    constexpr long long Z_CHUNK = 1 << 16;   // floats
    std::vector<std::pair<long long, long long>> own;   // [begin, end) float offsets
    for (size_t k = 0; k < t->segs.size(); ++k) {
      if (!x.fused_seg[k]) continue;
      const Seg& sg = t->segs[k];
      long long off, len;
      seg_owned(ctx, sg, R, &off, &len);
      if (len > 0) own.push_back({(sg.g - t->grad_pool) + off, (sg.g - t->grad_pool) + off + len});
    }
    std::sort(own.begin(), own.end());
    auto push_range = [&](long long a, long long b) {
      for (long long i = a; i < b; i += Z_CHUNK)
        ch.push_back({0, i, (int)std::min<long long>(Z_CHUNK, b - i), R});
    };
    x.zf_first = (int)ch.size();
    for (const auto& r : own) push_range(r.first, r.second);
    x.zf_count = (int)ch.size() - x.zf_first;
    x.zr_first = (int)ch.size();
    long long at = 0;
    for (const auto& r : own) {
      push_range(at, r.first);
      at = r.second;
    }
    push_range(at, (long long)t->grad_floats);
    x.zr_count = (int)ch.size() - x.zr_first;
  }
  if ((s = dalloc(ctx, &x.d_chunks, ch.size())) != NE_OK) return s;
  NE_CUDA(cudaMemcpy(x.d_chunks, ch.data(), ch.size() * sizeof(PxChunk), cudaMemcpyHostToDevice));
  if ((s = dalloc(ctx, reinterpret_cast<uint8_t**>(&x.d_wsrc), sizeof(char*) * W)) != NE_OK ||
      (s = dalloc(ctx, reinterpret_cast<uint8_t**>(&x.d_asrc), sizeof(char*) * W)) != NE_OK)
    return s;
  NE_CUDA(cudaMemcpy(x.d_wsrc, wsrc.data(), sizeof(char*) * W, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(x.d_asrc, asrc.data(), sizeof(char*) * W, cudaMemcpyHostToDevice));
  x.ready = true;
  return NE_OK;
}

// The exchange is set up (it is at the first reduced micro-step; a call
// before that sets it up here, outside any capture).
static ne_status px_ready(ne_ctx* ctx) {
  if (ctx->comm->aborted)
    return fail(ctx, NE_ERR_STATE, "the exchange was aborted after a failed step");
  return ctx->comm->pxs.ready ? NE_OK : px_setup(ctx);
}

// CTAs of the exchange kernels on the comm stream (they share the SMs with
// the backward's GEMMs): NE_PX_CTAS, default 256.  Their NVLink bandwidth
// grows with the loads in flight, so fewer CTAs cost more than the SMs they
// free (2 ranks, Qwen3 S 256, 16 loads per thread: 64 CTAs 26.8, 128 25.7,
// 256 25.4 ms per step).
static int px_ctas() {
  static const int n = [] {
    const char* e = std::getenv("NE_PX_CTAS");
    const int v = e ? std::atoi(e) : 0;
    return v > 0 ? v : 256;
  }();
  return n;
}

// The compute stream waits for bucket b's weight all-gather of the last
// optimizer step (a no-op when there was none).  Inside a capture the wait is
// an external-event node: each replay waits for the event's latest record.
static ne_status px_weights_ready(ne_ctx* ctx, int b) {
  if (!ctx->comm || !ctx->comm->shard || !ctx->comm->px || !ctx->comm->pxs.ready) return NE_OK;
  const PxState& x = ctx->comm->pxs;
  if (b < 0 || b >= (int)x.ag_ev.size()) return NE_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  NE_CUDA(cudaStreamIsCapturing(ctx->st, &cs));
  NE_CUDA(cudaStreamWaitEvent(ctx->st, x.ag_ev[b],
                              cs == cudaStreamCaptureStatusNone ? 0u : cudaEventWaitExternal));
  return NE_OK;
}

// Publish bucket b's gradients (compute stream) and reduce this rank's part
// of them over the ranks (comm stream).
static ne_status px_bucket(ne_ctx* ctx, int b) {
  if (ctx->comm->aborted)
    return fail(ctx, NE_ERR_STATE, "the exchange was aborted after a failed step");
  PxState& x = ctx->comm->pxs;
  NE_CUDA(px_signal(x.flags, PX_READY0 + b, ctx->st));
  ne_status s = comm_fence_in(ctx);
  if (s != NE_OK) return s;
  const int first = x.fused_now ? x.rsf_first[b] : x.rs_first[b];
  const int count = x.fused_now ? x.rsf_count[b] : x.rs_count[b];
  NE_CUDA(px_reduce(x.T, x.d_chunks + first, count, PX_READY0 + b, px_ctas(), ctx->d_status,
                    ctx->comm->cs));
  return NE_OK;
}

// Whether segment k's dW product goes straight to its owners in this
// micro-step (the fused exchange), and the GEMM call that does it.
static GemmCall dw_call(ne_ctx* ctx, GemmCall c, int k) {
  if (!ctx->comm || !ctx->comm->px || !comm_active(ctx)) return c;
  const PxState& x = ctx->comm->pxs;
  if (!x.ready || !x.fused_now || k >= (int)x.fused_seg.size() || !x.fused_seg[k]) return c;
  c.epi = EPI_RESID_PEER;
  c.peer = &x.peer_out[k];
  return c;
}

// One bucket (segments [s0, s1)): reduce-scatter the owned segments, all-reduce
// the replicated ones, as one NCCL group on the comm stream.
static ne_status exchange_segments(ne_ctx* ctx, int s0, int s1) {
  TrainState* t = ctx->train;
  ne_status s = comm_group(ctx, true);
  if (s != NE_OK) return s;
  for (int k = s0; k < s1 && s == NE_OK; ++k) {
    const Seg& sg = t->segs[k];
    s = seg_sharded(ctx, sg) ? comm_reduce_scatter(ctx, sg.g, (size_t)shard_len(ctx, sg))
                             : comm_allreduce(ctx, sg.g, (size_t)sg.n);
  }
  const ne_status e = comm_group(ctx, false);
  return s != NE_OK ? s : e;
}

// In place all-gather of the owned parts of one array (seg_array selector:
// 0 masters, 1 m, 2 v, 3 gradients) of every sharded segment; 4 = the bf16
// compute copies.  Enqueued on the comm stream between fences.
static ne_status gather_owned(ne_ctx* ctx, int which) {
  TrainState* t = ctx->train;
  ne_status s = comm_fence_in(ctx);
  if (s != NE_OK) return s;
  if ((s = comm_group(ctx, true)) != NE_OK) return s;
  for (const Seg& sg : t->segs) {
    if (!seg_sharded(ctx, sg) || s != NE_OK) continue;
    const long long off = shard_off(ctx, sg), len = shard_len(ctx, sg);
    if (which == 4) {
      s = comm_allgather(ctx, sg.w16 + off, sg.w16, (size_t)len * 2);
    } else {
      float* a = which == 0 ? sg.w : which == 1 ? sg.m : which == 2 ? sg.v : sg.g;
      s = comm_allgather(ctx, a + off, a, (size_t)len * 4);
    }
  }
  const ne_status e = comm_group(ctx, false);
  if (s != NE_OK) return s;
  if (e != NE_OK) return e;
  return comm_fence_out(ctx);
}

static ne_status comm_after_lmhead(ne_ctx* ctx) {
  if (!comm_active(ctx)) return NE_OK;
  TrainState* t = ctx->train;
  if (px_active(ctx)) {
    if (!ctx->comm->pxs.ready) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      NE_CUDA(cudaStreamIsCapturing(ctx->st, &cs));
      if (cs != cudaStreamCaptureStatusNone)
        return fail(ctx, NE_ERR_STATE, "peer-memory exchange set up inside a capture");
    }
    ne_status s = px_ready(ctx);
    if (s != NE_OK) return s;
    PxState& x = ctx->comm->pxs;
    NE_CUDA(px_epoch(x.flags, ctx->st));
    // the first micro-step after the gradients were zeroed may add its dW
    // products into the owners' parts, once every owner has cleared them
    x.fused_now = x.fused && t->micro_steps == 0;
    if (x.fused_now) NE_CUDA(px_wait(x.T, PX_ZEROED, ctx->d_status, ctx->st));
    return px_bucket(ctx, 0);
  }
  ne_status s = comm_fence_in(ctx);
  if (s != NE_OK) return s;
  if (shard_active(ctx)) return exchange_segments(ctx, (int)t->segs.size() - 2, (int)t->segs.size());
  return comm_allreduce(ctx, t->grad_pool + t->tail_grad_off, t->grad_floats - t->tail_grad_off);
}

static ne_status comm_after_layer(ne_ctx* ctx, int l) {
  if (!comm_active(ctx)) return NE_OK;
  TrainState* t = ctx->train;
  if (px_active(ctx)) return px_bucket(ctx, 1 + l);
  ne_status s = comm_fence_in(ctx);
  if (s != NE_OK) return s;
  if (shard_active(ctx)) {
    const int s1 = l + 1 < (int)t->P.size() ? t->P[l + 1].seg0 : (int)t->segs.size() - 2;
    return exchange_segments(ctx, t->P[l].seg0, s1);
  }
  return comm_allreduce(ctx, t->grad_pool + (size_t)l * t->layer_grad_floats,
                        t->layer_grad_floats);
}

// Deterministic scatter of n (token id, dY row) pairs into the embedding gradient.
static ne_status embed_scatter(ne_ctx* ctx, const int32_t* ids, const float* dy, int n) {
  TrainState* t = ctx->train;
  const size_t need = embed_bwd_scratch_bytes(n);
  if (t->embed_scratch_bytes < need) {
    if (t->embed_scratch) NE_CUDA(cudaFree(t->embed_scratch));
    t->embed_scratch = nullptr;
    t->embed_scratch_bytes = 0;
    uint8_t* p = nullptr;
    ne_status s = dalloc(ctx, &p, need);
    if (s != NE_OK) return s;
    t->embed_scratch = p;
    t->embed_scratch_bytes = need;
  }
  NE_LAUNCH(launch_embed_bwd(ids, dy, n, ctx->cfg.vocab, ctx->cfg.dim, t->embed_g, t->embed_scratch,
                             t->embed_scratch_bytes, ctx->d_status, ctx->st));
  return NE_OK;
}

// Input-embedding gradient.  Reduced: gather every rank's (token id, dY row)
// pairs, wait for all buckets, then scatter-add all of them on every rank
// (the dense part of the embedding gradient was already summed).
static ne_status comm_embed_bwd(ne_ctx* ctx) {
  TrainState* t = ctx->train;
  const ne_model_cfg& m = ctx->cfg;
  const int M = t->M, D = m.dim, V = m.vocab;
  (void)V;
  if (!comm_active(ctx)) return embed_scatter(ctx, t->ids, t->dY, M);
  Comm* c = ctx->comm;
  if (px_active(ctx)) {
    // after this rank's reduce-scatters (comm stream order) and its last
    // layer's backward (fence): publish, then gather every rank's pairs
    PxState& x = c->pxs;
    const size_t ids_bytes = ((size_t)c->world * M * 4 + 255) & ~(size_t)255;
    ne_status s;
    if ((s = comm_fence_in(ctx)) != NE_OK) return s;
    NE_CUDA(px_signal(x.flags, PX_EMBED, c->cs));
    NE_CUDA(px_copy(x.T, x.d_asrc, static_cast<char*>(c->gather), x.d_chunks + x.em_first,
                    x.em_count, PX_EMBED, px_ctas(), ctx->d_status, c->cs));
    if ((s = comm_fence_out(ctx)) != NE_OK) return s;
    return embed_scatter(ctx, reinterpret_cast<int32_t*>(c->gather),
                         reinterpret_cast<float*>(static_cast<uint8_t*>(c->gather) + ids_bytes),
                         c->world * M);
  }
  const size_t ids_bytes = ((size_t)c->world * M * 4 + 255) & ~(size_t)255;
  const size_t need = ids_bytes + (size_t)c->world * M * D * 4;
  if (c->gather_bytes < need) {
    if (c->gather) NE_CUDA(cudaFree(c->gather));
    c->gather = nullptr;
    c->gather_bytes = 0;
    uint8_t* g = nullptr;
    ne_status s = dalloc(ctx, &g, need);
    if (s != NE_OK) return s;
    c->gather = g;
    c->gather_bytes = need;
  }
  int32_t* ids_all = reinterpret_cast<int32_t*>(c->gather);
  float* dy_all = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(c->gather) + ids_bytes);
  ne_status s;
  if ((s = comm_fence_in(ctx)) != NE_OK) return s;
  if ((s = comm_allgather(ctx, t->ids, ids_all, (size_t)M * 4)) != NE_OK) return s;
  if ((s = comm_allgather(ctx, t->dY, dy_all, (size_t)M * D * 4)) != NE_OK) return s;
  if ((s = comm_fence_out(ctx)) != NE_OK) return s;
  return embed_scatter(ctx, ids_all, dy_all, c->world * M);
}

// The tcgen05 attention forward serves head_dim 128; NE_ATTN_TC=0 selects the
// mma.sync kernel instead (both are complete implementations; for comparison).
static bool attn_tc_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("NE_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

// ---------------------------------------------------------------------------
// Per-layer entry points.  Each enqueues on the context stream and works on
// the training workspace; the composition below (ne_train_fwd_bwd_device) is
// the whole micro-step.  Activations saved for the backward pass live in
// t->A[layer]; the running residual gradient is t->dY (fp32) / t->dY16 (bf16).

#define NE_TRAIN_PRELUDE()                                                                   \
  if (!ctx || !ctx->train) return NE_ERR_STATE;                                              \
  TrainState* t = ctx->train;                                                                \
  const ne_model_cfg& m = ctx->cfg;                                                          \
  const int B = t->B, S = t->S, M = t->M, D = m.dim, F = m.hidden, Hq = m.n_heads,           \
            Hkv = m.kv_heads, hd = m.head_dim, V = m.vocab;                                  \
  const int qd = Hq * hd, kvd = Hkv * hd, qkv = qd + 2 * kvd;                                \
  const float alpha = m.res_alpha;                                                           \
  cudaStream_t st = ctx->st;                                                                 \
  ne_status s = NE_OK;                                                                       \
  (void)B; (void)S; (void)M; (void)D; (void)F; (void)Hq; (void)Hkv; (void)hd; (void)V;       \
  (void)qd; (void)kvd; (void)qkv; (void)alpha; (void)st; (void)s;                            \
  NE_CUDA(cudaSetDevice(ctx->device))

#define NE_LAYER_CHECK(layer) \
  if ((layer) < 0 || (layer) >= m.n_layers) return fail(ctx, NE_ERR_INVALID, "layer out of range")

// Split d_tokens [B, S+1] into inputs / targets, embed, first RMSNorm
// (embed_lookup, cpu_ops.h:433-439; rmsnorm, cpu_ops.h:20-60).
static ne_status split_tokens(ne_ctx* ctx, const int32_t* d_tokens) {
  TrainState* t = ctx->train;
  split_tokens_kernel<<<(t->M + 255) / 256, 256, 0, ctx->st>>>(d_tokens, t->B, t->S, t->ids,
                                                               t->tgt);
  NE_CUDA(cudaGetLastError());
  return NE_OK;
}

// embed + first norm of the split batch (t->ids)
static ne_status embed_fwd_ids(ne_ctx* ctx) {
  NE_TRAIN_PRELUDE();
  // the embedding / final norm (bucket 0) and layer 0's gains (bucket 1)
  if ((s = px_weights_ready(ctx, 0)) != NE_OK || (s = px_weights_ready(ctx, 1)) != NE_OK) return s;
  NE_LAUNCH(launch_embed_rmsnorm(t->ids, t->embed_w, 1, V, D, ctx->L[0].rms_att, m.rms_eps,
                                 t->A[0].X, t->A[0].XN, M, ctx->d_status, st));
  // the attention residual of layer 0 accumulates onto a copy of x
  NE_CUDA(cudaMemcpyAsync(t->A[0].X2, t->A[0].X, (size_t)M * D * 4, cudaMemcpyDeviceToDevice, st));
  return NE_OK;
}

NE_API ne_status ne_embed_fwd(ne_ctx* ctx, const int32_t* d_tokens) {
  if (!ctx || !ctx->train) return NE_ERR_STATE;
  if (!d_tokens) return NE_ERR_INVALID;
  NE_CUDA(cudaSetDevice(ctx->device));
  ne_status s = split_tokens(ctx, d_tokens);
  return s != NE_OK ? s : embed_fwd_ids(ctx);
}

// Attention half of a layer (sdpaFwd, mil_dynamic.h:57-234): fused QKV
// projection, per-head QK-norm, RoPE, causal GQA attention, Wo projection and
// the scaled residual x2 = x + alpha*o (residual_cvt_f16, io.h:25-37), then the
// FFN's RMSNorm of x2.
NE_API ne_status ne_attn_fwd(ne_ctx* ctx, int l) {
  NE_TRAIN_PRELUDE();
  NE_LAYER_CHECK(l);
  if ((s = px_weights_ready(ctx, 1 + l)) != NE_OK) return s;
  const LayerW& w = ctx->L[l];
  TrainActs& a = t->A[l];
  if ((s = gemm(ctx, gc(a.XN, D, M, 0, w.wqkv, D, qkv, 0, D, EPI_F32, a.QKVR, qkv))) != NE_OK)
    return s;
  NE_LAUNCH(launch_qkv_post(a.QKVR, 1, 0, M, S, nullptr, 0, Hq, Hkv, hd,
                            m.qk_norm ? w.q_norm : nullptr, m.qk_norm ? w.k_norm : nullptr,
                            m.qk_eps, ctx->rope_cs, a.Q, 2, a.K, a.V, S, ctx->d_status, st, 1));
  if ((hd == 128 || (hd == 64 && attn_tc64())) && attn_tc_enabled())
    NE_LAUNCH(launch_attn_fwd_tc(a.Q, a.K, a.V, B, S, Hq, Hkv, hd, S, a.O, a.LSE, ctx->d_status, st));
  else
    NE_LAUNCH(launch_prefill_attn_bf16(a.Q, a.K, a.V, B, S, 0, Hq, Hkv, hd, S, a.O, st, a.LSE));
  // x2 (seeded with x by the preceding norm) += alpha * o.Wo^T
  if ((s = gemm(ctx, gc(a.O, qd, M, 0, w.wo, qd, D, 0, qd, EPI_RESID, a.X2, D, alpha))) != NE_OK)
    return s;
  // FFN norm of x2; x2 also seeds the FFN residual sum x_next
  float* xnext = (l + 1 < m.n_layers) ? t->A[l + 1].X : t->XL;
  NE_LAUNCH(launch_resid_rmsnorm(a.X2, nullptr, 0, 0, 1.f, D, w.rms_ffn, m.rms_eps, a.X2N, M, st,
                                 xnext));
  return NE_OK;
}

// FFN half of a layer (ffnFused, mil_dynamic.h:238-306): SwiGLU over the
// interleaved W1/W3 projection, W2, residual x_next = x2 + alpha*ffn, then the
// RMSNorm the next consumer needs (next layer's attention norm, or the final
// norm before the classifier).
NE_API ne_status ne_ffn_fwd(ne_ctx* ctx, int l) {
  NE_TRAIN_PRELUDE();
  NE_LAYER_CHECK(l);
  // this layer's matrices, and the gain of the norm that follows (next layer / final)
  if ((s = px_weights_ready(ctx, 1 + l)) != NE_OK ||
      (s = px_weights_ready(ctx, l + 1 < m.n_layers ? 2 + l : 0)) != NE_OK)
    return s;
  const LayerW& w = ctx->L[l];
  TrainActs& a = t->A[l];
  GemmCall c = gc(a.X2N, D, M, 0, w.w13, D, 2 * F, 0, D, EPI_SWIGLU, a.GATE, F);
  c.aux1 = a.H13;
  if ((s = gemm(ctx, c)) != NE_OK) return s;
  // x_next (seeded with x2 by the FFN norm) += alpha * gate.W2^T
  float* xnext = (l + 1 < m.n_layers) ? t->A[l + 1].X : t->XL;
  if ((s = gemm(ctx, gc(a.GATE, F, M, 0, w.w2, F, D, 0, F, EPI_RESID, xnext, D, alpha))) != NE_OK)
    return s;
  const bool last = l + 1 == m.n_layers;
  const float* g = last ? ctx->rms_final : ctx->L[l + 1].rms_att;
  __nv_bfloat16* xn = last ? t->XNF : t->A[l + 1].XN;
  NE_LAUNCH(launch_resid_rmsnorm(xnext, nullptr, 0, 0, 1.f, D, g, m.rms_eps, xn, M, st,
                                 last ? nullptr : t->A[l + 1].X2));
  return NE_OK;
}

// Classifier over the tied embedding (train.m:495-505), mean cross-entropy
// (cpu_ops.h:348-382), the classifier's backward (dX and the dense part of
// dE), and the final RMSNorm's backward, leaving dY for the last layer.
// d_loss (device, optional) receives the batch's mean loss.
NE_API ne_status ne_lmhead_ce_fwd_bwd(ne_ctx* ctx, float* d_loss) {
  NE_TRAIN_PRELUDE();
  const float ce_scale = 1.0f / (float)M;
  // classifier rows: the whole tied embedding, or its compacted rows
  const bool cmp = t->CV > 0;
  const int Vc = cmp ? t->CV : V;           // classes of the softmax
  const int ldl = cmp ? t->CVp : V;         // logits row stride = classifier rows
  const __nv_bfloat16* Wcls = cmp ? t->Ec : ctx->embed;
  float* dWcls = cmp ? t->dEc : t->embed_g;
  if (cmp) NE_LAUNCH(launch_gather_rows(ctx->embed, t->d_c2f, t->CV, D, t->Ec, st));
  const int nck = (Vc + 31) / 32;
  for (int r0 = 0; r0 < M; r0 += t->Mc) {
    const int rows = std::min(t->Mc, M - r0);
    const __nv_bfloat16* xnf = t->XNF + (size_t)r0 * D;
    GemmCall cl = gc(xnf, D, rows, 0, Wcls, D, Vc, 0, D, EPI_F32_STATS, t->logits, ldl);
    cl.aux1 = t->ce_stats;
    cl.aux_ld = nck;
    if ((s = gemm(ctx, cl)) != NE_OK) return s;
    NE_LAUNCH(launch_ce_rows(t->logits, ldl, t->ce_stats, nck, t->tgt + r0,
                             cmp ? t->d_f2c : nullptr, rows, Vc, ce_scale, t->loss_rows + r0,
                             t->dlogits, ctx->d_status, st));
    // dXNF = dlogits . Wcls   (Wcls read MN-major as [classes (K), D (N)])
    if ((s = gemm(ctx, gc(t->dlogits, ldl, rows, 0, Wcls, D, D, 1, ldl, EPI_F32,
                          t->dXF + (size_t)r0 * D, D))) != NE_OK)
      return s;
    // dWcls += dlogits^T . XNF   (both MN-major)
    if ((s = gemm(ctx, gc(t->dlogits, ldl, ldl, 1, xnf, D, D, 1, rows, EPI_RESID, dWcls, D))) !=
        NE_OK)
      return s;
  }
  if (cmp) NE_LAUNCH(launch_scatter_add_rows(t->dEc, t->d_c2f, t->CV, D, t->embed_g, st));
  NE_LAUNCH(launch_rmsnorm_bwd(t->dXF, t->XL, ctx->rms_final, m.rms_eps, M, D, nullptr, t->dY,
                               t->dY16, t->rmsf_g, st));
  if (d_loss) {
    NE_CUDA(cudaMemsetAsync(t->red + 1, 0, sizeof(double), st));
    sum_rows_kernel<<<64, 256, 0, st>>>(t->loss_rows, M, t->red + 1);
    NE_CUDA(cudaGetLastError());
    // d_loss = sum / M  (a 1-thread kernel keeps it on the device)
    mean_from_sum_kernel<<<1, 1, 0, st>>>(t->red + 1, M, d_loss);
    NE_CUDA(cudaGetLastError());
  }
  return comm_after_lmhead(ctx);
}

// FFN backward of a layer (ffnBwdFull, mil_dynamic.h:320-409): d_gate -> dh1,
// dh3 through the SwiGLU-backward epilogue, dW2, dW1/dW3, dX through W1/W3,
// and the FFN RMSNorm's backward plus the residual (rmsnorm_bwd_add,
// cpu_ops.h:108-261), leaving the gradient at x2 in t->dX2 / t->dX216.
NE_API ne_status ne_ffn_bwd(ne_ctx* ctx, int l) {
  NE_TRAIN_PRELUDE();
  NE_LAYER_CHECK(l);
  const LayerW& w = ctx->L[l];
  const TrainActs& a = t->A[l];
  const TrainLayerP& p = t->P[l];
  GemmCall c = gc(t->dY16, D, M, 0, w.w2, F, F, 1, D, EPI_SWIGLU_BWD, t->DH13, 2 * F, alpha);
  c.aux3 = a.H13;
  c.aux_ld = F;
  if ((s = gemm(ctx, c)) != NE_OK) return s;
  if ((s = gemm(ctx, dw_call(ctx, gc(t->dY16, D, D, 1, a.GATE, F, F, 1, M, EPI_RESID, p.g2, F,
                                      alpha), p.seg0 + 3))) != NE_OK)
    return s;
  if ((s = gemm(ctx, dw_call(ctx, gc(t->DH13, 2 * F, 2 * F, 1, a.X2N, D, D, 1, M, EPI_RESID, p.g13,
                                      D), p.seg0 + 2))) != NE_OK)
    return s;
  if ((s = gemm(ctx, gc(t->DH13, 2 * F, M, 0, w.w13, D, D, 1, 2 * F, EPI_F32, t->dXF, D))) !=
      NE_OK)
    return s;
  NE_LAUNCH(launch_rmsnorm_bwd(t->dXF, a.X2, w.rms_ffn, m.rms_eps, M, D, t->dY, t->dX2,
                               t->dX216, p.g_ffn, st));
  return NE_OK;
}

// Attention backward of a layer: dO = dx2 . Wo (wotBwd, mil_dynamic.h:412),
// dWo, SDPA backward (sdpaBwd1/2, mil_dynamic.h:583-707, with the GQA group
// sum of gqa_reduce_kv_f16, cpu_ops.h:585), RoPE and QK-norm backward
// (rope_backward_inplace_f16, cpu_ops.h:510-537), dX through Wq/Wk/Wv (qkvBwd,
// mil_dynamic.h:516-576), dWq/dWk/dWv and the attention RMSNorm's backward
// plus the residual, leaving dY for the layer below.  The layer's gradients
// are final afterwards (the data-parallel bucket of this layer may start).
NE_API ne_status ne_attn_bwd(ne_ctx* ctx, int l) {
  NE_TRAIN_PRELUDE();
  NE_LAYER_CHECK(l);
  const LayerW& w = ctx->L[l];
  const TrainActs& a = t->A[l];
  const TrainLayerP& p = t->P[l];
  GemmCall c = gc(t->dX216, D, M, 0, w.wo, qd, qd, 1, D, EPI_BF16, t->dO, qd, alpha);
  if ((s = gemm(ctx, c)) != NE_OK) return s;
  if ((s = gemm(ctx, dw_call(ctx, gc(t->dX216, D, D, 1, a.O, qd, qd, 1, M, EPI_RESID, p.go, qd,
                                      alpha), p.seg0 + 1))) != NE_OK)
    return s;
  NE_LAUNCH(launch_attn_bwd(a.Q, a.K, a.V, a.O, t->dO, a.LSE, t->Dl, B, S, Hq, Hkv, hd, S, a.QKVR,
                            m.qk_norm ? w.q_norm : nullptr, m.qk_norm ? w.k_norm : nullptr,
                            m.qk_eps, ctx->rope_cs, t->DQKV, p.g_qn, p.g_kn, ctx->d_status, st));
  ctx->launches += 1;
  if ((s = gemm(ctx, gc(t->DQKV, qkv, M, 0, w.wqkv, D, D, 1, qkv, EPI_F32, t->dXF, D))) != NE_OK)
    return s;
  if ((s = gemm(ctx, dw_call(ctx, gc(t->DQKV, qkv, qkv, 1, a.XN, D, D, 1, M, EPI_RESID, p.gqkv, D),
                             p.seg0))) != NE_OK)
    return s;
  NE_LAUNCH(launch_rmsnorm_bwd(t->dXF, a.X, w.rms_att, m.rms_eps, M, D, t->dX2, t->dY, t->dY16,
                               p.g_att, st));
  return comm_after_layer(ctx, l);
}

// Scatter-add of the input-embedding gradient (embed_backward,
// cpu_ops.h:441-447).  With data-parallel reduction active, every rank's
// (token, dY row) pairs are gathered first and added on every rank.
NE_API ne_status ne_embed_bwd(ne_ctx* ctx) {
  NE_TRAIN_PRELUDE();
  return comm_embed_bwd(ctx);
}

// Forward + backward of one batch d_tokens [B, S+1] (inputs tokens[:, :S],
// targets tokens[:, 1:]); gradients ACCUMULATE into the gradient buffers
// (mean cross-entropy over the B*S targets of this batch).  *d_loss (device,
// optional) receives the batch's mean loss.
static ne_status step_body(ne_ctx* ctx, float* d_loss) {
  const int L = ctx->cfg.n_layers;
  ne_status s;
  if ((s = embed_fwd_ids(ctx)) != NE_OK) return s;
  for (int l = 0; l < L; ++l) {
    if ((s = ne_attn_fwd(ctx, l)) != NE_OK) return s;
    if ((s = ne_ffn_fwd(ctx, l)) != NE_OK) return s;
  }
  if ((s = ne_lmhead_ce_fwd_bwd(ctx, d_loss)) != NE_OK) return s;
  for (int l = L - 1; l >= 0; --l) {
    if ((s = ne_ffn_bwd(ctx, l)) != NE_OK) return s;
    if ((s = ne_attn_bwd(ctx, l)) != NE_OK) return s;
  }
  return ne_embed_bwd(ctx);
}

// Whether the micro-step runs as a captured graph: on by default (NE_TRAIN_GRAPH=0
// turns it off).  With gradients exchanged over NCCL the comm stream's
// buckets are captured into the same graph (the first, eager micro-step has
// allocated the exchange buffers) unless NE_TRAIN_GRAPH_COMM=0.
static bool use_step_graph(const ne_ctx* ctx) {
  static const bool on = [] {
    const char* e = std::getenv("NE_TRAIN_GRAPH");
    return !(e && e[0] == '0');
  }();
  static const bool with_comm = [] {
    const char* e = std::getenv("NE_TRAIN_GRAPH_COMM");
    return !(e && e[0] == '0');
  }();
  return on && (with_comm || !comm_active(ctx));
}

NE_API ne_status ne_train_fwd_bwd_device(ne_ctx* ctx, const int32_t* d_tokens, float* d_loss) {
  if (!ctx || !ctx->train || !d_tokens) return NE_ERR_STATE;
  NE_FAULT_POINT(ctx, "ne_train_fwd_bwd_device");
  TrainState* t = ctx->train;
  NE_CUDA(cudaSetDevice(ctx->device));
  if (comm_active(ctx) && ctx->comm->aborted)   // also keeps a captured exchange from replaying
    return fail(ctx, NE_ERR_STATE, "the exchange was aborted after a failed step");
  ne_status s = split_tokens(ctx, d_tokens);
  if (s != NE_OK) return s;
  if (ctx->comm) ctx->comm->pxs.owned_clean = false;   // the step writes the gradients
  // The first micro-step runs eagerly (kernel attributes and modules get
  // loaded outside any capture); later ones replay the captured graph.
  if (!use_step_graph(ctx) || t->steps_run == 0) {
    if ((s = step_body(ctx, d_loss)) != NE_OK) return s;
  } else {
    // The graph always writes the loss to its own slot; copied out below.
    float* g_loss = reinterpret_cast<float*>(t->red + 3);
    const bool fused = comm_active(ctx) && ctx->comm->px && ctx->comm->pxs.ready &&
                       ctx->comm->pxs.fused && t->micro_steps == 0;
    const int gi = !comm_active(ctx) ? 0 : fused ? 2 : 1;
    cudaGraphExec_t& sgraph = t->step_graphs[gi];
    if (sgraph && t->step_graph_rope[gi] != ctx->rope_cs) {
      NE_CUDA(cudaGraphExecDestroy(sgraph));
      sgraph = nullptr;
    }
    if (!sgraph) {
      cudaGraph_t g = nullptr;
      NE_CUDA(cudaStreamBeginCapture(ctx->st, cudaStreamCaptureModeThreadLocal));
      const ne_status sb = step_body(ctx, g_loss);
      const cudaError_t ec = cudaStreamEndCapture(ctx->st, &g);
      if (sb != NE_OK) {
        if (g) cudaGraphDestroy(g);
        return sb;
      }
      if (ec != cudaSuccess)
        return fail(ctx, NE_ERR_CUDA, std::string("step capture: ") + cudaGetErrorString(ec));
      const cudaError_t ei = cudaGraphInstantiate(&sgraph, g, 0);
      cudaGraphDestroy(g);
      if (ei != cudaSuccess) {
        sgraph = nullptr;
        return fail(ctx, NE_ERR_CUDA, std::string("step graph: ") + cudaGetErrorString(ei));
      }
      t->step_graph_rope[gi] = ctx->rope_cs;
    }
    NE_CUDA(cudaGraphLaunch(sgraph, ctx->st));
    if (d_loss)
      NE_CUDA(cudaMemcpyAsync(d_loss, g_loss, sizeof(float), cudaMemcpyDeviceToDevice, ctx->st));
  }
  t->micro_steps++;
  t->steps_run++;
  return NE_OK;
}

// Token-major RMSNorm (rmsnorm, cpu_ops.h:20-60): out [rows, D] (bf16) =
// x / sqrt(mean(x^2) + eps) * w, for caller-owned device buffers.
NE_API ne_status ne_rmsnorm_fwd(ne_ctx* ctx, const float* d_x, const float* d_w, int rows,
                                void* d_out_bf16) {
  if (!ctx || !d_x || !d_w || !d_out_bf16 || rows <= 0) return NE_ERR_INVALID;
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_LAUNCH(launch_resid_rmsnorm(const_cast<float*>(d_x), nullptr, 0, 0, 1.f, ctx->cfg.dim, d_w,
                                 ctx->cfg.rms_eps, reinterpret_cast<__nv_bfloat16*>(d_out_bf16),
                                 rows, ctx->st));
  return NE_OK;
}

// RMSNorm backward with residual (rmsnorm_bwd / rmsnorm_bwd_add,
// cpu_ops.h:108-261) in token-major layout: d_dx = d(rmsnorm)/dx . d_dy
// (+ d_residual when not NULL); d_dw (optional) accumulates the gain gradient.
// The exact derivative of x*w/rms is used for every gain value.
NE_API ne_status ne_rmsnorm_bwd_add(ne_ctx* ctx, const float* d_dy, const float* d_x,
                                    const float* d_w, int rows, const float* d_residual,
                                    float* d_dx, float* d_dw) {
  if (!ctx || !d_dy || !d_x || !d_w || !d_dx || rows <= 0) return NE_ERR_INVALID;
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_LAUNCH(launch_rmsnorm_bwd(d_dy, d_x, d_w, ctx->cfg.rms_eps, rows, ctx->cfg.dim, d_residual,
                               d_dx, nullptr, d_dw, ctx->st));
  return NE_OK;
}

// Host tokens -> the page-locked stage -> t->tok (ordered on the stream).
static ne_status stage_tokens(ne_ctx* ctx, const int32_t* h_tokens) {
  TrainState* t = ctx->train;
  const size_t bytes = (size_t)t->B * (t->S + 1) * 4;
  std::memcpy(t->h_stage, h_tokens, bytes);   // the stage is idle: every host call synchronises
  NE_CUDA(cudaMemcpyAsync(t->tok, t->h_stage, bytes, cudaMemcpyHostToDevice, ctx->st));
  return NE_OK;
}

// The loss (if asked for) through the stage, then the bounded synchronisation.
static ne_status finish_host_call(ne_ctx* ctx, const float* d_loss, float* h_loss) {
  TrainState* t = ctx->train;
  float* staged = reinterpret_cast<float*>(t->h_stage + t->h_stage_tok);
  if (d_loss) NE_CUDA(cudaMemcpyAsync(staged, d_loss, 4, cudaMemcpyDeviceToHost, ctx->st));
  const ne_status s = ne_sync(ctx);
  if (s == NE_OK && d_loss) *h_loss = *staged;
  return s;
}

NE_API ne_status ne_train_fwd_bwd(ne_ctx* ctx, const int32_t* h_tokens, float* h_loss) {
  if (!ctx || !ctx->train || !h_tokens) return NE_ERR_STATE;
  NE_FAULT_POINT(ctx, "ne_train_fwd_bwd");
  TrainState* t = ctx->train;
  NE_CUDA(cudaSetDevice(ctx->device));
  ne_status s = stage_tokens(ctx, h_tokens);
  if (s != NE_OK) return s;
  float* d_loss = reinterpret_cast<float*>(t->red + 2);
  if ((s = ne_train_fwd_bwd_device(ctx, t->tok, h_loss ? d_loss : nullptr)) != NE_OK) return s;
  return finish_host_call(ctx, h_loss ? d_loss : nullptr, h_loss);
}

// One micro-step like ne_train_fwd_bwd, run without the captured graph and
// with an event between consecutive entry points, so the device time of each
// stage can be reported (the per-phase timing line of train.m:763-768).
// h_ms[NE_TRAIN_PHASES] receives, in ms: 0 embedding forward, 1 attention
// forward (all layers), 2 FFN forward, 3 classifier + cross-entropy + its
// backward, 4 FFN backward, 5 attention backward, 6 embedding backward (with
// the wait for the gradient exchange), 7 the whole micro-step.
NE_API ne_status ne_train_fwd_bwd_timed(ne_ctx* ctx, const int32_t* h_tokens, float* h_loss,
                                        float* h_ms) {
  if (!ctx || !ctx->train || !h_tokens || !h_ms) return NE_ERR_INVALID;
  NE_FAULT_POINT(ctx, "ne_train_fwd_bwd_timed");
  TrainState* t = ctx->train;
  const int L = ctx->cfg.n_layers;
  NE_CUDA(cudaSetDevice(ctx->device));
  const size_t nev = 4 * (size_t)L + 4;
  if (t->phase_ev.size() != nev) {
    for (cudaEvent_t e : t->phase_ev)
      if (e) cudaEventDestroy(e);
    t->phase_ev.assign(nev, nullptr);
    for (cudaEvent_t& e : t->phase_ev) NE_CUDA(cudaEventCreate(&e));
  }
  ne_status s = stage_tokens(ctx, h_tokens);
  if (s != NE_OK) return s;
  float* d_loss = reinterpret_cast<float*>(t->red + 2);
  if ((s = split_tokens(ctx, t->tok)) != NE_OK) return s;
  if (ctx->comm) ctx->comm->pxs.owned_clean = false;
  std::vector<int> phase;   // phase of the interval that ends at event k + 1
  size_t k = 0;
  auto mark = [&](int ph) -> ne_status {
    NE_CUDA(cudaEventRecord(t->phase_ev[k++], ctx->st));
    if (ph >= 0) phase.push_back(ph);
    return NE_OK;
  };
  if ((s = mark(-1)) != NE_OK) return s;
  if ((s = embed_fwd_ids(ctx)) != NE_OK || (s = mark(0)) != NE_OK) return s;
  for (int l = 0; l < L; ++l) {
    if ((s = ne_attn_fwd(ctx, l)) != NE_OK || (s = mark(1)) != NE_OK) return s;
    if ((s = ne_ffn_fwd(ctx, l)) != NE_OK || (s = mark(2)) != NE_OK) return s;
  }
  if ((s = ne_lmhead_ce_fwd_bwd(ctx, d_loss)) != NE_OK || (s = mark(3)) != NE_OK) return s;
  for (int l = L - 1; l >= 0; --l) {
    if ((s = ne_ffn_bwd(ctx, l)) != NE_OK || (s = mark(4)) != NE_OK) return s;
    if ((s = ne_attn_bwd(ctx, l)) != NE_OK || (s = mark(5)) != NE_OK) return s;
  }
  if ((s = ne_embed_bwd(ctx)) != NE_OK || (s = mark(6)) != NE_OK) return s;
  t->micro_steps++;
  t->steps_run++;
  if ((s = finish_host_call(ctx, h_loss ? d_loss : nullptr, h_loss)) != NE_OK) return s;
  for (int i = 0; i < NE_TRAIN_PHASES; ++i) h_ms[i] = 0.f;
  for (size_t i = 0; i < phase.size(); ++i) {
    float ms = 0.f;
    NE_CUDA(cudaEventElapsedTime(&ms, t->phase_ev[i], t->phase_ev[i + 1]));
    h_ms[phase[i]] += ms;
  }
  NE_CUDA(cudaEventElapsedTime(&h_ms[7], t->phase_ev[0], t->phase_ev[phase.size()]));
  return NE_OK;
}

// Smallest and largest value of the final residual stream x (before the
// final norm) and of the gradient the last micro-step left at the embedding
// output: h_out = {x_min, x_max, dy_min, dy_max} (train.m:771-776).
NE_API ne_status ne_train_value_ranges(ne_ctx* ctx, float* h_out) {
  if (!ctx || !ctx->train || !h_out) return NE_ERR_INVALID;
  TrainState* t = ctx->train;
  NE_CUDA(cudaSetDevice(ctx->device));
  if (!t->range_out) {
    ne_status s = dalloc(ctx, &t->range_out, 4);
    if (s != NE_OK) return s;
  }
  const long long n = (long long)t->M * ctx->cfg.dim;
  NE_LAUNCH(launch_minmax(t->XL, n, t->range_out, ctx->st));
  NE_LAUNCH(launch_minmax(t->dY, n, t->range_out + 2, ctx->st));
  NE_CUDA(cudaMemcpyAsync(h_out, t->range_out, 4 * sizeof(float), cudaMemcpyDeviceToHost, ctx->st));
  return ne_sync(ctx);
}

// Sum the whole gradient pool over the communicator's ranks now (for callers
// that drive the per-layer entry points with reduction off); enqueued on the
// comm stream, ordered after and before the compute stream's work.
NE_API ne_status ne_grad_allreduce_async(ne_ctx* ctx) {
  if (!ctx || !ctx->train || !ctx->comm) return NE_ERR_STATE;
  if (ctx->comm->world == 1) return NE_OK;
  NE_CUDA(cudaSetDevice(ctx->device));
  ne_status s;
  if ((s = comm_fence_in(ctx)) != NE_OK) return s;
  if ((s = comm_allreduce(ctx, ctx->train->grad_pool, ctx->train->grad_floats)) != NE_OK) return s;
  return comm_fence_out(ctx);
}

NE_API ne_status ne_train_grad_pool(ne_ctx* ctx, float** d_grads, size_t* n_floats) {
  if (!ctx || !ctx->train || !d_grads || !n_floats) return NE_ERR_STATE;
  *d_grads = ctx->train->grad_pool;
  *n_floats = ctx->train->grad_floats;
  return NE_OK;
}

// Global L2 norm of the accumulated gradients times grad_scale (train.m:805-826).
// Upload the segment table (with the weight decay of this step) when it changed.
static ne_status upload_segs(ne_ctx* ctx, float weight_decay) {
  TrainState* t = ctx->train;
  if (!t->d_chunks) {
    // the rank's work: its part of each sharded segment, every replicated
    // segment (whose norm share only rank 0 counts)
    const bool sharded = shard_mode(ctx);
    const bool count_replicated = !sharded || ctx->comm->rank == 0;
    std::vector<OptChunk> hc;
    for (size_t k = 0; k < t->segs.size(); ++k) {
      const Seg& sg = t->segs[k];
      const bool own = seg_sharded(ctx, sg);
      const long long b0 = own ? shard_off(ctx, sg) : 0;
      const long long b1 = own ? b0 + shard_len(ctx, sg) : sg.n;
      auto a16 = [&](const float* p) { return (reinterpret_cast<uintptr_t>(p + b0) & 15u) == 0; };
      const int vec = a16(sg.w) && a16(sg.g) && a16(sg.m) && a16(sg.v) &&
                      (sg.w16 == nullptr || (reinterpret_cast<uintptr_t>(sg.w16 + b0) & 7u) == 0);
      const int norm = (own || count_replicated) ? 1 : 0;
      for (long long off = b0; off < b1; off += OPT_CHUNK)
        hc.push_back({(int)k, vec, off, (int)std::min<long long>(OPT_CHUNK, b1 - off), norm});
    }
    t->nchunks = (int)hc.size();
    ne_status s;
    if ((s = dalloc(ctx, &t->d_chunks, hc.size())) != NE_OK ||
        (s = dalloc(ctx, &t->opt_partial, hc.size())) != NE_OK ||
        (s = dalloc(ctx, &t->opt_ticket, 1)) != NE_OK ||
        (!t->norm_out && (s = dalloc(ctx, &t->norm_out, 4)) != NE_OK))
      return s;
    NE_CUDA(cudaMemcpyAsync(t->d_chunks, hc.data(), hc.size() * sizeof(OptChunk),
                            cudaMemcpyHostToDevice, ctx->st));
  }
  if (t->d_segs && t->d_segs_wd == weight_decay) return NE_OK;
  std::vector<AdamSeg> hs;
  for (const Seg& sg : t->segs)
    hs.push_back({sg.w, sg.g, sg.m, sg.v, sg.w16, sg.n, sg.wd < 0.f ? weight_decay : 0.f});
  if (!t->d_segs) {
    ne_status s = dalloc(ctx, &t->d_segs, hs.size());
    if (s != NE_OK) return s;
  }
  NE_CUDA(cudaMemcpyAsync(t->d_segs, hs.data(), hs.size() * sizeof(AdamSeg), cudaMemcpyHostToDevice,
                          ctx->st));
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  t->d_segs_wd = weight_decay;
  return NE_OK;
}

// Global gradient norm (train.m:805-826), times grad_scale; synchronises.
// The global gradient norm into t->norm_out ([0] norm, [1] factor): in sharded
// mode each rank's sum of squares (its parts + rank 0's replicated segments)
// is added over the ranks before the norm and the clip factor are formed.
static ne_status enqueue_norm(ne_ctx* ctx, float grad_scale, float grad_clip) {
  TrainState* t = ctx->train;
  const bool sharded = shard_mode(ctx);
  NE_LAUNCH(launch_sumsq_chunks(t->d_segs, t->d_chunks, t->nchunks, t->opt_partial, t->opt_ticket,
                                grad_scale, grad_clip, t->norm_out, ctx->st, sharded ? 1 : 0));
  if (!sharded) return NE_OK;
  ne_status s;
  if (ctx->comm->px) {
    if ((s = px_ready(ctx)) != NE_OK) return s;
    NE_CUDA(px_norm(ctx->comm->pxs.T, t->norm_out, ctx->d_status, ctx->st));
  } else if ((s = comm_fence_in(ctx)) != NE_OK ||
             (s = comm_allreduce(ctx, t->norm_out + 2, 1)) != NE_OK ||
             (s = comm_fence_out(ctx)) != NE_OK) {
    return s;
  }
  NE_LAUNCH(launch_norm_finish(t->norm_out, grad_scale, grad_clip, ctx->st));
  return NE_OK;
}

NE_API ne_status ne_train_grad_norm(ne_ctx* ctx, float grad_scale, float* h_norm) {
  if (!ctx || !ctx->train || !h_norm) return NE_ERR_STATE;
  TrainState* t = ctx->train;
  ne_status s = upload_segs(ctx, t->d_segs ? t->d_segs_wd : 0.f);
  if (s != NE_OK) return s;
  if ((s = enqueue_norm(ctx, grad_scale, 0.f)) != NE_OK) return s;
  NE_CUDA(cudaMemcpyAsync(h_norm, t->norm_out, sizeof(float), cudaMemcpyDeviceToHost, ctx->st));
  return ne_sync(ctx);
}

// AdamW over every trainable tensor (train.m:782-897, cpu_ops.h:266-303):
// gradients are multiplied by cfg->grad_scale (1/accum in the reference), the
// global norm of the result is clipped to cfg->grad_clip (when > 0), then
// decoupled AdamW with bias correction at step t (1-based); weight decay on
// matrices and the embedding, none on the gains.  Gradients are zeroed
// afterwards.  The norm and the clip factor stay on the device (no host round
// trip between them and the update); *h_grad_norm, when not NULL, receives
// the pre-clip norm, which makes this call wait for the step to finish.
NE_API ne_status ne_adamw_step(ne_ctx* ctx, const ne_adam_cfg* cfg, int t_step, float* h_grad_norm) {
  if (!ctx || !ctx->train || !cfg || t_step <= 0) return NE_ERR_INVALID;
  NE_FAULT_POINT(ctx, "ne_adamw_step");
  TrainState* t = ctx->train;
  ne_status s = upload_segs(ctx, cfg->weight_decay);
  if (s != NE_OK) return s;
  const float bc1 = 1.0f - std::pow(cfg->beta1, (float)t_step);
  const float bc2 = 1.0f - std::pow(cfg->beta2, (float)t_step);
  if ((s = enqueue_norm(ctx, cfg->grad_scale, cfg->grad_clip)) != NE_OK) return s;
  NE_LAUNCH(launch_adamw_chunks(t->d_segs, t->d_chunks, t->nchunks, cfg->lr, cfg->beta1,
                                cfg->beta2, cfg->eps, 1.0f / bc1, 1.0f / bc2, t->norm_out, ctx->st));
  if (shard_mode(ctx)) {
    // every rank needs the whole updated compute copy; the fp32 masters and
    // moments stay with their owners until ne_train_gather_state
    if (ctx->comm->px) {
      // the other ranks' updated parts arrive on the comm stream, bucket by
      // bucket, while the next micro-step's forward runs (each layer waits for
      // its bucket's event); the gradients may be zeroed once every rank has
      // published, i.e. finished reading them
      PxState& x = ctx->comm->pxs;
      if (x.fused) {
        // only this rank reads its owned parts: clear them now and let the
        // other ranks' next fused exchange add into them
        NE_CUDA(px_zero(t->grad_pool, x.d_chunks + x.zf_first, x.zf_count, ctx->st));
        NE_CUDA(px_signal_next(x.flags, PX_ZEROED, ctx->st));
        x.owned_clean = true;
      }
      NE_CUDA(px_signal(x.flags, PX_W16, ctx->st));
      if ((s = comm_fence_in(ctx)) != NE_OK) return s;
      for (int b = 0; b < (int)x.ag_ev.size(); ++b) {
        NE_CUDA(px_copy(x.T, x.d_wsrc, static_cast<char*>(ctx->wpool),
                        x.d_chunks + x.ag_bfirst[b], x.ag_bcount[b], PX_W16, px_ctas(),
                        ctx->d_status, ctx->comm->cs));
        NE_CUDA(cudaEventRecord(x.ag_ev[b], ctx->comm->cs));
      }
      NE_CUDA(px_wait(x.T, PX_W16, ctx->d_status, ctx->st));
    } else if ((s = gather_owned(ctx, 4)) != NE_OK) {
      return s;
    }
    t->state_gathered = false;
  }
  if ((s = ne_train_zero_grads(ctx)) != NE_OK) return s;
  if (h_grad_norm) {
    NE_CUDA(cudaMemcpyAsync(h_grad_norm, t->norm_out, sizeof(float), cudaMemcpyDeviceToHost,
                            ctx->st));
    return ne_sync(ctx);
  }
  return NE_OK;
}

// Sharded mode: all-gather the owned parts of the fp32 masters and both Adam
// moments (which = 0) and of the gradients (which = 1), so checkpoints and the
// state getters see whole tensors.  Collective: every rank calls it.
NE_API ne_status ne_train_gather_state(ne_ctx* ctx, int which) {
  if (!ctx || !ctx->train || which < 0 || which > 1) return NE_ERR_INVALID;
  NE_CUDA(cudaSetDevice(ctx->device));
  if (!shard_mode(ctx)) return NE_OK;
  ne_status s;
  if (ctx->comm->px) {
    // not on the step's path: NCCL broadcasts of each rank's parts (the
    // parts differ in length by a few elements, which rules out all-gather)
    TrainState* t = ctx->train;
    if ((s = comm_sync(ctx)) != NE_OK || (s = comm_fence_in(ctx)) != NE_OK ||
        (s = comm_group(ctx, true)) != NE_OK)
      return s;
    for (int a = (which == 1 ? 3 : 0); a < (which == 1 ? 4 : 3) && s == NE_OK; ++a) {
      for (const Seg& sg : t->segs) {
        if (a == 0 && sg.w16 == nullptr) continue;   // the gains' masters are all-gathered each step
        float* arr = a == 0 ? sg.w : a == 1 ? sg.m : a == 2 ? sg.v : sg.g;
        for (int p = 0; p < ctx->comm->world && s == NE_OK; ++p) {
          long long off, len;
          seg_owned(ctx, sg, p, &off, &len);
          if (len > 0) s = comm_broadcast(ctx, arr + off, (size_t)len * 4, p);
        }
      }
    }
    const ne_status e = comm_group(ctx, false);
    if (s != NE_OK) return s;
    if (e != NE_OK) return e;
    if ((s = comm_fence_out(ctx)) != NE_OK) return s;
    if (which == 0) t->state_gathered = true;
    return ne_sync(ctx);
  }
  if (which == 1) {
    if ((s = gather_owned(ctx, 3)) != NE_OK) return s;
  } else {
    for (int a = 0; a < 3; ++a)
      if ((s = gather_owned(ctx, a)) != NE_OK) return s;
    ctx->train->state_gathered = true;
  }
  return ne_sync(ctx);
}

// The ZeRO-1 partition of the peer-memory exchange (host arithmetic only).
NE_API ne_status ne_shard_range(long long n, int world, int rank, long long* off, long long* len) {
  if (n < 0 || world < 1 || rank < 0 || rank >= world || !off || !len) return NE_ERR_INVALID;
  ne_status fs;
  if (fault_point("ne_shard_range", &fs)) return fs;
  px_part(n, world, rank, off, len);
  return NE_OK;
}

// Learning-rate schedule of train.m:851-858: linear warmup, then cosine decay
// to min_lr_frac * max_lr.
NE_API float ne_lr_schedule(int step, float max_lr, int warmup_steps, int total_steps,
                            float min_lr_frac) {
  if (step < warmup_steps) return max_lr * ((float)(step + 1)) / warmup_steps;
  const float decay_ratio = (float)(step - warmup_steps) / (float)(total_steps - warmup_steps);
  const float min_lr = max_lr * min_lr_frac;
  // cosf of a double product, as train.m:857 writes cosf(M_PI * decay_ratio)
  return min_lr +
         0.5f * (1.0f + cosf((float)(3.14159265358979323846 * (double)decay_ratio))) *
             (max_lr - min_lr);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// v4 checkpoint with the full training state (train.m:97-165): the layout is
// the reference's byte for byte; the fp32 masters and both Adam moments come
// from the device pools, W1/W3 (and their moments) are separated from the
// interleaved device layout.  When the model has QK-norm, the trailing "QKN1"
// block follows (q_norm, k_norm per layer, then m, v of each), which v4
// readers ignore.
namespace {

struct TensorRef {
  int seg;          // index into TrainState::segs
  size_t off, n;    // element offset inside the segment, element count
  int w13;          // 0 plain, 1 = W1 rows, 2 = W3 rows of the interleaved block
};

// The nine v4 tensors of layer l in file order.
std::vector<TensorRef> layer_tensors(const ne_ctx* ctx, int l) {
  const ne_model_cfg& m = ctx->cfg;
  const size_t D = m.dim, F = m.hidden, qd = (size_t)m.n_heads * m.head_dim,
               kvd = (size_t)m.kv_heads * m.head_dim;
  const int s0 = ctx->train->P[l].seg0;
  return {{s0, 0, qd * D, 0},          {s0, qd * D, kvd * D, 0}, {s0, (qd + kvd) * D, kvd * D, 0},
          {s0 + 1, 0, D * qd, 0},      {s0 + 2, 0, F * D, 1},    {s0 + 3, 0, D * F, 0},
          {s0 + 2, 0, F * D, 2},       {s0 + 4, 0, D, 0},        {s0 + 5, 0, D, 0}};
}

// which: 0 weights (masters / gains), 1 Adam m, 2 Adam v, 3 gradients
float* seg_array(const Seg& sg, int which) {
  return which == 0 ? sg.w : which == 1 ? sg.m : which == 2 ? sg.v : sg.g;
}

// Copy a tensor (which as in seg_array) between the device and host[n].
ne_status xfer(ne_ctx* ctx, const TensorRef& r, int which, float* host, bool to_host) {
  const Seg& sg = ctx->train->segs[r.seg];
  float* dev = seg_array(sg, which);
  if (!r.w13) {
    NE_CUDA(cudaMemcpy(to_host ? (void*)host : (void*)(dev + r.off),
                       to_host ? (const void*)(dev + r.off) : (const void*)host, r.n * 4,
                       to_host ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice));
    return NE_OK;
  }
  // W1 / W3 rows live in 16-row blocks of the [2F, D] device array
  const size_t D = ctx->cfg.dim, F = ctx->cfg.hidden;
  const bool is_w3 = r.w13 == 2;
  for (size_t f0 = 0; f0 < F; f0 += 16) {
    const size_t rows = std::min<size_t>(16, F - f0);
    float* d = dev + w13_row(f0, is_w3) * D;
    float* h = host + f0 * D;
    NE_CUDA(cudaMemcpy(to_host ? (void*)h : (void*)d, to_host ? (const void*)d : (const void*)h,
                       rows * D * 4, to_host ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice));
  }
  return NE_OK;
}

}  // namespace

extern "C" NE_API ne_status ne_save_ckpt_v4(ne_ctx* ctx, const char* path, const ne_ckpt_info* info) {
  if (!ctx || !path) return NE_ERR_INVALID;
  NE_FAULT_POINT(ctx, "ne_save_ckpt_v4");
  if (!ctx->train) return fail(ctx, NE_ERR_STATE, "ne_save_ckpt_v4 needs the training state");
  if (!ctx->train->state_gathered)
    return fail(ctx, NE_ERR_STATE, "sharded optimizer state: ne_train_gather_state on every rank first");
  const ne_model_cfg& m = ctx->cfg;
  TrainState* t = ctx->train;
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  FILE* f = fopen(path, "wb");
  if (!f) return fail(ctx, NE_ERR_IO, std::string("cannot open ") + path);
  struct Closer {
    FILE* f;
    ~Closer() {
      if (f) fclose(f);
    }
  } closer{f};
  CkptHdr h;
  std::memset(&h, 0, sizeof(h));
  h.magic = kCkptMagic;
  h.version = 4;
  h.n_layers = m.n_layers;
  h.vocab_size = m.vocab;
  h.dim = m.dim;
  h.hidden_dim = m.hidden;
  h.n_heads = m.n_heads;
  h.seq_len = t->S;
  h.kv_heads = m.kv_heads;
  h.head_dim = m.head_dim;
  h.q_dim = m.n_heads * m.head_dim;
  if (info) {
    h.step = info->step;
    h.total_steps = info->total_steps;
    if (info->seq_len > 0) h.seq_len = info->seq_len;
    h.lr = info->lr;
    h.loss = info->loss;
    h.cum_compile = info->cum_compile;
    h.cum_train = info->cum_train;
    h.cum_wall = info->cum_wall;
    h.cum_steps = info->cum_steps;
    h.cum_batches = info->cum_batches;
    h.adam_t = info->adam_t;
  }
  auto put = [&](const std::vector<float>& v, size_t n) { return fwrite(v.data(), 4, n, f) == n; };
  if (fwrite(&h, sizeof(h), 1, f) != 1) return fail(ctx, NE_ERR_IO, "write failed");
  std::vector<float> buf;
  ne_status s;
  for (int l = 0; l < m.n_layers; ++l) {
    const std::vector<TensorRef> tr = layer_tensors(ctx, l);
    auto emit = [&](const TensorRef& r, int which) -> ne_status {
      buf.resize(r.n);
      ne_status e = xfer(ctx, r, which, buf.data(), true);
      if (e != NE_OK) return e;
      return put(buf, r.n) ? NE_OK : fail(ctx, NE_ERR_IO, "write failed");
    };
    for (const TensorRef& r : tr)          // the nine weights
      if ((s = emit(r, 0)) != NE_OK) return s;
    for (const TensorRef& r : tr)          // then (m, v) of each
      if ((s = emit(r, 1)) != NE_OK || (s = emit(r, 2)) != NE_OK) return s;
  }
  for (int k = 0; k < 2; ++k) {   // rms_final, then the embedding: value, m, v
    const Seg& sg = t->segs[t->segs.size() - 2 + k];
    for (int which = 0; which < 3; ++which) {
      buf.resize((size_t)sg.n);
      NE_CUDA(cudaMemcpy(buf.data(), seg_array(sg, which), (size_t)sg.n * 4, cudaMemcpyDeviceToHost));
      if (!put(buf, (size_t)sg.n)) return fail(ctx, NE_ERR_IO, "write failed");
    }
  }
  if (m.qk_norm) {
    const int nl = m.n_layers, hd = m.head_dim;
    if (fwrite("QKN1", 1, 4, f) != 4 || fwrite(&nl, 4, 1, f) != 1 || fwrite(&hd, 4, 1, f) != 1)
      return fail(ctx, NE_ERR_IO, "write failed");
    for (int l = 0; l < nl; ++l) {
      const int s0 = t->P[l].seg0;
      const Seg* qk[2] = {&t->segs[s0 + 6], &t->segs[s0 + 7]};
      buf.resize(hd);
      auto emit = [&](const Seg& sg, int which) -> ne_status {
        NE_CUDA(cudaMemcpy(buf.data(), seg_array(sg, which), (size_t)hd * 4,
                           cudaMemcpyDeviceToHost));
        return put(buf, hd) ? NE_OK : fail(ctx, NE_ERR_IO, "write failed");
      };
      // q_norm, k_norm, then (m, v) of each
      if ((s = emit(*qk[0], 0)) != NE_OK || (s = emit(*qk[1], 0)) != NE_OK) return s;
      for (int i = 0; i < 2; ++i)
        if ((s = emit(*qk[i], 1)) != NE_OK || (s = emit(*qk[i], 2)) != NE_OK) return s;
    }
  }
  if (fflush(f) != 0) return fail(ctx, NE_ERR_IO, "write failed");
  return NE_OK;
}

namespace ne {

ne_status train_ckpt_load(ne_ctx* ctx, const char* path, ne_ckpt_info* info, bool* handled) {
  *handled = false;
  if (!ctx->train) return NE_OK;
  *handled = true;
  const ne_model_cfg& m = ctx->cfg;
  TrainState* t = ctx->train;
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  FILE* f = fopen(path, "rb");
  if (!f) return NE_ERR_IO;
  struct Closer {
    FILE* f;
    ~Closer() {
      if (f) fclose(f);
    }
  } closer{f};
  CkptHdr h;
  if (fread(&h, sizeof(h), 1, f) != 1) return NE_ERR_FORMAT;
  if (h.magic != kCkptMagic || h.version != 4) return NE_ERR_FORMAT;
  if (h.n_layers != m.n_layers || h.vocab_size != m.vocab || h.dim != m.dim ||
      h.hidden_dim != m.hidden || h.n_heads != m.n_heads || h.kv_heads != m.kv_heads ||
      h.head_dim != m.head_dim || h.q_dim != m.n_heads * m.head_dim)
    return NE_ERR_FORMAT;
  auto get = [&](std::vector<float>& v, size_t n) {
    v.resize(n);
    return fread(v.data(), 4, n, f) == n;
  };
  std::vector<float> buf;
  ne_status s;
  for (int l = 0; l < m.n_layers; ++l) {
    const std::vector<TensorRef> tr = layer_tensors(ctx, l);
    for (const TensorRef& r : tr) {
      if (!get(buf, r.n)) return NE_ERR_FORMAT;
      if ((s = xfer(ctx, r, 0, buf.data(), false)) != NE_OK) return s;
    }
    for (const TensorRef& r : tr)
      for (int which = 1; which <= 2; ++which) {
        if (!get(buf, r.n)) return NE_ERR_FORMAT;
        if ((s = xfer(ctx, r, which, buf.data(), false)) != NE_OK) return s;
      }
  }
  for (int k = 0; k < 2; ++k) {
    const Seg& sg = t->segs[t->segs.size() - 2 + k];
    for (int which = 0; which < 3; ++which) {
      if (!get(buf, (size_t)sg.n)) return NE_ERR_FORMAT;
      NE_CUDA(cudaMemcpy(seg_array(sg, which), buf.data(), (size_t)sg.n * 4, cudaMemcpyHostToDevice));
    }
  }
  bool has_qk = false;
  char magic[4];
  if (fread(magic, 1, 4, f) == 4 && std::memcmp(magic, "QKN1", 4) == 0) {
    int nl = 0, hd = 0;
    if (fread(&nl, 4, 1, f) != 1 || fread(&hd, 4, 1, f) != 1) return NE_ERR_FORMAT;
    if (nl != m.n_layers || hd != m.head_dim || !m.qk_norm) return NE_ERR_FORMAT;
    for (int l = 0; l < nl; ++l) {
      const int s0 = t->P[l].seg0;
      const Seg* qk[2] = {&t->segs[s0 + 6], &t->segs[s0 + 7]};
      for (int i = 0; i < 2; ++i) {
        if (!get(buf, hd)) return NE_ERR_FORMAT;
        NE_CUDA(cudaMemcpy(qk[i]->w, buf.data(), (size_t)hd * 4, cudaMemcpyHostToDevice));
      }
      for (int i = 0; i < 2; ++i)
        for (int which = 1; which <= 2; ++which) {
          if (!get(buf, hd)) return NE_ERR_FORMAT;
          NE_CUDA(cudaMemcpy(seg_array(*qk[i], which), buf.data(), (size_t)hd * 4,
                             cudaMemcpyHostToDevice));
        }
    }
    has_qk = true;
  } else if (m.qk_norm) {
    // a reference checkpoint has no QK-norm block: unit gains, zero moments
    std::vector<float> ones(m.head_dim, 1.0f), zeros(m.head_dim, 0.0f);
    for (int l = 0; l < m.n_layers; ++l) {
      const int s0 = t->P[l].seg0;
      for (int i = 0; i < 2; ++i) {
        const Seg& sg = t->segs[s0 + 6 + i];
        NE_CUDA(cudaMemcpy(sg.w, ones.data(), (size_t)m.head_dim * 4, cudaMemcpyHostToDevice));
        NE_CUDA(cudaMemcpy(sg.m, zeros.data(), (size_t)m.head_dim * 4, cudaMemcpyHostToDevice));
        NE_CUDA(cudaMemcpy(sg.v, zeros.data(), (size_t)m.head_dim * 4, cudaMemcpyHostToDevice));
      }
    }
  }
  if ((s = ne_train_sync_weights(ctx)) != NE_OK) return s;
  if (info) {
    info->step = h.step;
    info->total_steps = h.total_steps;
    info->seq_len = h.seq_len;
    info->adam_t = h.adam_t;
    info->lr = h.lr;
    info->loss = h.loss;
    info->cum_compile = h.cum_compile;
    info->cum_train = h.cum_train;
    info->cum_wall = h.cum_wall;
    info->cum_steps = h.cum_steps;
    info->cum_batches = h.cum_batches;
    info->has_qk_norm = has_qk ? 1 : 0;
  }
  t->state_gathered = true;   // every part came from the file
  return NE_OK;
}

}  // namespace ne

// Copy one layer's tensors to host buffers in the v4 layout: which = 0
// gradients, 1 fp32 master weights, 2 Adam m, 3 Adam v.  Layer -1 =
// (rms_final, embedding) into (h_rms_att, h_wq).  Any pointer may be NULL.
extern "C" NE_API ne_status ne_train_get_layer(ne_ctx* ctx, int layer, int which, float* h_wq,
                                               float* h_wk, float* h_wv, float* h_wo,
                                               float* h_w1, float* h_w2, float* h_w3,
                                               float* h_rms_att, float* h_rms_ffn,
                                               float* h_q_norm, float* h_k_norm) {
  if (!ctx || !ctx->train || which < 0 || which > 3) return NE_ERR_INVALID;
  TrainState* t = ctx->train;
  const ne_model_cfg& m = ctx->cfg;
  if (layer < -1 || layer >= m.n_layers) return NE_ERR_INVALID;
  if (which != 0 && !t->state_gathered)   // which 0 = gradients (see ne_train_gather_state)
    return fail(ctx, NE_ERR_STATE, "sharded optimizer state: ne_train_gather_state on every rank first");
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  const int arr = which == 0 ? 3 : which - 1;   // seg_array selector
  ne_status s;
  if (layer == -1) {
    float* dst[2] = {h_rms_att, h_wq};
    for (int k = 0; k < 2; ++k) {
      const Seg& sg = t->segs[t->segs.size() - 2 + k];
      if (dst[k])
        NE_CUDA(cudaMemcpy(dst[k], seg_array(sg, arr), (size_t)sg.n * 4, cudaMemcpyDeviceToHost));
    }
    return NE_OK;
  }
  const std::vector<TensorRef> tr = layer_tensors(ctx, layer);
  float* dst[9] = {h_wq, h_wk, h_wv, h_wo, h_w1, h_w2, h_w3, h_rms_att, h_rms_ffn};
  for (int k = 0; k < 9; ++k)
    if (dst[k] && (s = xfer(ctx, tr[k], arr, dst[k], true)) != NE_OK) return s;
  if (m.qk_norm) {
    const int s0 = t->P[layer].seg0;
    float* qk[2] = {h_q_norm, h_k_norm};
    for (int i = 0; i < 2; ++i)
      if (qk[i])
        NE_CUDA(cudaMemcpy(qk[i], seg_array(t->segs[s0 + 6 + i], arr), (size_t)m.head_dim * 4,
                           cudaMemcpyDeviceToHost));
  }
  return NE_OK;
}

// Causal GQA scaled-dot-product attention on caller-owned device buffers (the
// reference's sdpaFwd core, mil_dynamic.h:184-198): Q [B*S][Hq*hd] bf16 (token
// major), K / V [B][Hkv][S][hd] bf16; out [B*S][Hq*hd] bf16; lse (optional)
// [B][Hq][S] fp32 row log-sum-exp of the scaled scores, log2 domain.
extern "C" NE_API ne_status ne_sdpa_fwd_device(ne_ctx* ctx, const void* d_q, const void* d_k,
                                               const void* d_v, int B, int S, void* d_out,
                                               float* d_lse) {
  if (!ctx || !d_q || !d_k || !d_v || !d_out || B <= 0 || S <= 0) return NE_ERR_INVALID;
  const ne_model_cfg& m = ctx->cfg;
  NE_CUDA(cudaSetDevice(ctx->device));
  const auto* q = static_cast<const __nv_bfloat16*>(d_q);
  const auto* k = static_cast<const __nv_bfloat16*>(d_k);
  const auto* v = static_cast<const __nv_bfloat16*>(d_v);
  auto* o = static_cast<__nv_bfloat16*>(d_out);
  if ((m.head_dim == 128 || (m.head_dim == 64 && attn_tc64())) && attn_tc_enabled())
    NE_LAUNCH(launch_attn_fwd_tc(q, k, v, B, S, m.n_heads, m.kv_heads, m.head_dim, S, o, d_lse,
                                 ctx->d_status, ctx->st));
  else
    NE_LAUNCH(launch_prefill_attn_bf16(q, k, v, B, S, 0, m.n_heads, m.kv_heads, m.head_dim, S, o,
                                       ctx->st, d_lse));
  return NE_OK;
}

// Vocabulary compaction (vocab_map_build / vocab_compact_embed /
// vocab_scatter_grads, cpu_ops.h:385-431): the classifier and its softmax run
// over the CV rows h_c2f[0..CV) of the tied embedding (the tokens present in
// the training data, in increasing id order when built as the reference does);
// targets must be among them.  Their gradient is added back into the full
// embedding gradient.  CV = 0 (or NULL) restores the full vocabulary.
extern "C" NE_API ne_status ne_train_set_vocab_map(ne_ctx* ctx, const int32_t* h_c2f, int CV) {
  if (!ctx || !ctx->train) return NE_ERR_STATE;
  TrainState* t = ctx->train;
  const ne_model_cfg& m = ctx->cfg;
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  for (void* p : {(void*)t->d_c2f, (void*)t->d_f2c, (void*)t->Ec, (void*)t->dEc})
    if (p) NE_CUDA(cudaFree(p));
  t->d_c2f = t->d_f2c = nullptr;
  t->Ec = nullptr;
  t->dEc = nullptr;
  t->CV = t->CVp = 0;
  for (cudaGraphExec_t& g : t->step_graphs) {   // the captured steps used the previous classifier
    if (g) NE_CUDA(cudaGraphExecDestroy(g));
    g = nullptr;
  }
  if (!h_c2f || CV <= 0) return NE_OK;
  if (CV > m.vocab) return fail(ctx, NE_ERR_INVALID, "vocab map larger than the vocabulary");
  std::vector<int32_t> f2c(m.vocab, -1);
  for (int c = 0; c < CV; ++c) {
    const int32_t v = h_c2f[c];
    if (v < 0 || v >= m.vocab || f2c[v] >= 0)
      return fail(ctx, NE_ERR_INVALID, "vocab map entries must be distinct ids < vocab");
    f2c[v] = c;
  }
  const int CVp = (CV + 63) / 64 * 64;
  const size_t D = m.dim;
  ne_status s;
  if ((s = dalloc(ctx, &t->d_c2f, (size_t)CV)) != NE_OK || (s = dalloc(ctx, &t->d_f2c, (size_t)m.vocab)) ||
      (s = dalloc(ctx, &t->Ec, (size_t)CVp * D)) || (s = dalloc(ctx, &t->dEc, (size_t)CVp * D)))
    return s;
  NE_CUDA(cudaMemcpy(t->d_c2f, h_c2f, (size_t)CV * 4, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(t->d_f2c, f2c.data(), (size_t)m.vocab * 4, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemset(t->Ec, 0, (size_t)CVp * D * 2));     // padding rows stay zero
  NE_CUDA(cudaMemset(t->dEc, 0, (size_t)CVp * D * 4));
  // padding columns of dlogits are never written by the cross-entropy kernel
  NE_CUDA(cudaMemset(t->dlogits, 0, (size_t)t->Mc * m.vocab * 2));
  t->CV = CV;
  t->CVp = CVp;
  return NE_OK;
}
