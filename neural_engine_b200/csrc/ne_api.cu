// ne_api.cu -- C ABI of libne.so: context, weights, KV cache, token loop.
//
// Per-layer flow of one decode step (B sequences at one position), the
// device counterpart of tools/generate.py:141-200 (and of the forward half
// of train.m:413-488):
//   embed_rmsnorm                       x = E[tok]; xn = rmsnorm(x, g_att[0])
//   for each layer:
//     GEMM  Wqkv . xn   (swap-AB, split-K partials)   generate.py:151-153
//     qkv_post  (sum splits, QK-norm, RoPE, KV append) generate.py:156-162
//     decode_attention (split-KV over the fp16 cache)  generate.py:164-181
//     GEMM  Wo . attn                                  generate.py:184
//     resid_rmsnorm  x += alpha*sum; xn = rmsnorm(x, g_ffn)
//     GEMM  W13 . xn                                   generate.py:188-189
//     swiglu_split                                     generate.py:190
//     GEMM  W2 . gate                                  generate.py:191
//     resid_rmsnorm  x += alpha*sum; xn = rmsnorm(x, next gain)
//   GEMM  E . xn  -> logits (tied LM head)             generate.py:194-195
//   argmax -> next token (+ device position/step advance)  generate.py:200
// The whole step is captured once per batch size as a CUDA graph and
// replayed; the position lives in device memory so replays need no host work.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/ne.h"
#include "ne_comm.h"
#include "ne_ctx.h"
#include "ne_device.cuh"
#include "ne_internal.h"
#include "ne_fault.h"

using namespace ne;

namespace {

// Decode-GEMM helper (weight-major, batch <= 256 rows in one N tile):
//   out[rows][n_out] += alpha * act[rows, K] . W[n_out, K]^T
// through the TMA add, split-K across the SMs (the partial sums meet in L2).
GemmCall decode_call(ne_ctx* ctx, const __nv_bfloat16* W, int n_out, int K,
                     const __nv_bfloat16* act, long long ld_act, int rows, float* out,
                     float alpha) {
  GemmCall c;
  c.A = W; c.lda = K; c.M = n_out;
  c.B = act; c.ldb = ld_act; c.N = rows;
  c.K = K;
  c.epi = EPI_F32T_ADD;
  c.out = out; c.ld = n_out;
  c.alpha = alpha;
  c.splits = 0;
  c.prefetch_a = 1;   // A = weights: loaded while the producer of `act` finishes
  // Batch tiles of 128 rows: against one 256-row tile they take half the K
  // splits for the same CTA count, so half the partial sums go through the
  // L2 add (measured at B 256: 4.71 against 4.79 ms per step; 64-row tiles
  // 4.88).  NE_DECODE_BN = 64 / 128 / 256 overrides (tuning).
  static const int bn_cfg = [] {
    const char* e = std::getenv("NE_DECODE_BN");
    const int v = e ? std::atoi(e) : 128;
    return (v == 64 || v == 128 || v == 256) ? v : 128;
  }();
  if (rows > bn_cfg) c.bn = bn_cfg;
  c.splits = gemm_pick_splits(c, ctx->num_sms);
  return c;
}

ne_status gemm_decode(ne_ctx* ctx, const __nv_bfloat16* W, int n_out, int K,
                      const __nv_bfloat16* act, long long ld_act, int rows, float* out,
                      float alpha) {
  const GemmCall c = decode_call(ctx, W, n_out, K, act, ld_act, rows, out, alpha);
  NE_LAUNCH(gemm_run(c, ctx->d_status, ctx->st));
  return NE_OK;
}

// The W1/W3 projection of a decode step writes the SwiGLU gate directly
// (EPI_SWIGLU_T) when its tiles fill the SMs without splitting K (B > 128 on
// 148 SMs): no fp32 h1/h3 sums in HBM and no separate SwiGLU kernel.
// NE_DECODE_SWIGLU=0 keeps the split projection + swiglu_split pair.
bool decode_swiglu_fused(ne_ctx* ctx, int rows) {
  static const bool on = [] {
    const char* e = std::getenv("NE_DECODE_SWIGLU");
    return !(e && e[0] == '0');
  }();
  const ne_model_cfg& m = ctx->cfg;
  if (!on || m.hidden % 16) return false;
  const GemmCall c =
      decode_call(ctx, ctx->L[0].w13, 2 * m.hidden, m.dim, ctx->xn, m.dim, rows, ctx->part, 1.f);
  return c.splits == 1;
}

ne_status gemm_decode_swiglu(ne_ctx* ctx, const __nv_bfloat16* W13, const __nv_bfloat16* act,
                             long long ld_act, int rows, __nv_bfloat16* gate) {
  const ne_model_cfg& m = ctx->cfg;
  GemmCall c = decode_call(ctx, W13, 2 * m.hidden, m.dim, act, ld_act, rows, nullptr, 1.f);
  c.epi = EPI_SWIGLU_T;
  c.out = gate;
  c.ld = m.hidden;
  c.splits = 1;
  NE_LAUNCH(gemm_run(c, ctx->d_status, ctx->st));
  return NE_OK;
}

// The greedy LM head: act . E^T reduced on the fly to each row's best
// (logit, id) key in ctx->argmax_keys (launch_argmax_keys finishes the step).
ne_status gemm_lm_head_argmax(ne_ctx* ctx, const __nv_bfloat16* act, long long ld_act, int rows) {
  GemmCall c;
  c.A = ctx->embed; c.lda = ctx->cfg.dim; c.M = ctx->cfg.vocab;
  c.B = act; c.ldb = ld_act; c.N = rows;
  c.K = ctx->cfg.dim;
  c.epi = EPI_ARGMAX_T;
  c.aux1 = ctx->argmax_keys;
  c.splits = 1;
  c.prefetch_a = 1;
  NE_LAUNCH(gemm_run(c, ctx->d_status, ctx->st));
  return NE_OK;
}

// The tied LM head: out[rows][V] = act . E^T (plain transposed store; the
// vocabulary gives enough tiles without splitting K).
ne_status gemm_lm_head(ne_ctx* ctx, const __nv_bfloat16* act, long long ld_act, int rows,
                       float* out) {
  GemmCall c;
  c.A = ctx->embed; c.lda = ctx->cfg.dim; c.M = ctx->cfg.vocab;
  c.B = act; c.ldb = ld_act; c.N = rows;
  c.K = ctx->cfg.dim;
  c.epi = EPI_F32T;
  c.out = out; c.ld = ctx->cfg.vocab; c.split_stride = (long long)rows * ctx->cfg.vocab;
  c.splits = 1;
  c.prefetch_a = 1;
  NE_LAUNCH(gemm_run(c, ctx->d_status, ctx->st));
  return NE_OK;
}

ne_status gemm_tokens(ne_ctx* ctx, const __nv_bfloat16* act, long long ld_act, int rows,
                      const __nv_bfloat16* W, int n_out, int K, int epi, void* out, long long ld,
                      float alpha) {
  GemmCall c;
  c.A = act; c.lda = ld_act; c.M = rows;
  c.B = W; c.ldb = K; c.N = n_out;
  c.K = K;
  c.epi = epi;
  c.out = out; c.ld = ld; c.split_stride = 0;
  c.alpha = alpha;
  c.splits = 1;
  c.bn = 256;
  NE_LAUNCH(gemm_run(c, ctx->d_status, ctx->st));
  return NE_OK;
}

ne_status check_status(ne_ctx* ctx) {
  int h = 0;
  NE_CUDA(cudaMemcpy(&h, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (h == DEV_ERR_TIMEOUT) return fail(ctx, NE_ERR_TIMEOUT, "a kernel wait timed out");
  if (h == DEV_ERR_BOUNDS) return fail(ctx, NE_ERR_BOUNDS, "token id or position out of range");
  if (h != 0) return fail(ctx, NE_ERR_CUDA, "device status " + std::to_string(h));
  return NE_OK;
}

// Record an event closing a kernel group when profiling is on.
void prof_mark(ne_ctx* ctx, int group) {
  if (!ctx->prof_on || ctx->prof_n >= (int)ctx->prof_events.size()) return;
  cudaEventRecord(ctx->prof_events[ctx->prof_n], ctx->st);
  ctx->prof_groups[ctx->prof_n] = group;
  ctx->prof_n++;
}

bool ready(ne_ctx* ctx) { return ctx->global_set && ctx->layer_set_count == (unsigned)ctx->cfg.n_layers; }

// ------------------------------------------------------------------ decode step
// Enqueue one step for B sequences.  Token input: ctx->tok; position: state[0].
ne_status enqueue_decode_step(ne_ctx* ctx, int B, int32_t* d_out_tokens, bool keep_logits) {
  const ne_model_cfg& m = ctx->cfg;
  const int D = m.dim, F = m.hidden, Hq = m.n_heads, Hkv = m.kv_heads, hd = m.head_dim;
  const int qkv_dim = ctx->qkv_dim(), q_dim = ctx->q_dim();
  ne_status s;
  prof_mark(ctx, 9);
  NE_LAUNCH(launch_embed_rmsnorm(ctx->tok, ctx->embed, 0, m.vocab, D, ctx->L[0].rms_att, m.rms_eps,
                                 ctx->x, ctx->xn, B, ctx->d_status, ctx->st));
  prof_mark(ctx, 9);
  const size_t kv_layer = ctx->layer_kv_elems();
  const bool swiglu_fused = decode_swiglu_fused(ctx, B);
  // ctx->part holds the QKV and (unless fused) W1/W3 sums (zero between uses:
  // their consumers clear what they read); the Wo and W2 projections add
  // alpha * acc straight into the fp32 residual stream x.
  for (int l = 0; l < m.n_layers; ++l) {
    const LayerW& w = ctx->L[l];
    if ((s = gemm_decode(ctx, w.wqkv, qkv_dim, D, ctx->xn, D, B, ctx->part, 1.f)) != NE_OK)
      return s;
    prof_mark(ctx, 0);
    __half* kc = ctx->kcache + kv_layer * l;
    __half* vc = ctx->vcache + kv_layer * l;
    NE_LAUNCH(launch_qkv_post(ctx->part, 1, 0, B, 1, ctx->state, 0, Hq, Hkv, hd,
                              m.qk_norm ? w.q_norm : nullptr, m.qk_norm ? w.k_norm : nullptr,
                              m.qk_eps, ctx->rope_cs, ctx->q, 0, kc, vc, ctx->max_seq,
                              ctx->d_status, ctx->st, 0, 1));
    prof_mark(ctx, 1);
    NE_LAUNCH(launch_decode_attn(ctx->q, kc, vc, B, Hq, Hkv, hd, ctx->max_seq, ctx->state,
                                 ctx->attn_po, ctx->attn_ml, ctx->attn_cnt, ctx->attn,
                                 ctx->d_status, ctx->st));
    prof_mark(ctx, 2);
    if ((s = gemm_decode(ctx, w.wo, D, q_dim, ctx->attn, q_dim, B, ctx->x, m.res_alpha)) != NE_OK)
      return s;
    prof_mark(ctx, 3);
    NE_LAUNCH(launch_resid_rmsnorm(ctx->x, nullptr, 0, 0, 1.f, D, w.rms_ffn, m.rms_eps, ctx->xn, B,
                                   ctx->st));
    prof_mark(ctx, 4);
    if (swiglu_fused) {
      if ((s = gemm_decode_swiglu(ctx, w.w13, ctx->xn, D, B, ctx->gate)) != NE_OK) return s;
      prof_mark(ctx, 5);
    } else {
      if ((s = gemm_decode(ctx, w.w13, 2 * F, D, ctx->xn, D, B, ctx->part, 1.f)) != NE_OK)
        return s;
      prof_mark(ctx, 5);
      NE_LAUNCH(launch_swiglu_split(ctx->part, 1, 0, B, F, ctx->gate, ctx->st, 1));
      prof_mark(ctx, 6);
    }
    if ((s = gemm_decode(ctx, w.w2, D, F, ctx->gate, F, B, ctx->x, m.res_alpha)) != NE_OK) return s;
    prof_mark(ctx, 7);
    const float* next_g = (l + 1 < m.n_layers) ? ctx->L[l + 1].rms_att : ctx->rms_final;
    NE_LAUNCH(launch_resid_rmsnorm(ctx->x, nullptr, 0, 0, 1.f, D, next_g, m.rms_eps, ctx->xn, B,
                                   ctx->st));
    prof_mark(ctx, 4);
  }
  if (keep_logits) {
    if ((s = gemm_lm_head(ctx, ctx->xn, D, B, ctx->logits)) != NE_OK) return s;
    prof_mark(ctx, 8);
    NE_LAUNCH(launch_argmax(ctx->logits, B, m.vocab, ctx->tok, d_out_tokens, ctx->state, 1,
                            ctx->st));
    ctx->launches++;  // state advance kernel
  } else {
    // greedy: the LM head keeps only each row's best (logit, id); no logits in HBM
    if ((s = gemm_lm_head_argmax(ctx, ctx->xn, D, B)) != NE_OK) return s;
    prof_mark(ctx, 8);
    NE_LAUNCH(launch_argmax_keys(ctx->argmax_keys, B, ctx->tok, d_out_tokens, ctx->state,
                                 ctx->st));
  }
  prof_mark(ctx, 9);
  return NE_OK;
}

ne_status get_graph(ne_ctx* ctx, int B, bool keep_logits, DecodeGraph** out) {
  const int key = 2 * B + (keep_logits ? 1 : 0);
  auto it = ctx->graphs.find(key);
  if (it != ctx->graphs.end()) {
    *out = &it->second;
    return NE_OK;
  }
  DecodeGraph g;
  ctx->launches = 0;
  NE_CUDA(cudaStreamBeginCapture(ctx->st, cudaStreamCaptureModeThreadLocal));
  ne_status s = enqueue_decode_step(ctx, B, ctx->out_tokens, keep_logits);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->st, &graph);
  if (s != NE_OK) {
    if (graph) cudaGraphDestroy(graph);
    return s;
  }
  if (e != cudaSuccess)
    return fail(ctx, NE_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
  e = cudaGraphInstantiate(&g.exec, graph, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(graph);
    return fail(ctx, NE_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
  }
  g.graph = graph;
  g.kernels = ctx->launches;
  ctx->graphs[key] = g;
  *out = &ctx->graphs[key];
  return NE_OK;
}

// ------------------------------------------------------------------ prefill
// Prompt tokens d_tokens [B, S] at positions pos0..pos0+S-1; next token per
// sequence to d_next [B]; last-position logits stay in ctx->logits [B, V].
ne_status enqueue_prefill(ne_ctx* ctx, const int32_t* d_tokens, int B, int S, int pos0,
                          int32_t* d_next) {
  const ne_model_cfg& m = ctx->cfg;
  const int D = m.dim, F = m.hidden, Hq = m.n_heads, Hkv = m.kv_heads, hd = m.head_dim;
  const int qkv_dim = ctx->qkv_dim(), q_dim = ctx->q_dim();
  const size_t kv_layer = ctx->layer_kv_elems();
  const size_t kv_seq = (size_t)Hkv * ctx->max_seq * hd;
  ne_status s;
  // A prompt that starts at position 0 with head_dim 128 runs its attention on
  // the tcgen05 kernel (fp16 operands, TMEM accumulators); a continuation
  // (pos0 > 0, keys before the chunk already cached) and other head sizes on
  // the mma.sync kernel.  NE_PREFILL_TC=0 keeps the mma.sync kernel throughout.
  static const bool tc_on = [] {
    const char* e = getenv("NE_PREFILL_TC");
    return !(e && e[0] == '0');
  }();
  const bool tc_attn = tc_on && pos0 == 0 && (hd == 128 || (hd == 64 && attn_tc64()));
  const int seqs_per_chunk = std::max(1, ctx->pf_rows / S);
  for (int b0 = 0; b0 < B; b0 += seqs_per_chunk) {
    const int nb = std::min(seqs_per_chunk, B - b0);
    const int rows = nb * S;
    NE_LAUNCH(launch_embed_rmsnorm(d_tokens + (size_t)b0 * S, ctx->embed, 0, m.vocab, D,
                                   ctx->L[0].rms_att, m.rms_eps, ctx->pf_x, ctx->pf_xn, rows,
                                   ctx->d_status, ctx->st));
    for (int l = 0; l < m.n_layers; ++l) {
      const LayerW& w = ctx->L[l];
      __half* kc = ctx->kcache + kv_layer * l + kv_seq * b0;
      __half* vc = ctx->vcache + kv_layer * l + kv_seq * b0;
      if ((s = gemm_tokens(ctx, ctx->pf_xn, D, rows, w.wqkv, qkv_dim, D, EPI_F32, ctx->pf_qkv,
                           qkv_dim, 1.f)) != NE_OK)
        return s;
      NE_LAUNCH(launch_qkv_post(ctx->pf_qkv, 1, 0, rows, S, nullptr, pos0, Hq, Hkv, hd,
                                m.qk_norm ? w.q_norm : nullptr, m.qk_norm ? w.k_norm : nullptr,
                                m.qk_eps, ctx->rope_cs, ctx->pf_q, 1, kc, vc, ctx->max_seq,
                                ctx->d_status, ctx->st));
      if (tc_attn)
        NE_LAUNCH(launch_attn_fwd_tc_f16(ctx->pf_q, kc, vc, nb, S, Hq, Hkv, hd, ctx->max_seq,
                                         ctx->pf_o, ctx->d_status, ctx->st));
      else
        NE_LAUNCH(launch_prefill_attn(ctx->pf_q, kc, vc, nb, S, pos0, Hq, Hkv, hd, ctx->max_seq,
                                      ctx->pf_o, ctx->st));
      if ((s = gemm_tokens(ctx, ctx->pf_o, q_dim, rows, w.wo, D, q_dim, EPI_RESID, ctx->pf_x, D,
                           m.res_alpha)) != NE_OK)
        return s;
      NE_LAUNCH(launch_resid_rmsnorm(ctx->pf_x, nullptr, 0, 0, 1.f, D, w.rms_ffn, m.rms_eps,
                                     ctx->pf_xn, rows, ctx->st));
      if ((s = gemm_tokens(ctx, ctx->pf_xn, D, rows, w.w13, 2 * F, D, EPI_SWIGLU, ctx->pf_gate, F,
                           1.f)) != NE_OK)
        return s;
      if ((s = gemm_tokens(ctx, ctx->pf_gate, F, rows, w.w2, D, F, EPI_RESID, ctx->pf_x, D,
                           m.res_alpha)) != NE_OK)
        return s;
      const float* next_g = (l + 1 < m.n_layers) ? ctx->L[l + 1].rms_att : ctx->rms_final;
      NE_LAUNCH(launch_resid_rmsnorm(ctx->pf_x, nullptr, 0, 0, 1.f, D, next_g, m.rms_eps,
                                     ctx->pf_xn, rows, ctx->st));
    }
    // LM head on the last position of each sequence: rows (S-1), (2S-1), ...
    if ((s = gemm_lm_head(ctx, ctx->pf_xn + (size_t)(S - 1) * D, (long long)S * D, nb,
                          ctx->logits + (size_t)b0 * m.vocab)) != NE_OK)
      return s;
  }
  NE_LAUNCH(launch_argmax(ctx->logits, B, m.vocab, d_next, nullptr, ctx->state, 0, ctx->st));
  return NE_OK;
}

ne_status free_workspace(ne_ctx* ctx) {
  for (auto& kv : ctx->graphs) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
  }
  ctx->graphs.clear();
  for (cudaEvent_t e : ctx->prof_events) cudaEventDestroy(e);
  ctx->prof_events.clear();
  void* ptrs[] = {ctx->kcache, ctx->vcache, ctx->rope_cs, ctx->x, ctx->xn, ctx->part, ctx->q,
                  ctx->attn, ctx->attn_po, ctx->attn_ml, ctx->attn_cnt, ctx->gate, ctx->logits,
                  ctx->argmax_keys, ctx->tok,
                  ctx->state, ctx->out_tokens, ctx->pf_x, ctx->pf_xn, ctx->pf_qkv, ctx->pf_q,
                  ctx->pf_o, ctx->pf_gate, ctx->pf_tok};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  ctx->kcache = ctx->vcache = nullptr;
  ctx->rope_cs = nullptr;
  ctx->x = nullptr; ctx->xn = nullptr; ctx->part = nullptr; ctx->q = nullptr;
  ctx->attn = nullptr; ctx->attn_po = nullptr; ctx->attn_ml = nullptr; ctx->attn_cnt = nullptr;
  ctx->argmax_keys = nullptr;
  ctx->gate = nullptr;
  ctx->logits = nullptr; ctx->tok = nullptr; ctx->state = nullptr; ctx->out_tokens = nullptr;
  ctx->pf_x = nullptr; ctx->pf_xn = nullptr; ctx->pf_qkv = nullptr; ctx->pf_q = nullptr;
  ctx->pf_o = nullptr; ctx->pf_gate = nullptr; ctx->pf_tok = nullptr;
  ctx->max_batch = ctx->max_seq = 0;
  return NE_OK;
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

NE_API const char* ne_version(void) { return "neural-engine-b200 0.1 (sm_100a)"; }

NE_API const char* ne_status_str(ne_status s) {
  switch (s) {
    case NE_OK: return "ok";
    case NE_ERR_INVALID: return "invalid argument";
    case NE_ERR_CUDA: return "cuda error";
    case NE_ERR_OOM: return "out of device memory";
    case NE_ERR_IO: return "i/o error";
    case NE_ERR_FORMAT: return "bad checkpoint format";
    case NE_ERR_TIMEOUT: return "device wait timed out";
    case NE_ERR_UNSUPPORTED: return "unsupported shape or option";
    case NE_ERR_STATE: return "call out of order";
    case NE_ERR_BOUNDS: return "index out of range";
  }
  return "unknown status";
}

NE_API const char* ne_last_error(const ne_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

NE_API ne_status ne_init(ne_ctx** out, const ne_model_cfg* cfg, int device) {
  if (!out || !cfg) return NE_ERR_INVALID;
  *out = nullptr;
  const ne_model_cfg& m = *cfg;
  if (m.n_layers <= 0 || m.dim <= 0 || m.hidden <= 0 || m.n_heads <= 0 || m.kv_heads <= 0 ||
      m.vocab <= 0 || m.n_heads % m.kv_heads != 0)
    return NE_ERR_INVALID;
  if (m.head_dim != 64 && m.head_dim != 128) return NE_ERR_UNSUPPORTED;
  const int group = m.n_heads / m.kv_heads;
  if (group != 1 && group != 2) return NE_ERR_UNSUPPORTED;
  if (m.dim % 64 || m.hidden % 64 || (m.n_heads * m.head_dim) % 64) return NE_ERR_UNSUPPORTED;
  ne_ctx* ctx = new ne_ctx();
  ctx->cfg = m;
  ctx->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    delete ctx;
    return NE_ERR_CUDA;
  }
  cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10) {
    delete ctx;
    return NE_ERR_UNSUPPORTED;  // built for sm_100a only
  }
  if (cudaStreamCreateWithFlags(&ctx->st, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->d_status, sizeof(int)) != cudaSuccess) {
    delete ctx;
    return NE_ERR_CUDA;
  }
  cudaMemset(ctx->d_status, 0, sizeof(int));
  // weight pool: every tensor 256-byte aligned (TMA needs 16)
  const size_t D = m.dim, F = m.hidden, qd = (size_t)m.n_heads * m.head_dim,
               kvd = (size_t)m.kv_heads * m.head_dim;
  auto rnd = [](size_t nbytes) { return (nbytes + 255) & ~(size_t)255; };
  const size_t per_layer = rnd((qd + 2 * kvd) * D * 2) + rnd(D * qd * 2) + rnd(2 * F * D * 2) +
                           rnd(D * F * 2) + 2 * rnd(D * 4) + 2 * rnd((size_t)m.head_dim * 4);
  const size_t bytes = per_layer * m.n_layers + rnd(D * 4) + rnd((size_t)m.vocab * D * 2);
  if (cudaMalloc(&ctx->wpool, bytes) != cudaSuccess) {
    cudaFree(ctx->d_status);
    cudaStreamDestroy(ctx->st);
    delete ctx;
    return NE_ERR_OOM;
  }
  uint8_t* p = reinterpret_cast<uint8_t*>(ctx->wpool);
  auto take = [&](size_t nbytes) {
    uint8_t* r = p;
    p += rnd(nbytes);
    return r;
  };
  ctx->L.resize(m.n_layers);
  ctx->layer_set.assign(m.n_layers, 0);
  for (int l = 0; l < m.n_layers; ++l) {
    LayerW& w = ctx->L[l];
    w.wqkv = reinterpret_cast<__nv_bfloat16*>(take((qd + 2 * kvd) * D * 2));
    w.wo = reinterpret_cast<__nv_bfloat16*>(take(D * qd * 2));
    w.w13 = reinterpret_cast<__nv_bfloat16*>(take(2 * F * D * 2));
    w.w2 = reinterpret_cast<__nv_bfloat16*>(take(D * F * 2));
    w.rms_att = reinterpret_cast<float*>(take(D * 4));
    w.rms_ffn = reinterpret_cast<float*>(take(D * 4));
    w.q_norm = reinterpret_cast<float*>(take(m.head_dim * 4));
    w.k_norm = reinterpret_cast<float*>(take(m.head_dim * 4));
  }
  ctx->rms_final = reinterpret_cast<float*>(take(D * 4));
  ctx->embed = reinterpret_cast<__nv_bfloat16*>(take((size_t)m.vocab * D * 2));
  *out = ctx;
  return NE_OK;
}

NE_API void ne_free(ne_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->st);
  free_train(ctx);   // first: a captured training step may hold NCCL calls of the communicator
  comm_free(ctx);
  free_workspace(ctx);
  if (ctx->wpool) cudaFree(ctx->wpool);
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (ctx->st) cudaStreamDestroy(ctx->st);
  delete ctx;
}

NE_API ne_status ne_sync(ne_ctx* ctx) {
  if (!ctx) return NE_ERR_INVALID;
  if (ctx->comm && ctx->comm->world > 1) {
    // bounded: a gradient exchange that cannot finish aborts the communicator
    ne_status s = comm_sync(ctx);
    if (s != NE_OK) return s;
    s = check_status(ctx);
    // a wait of the peer-memory exchange that ran out leaves the ranks out of
    // step: no further exchange on this communicator
    if (s == NE_ERR_TIMEOUT) ctx->comm->aborted = true;
    return s;
  }
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  return check_status(ctx);
}

NE_API ne_status ne_get_cfg(const ne_ctx* ctx, ne_model_cfg* out) {
  if (!ctx || !out) return NE_ERR_INVALID;
  *out = ctx->cfg;
  return NE_OK;
}

NE_API ne_status ne_set_layer_weights(ne_ctx* ctx, int layer, const float* wq, const float* wk,
                                      const float* wv, const float* wo, const float* w1,
                                      const float* w2, const float* w3, const float* rms_att,
                                      const float* rms_ffn, const float* q_norm,
                                      const float* k_norm) {
  if (!ctx) return NE_ERR_INVALID;
  const ne_model_cfg& m = ctx->cfg;
  if (layer < 0 || layer >= m.n_layers || !wq || !wk || !wv || !wo || !w1 || !w2 || !w3 ||
      !rms_att || !rms_ffn)
    return fail(ctx, NE_ERR_INVALID, "ne_set_layer_weights: bad layer or null tensor");
  NE_CUDA(cudaSetDevice(ctx->device));
  const size_t D = m.dim, F = m.hidden, qd = ctx->q_dim(), kvd = ctx->kv_dim();
  const LayerW& w = ctx->L[layer];
  std::vector<uint16_t> buf((qd + 2 * kvd) * D);
  to_bf16(buf.data(), wq, qd * D);
  to_bf16(buf.data() + qd * D, wk, kvd * D);
  to_bf16(buf.data() + (qd + kvd) * D, wv, kvd * D);
  NE_CUDA(cudaMemcpy(w.wqkv, buf.data(), buf.size() * 2, cudaMemcpyHostToDevice));
  buf.resize(D * qd);
  to_bf16(buf.data(), wo, D * qd);
  NE_CUDA(cudaMemcpy(w.wo, buf.data(), D * qd * 2, cudaMemcpyHostToDevice));
  // W1/W3 interleaved in blocks of 16 rows: [W1 rows 16c..16c+15, W3 rows 16c..16c+15] ...
  buf.resize(2 * F * D);
  for (size_t r = 0; r < F; ++r) {
    const size_t blk = r / 16, off = r % 16;
    to_bf16(buf.data() + (blk * 32 + off) * D, w1 + r * D, D);
    to_bf16(buf.data() + (blk * 32 + 16 + off) * D, w3 + r * D, D);
  }
  NE_CUDA(cudaMemcpy(w.w13, buf.data(), 2 * F * D * 2, cudaMemcpyHostToDevice));
  buf.resize(D * F);
  to_bf16(buf.data(), w2, D * F);
  NE_CUDA(cudaMemcpy(w.w2, buf.data(), D * F * 2, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(w.rms_att, rms_att, D * 4, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(w.rms_ffn, rms_ffn, D * 4, cudaMemcpyHostToDevice));
  std::vector<float> ones(m.head_dim, 1.0f);
  NE_CUDA(cudaMemcpy(w.q_norm, q_norm ? q_norm : ones.data(), m.head_dim * 4, cudaMemcpyHostToDevice));
  NE_CUDA(cudaMemcpy(w.k_norm, k_norm ? k_norm : ones.data(), m.head_dim * 4, cudaMemcpyHostToDevice));
  if (!ctx->layer_set[layer]) {
    ctx->layer_set[layer] = 1;
    ctx->layer_set_count++;
  }
  return NE_OK;
}

NE_API ne_status ne_set_global_weights(ne_ctx* ctx, const float* rms_final, const float* embed) {
  if (!ctx || !rms_final || !embed) return NE_ERR_INVALID;
  const ne_model_cfg& m = ctx->cfg;
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaMemcpy(ctx->rms_final, rms_final, (size_t)m.dim * 4, cudaMemcpyHostToDevice));
  const size_t n = (size_t)m.vocab * m.dim;
  const size_t chunk = (size_t)1 << 24;
  std::vector<uint16_t> buf(std::min(n, chunk));
  for (size_t o = 0; o < n; o += chunk) {
    const size_t k = std::min(chunk, n - o);
    to_bf16(buf.data(), embed + o, k);
    NE_CUDA(cudaMemcpy(reinterpret_cast<uint16_t*>(ctx->embed) + o, buf.data(), k * 2,
                       cudaMemcpyHostToDevice));
  }
  ctx->global_set = true;
  return NE_OK;
}

NE_API ne_status ne_kv_alloc(ne_ctx* ctx, int max_batch, int max_seq) {
  if (!ctx || max_batch <= 0 || max_seq <= 0) return NE_ERR_INVALID;
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  free_workspace(ctx);
  const ne_model_cfg& m = ctx->cfg;
  const int D = m.dim, F = m.hidden, Hq = m.n_heads, hd = m.head_dim;
  ctx->max_batch = max_batch;
  ctx->max_seq = max_seq;
  ne_status s;
  const size_t kv = ctx->layer_kv_elems() * m.n_layers;
  if ((s = dalloc(ctx, &ctx->kcache, kv)) || (s = dalloc(ctx, &ctx->vcache, kv))) return s;
  // RoPE table in float64 on the host, stored fp32 (cos, sin):
  // freq_i = 1 / theta^(2i/hd); angle = pos * freq_i   (generate.py:103-105)
  {
    std::vector<float2> cs((size_t)max_seq * (hd / 2));
    for (int pidx = 0; pidx < max_seq; ++pidx)
      for (int i = 0; i < hd / 2; ++i) {
        const double freq = 1.0 / std::pow((double)m.rope_theta, 2.0 * i / hd);
        const double ang = (double)pidx * freq;
        cs[(size_t)pidx * (hd / 2) + i] = make_float2((float)std::cos(ang), (float)std::sin(ang));
      }
    if ((s = dalloc(ctx, &ctx->rope_cs, cs.size()))) return s;
    NE_CUDA(cudaMemcpy(ctx->rope_cs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice));
  }
  // decode accumulators of the QKV and W1/W3 projections (zero between uses)
  const int qkv_dim = ctx->qkv_dim(), q_dim = ctx->q_dim();
  const size_t part = (size_t)max_batch * std::max(qkv_dim, 2 * F);
  ctx->part_elems = part;
  const size_t attn_slots = decode_attn_partial_slots(max_batch, m.kv_heads, ctx->num_sms);
  const size_t group = (size_t)(Hq / m.kv_heads);
  // the attention partial buffers are sized for max_batch, so captured
  // graphs stay valid for every batch size up to it
  const size_t B = max_batch;
  if ((s = dalloc(ctx, &ctx->x, B * D)) || (s = dalloc(ctx, &ctx->xn, B * D)) ||
      (s = dalloc(ctx, &ctx->part, part)) || (s = dalloc(ctx, &ctx->q, B * Hq * hd)) ||
      (s = dalloc(ctx, &ctx->attn, B * q_dim)) ||
      (s = dalloc(ctx, &ctx->attn_po, attn_slots * group * hd)) ||
      (s = dalloc(ctx, &ctx->attn_ml, attn_slots * group * 2)) ||
      (s = dalloc(ctx, &ctx->attn_cnt, B * m.kv_heads)) ||
      (s = dalloc(ctx, &ctx->argmax_keys, B)) ||
      (s = dalloc(ctx, &ctx->gate, B * F)) || (s = dalloc(ctx, &ctx->logits, B * m.vocab)) ||
      (s = dalloc(ctx, &ctx->tok, B)) || (s = dalloc(ctx, &ctx->state, 2)) ||
      (s = dalloc(ctx, &ctx->out_tokens, (size_t)max_seq * B)))
    return s;
  // prefill chunk: up to 16384 rows (at least one full sequence)
  ctx->pf_rows = std::max(max_seq, std::min(16384, max_batch * max_seq));
  const size_t R = ctx->pf_rows;
  if ((s = dalloc(ctx, &ctx->pf_x, R * D)) || (s = dalloc(ctx, &ctx->pf_xn, R * D)) ||
      (s = dalloc(ctx, &ctx->pf_qkv, R * qkv_dim)) || (s = dalloc(ctx, &ctx->pf_q, R * q_dim)) ||
      (s = dalloc(ctx, &ctx->pf_o, R * q_dim)) || (s = dalloc(ctx, &ctx->pf_gate, R * F)) ||
      (s = dalloc(ctx, &ctx->pf_tok, (size_t)max_batch * max_seq)))
    return s;
  NE_CUDA(cudaMemset(ctx->kcache, 0, kv * sizeof(__half)));
  NE_CUDA(cudaMemset(ctx->vcache, 0, kv * sizeof(__half)));
  NE_CUDA(cudaMemset(ctx->state, 0, 2 * sizeof(int)));
  NE_CUDA(cudaMemset(ctx->part, 0, part * sizeof(float)));
  NE_CUDA(cudaMemset(ctx->attn_cnt, 0, B * m.kv_heads * sizeof(int)));
  NE_CUDA(cudaMemset(ctx->argmax_keys, 0, B * sizeof(unsigned long long)));
  return NE_OK;
}

NE_API ne_status ne_kv_reset(ne_ctx* ctx) {
  if (!ctx) return NE_ERR_INVALID;
  if (!ctx->kcache) return fail(ctx, NE_ERR_STATE, "ne_kv_alloc not called");
  NE_CUDA(cudaSetDevice(ctx->device));
  const ne_model_cfg& m = ctx->cfg;
  const size_t B = ctx->max_batch;
  const size_t kv = ctx->layer_kv_elems() * m.n_layers;
  const size_t part = B * std::max(ctx->qkv_dim(), 2 * m.hidden);
  // the same state ne_kv_alloc leaves, enqueued after the work already on the
  // context's stream; buffers and captured graphs stay as they are
  NE_CUDA(cudaMemsetAsync(ctx->kcache, 0, kv * sizeof(__half), ctx->st));
  NE_CUDA(cudaMemsetAsync(ctx->vcache, 0, kv * sizeof(__half), ctx->st));
  NE_CUDA(cudaMemsetAsync(ctx->state, 0, 2 * sizeof(int), ctx->st));
  NE_CUDA(cudaMemsetAsync(ctx->part, 0, part * sizeof(float), ctx->st));
  NE_CUDA(cudaMemsetAsync(ctx->attn_cnt, 0, B * m.kv_heads * sizeof(int), ctx->st));
  NE_CUDA(cudaMemsetAsync(ctx->argmax_keys, 0, B * sizeof(unsigned long long), ctx->st));
  return NE_OK;
}

NE_API ne_status ne_prefill_device(ne_ctx* ctx, const int32_t* d_tokens, int B, int S, int pos0,
                                   int32_t* d_next) {
  if (!ctx || !d_tokens || !d_next || B <= 0 || S <= 0 || pos0 < 0) return NE_ERR_INVALID;
  NE_FAULT_POINT(ctx, "ne_prefill_device");
  if (!ready(ctx)) return fail(ctx, NE_ERR_STATE, "weights not set");
  if (!ctx->kcache) return fail(ctx, NE_ERR_STATE, "ne_kv_alloc not called");
  if (B > ctx->max_batch || pos0 + S > ctx->max_seq)
    return fail(ctx, NE_ERR_INVALID, "batch or sequence exceeds the allocated KV cache");
  ctx->launches = 0;
  return enqueue_prefill(ctx, d_tokens, B, S, pos0, d_next);
}

NE_API ne_status ne_prefill(ne_ctx* ctx, const int32_t* h_tokens, int B, int S, int pos0,
                            int32_t* h_next, float* h_logits) {
  if (!ctx || !h_tokens) return NE_ERR_INVALID;
  NE_FAULT_POINT(ctx, "ne_prefill");
  if (!ctx->kcache) return fail(ctx, NE_ERR_STATE, "ne_kv_alloc not called");
  if (B <= 0 || S <= 0 || B > ctx->max_batch || pos0 < 0 || pos0 + S > ctx->max_seq)
    return fail(ctx, NE_ERR_INVALID, "batch or sequence exceeds the allocated KV cache");
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaMemcpyAsync(ctx->pf_tok, h_tokens, (size_t)B * S * sizeof(int32_t),
                          cudaMemcpyHostToDevice, ctx->st));
  ne_status s = ne_prefill_device(ctx, ctx->pf_tok, B, S, pos0, ctx->tok);
  if (s != NE_OK) return s;
  if (h_next)
    NE_CUDA(cudaMemcpyAsync(h_next, ctx->tok, (size_t)B * sizeof(int32_t), cudaMemcpyDeviceToHost,
                            ctx->st));
  if (h_logits)
    NE_CUDA(cudaMemcpyAsync(h_logits, ctx->logits, (size_t)B * ctx->cfg.vocab * sizeof(float),
                            cudaMemcpyDeviceToHost, ctx->st));
  return ne_sync(ctx);
}

// The graph-replayed token loop; keep_logits leaves the last step's logits in
// ctx->logits (the sampling path), otherwise the greedy LM head runs fused.
ne_status decode_loop(ne_ctx* ctx, const int32_t* d_tok, int B, int pos0, int n_steps,
                      int32_t* d_out, bool keep_logits);

NE_API ne_status ne_decode_loop_device(ne_ctx* ctx, const int32_t* d_tok, int B, int pos0,
                                       int n_steps, int32_t* d_out) {
  return decode_loop(ctx, d_tok, B, pos0, n_steps, d_out, false);
}

ne_status decode_loop(ne_ctx* ctx, const int32_t* d_tok, int B, int pos0, int n_steps,
                      int32_t* d_out, bool keep_logits) {
  if (!ctx || !d_tok || B <= 0 || n_steps < 0 || pos0 < 0) return NE_ERR_INVALID;
  if (!ready(ctx)) return fail(ctx, NE_ERR_STATE, "weights not set");
  if (!ctx->kcache) return fail(ctx, NE_ERR_STATE, "ne_kv_alloc not called");
  if (B > ctx->max_batch || pos0 + n_steps > ctx->max_seq)
    return fail(ctx, NE_ERR_INVALID, "batch or positions exceed the allocated KV cache");
  DecodeGraph* g = nullptr;
  ne_status s = get_graph(ctx, B, keep_logits, &g);
  if (s != NE_OK) return s;
  const int st0[2] = {pos0, 0};
  if (d_tok != ctx->tok)
    NE_CUDA(cudaMemcpyAsync(ctx->tok, d_tok, (size_t)B * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                            ctx->st));
  // the state is written through a pinned-free path: a tiny H2D copy of 8 bytes
  NE_CUDA(cudaMemcpyAsync(ctx->state, st0, sizeof(st0), cudaMemcpyHostToDevice, ctx->st));
  for (int i = 0; i < n_steps; ++i) NE_CUDA(cudaGraphLaunch(g->exec, ctx->st));
  if (d_out && n_steps > 0 && d_out != ctx->out_tokens)
    NE_CUDA(cudaMemcpyAsync(d_out, ctx->out_tokens, (size_t)n_steps * B * sizeof(int32_t),
                            cudaMemcpyDeviceToDevice, ctx->st));
  return NE_OK;
}

NE_API ne_status ne_gemm_device(ne_ctx* ctx, const void* d_A, long long lda, int M, const void* d_B,
                                long long ldb, int N, int K, int epi, void* d_out, long long ld,
                                float alpha) {
  if (!ctx || !d_A || !d_B || !d_out || M <= 0 || N <= 0 || K <= 0 || epi < 0 || epi > 4)
    return NE_ERR_INVALID;
  if (K % 64) return fail(ctx, NE_ERR_UNSUPPORTED, "K must be a multiple of 64");
  NE_CUDA(cudaSetDevice(ctx->device));
  GemmCall c;
  c.A = d_A; c.lda = lda; c.M = M;
  c.B = d_B; c.ldb = ldb; c.N = N;
  c.K = K; c.epi = epi; c.out = d_out; c.ld = ld; c.alpha = alpha;
  c.splits = 1;
  cudaError_t e = gemm_run(c, ctx->d_status, ctx->st);
  if (e != cudaSuccess) return fail(ctx, NE_ERR_CUDA, std::string("gemm: ") + cudaGetErrorString(e));
  return NE_OK;
}

NE_API ne_status ne_gemm_device_ex(ne_ctx* ctx, const void* d_A, long long lda, int M,
                                   const void* d_B, long long ldb, int N, int K, int epi,
                                   void* d_out, long long ld, float alpha, int bn, int splits,
                                   long long split_stride, int* h_splits) {
  if (!ctx || !d_A || !d_B || !d_out || M <= 0 || N <= 0 || K <= 0 || epi < 0 || epi > 4 ||
      splits < 0)
    return NE_ERR_INVALID;
  if (bn != 0 && bn != 16 && bn != 32 && bn != 64 && bn != 128 && bn != 256)
    return fail(ctx, NE_ERR_UNSUPPORTED, "bn must be 16, 32, 64, 128 or 256");
  if (K % 64) return fail(ctx, NE_ERR_UNSUPPORTED, "K must be a multiple of 64");
  if (splits != 1 && epi != EPI_F32T && epi != EPI_F32)
    return fail(ctx, NE_ERR_UNSUPPORTED, "split-K needs an fp32 slab epilogue (epi 0 or 1)");
  NE_CUDA(cudaSetDevice(ctx->device));
  GemmCall c;
  c.A = d_A; c.lda = lda; c.M = M;
  c.B = d_B; c.ldb = ldb; c.N = N;
  c.K = K; c.epi = epi; c.out = d_out; c.ld = ld; c.alpha = alpha;
  c.bn = bn;
  c.splits = splits;
  c.split_stride = split_stride;
  const int sp = gemm_pick_splits(c, ctx->num_sms);
  if ((K / 64) % sp) return fail(ctx, NE_ERR_UNSUPPORTED, "splits must divide K/64");
  c.splits = sp;
  if (h_splits) *h_splits = sp;
  cudaError_t e = gemm_run(c, ctx->d_status, ctx->st);
  if (e != cudaSuccess) return fail(ctx, NE_ERR_CUDA, std::string("gemm: ") + cudaGetErrorString(e));
  return NE_OK;
}

NE_API void* ne_get_stream(const ne_ctx* ctx) { return ctx ? (void*)ctx->st : nullptr; }

NE_API ne_status ne_profile_decode_step(ne_ctx* ctx, int B, int pos, float* h_ms) {
  if (!ctx || !h_ms || B <= 0) return NE_ERR_INVALID;
  if (!ready(ctx)) return fail(ctx, NE_ERR_STATE, "weights not set");
  if (!ctx->kcache) return fail(ctx, NE_ERR_STATE, "ne_kv_alloc not called");
  if (B > ctx->max_batch || pos < 0 || pos >= ctx->max_seq)
    return fail(ctx, NE_ERR_INVALID, "batch or position exceeds the allocated KV cache");
  NE_CUDA(cudaSetDevice(ctx->device));
  const int need = 4 + 9 * ctx->cfg.n_layers + 8;
  while ((int)ctx->prof_events.size() < need) {
    cudaEvent_t e;
    NE_CUDA(cudaEventCreate(&e));
    ctx->prof_events.push_back(e);
  }
  ctx->prof_groups.assign(ctx->prof_events.size(), 0);
  const int st0[2] = {pos, 0};
  NE_CUDA(cudaMemcpyAsync(ctx->state, st0, sizeof(st0), cudaMemcpyHostToDevice, ctx->st));
  ctx->prof_on = true;
  ctx->prof_n = 0;
  ctx->launches = 0;
  ne_status s = enqueue_decode_step(ctx, B, nullptr, false);
  ctx->prof_on = false;
  if (s != NE_OK) return s;
  NE_CUDA(cudaStreamSynchronize(ctx->st));
  for (int i = 1; i < ctx->prof_n; ++i) {
    float ms = 0.f;
    NE_CUDA(cudaEventElapsedTime(&ms, ctx->prof_events[i - 1], ctx->prof_events[i]));
    const int g = ctx->prof_groups[i];
    if (g >= 0 && g < NE_PROF_GROUPS) h_ms[g] += ms;
  }
  return check_status(ctx);
}

NE_API ne_status ne_gemm(ne_ctx* ctx, const ne_gemm_desc* d) {
  if (!ctx || !d || !d->a || !d->b || !d->out || d->M <= 0 || d->N <= 0 || d->K <= 0 ||
      d->epi < 0 || (d->epi > 8 && d->epi != EPI_SWIGLU_T))
    return NE_ERR_INVALID;
  if (d->K % 64) return fail(ctx, NE_ERR_UNSUPPORTED, "K must be a multiple of 64");
  if (d->a_mn && !d->b_mn) return fail(ctx, NE_ERR_UNSUPPORTED, "MN-major A needs MN-major B");
  NE_CUDA(cudaSetDevice(ctx->device));
  GemmCall c;
  c.A = d->a; c.lda = d->lda; c.M = d->M; c.a_mn = d->a_mn;
  c.B = d->b; c.ldb = d->ldb; c.N = d->N; c.b_mn = d->b_mn;
  c.K = d->K; c.epi = d->epi; c.out = d->out; c.ld = d->ld; c.alpha = d->alpha;
  c.bn = d->bn; c.half_out = d->half_out; c.splits = 1;
  if (d->epi == EPI_F32T_ADD) c.splits = gemm_pick_splits(c, ctx->num_sms);
  if (d->epi == EPI_ADD) c.aux3 = d->aux0;
  if (d->epi == EPI_SWIGLU_BWD) { c.aux3 = d->aux0; c.aux_ld = d->aux_ld; }
  if (d->epi == EPI_SWIGLU) c.aux1 = const_cast<void*>(d->aux0);
  if (d->epi == EPI_F32_STATS) { c.aux1 = const_cast<void*>(d->aux0); c.aux_ld = d->aux_ld; }
  cudaError_t e = gemm_run(c, ctx->d_status, ctx->st);
  if (e != cudaSuccess) return fail(ctx, NE_ERR_CUDA, std::string("gemm: ") + cudaGetErrorString(e));
  return NE_OK;
}

NE_API int ne_decode_kernels_per_step(const ne_ctx* ctx, int B) {
  if (!ctx) return 0;
  auto it = ctx->graphs.find(2 * B);   // the greedy loop's graph
  return it == ctx->graphs.end() ? 0 : it->second.kernels;
}

NE_API ne_status ne_decode_step(ne_ctx* ctx, const int32_t* h_tok, int B, int pos, int32_t* h_next,
                                float* h_logits) {
  if (!ctx || !h_tok) return NE_ERR_INVALID;
  NE_FAULT_POINT(ctx, "ne_decode_step");
  if (!ctx->kcache) return fail(ctx, NE_ERR_STATE, "ne_kv_alloc not called");
  if (B <= 0 || B > ctx->max_batch || pos < 0 || pos >= ctx->max_seq)
    return fail(ctx, NE_ERR_INVALID, "batch or position exceeds the allocated KV cache");
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaMemcpyAsync(ctx->tok, h_tok, (size_t)B * sizeof(int32_t), cudaMemcpyHostToDevice,
                          ctx->st));
  ne_status s = decode_loop(ctx, ctx->tok, B, pos, 1, nullptr, h_logits != nullptr);
  if (s != NE_OK) return s;
  if (h_next)
    NE_CUDA(cudaMemcpyAsync(h_next, ctx->tok, (size_t)B * sizeof(int32_t), cudaMemcpyDeviceToHost,
                            ctx->st));
  if (h_logits)
    NE_CUDA(cudaMemcpyAsync(h_logits, ctx->logits, (size_t)B * ctx->cfg.vocab * sizeof(float),
                            cudaMemcpyDeviceToHost, ctx->st));
  return ne_sync(ctx);
}

NE_API ne_status ne_generate(ne_ctx* ctx, const int32_t* h_prompt, int B, int P, int n_new,
                             int32_t* h_out) {
  if (!ctx || !h_prompt || !h_out || B <= 0 || P <= 0 || n_new <= 0) return NE_ERR_INVALID;
  NE_FAULT_POINT(ctx, "ne_generate");
  if (!ctx->kcache) return fail(ctx, NE_ERR_STATE, "ne_kv_alloc not called");
  if (B > ctx->max_batch || P + n_new - 1 > ctx->max_seq)
    return fail(ctx, NE_ERR_INVALID, "batch or sequence exceeds the allocated KV cache");
  NE_CUDA(cudaSetDevice(ctx->device));
  NE_CUDA(cudaMemcpyAsync(ctx->pf_tok, h_prompt, (size_t)B * P * sizeof(int32_t),
                          cudaMemcpyHostToDevice, ctx->st));
  ne_status s = ne_prefill_device(ctx, ctx->pf_tok, B, P, 0, ctx->tok);
  if (s != NE_OK) return s;
  // first generated token comes from the prompt pass; copy it to row 0 of the
  // output ring, then n_new-1 decode steps write rows 1.. (state step starts at 1)
  NE_CUDA(cudaMemcpyAsync(ctx->out_tokens, ctx->tok, (size_t)B * sizeof(int32_t),
                          cudaMemcpyDeviceToDevice, ctx->st));
  if (n_new > 1) {
    DecodeGraph* g = nullptr;
    if ((s = get_graph(ctx, B, false, &g)) != NE_OK) return s;
    const int st0[2] = {P, 1};
    NE_CUDA(cudaMemcpyAsync(ctx->state, st0, sizeof(st0), cudaMemcpyHostToDevice, ctx->st));
    for (int i = 1; i < n_new; ++i) NE_CUDA(cudaGraphLaunch(g->exec, ctx->st));
  }
  std::vector<int32_t> tmp((size_t)n_new * B);
  NE_CUDA(cudaMemcpyAsync(tmp.data(), ctx->out_tokens, tmp.size() * sizeof(int32_t),
                          cudaMemcpyDeviceToHost, ctx->st));
  if ((s = ne_sync(ctx)) != NE_OK) return s;
  for (int b = 0; b < B; ++b)
    for (int i = 0; i < n_new; ++i) h_out[(size_t)b * n_new + i] = tmp[(size_t)i * B + b];
  return NE_OK;
}

}  // extern "C"
