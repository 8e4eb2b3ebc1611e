// ne_ctx.h -- the context behind the C ABI's opaque ne_ctx*, shared by the
// library's host translation units (ne_api.cu: weights, KV cache, token loop;
// ne_train.cu: training step).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/ne.h"
#include "ne_device.cuh"
#include "ne_internal.h"

namespace ne {
struct TrainState;                      // ne_train.cu
void free_train(ne_ctx* ctx);           // ne_train.cu
struct Comm;                            // comm.cu
void comm_free(ne_ctx* ctx);            // comm.cu
}  // namespace ne

namespace ne {

struct LayerW {
  __nv_bfloat16* wqkv = nullptr;  // [q_dim + 2*kv_dim, D]: Wq rows, Wk rows, Wv rows
  __nv_bfloat16* wo = nullptr;    // [D, q_dim]
  __nv_bfloat16* w13 = nullptr;   // [2F, D]: W1/W3 interleaved in 16-row blocks
  __nv_bfloat16* w2 = nullptr;    // [D, F]
  float* rms_att = nullptr;
  float* rms_ffn = nullptr;
  float* q_norm = nullptr;        // [hd]
  float* k_norm = nullptr;        // [hd]
};

struct DecodeGraph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int kernels = 0;
};

}  // namespace ne

struct ne_ctx {
  ne_model_cfg cfg{};
  int device = 0;
  int num_sms = 148;
  cudaStream_t st = nullptr;
  std::string err;
  int* d_status = nullptr;
  int launches = 0;  // kernels enqueued by the current enqueue_* call
  ne::TrainState* train = nullptr;  // training buffers (ne_train_alloc)
  ne::Comm* comm = nullptr;         // NCCL gradient exchange (ne_comm_init)
  int comm_timeout_ms = 0;          // ne_comm_set_timeout (0: NE_COMM_TIMEOUT_MS or 120 s)

  // weights
  void* wpool = nullptr;
  std::vector<ne::LayerW> L;
  float* rms_final = nullptr;
  __nv_bfloat16* embed = nullptr;  // [V, D]
  unsigned layer_set_count = 0;
  std::vector<char> layer_set;
  bool global_set = false;

  // KV cache + workspaces
  int max_batch = 0, max_seq = 0;
  __half* kcache = nullptr;  // [L][maxB][Hkv][maxT][hd]
  __half* vcache = nullptr;
  float2* rope_cs = nullptr;  // [maxT][hd/2] (cos, sin)
  // decode workspace
  float* x = nullptr;            // [maxB, D]
  __nv_bfloat16* xn = nullptr;   // [maxB, D]
  float* part = nullptr;         // decode QKV / W1-W3 accumulators (zero between uses)
  size_t part_elems = 0;
  float* q = nullptr;            // [maxB, Hq, hd]
  __nv_bfloat16* attn = nullptr; // [maxB, q_dim]
  float* attn_po = nullptr;      // [segment slots][group][hd]  (decode attention partials)
  float* attn_ml = nullptr;      // [segment slots][group][2]
  int* attn_cnt = nullptr;       // [maxB * Hkv] segment tickets per (sequence, kv-head)
  unsigned long long* argmax_keys = nullptr;   // [maxB] greedy LM head: best (logit, id) keys
  __nv_bfloat16* gate = nullptr; // [maxB, F]
  float* logits = nullptr;       // [maxB, V]
  int32_t* tok = nullptr;        // [maxB]
  int* state = nullptr;          // [pos, step]
  int32_t* out_tokens = nullptr; // [maxT, maxB]
  // prefill workspace (rows = sequences_per_chunk * S)
  int pf_rows = 0;
  float* pf_x = nullptr;
  __nv_bfloat16* pf_xn = nullptr;
  float* pf_qkv = nullptr;
  __half* pf_q = nullptr;
  __nv_bfloat16* pf_o = nullptr;
  __nv_bfloat16* pf_gate = nullptr;
  int32_t* pf_tok = nullptr;

  std::map<int, ne::DecodeGraph> graphs;   // key: 2 * batch + (logits kept)

  // instrumented-step profiling (ne_profile_decode_step)
  bool prof_on = false;
  std::vector<cudaEvent_t> prof_events;
  std::vector<int> prof_groups;
  int prof_n = 0;

  int qkv_dim() const { return (cfg.n_heads + 2 * cfg.kv_heads) * cfg.head_dim; }
  int q_dim() const { return cfg.n_heads * cfg.head_dim; }
  int kv_dim() const { return cfg.kv_heads * cfg.head_dim; }
  size_t layer_kv_elems() const {
    return (size_t)max_batch * cfg.kv_heads * max_seq * cfg.head_dim;
  }
};

namespace ne {

inline ne_status fail(ne_ctx* c, ne_status s, const std::string& msg) {
  if (c) c->err = msg;
  return s;
}

#define NE_CUDA(call)                                                                    \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail(ctx, NE_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

#define NE_LAUNCH(call)                                                                  \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail(ctx, NE_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    ctx->launches++;                                                                     \
  } while (0)

template <class T>
inline ne_status dalloc(ne_ctx* ctx, T** p, size_t n) {
  if (n == 0) n = 1;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T));
  if (e != cudaSuccess) {
    *p = nullptr;
    return fail(ctx, NE_ERR_OOM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  }
  return NE_OK;
}

inline uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  const uint32_t rounding = ((u >> 16) & 1u) + 0x7fffu;
  return (uint16_t)((u + rounding) >> 16);
}

inline void to_bf16(uint16_t* dst, const float* src, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = f32_to_bf16_bits(src[i]);
}


}  // namespace ne
