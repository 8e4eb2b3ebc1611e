// ne_internal.h -- declarations shared by the library's translation units.
#pragma once
#include <cstdlib>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ne {

// ------------------------------------------------------------------ GEMM
enum GemmEpi : int {
  EPI_F32T = 0,    // fp32, transposed store  out[split][n][m]   (swap-AB decode)
  EPI_F32 = 1,     // fp32, row-major        out[split][m][n]
  EPI_BF16 = 2,    // bf16, row-major        out[m][n]
  EPI_RESID = 3,   // fp32 residual          x[m][n] += alpha * acc
  EPI_SWIGLU = 4,  // bf16 silu(h1)*h3 from a W1/W3 16-row-interleaved operand (aux1: h13 save)
  EPI_ADD = 5,     // fp32 out[m][n] = in[m][n] + alpha * acc
  EPI_SWIGLU_BWD = 6,  // bf16 dh1/dh3 (interleaved) from d_gate and the saved h13 (aux3)
  EPI_F32_STATS = 7,   // fp32 row-major + per-32-column (max, sum exp) into aux1 [m][aux_ld]
  EPI_F32T_ADD = 8,    // swap-AB: out[n][m] += alpha * acc through the TMA add (split-K safe)
  EPI_ARGMAX_T = 9,    // swap-AB: atomicMax of (logit, ~m) keys into aux1 [N] (greedy LM head)
  EPI_SWIGLU_T = 10,   // swap-AB, K not split: bf16 out[n][m/2] = silu(h1)*h3 of a W1/W3 16-row-interleaved A
  EPI_RESID_PEER = 11, // fp32 x[m][n] += alpha * acc added into the rank that owns element
                       // m*ld + n (GemmCall::peer): the dW products of the peer-memory exchange
};

// Output of EPI_RESID_PEER: each rank's copy of the [M, ld] fp32 matrix (this
// rank's: local) and the element boundaries of the ranks' parts (multiples of
// 64, bound[world] = M * ld).
constexpr int GEMM_PEER_MAX = 8;
struct GemmPeerOut {
  float* dst[GEMM_PEER_MAX];
  long long bound[GEMM_PEER_MAX + 1];
  const unsigned* abort = nullptr;   // this rank's abort word: set, no adds into other ranks
  int world = 1;
  int rank = 0;
};

struct GemmCall {
  const void* A = nullptr;  // [M, K] row-major (K contiguous), leading dim lda (elements)
  long long lda = 0;
  int M = 0;
  const void* B = nullptr;  // [N, K] row-major, leading dim ldb
  long long ldb = 0;
  int N = 0;
  int K = 0;
  int epi = EPI_F32;
  void* out = nullptr;
  long long ld = 0;             // output leading dim (elements)
  long long split_stride = 0;   // elements between split slabs (split-capable epilogues)
  float alpha = 1.0f;
  void* aux1 = nullptr;         // SwiGLU: h13 store [M, N] (optional); stats (epi 7)
  void* aux2 = nullptr;         // unused
  int splits = 1;               // split-K factor (0 = choose)
  int bn = 0;                   // N tile (0 = choose)
  int ab_fp16 = 0;              // 1: fp16 operands, 0: bf16
  int max_ctas = 0;             // 0 = number of SMs
  int prefetch_a = 0;           // A is not written by the preceding kernel (PDL overlap)
  int a_mn = 0;                 // A stored MN-major: [K, M] row-major, lda >= M
  int b_mn = 0;                 // B stored MN-major: [K, N] row-major, ldb >= N
  int half_out = 0;             // EPI_BF16: write fp16 instead of bf16
  const void* aux3 = nullptr;   // EPI_ADD: input; EPI_SWIGLU_BWD: h13 [M, 2F]
  long long aux_ld = 0;         // EPI_SWIGLU_BWD: F
  int atomic = 0;               // EPI_RESID: accumulate with atomics (allows split-K)
  const GemmPeerOut* peer = nullptr;   // EPI_RESID_PEER: where each element goes
};

// Returns the split-K factor gemm_run would use for `c` (resolving splits == 0).
// Whether gemm_run takes CTA-pair tiles (256 x 256 over two SMs) for this call.
bool gemm_pair_tiles(const GemmCall& c);
int gemm_pick_splits(const GemmCall& c, int num_sms);
cudaError_t gemm_run(const GemmCall& c, int* status, cudaStream_t st);
int device_num_sms();

// ------------------------------------------------------------------ elementwise
cudaError_t launch_embed_rmsnorm(const int32_t* tok, const void* table, int table_f32, int V, int D,
                                 const float* g, float eps, float* x, __nv_bfloat16* xn, int rows,
                                 int* status, cudaStream_t st);
// x[r] += alpha * sum of nsplit slabs (nsplit may be 0); xn = rmsnorm(x) (bf16);
// copy (optional) receives the resulting x, e.g. to seed the next residual sum.
cudaError_t launch_resid_rmsnorm(float* x, const float* P, int nsplit, long long split_stride,
                                 float alpha, int D, const float* g, float eps, __nv_bfloat16* xn,
                                 int rows, cudaStream_t st, float* copy = nullptr);
// q_type: 0 = fp32 q, 1 = fp16 q (with fp16 K/V); kv_bf16: q, K and V all bf16
// (training path).
cudaError_t launch_qkv_post(const float* qkv, int nsplit, long long split_stride, int rows,
                            int S_rows, const int* d_pos, int pos0, int Hq, int Hkv, int hd,
                            const float* qn, const float* kn, float qk_eps, const float2* rope_cs,
                            void* q_out, int q_type, void* kc, void* vc, int Tmax, int* status,
                            cudaStream_t st, int kv_bf16 = 0, int zero_src = 0);
// zero_src: clear the consumed sums (the decode accumulators are reused by the
// next projection's TMA add)
cudaError_t launch_swiglu_split(float* P, int nsplit, long long split_stride, int rows, int F,
                                __nv_bfloat16* gate, cudaStream_t st, int zero_src = 0);
// Turns the keys of EPI_ARGMAX_T into next_tok[r] (and out_tokens[step][r]),
// clears the keys for the next step and advances [pos, step].
cudaError_t launch_argmax_keys(unsigned long long* keys, int rows, int32_t* next_tok,
                               int32_t* out_tokens, int* d_state, cudaStream_t st);
cudaError_t launch_argmax(const float* logits, int rows, int V, int32_t* next_tok,
                          int32_t* out_tokens, int* d_state, int adv_state, cudaStream_t st);
// Segment slots (each GROUP x (hd + 2) floats) the decode-attention partial
// buffers must hold for batch B.
size_t decode_attn_partial_slots(int B, int Hkv, int num_sms);
cudaError_t launch_decode_attn(const float* q, const __half* kc, const __half* vc, int B, int Hq,
                               int Hkv, int hd, int Tmax, const int* d_pos, float* part_o,
                               float* part_ml, int* pair_cnt, __nv_bfloat16* out, int* status,
                               cudaStream_t st);

// ------------------------------------------------------------------ prefill attention
// q: fp16 [B*S][Hq][hd] (row = b*S + s, position pos0 + s); cache fp16
// [B][Hkv][Tmax][hd] holding positions 0 .. pos0+S-1; out bf16 [B*S][Hq*hd].
cudaError_t launch_prefill_attn_bf16(const __nv_bfloat16* q, const __nv_bfloat16* kc,
                                     const __nv_bfloat16* vc, int B, int S, int pos0, int Hq,
                                     int Hkv, int hd, int Tmax, __nv_bfloat16* out, cudaStream_t st,
                                     float* lse);
// lse (optional): log2-domain log-sum-exp per (b, head, row) [B][Hq][S].
cudaError_t launch_prefill_attn(const __half* q, const __half* kc, const __half* vc, int B, int S,
                                int pos0, int Hq, int Hkv, int hd, int Tmax, __nv_bfloat16* out,
                                cudaStream_t st, float* lse = nullptr);

// ------------------------------------------------------------------ training
// One trainable tensor for the multi-tensor AdamW / norm kernels (device array).
struct AdamSeg {
  float* w;
  const float* g;
  float* m;
  float* v;
  __nv_bfloat16* w16;
  long long n;
  float wd;
};
// One chunk of at most OPT_CHUNK elements of segment `seg`, starting at `off`;
// vec = 1 when the segment's four fp32 pointers are 16-byte aligned (and its
// bf16 copy 8-byte aligned), so the chunk may use vector accesses.
constexpr int OPT_CHUNK = 16384;
struct OptChunk {
  int seg;
  int vec;
  long long off;
  int n;      // elements in this chunk (<= OPT_CHUNK)
  int norm;   // 1: counts in this rank's share of the global gradient norm
};
// norm_out: [0] pre-clip norm, [1] gradient factor, [2] this rank's sum of
// squares.  partial_only = 1 stops after [2] (sharded optimizer state: the
// sums are added over ranks first, then launch_norm_finish fills [0], [1]).
cudaError_t launch_sumsq_chunks(const AdamSeg* segs, const OptChunk* chunks, int nchunks,
                                float* partial, unsigned* ticket, float grad_scale,
                                float grad_clip, float* norm_out, cudaStream_t st,
                                int partial_only = 0);
cudaError_t launch_norm_finish(float* norm_out, float grad_scale, float grad_clip, cudaStream_t st);
cudaError_t launch_adamw_chunks(const AdamSeg* segs, const OptChunk* chunks, int nchunks,
                                float lr, float b1, float b2, float eps, float inv_bc1,
                                float inv_bc2, const float* norm_out, cudaStream_t st);
// Whether head dim 64 takes the tcgen05 attention kernels (NE_ATTN_TC64=1);
// by default it keeps the mma.sync ones, measured faster at that width (the
// element-wise work per 128 x 128 tile is the same as at 128, the products
// half as long).
inline bool attn_tc64() {
  static const bool on = [] {
    const char* e = std::getenv("NE_ATTN_TC64");
    return e && e[0] == '1';
  }();
  return on;
}
// Causal GQA attention forward on the tcgen05 tensor cores (head_dim 128 or
// 64, bf16): Q [B*S][Hq*hd], K / V [B][Hkv][Tmax][hd]; out [B*S][Hq*hd] bf16 and
// the row log-sum-exp lse [B][Hq][S] (log2 domain).
cudaError_t launch_attn_fwd_tc(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                               const __nv_bfloat16* V, int B, int S, int Hq, int Hkv, int hd,
                               int Tmax, __nv_bfloat16* out, float* lse, int* status,
                               cudaStream_t st);
// The same kernel over fp16 operands (the token loop's prompt pass: fp16 Q and
// the fp16 KV cache, K / V rows [b][kv_head][Tmax][hd]); positions start at 0.
cudaError_t launch_attn_fwd_tc_f16(const __half* Q, const __half* K, const __half* V, int B,
                                   int S, int Hq, int Hkv, int hd, int Tmax,
                                   __nv_bfloat16* out, int* status, cudaStream_t st);
// Causal GQA attention backward; dQ and dK leave through the RoPE and QK-norm
// backward (qn / kn may be NULL: no QK-norm; the raw projection qkv_raw gives
// the pre-norm rows) and dQ, dK, dV are written bf16 into dqkv [B*S][qkv_dim];
// the gain gradients add into dqn / dkn.  Dl: [B][Hq][S] scratch.
cudaError_t launch_attn_bwd(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                            const __nv_bfloat16* V, const __nv_bfloat16* O,
                            const __nv_bfloat16* dO, const float* LSE, float* Dl, int B, int S,
                            int Hq, int Hkv, int hd, int Tmax, const float* qkv_raw,
                            const float* qn, const float* kn, float qk_eps, const float2* rope_cs,
                            __nv_bfloat16* dqkv, float* dqn, float* dkn, int* status,
                            cudaStream_t st);
// tcgen05 variant (head_dim 128 or 64), chosen by launch_attn_bwd; tc_dq =
// false computes dQ (and D) with the mma.sync kernel and dK / dV with tcgen05.
cudaError_t launch_attn_bwd_tc(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                               const __nv_bfloat16* V, const __nv_bfloat16* O,
                               const __nv_bfloat16* dO, const float* LSE, float* Dl, int B, int S,
                               int Hq, int Hkv, int hd, int Tmax, const float* qkv_raw,
                               const float* qn, const float* kn, float qk_eps,
                               const float2* rope_cs, __nv_bfloat16* dqkv, float* dqn, float* dkn,
                               int* status, cudaStream_t st, bool tc_dq);
// mma.sync dQ kernel alone (also publishes D); head_dim 128 or 64.
cudaError_t launch_attn_dq_mma(const __nv_bfloat16* Q, const __nv_bfloat16* K,
                               const __nv_bfloat16* V, const __nv_bfloat16* O,
                               const __nv_bfloat16* dO, const float* LSE, float* Dl, int B, int S,
                               int Hq, int Hkv, int hd, int Tmax, const float* qkv_raw,
                               const float* qn,
                               float qk_eps, const float2* rope_cs, __nv_bfloat16* dqkv,
                               float* dqn, cudaStream_t st);
cudaError_t launch_rmsnorm_bwd(const float* dy, const float* x, const float* w, float eps, int M,
                               int D, const float* residual, float* dx, __nv_bfloat16* dx16,
                               float* dw, cudaStream_t st);
// Cross-entropy rows: logits [rows][ld] (V valid columns) with the GEMM's
// softmax chunk statistics; remap (optional) maps target ids to columns.
cudaError_t launch_ce_rows(const float* logits, int ld, const float2* stats, int stats_ld,
                           const int32_t* tgt, const int32_t* remap, int rows, int V, float scale,
                           float* loss, __nv_bfloat16* dlogits, int* status, cudaStream_t st);
// dst[r] = src[idx[r]] (bf16 rows of D) / dst[idx[r]] += src[r], src[r] = 0 (fp32)
cudaError_t launch_gather_rows(const __nv_bfloat16* src, const int32_t* idx, int n, int D,
                               __nv_bfloat16* dst, cudaStream_t st);
cudaError_t launch_scatter_add_rows(float* src, const int32_t* idx, int n, int D, float* dst,
                                    cudaStream_t st);

// Deterministic dE[tok[r]] += dy[r] over n rows (embed_bwd.cu); scratch of at
// least embed_bwd_scratch_bytes(n) bytes.
size_t embed_bwd_scratch_bytes(int n);
cudaError_t launch_embed_bwd(const int32_t* tok, const float* dy, int n, int V, int D, float* dE,
                             void* scratch, size_t scratch_bytes, int* status, cudaStream_t st);
cudaError_t launch_f32_to_bf16(const float* a, __nv_bfloat16* b, long long n, cudaStream_t st);
// out[0] = min, out[1] = max of a[0..n)
cudaError_t launch_minmax(const float* a, long long n, float* out, cudaStream_t st);

}  // namespace ne
