/* ne.h -- C ABI of libne.so, the B200 (sm_100a) implementation of the
 * per-layer transformer step of the reference's training_dynamic pipeline
 * (ane-training/training/training_dynamic/) and of its numpy token loop
 * (tools/generate.py).
 *
 * Conventions
 *   - Every entry point returns ne_status; nothing aborts.  ne_last_error()
 *     gives a human-readable reason for the last failure on a context.
 *   - Sizes are in elements.  Pointers named h_* are caller-owned HOST
 *     buffers; pointers named d_* are DEVICE buffers on the context's GPU.
 *   - A context owns one GPU, one CUDA stream and all device memory it uses;
 *     it is single-threaded (one host thread per context).  Calls that return
 *     data to host memory synchronise the stream; the *_device variants only
 *     enqueue work.
 *   - Weights are row-major [out, in] fp32 on the host, exactly the tensors
 *     of the v4 checkpoint (config.h:26-33, train.m:110-130); the device keeps
 *     bf16 compute copies.
 *   - Activations are token-major [tokens, features].  The KV cache is fp16,
 *     [layer][sequence][kv_head][position][head_dim].
 */
#ifndef NE_H_
#define NE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NE_API __attribute__((visibility("default")))
#else
#define NE_API
#endif

typedef enum ne_status {
  NE_OK = 0,
  NE_ERR_INVALID = 1,     /* bad argument or shape */
  NE_ERR_CUDA = 2,        /* CUDA runtime / launch error */
  NE_ERR_OOM = 3,         /* device allocation failed */
  NE_ERR_IO = 4,          /* file open / read / write failed */
  NE_ERR_FORMAT = 5,      /* checkpoint magic / version / size mismatch */
  NE_ERR_TIMEOUT = 6,     /* a kernel's bounded wait expired (status word set on device) */
  NE_ERR_UNSUPPORTED = 7, /* shape or option the kernels are not built for */
  NE_ERR_STATE = 8,       /* call out of order (e.g. decode before ne_kv_alloc) */
  NE_ERR_BOUNDS = 9       /* a kernel saw an out-of-range token id or position */
} ne_status;

/* Model description.  The reference fixes the model at compile time
 * (models/qwen3_06b.h:6-16, models/stories110m.h:6-16) and hard-codes
 * eps 1e-5, RoPE theta 10000, no QK-norm and residual alpha 1/sqrt(2L) in
 * training (train.m:181) but 1 in generate.py; here they are run-time fields. */
typedef struct ne_model_cfg {
  int n_layers;
  int dim;
  int hidden;
  int n_heads;
  int kv_heads;
  int head_dim;      /* 64 or 128 */
  int vocab;
  float rms_eps;     /* RMSNorm eps (generate.py:81) */
  float rope_theta;  /* RoPE base (generate.py:103) */
  int qk_norm;       /* 1: per-head RMSNorm of q and k before RoPE (Qwen3) */
  float qk_eps;
  float res_alpha;   /* residual branch scale x += alpha * f(x) */
} ne_model_cfg;

/* Subset of the v4 checkpoint header (config.h:83-91) returned by the loader. */
typedef struct ne_ckpt_info {
  int step, total_steps, seq_len, adam_t;
  float lr, loss;
  double cum_compile, cum_train, cum_wall;
  int cum_steps, cum_batches;
  int has_qk_norm;   /* the trailing QKN1 extension block was present */
} ne_ckpt_info;

typedef struct ne_ctx ne_ctx;

/* ---- context -------------------------------------------------------------
 * Replaces the reference's ane_init + compile_dynamic_kernels
 * (config.h:99-107, train.m:25-94): there is nothing to compile at run time. */
NE_API ne_status ne_init(ne_ctx** out, const ne_model_cfg* cfg, int device);
NE_API void ne_free(ne_ctx* ctx);
NE_API const char* ne_last_error(const ne_ctx* ctx);
NE_API const char* ne_status_str(ne_status s);
NE_API ne_status ne_sync(ne_ctx* ctx);
NE_API ne_status ne_get_cfg(const ne_ctx* ctx, ne_model_cfg* out);
/* Version string of the library build. */
NE_API const char* ne_version(void);

/* ---- weights -------------------------------------------------------------
 * Replaces the weight staging into per-layer IOSurfaces
 * (io.h:263-409 stage_*_weights; train.m:331-339).  Host fp32 tensors in the
 * v4 layout; q_norm / k_norm [head_dim] may be NULL (gains of 1). */
NE_API ne_status ne_set_layer_weights(ne_ctx* ctx, int layer, const float* h_wq, const float* h_wk,
                                      const float* h_wv, const float* h_wo, const float* h_w1,
                                      const float* h_w2, const float* h_w3, const float* h_rms_att,
                                      const float* h_rms_ffn, const float* h_q_norm,
                                      const float* h_k_norm);
/* rms_final [dim]; embed [vocab, dim] (tied: also the LM head, generate.py:195). */
NE_API ne_status ne_set_global_weights(ne_ctx* ctx, const float* h_rms_final, const float* h_embed);

/* v4 checkpoint (train.m:97-165 save/load_checkpoint; config.h:83-91).  The
 * header's model fields must match the context's configuration.  Without
 * training state the weights are loaded (Adam moments skipped); after
 * ne_train_alloc the fp32 masters, gains and Adam moments are restored exactly
 * (resume), and the bf16 compute copies refreshed.  A file without the QKN1
 * block gives unit QK-norm gains. */
NE_API ne_status ne_load_ckpt_v4(ne_ctx* ctx, const char* path, ne_ckpt_info* info);
/* Write the full training state (needs ne_train_alloc) in the reference's v4
 * layout, byte for byte (train.m:97-131); the header takes step, total_steps,
 * lr, loss, cum_*, adam_t (and seq_len if > 0) from info.  With QK-norm the
 * QKN1 block follows (q_norm, k_norm per layer, then m, v of each), which v4
 * readers ignore. */
NE_API ne_status ne_save_ckpt_v4(ne_ctx* ctx, const char* path, const ne_ckpt_info* info);

/* Host only (no context, no GPU): read and check a v4 checkpoint's header and
 * size before anything is loaded.  NE_ERR_IO when the file cannot be opened;
 * NE_ERR_FORMAT for a wrong magic or version, a header whose shapes are not a
 * model (non-positive sizes, q_dim != n_heads * head_dim, n_heads not a
 * multiple of kv_heads) and a file shorter than the body its header implies
 * (a truncated checkpoint), the QKN1 block included when it is present.
 * cfg (optional) receives n_layers, dim, hidden, n_heads, kv_heads, head_dim,
 * vocab and qk_norm (the QKN1 block was present); its other fields are left
 * as they were.  ne_load_ckpt_v4 runs the same checks, against the context's
 * model, before it changes any weight or optimizer state. */
NE_API ne_status ne_ckpt_probe(const char* path, ne_model_cfg* cfg, ne_ckpt_info* info);

/* Host-side fault injection (tests of the callers' failure paths; no GPU
 * fault is ever made).  The environment variable NE_FAULT_INJECT, read once,
 * holds comma-separated items "<entry>:<n>[:<status>]": the n-th call (from 1)
 * of the named entry point returns <status> (io, format, cuda, oom, timeout,
 * state; default cuda) before it does any work, with ne_last_error saying
 * "injected".  Entry points that take part: ne_ckpt_probe, ne_load_ckpt_v4,
 * ne_save_ckpt_v4, ne_train_fwd_bwd, ne_train_fwd_bwd_device,
 * ne_train_fwd_bwd_timed, ne_adamw_step, ne_prefill, ne_prefill_device,
 * ne_decode_step, ne_generate, ne_comm_init and ne_shard_range.
 * ne_fault_calls returns how many calls of `entry` were counted so far (0
 * when no item names it). */
NE_API int ne_fault_calls(const char* entry);

/* ---- token loop (tools/generate.py:113-228) ------------------------------
 * Allocates the fp16 KV cache and the decode / prefill workspaces for up to
 * max_batch sequences of up to max_seq positions. */
NE_API ne_status ne_kv_alloc(ne_ctx* ctx, int max_batch, int max_seq);

/* Start a new set of sequences in the allocated cache: clears the KV cache and
 * the decode state (position and step counters, accumulators) to what
 * ne_kv_alloc leaves, without freeing or reallocating anything.  Enqueued on
 * the context's stream after the work already there.  The reference builds a
 * fresh cache per generate() call (tools/generate.py:125-128); this is that
 * step for a long-lived context. */
NE_API ne_status ne_kv_reset(ne_ctx* ctx);

/* Process the prompt h_tokens [B, S] (positions pos0 .. pos0+S-1 of every
 * sequence) in one causal pass, filling the KV cache.  Writes the next token
 * (argmax, generate.py:200) into h_next [B] and, if non-NULL, the last
 * position's logits into h_logits [B, vocab]. */
NE_API ne_status ne_prefill(ne_ctx* ctx, const int32_t* h_tokens, int B, int S, int pos0,
                            int32_t* h_next, float* h_logits);

/* One KV-cached step: token h_tok [B] at position pos of every sequence
 * (generate.py:134-217 loop body).  h_next [B] receives the argmax token;
 * h_logits [B, vocab] (optional) the logits. */
NE_API ne_status ne_decode_step(ne_ctx* ctx, const int32_t* h_tok, int B, int pos, int32_t* h_next,
                                float* h_logits);

/* Greedy generation (temperature 0): prefill h_prompt [B, P], then n_new-1
 * decode steps; h_out [B, n_new] receives the generated tokens. */
NE_API ne_status ne_generate(ne_ctx* ctx, const int32_t* h_prompt, int B, int P, int n_new,
                             int32_t* h_out);

/* Device-resident variants (no host copies; enqueue only). */
NE_API ne_status ne_prefill_device(ne_ctx* ctx, const int32_t* d_tokens, int B, int S, int pos0,
                                   int32_t* d_next);
/* n_steps greedy steps starting from d_tok [B] at position pos0; token i of
 * sequence b is written to d_out[i * B + b].  Each step is one CUDA-graph
 * replay. */
NE_API ne_status ne_decode_loop_device(ne_ctx* ctx, const int32_t* d_tok, int B, int pos0,
                                       int n_steps, int32_t* d_out);

/* ---- dense contraction ---------------------------------------------------
 * out = op(A[M,K] . B[N,K]^T) on the context's stream, bf16 operands (both
 * K-major, row-major with leading dims lda / ldb), fp32 accumulation on the
 * tcgen05 tensor cores.  Library counterpart of the reference's cblas_sgemm
 * call sites (train.m:500-501 classifier, :514-523 classifier bwd / dEmbed,
 * :555-597 dW2/dW1/dW3, :629-655 dWo, :733-738 dWq/dWk/dWv).
 *   epi 0: fp32 out[n*ld + m]  (transposed)     epi 1: fp32 out[m*ld + n]
 *   epi 2: bf16 out[m*ld + n]                   epi 3: fp32 out[m*ld + n] += alpha*acc
 *   epi 4: bf16 SwiGLU of a W1/W3 16-row-interleaved B operand, out[m*ld + n/2]
 * K must be a multiple of 64; pointers 16-byte aligned. */
NE_API ne_status ne_gemm_device(ne_ctx* ctx, const void* d_A, long long lda, int M, const void* d_B,
                                long long ldb, int N, int K, int epi, void* d_out, long long ld,
                                float alpha);

/* As ne_gemm_device with explicit tiling: bn = N tile (16, 32, 64, 128 or 256;
 * 0 = automatic); splits = split-K factor (epi 0/1 only; 0 = automatic, 1 =
 * none).  With splits > 1 the output holds `splits` partial slabs, slab s at
 * d_out + s * split_stride elements; their sum is the product. *h_splits
 * (optional) receives the factor used. */
NE_API ne_status ne_gemm_device_ex(ne_ctx* ctx, const void* d_A, long long lda, int M,
                                   const void* d_B, long long ldb, int N, int K, int epi,
                                   void* d_out, long long ld, float alpha, int bn, int splits,
                                   long long split_stride, int* h_splits);

/* The dW product of the data-parallel training backward fused with its
 * reduce-scatter: fp32 acc = A^T . B with A [K, M] and B [K, N] bf16 stored
 * MN-major (lda >= M, ldb >= N), element (m, n) added, times alpha, into the
 * copy of the rank that owns flat index i = m*ld + n:
 *   h_dst[q][i] += alpha * acc   for h_bound[q] <= i < h_bound[q + 1].
 * world 1..8; h_bound[0] = 0 <= h_bound[1] <= ... <= h_bound[world] = M*ld,
 * every boundary a multiple of 64; ld a multiple of 64 and >= N; K a multiple
 * of 64; the copies 16-byte aligned.  h_dst[q] for q != rank may be another
 * GPU's memory (a CUDA IPC mapping over NVLink): those adds are system-scope
 * vector reductions.  The adds are atomic, so their order (and the fp32 sum's
 * rounding) is not fixed.  Replaces the dW cblas_sgemm + accumulation of
 * train.m:555-597, 629-655 and 733-738 together with the gradient exchange. */
NE_API ne_status ne_gemm_dw_owned(ne_ctx* ctx, const void* d_A, long long lda, int M,
                                  const void* d_B, long long ldb, int N, int K, float alpha,
                                  float* const* h_dst, const long long* h_bound, int world,
                                  int rank, long long ld);

/* The context's CUDA stream (a cudaStream_t), for events and interop. */
NE_API void* ne_get_stream(const ne_ctx* ctx);

/* Instrumented decode step: runs one step for B sequences at position pos
 * WITHOUT the graph, with CUDA events around every kernel group, and adds the
 * device time (ms) of each group to h_ms[NE_PROF_GROUPS]:
 *   0 QKV GEMM   1 qkv_post   2 decode attention (+combine)   3 Wo GEMM
 *   4 residual+RMSNorm   5 W1/W3 GEMM   6 SwiGLU   7 W2 GEMM   8 LM-head GEMM
 *   9 embed + argmax + state */
#define NE_PROF_GROUPS 10
NE_API ne_status ne_profile_decode_step(ne_ctx* ctx, int B, int pos, float* h_ms);

/* General form.  a_mn / b_mn: the operand is stored MN-major, i.e. A as
 * [K, M] (lda >= M) and B as [K, N] (ldb >= N) -- the transposed reads of the
 * reference's cblas_sgemm(CblasTrans, ...) calls (train.m:555-738) without a
 * transposed copy.  epi 4 as above; aux0 (optional) receives the raw
 * projection h13 [M, N] bf16 (W1/W3 16-row-interleaved columns).  epi 5: fp32
 * out = in + alpha*acc (aux0 = in, same ld); epi 6: SwiGLU backward of d_gate
 * = acc (aux0 = the saved h13 [M, 2*aux_ld] bf16; out = dh13 [M, 2*aux_ld]
 * bf16 in the same interleaved order).  epi 7: fp32
 * out as epi 1, plus for every row m and 32-column chunk c the pair
 * (max, sum of exp(acc - max)) over the chunk's columns < N, written as two
 * floats at aux0 + 2*(m*aux_ld + c) (the classifier's softmax statistics).
 * epi 8: out[n*ld + m] += alpha*acc (transposed like epi 0, accumulated
 * through element-wise TMA adds, so K is split across the SMs without
 * partial slabs; the decode projections).  epi 10: SwiGLU of a W1/W3
 * 16-row-interleaved A (rows [32c, 32c+16) = W1 rows [16c, 16c+16), the next
 * 16 the W3 rows), written transposed: bf16 out[n*ld + f] = silu(h1) * h3 for
 * feature f < M/2 (M a multiple of 32, K not split; the decode step's fused
 * W1/W3 projection). */
typedef struct ne_gemm_desc {
  const void* a; long long lda; int a_mn;
  const void* b; long long ldb; int b_mn;
  int M, N, K;
  int epi;
  void* out; long long ld;
  float alpha;
  const void* aux0; const void* aux1; long long aux_ld;
  int bn;            /* 0 = automatic */
  int half_out;      /* epi 2: write fp16 instead of bf16 */
} ne_gemm_desc;
NE_API ne_status ne_gemm(ne_ctx* ctx, const ne_gemm_desc* d);

/* Kernel launches enqueued by the last ne_decode_loop_device step graph
 * (per step), for launch accounting. */
NE_API int ne_decode_kernels_per_step(const ne_ctx* ctx, int B);

/* ---- training step (train.m:391-917) --------------------------------------
 * Typical loop (the reference's step loop with accum micro-steps):
 *   ne_train_alloc(ctx, B, S);                      once, after the weights are set
 *   for step: ne_train_fwd_bwd(ctx, tokens[B][S+1], &loss);   (accumulates grads)
 *             every accum steps: ne_adamw_step(ctx, &cfg, ++t, &norm);
 * Tokens: inputs tokens[:, :S], targets tokens[:, 1:] (train.m:395-401).
 * Loss = mean cross-entropy over the B*S targets (cpu_ops.h:348-382). */
typedef struct ne_adam_cfg {
  float lr;            /* this step's learning rate (see ne_lr_schedule) */
  float beta1, beta2;  /* 0.9, 0.95 in train.m:174 */
  float eps;           /* 1e-8, added after the sqrt (cpu_ops.h:295) */
  float weight_decay;  /* 0.1; applied to matrices and the embedding, not the gains */
  float grad_clip;     /* global-norm clip (train.m:833-849); <= 0 disables */
  float grad_scale;    /* multiplies the accumulated gradients first (1/accum) */
} ne_adam_cfg;

/* Allocate fp32 masters (initialised from the current weights), gradients,
 * Adam m/v and the saved activations for batches of B sequences of S tokens
 * (B*S a multiple of 64). */
NE_API ne_status ne_train_alloc(ne_ctx* ctx, int B, int S);
/* Load exact fp32 masters for one layer (v4 tensors); layer -1 loads the
 * embedding from h_wq.  Call ne_train_sync_weights afterwards. */
NE_API ne_status ne_train_set_masters(ne_ctx* ctx, int layer, const float* h_wq, const float* h_wk,
                                      const float* h_wv, const float* h_wo, const float* h_w1,
                                      const float* h_w2, const float* h_w3);
/* Refresh the bf16 compute copies from the fp32 masters. */
NE_API ne_status ne_train_sync_weights(ne_ctx* ctx);
NE_API ne_status ne_train_zero_grads(ne_ctx* ctx);
/* Forward + backward of one batch; gradients accumulate.  d_loss / h_loss
 * (optional) receive the batch's mean loss. */
NE_API ne_status ne_train_fwd_bwd_device(ne_ctx* ctx, const int32_t* d_tokens, float* d_loss);
NE_API ne_status ne_train_fwd_bwd(ne_ctx* ctx, const int32_t* h_tokens, float* h_loss);
/* One micro-step exactly as ne_train_fwd_bwd, run without the captured graph
 * and timed per stage with CUDA events (the per-phase "timing:" line of
 * train.m:763-768, which the reference prints every 10 steps).
 * h_ms[NE_TRAIN_PHASES] receives device milliseconds: 0 embedding forward,
 * 1 attention forward (all layers), 2 FFN forward, 3 classifier +
 * cross-entropy + classifier backward, 4 FFN backward, 5 attention backward,
 * 6 embedding backward (including the wait for the gradient exchange), 7 the
 * whole micro-step.  Synchronises. */
#define NE_TRAIN_PHASES 8
NE_API ne_status ne_train_fwd_bwd_timed(ne_ctx* ctx, const int32_t* h_tokens, float* h_loss,
                                        float* h_ms);
/* Value ranges the reference prints on its step line (train.m:771-776):
 * h_out[4] = {min, max} of the final residual stream x (before the final
 * norm) and {min, max} of the gradient at the embedding output, both from the
 * last micro-step.  Synchronises. */
NE_API ne_status ne_train_value_ranges(ne_ctx* ctx, float* h_out);
/* Vocabulary compaction (cpu_ops.h:385-431, applied by train.m to every run):
 * the classifier and its softmax use only the CV embedding rows h_c2f[0..CV)
 * (distinct ids; the reference takes the tokens present in the data, in
 * increasing order); every target must be one of them.  Their gradient is
 * added back into the tied embedding's.  CV = 0 / NULL: full vocabulary. */
NE_API ne_status ne_train_set_vocab_map(ne_ctx* ctx, const int32_t* h_c2f, int CV);
/* Global L2 norm of the accumulated gradients times grad_scale. */
NE_API ne_status ne_train_grad_norm(ne_ctx* ctx, float grad_scale, float* h_norm);
/* Unscale, clip, AdamW (bias correction at step t >= 1), refresh bf16 copies,
 * zero the gradients (train.m:782-904; cpu_ops.h:266-303).  The norm and the
 * clip factor are computed on the device.  h_grad_norm (optional) receives the
 * pre-clip norm and makes the call wait for the step; with NULL it only
 * enqueues work on the context's stream. */
NE_API ne_status ne_adamw_step(ne_ctx* ctx, const ne_adam_cfg* cfg, int t, float* h_grad_norm);
/* Warmup + cosine learning rate of train.m:851-858. */
NE_API float ne_lr_schedule(int step, float max_lr, int warmup_steps, int total_steps,
                            float min_lr_frac);
/* Copy a layer's gradients (which 0), fp32 masters (1), Adam m (2) or Adam v
 * (3) to host in the v4 layout; layer -1 gives rms_final in h_rms_att and the
 * embedding in h_wq.  NULL pointers are skipped. */
NE_API ne_status ne_train_get_layer(ne_ctx* ctx, int layer, int which, float* h_wq, float* h_wk,
                                    float* h_wv, float* h_wo, float* h_w1, float* h_w2,
                                    float* h_w3, float* h_rms_att, float* h_rms_ffn,
                                    float* h_q_norm, float* h_k_norm);

/* ---- per-layer entry points (the reference's kernel set) -----------------
 * The reference drives one compiled ANE kernel per stage from train.m; these
 * are the same stages on the training workspace of ne_train_alloc, enqueued
 * on the context stream.  One micro-step is exactly
 *   ne_embed_fwd(ctx, d_tokens);
 *   for l = 0 .. L-1:  ne_attn_fwd(ctx, l); ne_ffn_fwd(ctx, l);
 *   ne_lmhead_ce_fwd_bwd(ctx, d_loss);
 *   for l = L-1 .. 0:  ne_ffn_bwd(ctx, l); ne_attn_bwd(ctx, l);
 *   ne_embed_bwd(ctx);
 * which is what ne_train_fwd_bwd_device runs.  Gradients accumulate. */
/* embed_lookup (cpu_ops.h:433-439) + the first RMSNorm; d_tokens [B][S+1]. */
NE_API ne_status ne_embed_fwd(ne_ctx* ctx, const int32_t* d_tokens);
/* sdpaFwd (mil_dynamic.h:57-234): QKV, QK-norm, RoPE, causal GQA SDPA, Wo,
 * residual (io.h:25-37), FFN RMSNorm. */
NE_API ne_status ne_attn_fwd(ne_ctx* ctx, int layer);
/* ffnFused (mil_dynamic.h:238-306): SwiGLU FFN, residual, next RMSNorm. */
NE_API ne_status ne_ffn_fwd(ne_ctx* ctx, int layer);
/* Classifier (train.m:495-505), cross_entropy_loss (cpu_ops.h:348-382),
 * classifier backward, dense embedding gradient, final RMSNorm backward.
 * d_loss (device, optional): the batch's mean loss. */
NE_API ne_status ne_lmhead_ce_fwd_bwd(ne_ctx* ctx, float* d_loss);
/* ffnBwdFull (mil_dynamic.h:320-409) + dW1/dW2/dW3 + rmsnorm_bwd_add. */
NE_API ne_status ne_ffn_bwd(ne_ctx* ctx, int layer);
/* wotBwd + sdpaBwd1/2 + RoPE/QK-norm backward + qkvBwd (mil_dynamic.h:412-707)
 * + dWq/dWk/dWv/dWo + rmsnorm_bwd_add. */
NE_API ne_status ne_attn_bwd(ne_ctx* ctx, int layer);
/* embed_backward (cpu_ops.h:441-447). */
NE_API ne_status ne_embed_bwd(ne_ctx* ctx);
/* Token-major RMSNorm on caller-owned device buffers (rmsnorm, cpu_ops.h:20-60):
 * d_out [rows, dim] bf16.  And its backward (rmsnorm_bwd(_add),
 * cpu_ops.h:108-261): d_dx = J^T d_dy (+ d_residual if not NULL); d_dw
 * (optional) accumulates the gain gradient. */
NE_API ne_status ne_rmsnorm_fwd(ne_ctx* ctx, const float* d_x, const float* d_w, int rows,
                                void* d_out_bf16);
NE_API ne_status ne_rmsnorm_bwd_add(ne_ctx* ctx, const float* d_dy, const float* d_x,
                                    const float* d_w, int rows, const float* d_residual,
                                    float* d_dx, float* d_dw);

/* Causal GQA scaled-dot-product attention on device buffers (the core of
 * sdpaFwd, mil_dynamic.h:184-198): d_q [B*S][Hq*hd] bf16 (token major), d_k /
 * d_v [B][Hkv][S][hd] bf16; d_out [B*S][Hq*hd] bf16; d_lse (optional) [B][Hq][S]
 * fp32 log-sum-exp of the scaled scores in the log2 domain.  Enqueued on the
 * context stream. */
NE_API ne_status ne_sdpa_fwd_device(ne_ctx* ctx, const void* d_q, const void* d_k,
                                    const void* d_v, int B, int S, void* d_out, float* d_lse);

/* ---- data-parallel gradients (NCCL over NVLink; no reference counterpart:
 * the reference trains on one device) ---------------------------------------
 * Rank 0 makes an id with ne_comm_unique_id and shares it out of band; every
 * rank calls ne_comm_init with it.  Afterwards each ne_train_fwd_bwd(_device)
 * sums the gradients over ranks in buckets overlapped with its backward (one
 * bucket per layer, issued as soon as the layer's gradients are final), so
 * ne_adamw_step with grad_scale = 1/world takes the same step on every rank.
 * With gradient accumulation, turn reduction off (ne_comm_set_reduce(ctx, 0))
 * for all but the last micro-step of each optimizer step.  NCCL is loaded at
 * run time (libnccl.so.2); NE_ERR_UNSUPPORTED if it cannot be. */
#define NE_COMM_ID_BYTES 128
NE_API ne_status ne_comm_unique_id(void* id_out);
NE_API ne_status ne_comm_init(ne_ctx* ctx, const void* id, int rank, int world);
NE_API ne_status ne_comm_set_reduce(ne_ctx* ctx, int on);
/* Deadline, in ms, of every wait on the exchange: ne_comm_init waiting for all
 * ranks to join, and ne_sync (and the calls that synchronise) waiting for a
 * step's exchange.  0 restores the default (NE_COMM_TIMEOUT_MS, else 120 s).
 * When a deadline passes -- a rank that never joined or never entered an
 * exchange -- the communicator is aborted (its kernels return), the call
 * returns NE_ERR_TIMEOUT, and later exchanges return NE_ERR_STATE until
 * ne_comm_init builds a new communicator.  May be called before ne_comm_init. */
NE_API ne_status ne_comm_set_timeout(ne_ctx* ctx, int timeout_ms);
/* Sum the whole gradient pool over the ranks now (ordered on the stream). */
NE_API ne_status ne_grad_allreduce_async(ne_ctx* ctx);
/* ZeRO-1 (on = 1; no counterpart in the single-device reference).  Every
 * trainable tensor is owned in world parts (ne_shard_range): the gradient
 * buckets reduce-scatter (rank r keeps the sum of part r), the norm adds the
 * ranks' shares, AdamW updates only the owned parts, and the updated compute
 * copies (bf16 matrices, fp32 gains) are all-gathered.  The exchange runs on
 * the library's own kernels over NVLink peer memory: the ranks' buffers are
 * mapped through CUDA IPC at the first reduced micro-step (collective, outside
 * any capture), and the ranks order their reads by epoch flags whose waits
 * are bounded by the ne_comm_set_timeout deadline (NE_ERR_TIMEOUT).  At most
 * 8 ranks, one process per GPU of one node.  NE_COMM_PX=0 runs the same
 * scheme over NCCL collectives (equal parts of the matrices and the
 * embedding, replicated gains).  With gradient accumulation, turn reduction
 * on only for the last micro-step of each optimizer step.  The fp32 masters
 * and Adam moments of the other parts are then stale until
 * ne_train_gather_state(ctx, 0), which checkpoints and the state getters
 * require; gradients read back need ne_train_gather_state(ctx, 1).  Call
 * ne_train_gather_state(ctx, 0) before turning sharding off. */
NE_API ne_status ne_comm_set_sharding(ne_ctx* ctx, int on);
/* Collective (every rank, same order): all-gather the owned parts of the fp32
 * masters and both moments (which = 0) or of the reduced gradients (which =
 * 1).  A no-op without sharding. */
NE_API ne_status ne_train_gather_state(ne_ctx* ctx, int which);

/* Which part of an n-element tensor rank `rank` of `world` owns under ZeRO-1
 * over peer memory: [*off, *off + *len).  Part boundaries sit at multiples of
 * 64 elements (256-byte aligned fp32, 128-byte aligned bf16) and the last
 * rank takes the remainder, so every element is owned exactly once and every
 * rank computes the same table.  Host arithmetic only (no GPU). */
NE_API ne_status ne_shard_range(long long n, int world, int rank, long long* off, long long* len);

/* The contiguous fp32 gradient pool (every trainable tensor's gradient), for
 * data-parallel reduction by the caller (e.g. an NCCL all-reduce on the
 * context's stream between ne_train_fwd_bwd and ne_adamw_step). */
NE_API ne_status ne_train_grad_pool(ne_ctx* ctx, float** d_grads, size_t* n_floats);

/* ---- allocation-free split-K product --------------------------------------
 * No counterpart in the reference: an addition for callers that must not
 * allocate device memory -- code running inside an allocator hook or a memory
 * pool callback, plug-ins whose host process owns every device allocation,
 * start-up code that runs before the caller's allocator exists.  It needs no
 * ne_ctx (creating one allocates).
 *
 * d_out[m*ld + n] = sum_k A[m,k] * B[n,k] in fp32 (the same product as
 * ne_gemm_device with epi 1), bf16 operands as there, computed with `splits`
 * split-K slices whose partial slabs live in a static device array of
 * NE_NOALLOC_SCRATCH_FLOATS floats (8 MiB) that every GPU loading the library
 * holds until exit.  Nothing is allocated: no cudaMalloc / cudaFree / pools.
 *   - Returns NE_ERR_INVALID, before any GPU work, if splits * M * N >
 *     NE_NOALLOC_SCRATCH_FLOATS, if K is not a multiple of 64 or K/64 is not
 *     a multiple of `splits`, if lda or ldb is below K or not a multiple of 8,
 *     if d_A or d_B is not 16-byte aligned or d_out not 4-byte aligned, or if
 *     `stream` belongs to another device than the current one.
 *   - Runs on `stream` (a cudaStream_t; NULL = default stream) of the current
 *     device and synchronises it before returning (NE_ERR_TIMEOUT reports a
 *     kernel wait that expired).
 *   - The first call on a device looks up the array's device address; make it
 *     before any stream capture.
 *   - All calls share the one array: calls whose GPU work overlaps race. */
#define NE_NOALLOC_SCRATCH_FLOATS ((size_t)2 * 1024 * 1024)
NE_API ne_status ne_gemm_splitk_noalloc(const void* d_A, long long lda, int M, const void* d_B,
                                        long long ldb, int N, int K, int splits, float* d_out,
                                        long long ld, void* stream);

/* ---------------------------------------------------------------- measurement
 * Read-only streaming floor (no counterpart in the reference; a measuring aid
 * for the decode attention's roofline).  Reads `bytes` (a multiple of 16) of
 * device memory at d_src (16-byte aligned) once, through the decode attention's
 * data path -- 8 warps per SM, equal per-warp ranges, 3-stage rings of 8 KB
 * bulk copies -- with no arithmetic, XOR-folding one word per chunk into
 * d_sink[0]; d_sink[1] is set to 1 if a bounded wait ran out.  Enqueued on
 * `stream` (a cudaStream_t; NULL = default stream) without synchronising, so
 * a caller can time it with events. */
NE_API ne_status ne_stream_read(const void* d_src, long long bytes, unsigned int* d_sink,
                                void* stream);

#ifdef __cplusplus
}
#endif
#endif /* NE_H_ */
