// ne_ckpt.h -- the v4 checkpoint header (training_dynamic/config.h:83-91).
#pragma once

#include "../../include/ne.h"

namespace ne {

// 96 bytes with native alignment; written and read as one block.
struct CkptHdr {
  int magic, version, step, total_steps;
  int n_layers, vocab_size, dim, hidden_dim, n_heads, seq_len;
  float lr, loss;
  double cum_compile, cum_train, cum_wall;
  int cum_steps, cum_batches, adam_t;
  int kv_heads, head_dim, q_dim;
};
static_assert(sizeof(CkptHdr) == 96, "v4 header must be 96 bytes");
constexpr int kCkptMagic = 0x424C5A54;

// Opens `path` and checks its header and size (ne_ckpt_probe's checks; with
// `want`, also that the shapes are want's model).  Fills *hdr and *has_qk.
ne_status ckpt_check(const char* path, const ne_model_cfg* want, CkptHdr* hdr, bool* has_qk);

// With training state allocated, restores the fp32 masters, the gains and the
// Adam moments exactly (and refreshes the bf16 compute copies); sets *handled
// to false (and does nothing) when the context has no training state.
ne_status train_ckpt_load(ne_ctx* ctx, const char* path, ne_ckpt_info* info, bool* handled);

}  // namespace ne
