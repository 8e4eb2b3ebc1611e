// ckpt.cu -- v4 checkpoint reader (host code) feeding the device weights.
//
// Layout (ane-training/training/training_dynamic/config.h:83-91 header;
// train.m:110-130 body, read back by train.m:133-165):
//   CkptHdr (96 bytes)
//   per layer: Wq Wk Wv Wo W1 W2 W3 rms_att rms_ffn (fp32), then (m, v) of each
//   rms_final, m, v;  embed [V*D], m, v
//   optional trailing block "QKN1" (this library's extension; v4 readers stop
//   before it): int n_layers, head_dim; per layer q_norm, k_norm, then m, v of each.
#include <sys/stat.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/ne.h"
#include "ne_ckpt.h"
#include "ne_fault.h"

namespace {

using ne::CkptHdr;

struct File {
  FILE* f = nullptr;
  ~File() {
    if (f) fclose(f);
  }
};

bool read_f32(FILE* f, std::vector<float>& buf, size_t n) {
  buf.resize(n);
  return fread(buf.data(), 4, n, f) == n;
}

bool skip_f32(FILE* f, size_t n) { return fseeko(f, (off_t)(n * 4), SEEK_CUR) == 0; }

void fill_info(const CkptHdr& h, bool has_qk, ne_ckpt_info* info) {
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

}  // namespace

namespace ne {

ne_status ckpt_check(const char* path, const ne_model_cfg* want, CkptHdr* hdr, bool* has_qk) {
  File fh;
  fh.f = fopen(path, "rb");
  if (!fh.f) return NE_ERR_IO;
  FILE* f = fh.f;
  struct stat st;
  if (fstat(fileno(f), &st) != 0) return NE_ERR_IO;
  const uint64_t size = (uint64_t)st.st_size;
  CkptHdr& h = *hdr;
  if (fread(&h, sizeof(h), 1, f) != 1) return NE_ERR_FORMAT;
  if (h.magic != kCkptMagic || h.version != 4) return NE_ERR_FORMAT;
  // shapes of a model at all (a header with flipped bits usually fails here)
  const int lim = 1 << 24;
  const int dims[7] = {h.n_layers, h.vocab_size, h.dim, h.hidden_dim, h.n_heads, h.kv_heads,
                       h.head_dim};
  for (int d : dims)
    if (d <= 0 || d > lim) return NE_ERR_FORMAT;
  if (h.q_dim != h.n_heads * h.head_dim || h.n_heads % h.kv_heads != 0) return NE_ERR_FORMAT;
  if (want && (h.n_layers != want->n_layers || h.vocab_size != want->vocab ||
               h.dim != want->dim || h.hidden_dim != want->hidden ||
               h.n_heads != want->n_heads || h.kv_heads != want->kv_heads ||
               h.head_dim != want->head_dim))
    return NE_ERR_FORMAT;
  // body: (tensor, m, v) of every trainable tensor, train.m:110-130
  const uint64_t D = h.dim, F = h.hidden_dim, qd = h.q_dim, kvd = (uint64_t)h.kv_heads * h.head_dim;
  const uint64_t layer = qd * D + 2 * kvd * D + D * qd + 3 * F * D + 2 * D;
  const uint64_t body = 96 + 4 * 3 * ((uint64_t)h.n_layers * layer + D + (uint64_t)h.vocab_size * D);
  if (size < body) return NE_ERR_FORMAT;   // truncated
  *has_qk = false;
  if (size >= body + 12) {
    char magic[4];
    if (fseeko(f, (off_t)body, SEEK_SET) != 0 || fread(magic, 1, 4, f) != 4) return NE_ERR_FORMAT;
    if (std::memcmp(magic, "QKN1", 4) == 0) {
      int nl = 0, hd = 0;
      if (fread(&nl, 4, 1, f) != 1 || fread(&hd, 4, 1, f) != 1) return NE_ERR_FORMAT;
      if (nl != h.n_layers || hd != h.head_dim) return NE_ERR_FORMAT;
      if (size < body + 12 + 4 * 6 * (uint64_t)nl * hd) return NE_ERR_FORMAT;   // truncated
      *has_qk = true;
    }
  }
  return NE_OK;
}

}  // namespace ne

extern "C" NE_API ne_status ne_ckpt_probe(const char* path, ne_model_cfg* cfg, ne_ckpt_info* info) {
  ne_status fs;
  if (ne::fault_point("ne_ckpt_probe", &fs)) return fs;
  if (!path) return NE_ERR_INVALID;
  CkptHdr h;
  bool has_qk = false;
  const ne_status s = ne::ckpt_check(path, nullptr, &h, &has_qk);
  if (s != NE_OK) return s;
  if (cfg) {
    cfg->n_layers = h.n_layers;
    cfg->dim = h.dim;
    cfg->hidden = h.hidden_dim;
    cfg->n_heads = h.n_heads;
    cfg->kv_heads = h.kv_heads;
    cfg->head_dim = h.head_dim;
    cfg->vocab = h.vocab_size;
    cfg->qk_norm = has_qk ? 1 : 0;
  }
  if (info) fill_info(h, has_qk, info);
  return NE_OK;
}

extern "C" NE_API ne_status ne_load_ckpt_v4(ne_ctx* ctx, const char* path, ne_ckpt_info* info) {
  if (!ctx || !path) return NE_ERR_INVALID;
  ne_status fs;
  if (ne::fault_point("ne_load_ckpt_v4", &fs)) return fs;
  {
    // every check before any state changes: a truncated or corrupt file
    // leaves the context as it was
    ne_model_cfg m;
    if (ne_get_cfg(ctx, &m) != NE_OK) return NE_ERR_INVALID;
    CkptHdr h;
    bool qk = false;
    const ne_status cs = ne::ckpt_check(path, &m, &h, &qk);
    if (cs != NE_OK) return cs;
  }
  bool handled = false;
  ne_status ts = ne::train_ckpt_load(ctx, path, info, &handled);
  if (handled) return ts;
  ne_model_cfg m;
  if (ne_get_cfg(ctx, &m) != NE_OK) return NE_ERR_INVALID;
  File fh;
  fh.f = fopen(path, "rb");
  if (!fh.f) return NE_ERR_IO;
  FILE* f = fh.f;
  CkptHdr h;
  if (fread(&h, sizeof(h), 1, f) != 1) return NE_ERR_FORMAT;
  if (h.magic != 0x424C5A54 || h.version != 4) return NE_ERR_FORMAT;
  if (h.n_layers != m.n_layers || h.vocab_size != m.vocab || h.dim != m.dim ||
      h.hidden_dim != m.hidden || h.n_heads != m.n_heads || h.kv_heads != m.kv_heads ||
      h.head_dim != m.head_dim || h.q_dim != m.n_heads * m.head_dim)
    return NE_ERR_FORMAT;
  const size_t D = m.dim, F = m.hidden, qd = (size_t)h.q_dim, kvd = (size_t)m.kv_heads * m.head_dim;
  const size_t sz[9] = {qd * D, kvd * D, kvd * D, D * qd, F * D, D * F, F * D, D, D};
  std::vector<std::vector<float>> t(9);
  // Layer tensors are set once the optional QK-norm block is known, so read
  // every layer first (host memory: one fp32 copy of the transformer weights).
  std::vector<std::vector<std::vector<float>>> layers(m.n_layers);
  for (int l = 0; l < m.n_layers; ++l) {
    layers[l].resize(9);
    for (int k = 0; k < 9; ++k)
      if (!read_f32(f, layers[l][k], sz[k])) return NE_ERR_FORMAT;
    for (int k = 0; k < 9; ++k)
      if (!skip_f32(f, 2 * sz[k])) return NE_ERR_FORMAT;
  }
  std::vector<float> rms_final, embed;
  if (!read_f32(f, rms_final, D) || !skip_f32(f, 2 * D)) return NE_ERR_FORMAT;
  if (!read_f32(f, embed, (size_t)m.vocab * D)) return NE_ERR_FORMAT;
  if (!skip_f32(f, 2 * (size_t)m.vocab * D)) return NE_ERR_FORMAT;
  std::vector<std::vector<float>> qn(m.n_layers), kn(m.n_layers);
  bool has_qk = false;
  char magic[4];
  if (fread(magic, 1, 4, f) == 4 && std::memcmp(magic, "QKN1", 4) == 0) {
    int nl = 0, hd = 0;
    if (fread(&nl, 4, 1, f) != 1 || fread(&hd, 4, 1, f) != 1) return NE_ERR_FORMAT;
    if (nl != m.n_layers || hd != m.head_dim) return NE_ERR_FORMAT;
    for (int l = 0; l < nl; ++l) {
      if (!read_f32(f, qn[l], hd) || !read_f32(f, kn[l], hd) || !skip_f32(f, 4 * (size_t)hd))
        return NE_ERR_FORMAT;
    }
    has_qk = true;
  }
  for (int l = 0; l < m.n_layers; ++l) {
    auto& L = layers[l];
    ne_status s = ne_set_layer_weights(ctx, l, L[0].data(), L[1].data(), L[2].data(), L[3].data(),
                                       L[4].data(), L[5].data(), L[6].data(), L[7].data(),
                                       L[8].data(), has_qk ? qn[l].data() : nullptr,
                                       has_qk ? kn[l].data() : nullptr);
    if (s != NE_OK) return s;
    std::vector<std::vector<float>>().swap(L);
  }
  ne_status s = ne_set_global_weights(ctx, rms_final.data(), embed.data());
  if (s != NE_OK) return s;
  if (info) fill_info(h, has_qk, info);
  return NE_OK;
}
