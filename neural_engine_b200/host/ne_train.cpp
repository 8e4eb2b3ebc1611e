// ne_train -- command-line training driver over libne.so, a drop-in for the
// reference's training_dynamic/train.m driver (train.m:168-947).
//
// Same flags (--scratch, --resume, --steps, --lr, --accum, --warmup, --clip,
// --data), same checkpoint file and layout (ane_<model>_dyn_ckpt.bin, v4),
// same scratch initialisation (srand48(42), uniform scales, train.m:234-255),
// same data sampling (uint16 token file, srand48(42 + start_step), one window
// of SEQ+1 tokens per sequence, train.m:276-284 and 389-401), same schedule
// (warmup + cosine, train.m:851-858), optimizer step every --accum steps with
// global-norm clipping, checkpoint every 100 steps on a new best loss
// (train.m:908-916), and stdout lines the reference dashboard parses
// ("step N loss=...", "[ckpt saved, best_loss=...]").
//
// A "step" is one micro-step as in the reference: --batch sequences (1 in the
// reference) through forward + backward.  As in the reference the classifier
// runs over the token ids present in the data file (vocabulary compaction,
// cpu_ops.h:385-431; --no-compact-vocab uses the full vocabulary).  Gradients
// need no loss scaling (fp32 accumulation), so the update scales by 1/accum.
//
// Extensions: --model (qwen3_06b | stories110m | custom shape flags), --seq,
// --batch, --ckpt, --device, --synthetic (uniform random tokens, no data
// file), --qk-norm / --theta / --eps / --alpha (the reference's training
// model uses theta 1e4, eps 1e-5, no QK-norm, alpha = 1/sqrt(2L)), --dump-init
// and --print-windows (host-only checks, no GPU).  Data-parallel ranks come
// from RANK / WORLD_SIZE / LOCAL_RANK; rank 0 publishes the NCCL id through
// the file named by NE_COMM_ID_FILE.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "ne.h"

namespace {

struct Args {
  bool scratch = false, resume = false, synthetic = false, compact_vocab = true, print_vocab = false;
  bool zero1 = false;   // data parallel: ZeRO-1 (sharded optimizer state)
  bool data_u32 = false;   // token file of uint32 ids (vocabularies beyond 65,536)
  int steps = 10000, accum = 10, warmup = 100;
  float lr = 3e-4f, clip = 1.0f;
  std::string data = "../tinystories_data00.bin";
  std::string model = "qwen3_06b";
  std::string ckpt;
  std::string dump_init;
  int print_windows = 0;
  int seq = 0, batch = 1, device = -1, save_every = 100;
  int layers = 0, dim = 0, hidden = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0;
  int qk_norm = -1;
  float theta = 0.f, eps = 0.f, alpha = -1.f;
};

void usage() {
  std::printf(
      "usage: ne_train [--scratch | --resume] [--steps N] [--lr X] [--accum N] [--warmup N]\n"
      "                [--clip X] [--data FILE] [--data-u32] [--model qwen3_06b|stories110m]\n"
      "                [--seq S]\n"
      "                [--batch B] [--ckpt FILE] [--device D] [--synthetic] [--save-every N]\n"
      "                [--qk-norm 0|1] [--theta X] [--eps X] [--alpha X] [--no-compact-vocab]\n"
      "                [--zero1]   (with WORLD_SIZE > 1: reduce-scatter + sharded AdamW)\n"
      "                [--layers N --dim N --hidden N --heads N --kv-heads N --head-dim N\n"
      "                 --vocab N] [--dump-init FILE] [--print-windows N] [--print-vocab]\n");
}

bool parse(int argc, char** argv, Args& a) {
  for (int i = 1; i < argc; ++i) {
    const std::string s = argv[i];
    auto next = [&](const char* name) -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "%s needs a value\n", name);
        std::exit(2);
      }
      return argv[++i];
    };
    if (s == "--resume") a.resume = true;
    else if (s == "--scratch") a.scratch = true;
    else if (s == "--synthetic") a.synthetic = true;
    else if (s == "--no-compact-vocab") a.compact_vocab = false;
    else if (s == "--zero1") a.zero1 = true;
    else if (s == "--data-u32") a.data_u32 = true;
    else if (s == "--print-vocab") a.print_vocab = true;
    else if (s == "--steps") a.steps = std::atoi(next("--steps"));
    else if (s == "--lr") a.lr = (float)std::atof(next("--lr"));
    else if (s == "--accum") a.accum = std::atoi(next("--accum"));
    else if (s == "--warmup") a.warmup = std::atoi(next("--warmup"));
    else if (s == "--clip") a.clip = (float)std::atof(next("--clip"));
    else if (s == "--data") a.data = next("--data");
    else if (s == "--model") a.model = next("--model");
    else if (s == "--ckpt") a.ckpt = next("--ckpt");
    else if (s == "--seq") a.seq = std::atoi(next("--seq"));
    else if (s == "--batch") a.batch = std::atoi(next("--batch"));
    else if (s == "--device") a.device = std::atoi(next("--device"));
    else if (s == "--save-every") a.save_every = std::atoi(next("--save-every"));
    else if (s == "--qk-norm") a.qk_norm = std::atoi(next("--qk-norm"));
    else if (s == "--theta") a.theta = (float)std::atof(next("--theta"));
    else if (s == "--eps") a.eps = (float)std::atof(next("--eps"));
    else if (s == "--alpha") a.alpha = (float)std::atof(next("--alpha"));
    else if (s == "--layers") a.layers = std::atoi(next("--layers"));
    else if (s == "--dim") a.dim = std::atoi(next("--dim"));
    else if (s == "--hidden") a.hidden = std::atoi(next("--hidden"));
    else if (s == "--heads") a.heads = std::atoi(next("--heads"));
    else if (s == "--kv-heads") a.kv_heads = std::atoi(next("--kv-heads"));
    else if (s == "--head-dim") a.head_dim = std::atoi(next("--head-dim"));
    else if (s == "--vocab") a.vocab = std::atoi(next("--vocab"));
    else if (s == "--dump-init") a.dump_init = next("--dump-init");
    else if (s == "--print-windows") a.print_windows = std::atoi(next("--print-windows"));
    else if (s == "-h" || s == "--help") {
      usage();
      std::exit(0);
    } else {
      std::fprintf(stderr, "unknown argument %s\n", s.c_str());
      usage();
      return false;
    }
  }
  return true;
}

struct Model {
  std::string name, ckpt;
  ne_model_cfg cfg{};
  int seq = 256;
};

// Model presets (training_dynamic/models/*.h), with the reference training
// model's numerics: RMSNorm eps 1e-5, RoPE theta 1e4, no QK-norm,
// residual alpha = 1/sqrt(2 L) (train.m:181).
bool make_model(const Args& a, Model& m) {
  ne_model_cfg& c = m.cfg;
  if (a.model == "qwen3_06b") {
    m.name = "Qwen3-0.6B";
    m.ckpt = "ane_qwen3_06b_dyn_ckpt.bin";
    c.n_layers = 28; c.dim = 1024; c.hidden = 3072; c.n_heads = 16; c.kv_heads = 8;
    c.head_dim = 128; c.vocab = 151936;
  } else if (a.model == "stories110m") {
    m.name = "Stories110M";
    m.ckpt = "ane_stories110M_dyn_ckpt.bin";
    c.n_layers = 12; c.dim = 768; c.hidden = 2048; c.n_heads = 12; c.kv_heads = 12;
    c.head_dim = 64; c.vocab = 32000;
  } else if (a.model == "custom") {
    m.name = "custom";
    m.ckpt = "ane_custom_dyn_ckpt.bin";
  } else {
    std::fprintf(stderr, "unknown model %s\n", a.model.c_str());
    return false;
  }
  if (a.layers) c.n_layers = a.layers;
  if (a.dim) c.dim = a.dim;
  if (a.hidden) c.hidden = a.hidden;
  if (a.heads) c.n_heads = a.heads;
  if (a.kv_heads) c.kv_heads = a.kv_heads;
  if (a.head_dim) c.head_dim = a.head_dim;
  if (a.vocab) c.vocab = a.vocab;
  if (c.n_layers <= 0 || c.dim <= 0 || c.hidden <= 0 || c.n_heads <= 0 || c.kv_heads <= 0 ||
      c.head_dim <= 0 || c.vocab <= 0) {
    std::fprintf(stderr, "incomplete model shape\n");
    return false;
  }
  c.rms_eps = a.eps > 0.f ? a.eps : 1e-5f;
  c.rope_theta = a.theta > 0.f ? a.theta : 10000.0f;
  c.qk_norm = a.qk_norm > 0 ? 1 : 0;
  c.qk_eps = 1e-6f;
  c.res_alpha = a.alpha >= 0.f ? a.alpha : 1.0f / std::sqrt(2.0f * (float)c.n_layers);
  if (a.seq > 0) m.seq = a.seq;
  if (!a.ckpt.empty()) m.ckpt = a.ckpt;
  return true;
}

// Scratch initialisation in the reference's order and arithmetic
// (train.m:234-255): srand48(42); every matrix element scale * (2*drand48()-1)
// with the float scale promoted to double; gains 1.0; embedding 0.02 scale.
struct HostWeights {
  std::vector<std::vector<float>> wq, wk, wv, wo, w1, w2, w3, att, ffn;
  std::vector<float> rms_final, embed;
};

void scratch_init(const ne_model_cfg& c, HostWeights& w) {
  const size_t D = c.dim, F = c.hidden, qd = (size_t)c.n_heads * c.head_dim,
               kvd = (size_t)c.kv_heads * c.head_dim, L = c.n_layers, V = c.vocab;
  srand48(42);
  const float scale_d = 1.0f / sqrtf((float)D), scale_qd = 1.0f / sqrtf((float)qd),
              scale_h = 1.0f / sqrtf((float)F);
  const float res_scale = 1.0f / sqrtf(2.0f * (float)L);
  auto fill = [](std::vector<float>& v, size_t n, float scale) {
    v.resize(n);
    for (size_t i = 0; i < n; ++i) v[i] = (float)(scale * (2 * drand48() - 1));
  };
  for (auto* t : {&w.wq, &w.wk, &w.wv, &w.wo, &w.w1, &w.w2, &w.w3, &w.att, &w.ffn}) t->resize(L);
  for (size_t l = 0; l < L; ++l) {
    fill(w.wq[l], qd * D, scale_d);
    fill(w.wk[l], kvd * D, scale_d);
    fill(w.wv[l], kvd * D, scale_d);
    fill(w.wo[l], D * qd, scale_qd * res_scale);
    fill(w.w1[l], F * D, scale_h);
    fill(w.w2[l], D * F, scale_d * res_scale);
    fill(w.w3[l], F * D, scale_h);
    w.att[l].assign(D, 1.0f);
    w.ffn[l].assign(D, 1.0f);
  }
  w.rms_final.assign(D, 1.0f);
  const float escale = 0.02f;
  fill(w.embed, V * D, escale);
}

// v4 file with zero Adam moments (train.m:97-131 layout), for --dump-init.
bool write_init_ckpt(const std::string& path, const ne_model_cfg& c, const HostWeights& w, int seq) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) return false;
  struct Hdr {
    int magic, version, step, total_steps;
    int n_layers, vocab_size, dim, hidden_dim, n_heads, seq_len;
    float lr, loss;
    double cum_compile, cum_train, cum_wall;
    int cum_steps, cum_batches, adam_t;
    int kv_heads, head_dim, q_dim;
  } h;
  static_assert(sizeof(Hdr) == 96, "v4 header");
  std::memset(&h, 0, sizeof(h));
  h.magic = 0x424C5A54; h.version = 4; h.n_layers = c.n_layers; h.vocab_size = c.vocab;
  h.dim = c.dim; h.hidden_dim = c.hidden; h.n_heads = c.n_heads; h.seq_len = seq;
  h.kv_heads = c.kv_heads; h.head_dim = c.head_dim; h.q_dim = c.n_heads * c.head_dim;
  bool ok = std::fwrite(&h, sizeof(h), 1, f) == 1;
  auto put = [&](const std::vector<float>& v) {
    ok = ok && std::fwrite(v.data(), 4, v.size(), f) == v.size();
  };
  auto zeros = [&](size_t n) {
    std::vector<float> z(n, 0.f);
    put(z);
    put(z);
  };
  for (int l = 0; l < c.n_layers; ++l) {
    const std::vector<float>* t[9] = {&w.wq[l], &w.wk[l], &w.wv[l], &w.wo[l], &w.w1[l],
                                      &w.w2[l], &w.w3[l], &w.att[l], &w.ffn[l]};
    for (auto* p : t) put(*p);
    for (auto* p : t) zeros(p->size());
  }
  put(w.rms_final);
  zeros(w.rms_final.size());
  put(w.embed);
  zeros(w.embed.size());
  return std::fclose(f) == 0 && ok;
}

// Memory-mapped token file: uint16 ids as the reference writes them
// (tools/tokenize_data.py, read at train.m:276-284), or uint32 ids with
// --data-u32 for vocabularies beyond 65,536 (Qwen3's 151,936).
struct TokenFile {
  const void* base = nullptr;
  size_t n = 0, bytes = 0;
  int fd = -1;
  bool u32 = false;
  ~TokenFile() {
    if (base) munmap(const_cast<void*>(base), bytes);
    if (fd >= 0) close(fd);
  }
  bool open_file(const std::string& path, bool wide) {
    u32 = wide;
    fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return false;
    struct stat st;
    if (fstat(fd, &st) != 0) return false;
    bytes = (size_t)st.st_size;
    void* p = mmap(nullptr, bytes, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) return false;
    base = p;
    n = bytes / (u32 ? 4 : 2);
    return true;
  }
  // a file cut inside a token (its size not a whole number of tokens)
  bool truncated() const { return bytes % (u32 ? 4 : 2) != 0; }
  uint32_t operator[](size_t i) const {
    return u32 ? static_cast<const uint32_t*>(base)[i] : static_cast<const uint16_t*>(base)[i];
  }
};

// One micro-step's windows: for each sequence, pos = drand48() * (n - S - 1)
// and tokens [pos, pos + S] (train.m:395-401).  Synthetic data draws uniform
// token ids from the same generator instead.
void sample(const TokenFile& tf, bool synthetic, int V, int B, int S, std::vector<int32_t>& out,
            std::vector<size_t>* positions) {
  out.resize((size_t)B * (S + 1));
  for (int b = 0; b < B; ++b) {
    if (synthetic) {
      for (int t = 0; t <= S; ++t) out[(size_t)b * (S + 1) + t] = (int32_t)(drand48() * V);
      continue;
    }
    const size_t max_pos = tf.n - S - 1;
    const size_t pos = (size_t)(drand48() * max_pos);
    if (positions) positions->push_back(pos);
    for (int t = 0; t <= S; ++t) out[(size_t)b * (S + 1) + t] = (int32_t)tf[pos + t];
  }
}

// Vocabulary compaction map (vocab_map_build, cpu_ops.h:391-414): the token
// ids present in the data, in increasing order.
std::vector<int32_t> vocab_map(const TokenFile& tf, int V) {
  std::vector<char> used(V, 0);
  for (size_t i = 0; i < tf.n; ++i)
    if (tf[i] < (uint32_t)V) used[tf[i]] = 1;
  std::vector<int32_t> c2f;
  for (int v = 0; v < V; ++v)
    if (used[v]) c2f.push_back(v);
  return c2f;
}

double now_ms() {
  using namespace std::chrono;
  return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v ? std::atoi(v) : dflt;
}

#define CHECK(call)                                                                  \
  do {                                                                               \
    ne_status s_ = (call);                                                           \
    if (s_ != NE_OK) {                                                               \
      std::fprintf(stderr, "%s failed: %s (%s)\n", #call, ne_status_str(s_),         \
                   ctx ? ne_last_error(ctx) : "");                                   \
      return 1;                                                                      \
    }                                                                                \
  } while (0)

}  // namespace

int main(int argc, char** argv) {
  std::setbuf(stdout, nullptr);
  Args a;
  if (!parse(argc, argv, a)) return 2;
  Model mdl;
  if (!make_model(a, mdl)) return 2;
  const ne_model_cfg& c = mdl.cfg;
  const int S = mdl.seq, B = a.batch;
  if (B <= 0 || S <= 0 || a.accum <= 0 || a.steps <= 0) {
    std::fprintf(stderr, "batch, seq, accum and steps must be positive\n");
    return 2;
  }
  const int rank = env_int("RANK", 0), world = env_int("WORLD_SIZE", 1);
  const int device = a.device >= 0 ? a.device : env_int("LOCAL_RANK", 0);
  ne_ctx* ctx = nullptr;

  // ---- host-only modes (no GPU)
  if (!a.dump_init.empty()) {
    HostWeights w;
    scratch_init(c, w);
    if (!write_init_ckpt(a.dump_init, c, w, S)) {
      std::fprintf(stderr, "cannot write %s\n", a.dump_init.c_str());
      return 1;
    }
    return 0;
  }
  TokenFile tf;
  if (!a.synthetic) {
    if (!tf.open_file(a.data, a.data_u32)) {
      std::printf("Cannot open %s\n", a.data.c_str());
      return 1;
    }
    if (tf.truncated()) {
      std::printf("Token file truncated: %zu bytes is not a whole number of %d-byte tokens\n",
                  tf.bytes, a.data_u32 ? 4 : 2);
      return 1;
    }
    if (tf.n < (size_t)S + 2) {
      std::printf("Token file too short\n");
      return 1;
    }
  }
  std::vector<int32_t> c2f;
  if (!a.synthetic && a.compact_vocab) c2f = vocab_map(tf, c.vocab);
  if (a.print_vocab) {
    std::printf("%zu\n", c2f.size());
    for (int32_t v : c2f) std::printf("%d\n", v);
    return 0;
  }
  if (a.print_windows > 0) {
    srand48(42 + 0 + 1000L * rank);
    std::vector<int32_t> tok;
    for (int i = 0; i < a.print_windows; ++i) {
      std::vector<size_t> pos;
      sample(tf, a.synthetic, c.vocab, B, S, tok, &pos);
      for (size_t p : pos) std::printf("%zu\n", p);
      if (a.synthetic) std::printf("%d\n", tok[0]);
    }
    return 0;
  }

  // ---- data-parallel rendezvous (host only, before any GPU work): rank 0
  // publishes the NCCL id in a file, the others read it
  unsigned char id[NE_COMM_ID_BYTES];
  if (world > 1) {
    const char* idf = std::getenv("NE_COMM_ID_FILE");
    const std::string path = idf ? idf : "ne_comm_id.bin";
    if (rank == 0) {
      CHECK(ne_comm_unique_id(id));
      const std::string tmp = path + ".tmp";
      FILE* f = std::fopen(tmp.c_str(), "wb");
      if (!f || std::fwrite(id, 1, sizeof(id), f) != sizeof(id) || std::fclose(f) != 0 ||
          std::rename(tmp.c_str(), path.c_str()) != 0) {
        std::fprintf(stderr, "cannot publish the NCCL id to %s\n", path.c_str());
        return 1;
      }
    } else {
      // a rank 0 that never starts (or died) ends this rank's wait at the
      // communicator deadline (NE_COMM_TIMEOUT_MS, default 60 s)
      const int limit_ms = env_int("NE_COMM_TIMEOUT_MS", 60000);
      bool got = false;
      const double t0 = now_ms();
      while (!got) {
        FILE* f = std::fopen(path.c_str(), "rb");
        if (f) {
          got = std::fread(id, 1, sizeof(id), f) == sizeof(id);
          std::fclose(f);
        }
        if (got || now_ms() - t0 > limit_ms) break;
        std::this_thread::sleep_for(std::chrono::milliseconds(50));
      }
      if (!got) {
        std::fprintf(stderr, "rank %d: no NCCL id in %s after %d ms (rank 0 did not start)\n",
                     rank, path.c_str(), limit_ms);
        return 1;
      }
    }
  }

  // ---- the checkpoint to resume from, checked on the host before any GPU
  // work: a corrupt or truncated file is reported instead of half-loaded
  bool ckpt_usable = false;
  if (a.resume) {
    struct stat cst;
    if (stat(mdl.ckpt.c_str(), &cst) == 0) {
      ne_model_cfg hc = c;
      const ne_status ps = ne_ckpt_probe(mdl.ckpt.c_str(), &hc, nullptr);
      const bool same = hc.n_layers == c.n_layers && hc.dim == c.dim && hc.hidden == c.hidden &&
                        hc.n_heads == c.n_heads && hc.kv_heads == c.kv_heads &&
                        hc.head_dim == c.head_dim && hc.vocab == c.vocab;
      if (ps != NE_OK || !same) {
        std::printf("[RESUME FAILED] %s: %s\n", mdl.ckpt.c_str(),
                    ps == NE_ERR_FORMAT ? "bad header or truncated file"
                    : ps != NE_OK       ? ne_status_str(ps)
                                        : "a different model");
        if (!a.scratch) {
          std::printf("  ERROR: unusable checkpoint; remove it or pass --scratch.\n");
          return 1;
        }
      } else {
        ckpt_usable = true;
      }
    }
  }

  // ---- context and weights
  CHECK(ne_init(&ctx, &c, device));
  int start_step = 0, adam_t = 0, total_steps = a.steps;
  float lr = a.lr, resume_loss = 0.f;
  double cum_train = 0, cum_wall = 0;
  int cum_steps = 0;
  bool resuming = false;
  if (a.resume && ckpt_usable) {
    ne_ckpt_info info{};
    if (ne_load_ckpt_v4(ctx, mdl.ckpt.c_str(), &info) == NE_OK) {
      CHECK(ne_train_alloc(ctx, B, S));
      CHECK(ne_load_ckpt_v4(ctx, mdl.ckpt.c_str(), &info));   // masters + Adam moments
      start_step = info.step;
      total_steps = info.total_steps;
      lr = info.lr;
      resume_loss = info.loss;
      cum_train = info.cum_train;
      cum_wall = info.cum_wall;
      cum_steps = info.cum_steps;
      adam_t = info.adam_t;
      resuming = true;
      if (rank == 0) std::printf("[RESUMED step %d, loss=%.4f]\n", start_step, resume_loss);
    }
  }
  const double qd = (double)c.n_heads * c.head_dim, kvd = (double)c.kv_heads * c.head_dim;
  const double per_layer = qd * c.dim + 2 * kvd * c.dim + c.dim * qd + 3.0 * c.hidden * c.dim;
  if (!resuming) {
    if (rank == 0) {
      // train.m:222's banner, word for word: the reference's dashboard reads the
      // model name and layer count from it (dashboard.py RE_MODEL_NAME)
      std::printf("=== ANE Dynamic Training: %s (%d layers, GQA %d/%d heads) ===\n",
                  mdl.name.c_str(), c.n_layers, c.n_heads, c.kv_heads);
      std::printf("dim=%d q_dim=%d kv_dim=%d hd=%d hidden=%d seq=%d vocab=%d batch=%d\n", c.dim,
                  (int)qd, (int)kvd, c.head_dim, c.hidden, S, c.vocab, B);
      const double xf = c.n_layers * (per_layer + 2.0 * c.dim) / 1e6;
      const double em = (double)c.vocab * c.dim / 1e6;
      std::printf("Params: %.1fM (transformer %.1fM + embed %.1fM)\n", xf + em, xf, em);
      std::printf("Accum %d steps, LR=%g\n", a.accum, a.lr);
      const double fwd = 2.0 * c.n_layers * per_layer * S;
      std::printf("FLOPs/step: fwd=%.1fM total=%.1fM\n", fwd / 1e6, 3 * fwd / 1e6);
    }
    if (!a.scratch) {
      std::printf("  ERROR: no checkpoint to resume; use --scratch.\n");
      ne_free(ctx);
      return 1;
    }
    if (rank == 0) std::printf("  Training from scratch (random init)\n");
    HostWeights w;
    scratch_init(c, w);
    for (int l = 0; l < c.n_layers; ++l)
      CHECK(ne_set_layer_weights(ctx, l, w.wq[l].data(), w.wk[l].data(), w.wv[l].data(),
                                 w.wo[l].data(), w.w1[l].data(), w.w2[l].data(), w.w3[l].data(),
                                 w.att[l].data(), w.ffn[l].data(), nullptr, nullptr));
    CHECK(ne_set_global_weights(ctx, w.rms_final.data(), w.embed.data()));
    CHECK(ne_train_alloc(ctx, B, S));
    for (int l = 0; l < c.n_layers; ++l)
      CHECK(ne_train_set_masters(ctx, l, w.wq[l].data(), w.wk[l].data(), w.wv[l].data(),
                                 w.wo[l].data(), w.w1[l].data(), w.w2[l].data(), w.w3[l].data()));
    CHECK(ne_train_set_masters(ctx, -1, w.embed.data(), nullptr, nullptr, nullptr, nullptr,
                               nullptr, nullptr));
    CHECK(ne_train_sync_weights(ctx));
  }
  if (!a.synthetic && rank == 0)
    std::printf("Token data: %zu tokens (%.1f MB)\n", tf.n, tf.bytes / 1e6);
  if (!c2f.empty()) {
    CHECK(ne_train_set_vocab_map(ctx, c2f.data(), (int)c2f.size()));
    if (rank == 0)
      std::printf("Vocab compaction: %d \xe2\x86\x92 %zu active tokens (%.1fx reduction)\n", c.vocab,
                  c2f.size(), (float)c.vocab / (float)c2f.size());
  }

  // ---- data-parallel ranks
  if (world > 1) {
    CHECK(ne_comm_init(ctx, id, rank, world));
    if (a.zero1) CHECK(ne_comm_set_sharding(ctx, 1));
  }

  // ---- training loop (train.m:389-917)
  srand48(42 + start_step + 1000L * rank);
  float last_loss = 999.0f;
  float best_loss = resume_loss > 0 ? resume_loss : 999.0f;
  double total_train_ms = 0;
  int steps_done = 0;
  const double t_wall0 = now_ms();
  std::vector<int32_t> tok;
  for (int step = start_step; step < total_steps; ++step) {
    const double t0 = now_ms();
    sample(tf, a.synthetic, c.vocab, B, S, tok, nullptr);
    const bool update = (step + 1) % a.accum == 0 || step == total_steps - 1;
    if (world > 1) CHECK(ne_comm_set_reduce(ctx, update ? 1 : 0));
    float loss = 0.f;
    // every 10th step (train.m:763-777) runs the micro-step with per-stage
    // device timing; every rank takes the same path
    const bool log = step % 10 == 0 || step == start_step;
    float ph[NE_TRAIN_PHASES] = {0};
    if (log) CHECK(ne_train_fwd_bwd_timed(ctx, tok.data(), &loss, ph));
    else CHECK(ne_train_fwd_bwd(ctx, tok.data(), &loss));
    last_loss = loss;
    const double step_ms = now_ms() - t0;
    total_train_ms += step_ms;
    steps_done++;
    if (log) {
      float rg[4] = {0, 0, 0, 0};
      CHECK(ne_train_value_ranges(ctx, rg));
      if (rank == 0) {
        // train.m:766's fields: the forward / backward kernels take the ANE
        // stages' places; norms, residuals, RoPE and the GQA sums are fused
        // into them and there is no IOSurface staging, so those read 0; dwait
        // is the embedding backward with the wait for the gradient exchange
        const double fwd = ph[0] + ph[1] + ph[2], bwd = ph[4] + ph[5];
        const double timed = fwd + bwd + ph[3] + ph[6];
        std::printf("  timing: ane_fwd=%.1f io_fwd=%.1f rms=%.1f ane_bwd=%.1f io_bwd=%.1f "
                    "rms_bwd=%.1f cls=%.1f dw=%.1f dwait=%.1f resid=%.1f gqa=%.1f rope=%.1f "
                    "[gap=%.1f]\n",
                    fwd, 0.0, 0.0, bwd, 0.0, 0.0, (double)ph[3], 0.0, (double)ph[6], 0.0, 0.0, 0.0,
                    step_ms - timed > 0 ? step_ms - timed : 0.0);
        std::printf("  io_bwd: ffn_w=%.1f ffn_r=%.1f wot_w=%.1f s1=%.1f s2=%.1f s2r=%.1f "
                    "qkv_w=%.1f qkv_r=%.1f\n", 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0);
        std::printf("step %-4d loss=%.4f  lr=%.2e  %.1fms/step  x[%.2f,%.2f] dy[%.3e,%.3e]\n",
                    step, loss, lr, step_ms, rg[0], rg[1], rg[2], rg[3]);
      }
    }
    if (update) {
      const double ta = now_ms();
      adam_t++;
      lr = ne_lr_schedule(step, a.lr, a.warmup, total_steps, 0.1f);
      ne_adam_cfg ac{};
      ac.lr = lr;
      ac.beta1 = 0.9f;
      ac.beta2 = 0.95f;
      ac.eps = 1e-8f;
      ac.weight_decay = 0.1f;
      ac.grad_clip = a.clip;
      // gradients of `accum` micro-step means, summed over the ranks
      ac.grad_scale = 1.0f / (float)(a.accum * world);
      float norm = 0.f;
      CHECK(ne_adamw_step(ctx, &ac, adam_t, &norm));
      if (rank == 0) {
        if ((step + 1) % 10 == 0) std::printf("  grad_norm=%.4f\n", norm);
        std::printf("  [adam] step %d: %.1fms (update+restage+zero)\n", step, now_ms() - ta);
      }
      // sharded state: every rank takes part in gathering it at each save point
      if (a.zero1 && world > 1 && (step + 1) % a.save_every == 0)
        CHECK(ne_train_gather_state(ctx, 0));
      if (rank == 0 && (step + 1) % a.save_every == 0 && last_loss < best_loss) {
        best_loss = last_loss;
        ne_ckpt_info info{};
        info.step = step + 1;
        info.total_steps = total_steps;
        info.seq_len = S;
        info.lr = lr;
        info.loss = last_loss;
        info.cum_train = total_train_ms + cum_train;
        info.cum_wall = now_ms() - t_wall0 + cum_wall;
        info.cum_steps = steps_done + cum_steps;
        info.adam_t = adam_t;
        CHECK(ne_save_ckpt_v4(ctx, mdl.ckpt.c_str(), &info));
        std::printf("  [ckpt saved, best_loss=%.4f]\n", best_loss);
      }
    }
  }
  const double wall = now_ms() - t_wall0;
  if (rank == 0) {
    std::printf("\n=== Efficiency Report ===\n");
    std::printf("Total steps:  %d\n", steps_done);
    if (steps_done > 0)
      std::printf("Train time:   %.0fms (%.1fms/step)\n", total_train_ms, total_train_ms / steps_done);
    std::printf("Wall time:    %.1fs\n", (wall + cum_wall) / 1000);
  }
  ne_free(ctx);
  return 0;
}
