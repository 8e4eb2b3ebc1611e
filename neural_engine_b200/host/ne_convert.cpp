// ne_convert -- Hugging Face safetensors <-> v4 training checkpoint.
//
// The format adapters of the reference, ane-training/training/training_dynamic/
// tools/convert_hf.py (write_checkpoint, :58-171) and tools/export_hf.py
// (read_checkpoint / export_safetensors, :18-124), as one C++ tool that needs
// no Python packages and no network: it reads the model directory (config.json
// plus one or more *.safetensors files, F32 / BF16 / F16) and writes the v4
// file that ne_train --resume and ne_load_ckpt_v4 read, or the reverse.
//
//   ne_convert from-hf <model_dir> [-o ckpt.bin] [--steps N] [--seq S]
//                      [--qk-norm-block] [--rope-permute] [--hf-exact]
//   ne_convert to-hf <ckpt.bin> -o <dir> [--rope-permute] [--hf-exact]
//                    [--config config.json]
//
// Without flags the bytes written are those of the reference's converter:
// header {magic, 4, 0, steps, L, V, D, F, Hq, seq, 3e-4, 0, 0, 0, 0, 0, 0, 0,
// Hkv, hd, q_dim}, per layer q/k/v/o, gate (W1), down (W2), up (W3),
// input_layernorm, post_attention_layernorm, each followed later by zero Adam
// moments; then model.norm; then lm_head.weight when present, else
// model.embed_tokens.weight.  The reference drops Qwen3's QK-norm gains and
// keeps HF's RoPE layout (rotate_half: pairs (i, i + hd/2)) although its
// kernels rotate interleaved pairs (2i, 2i + 1).  Two options make the
// converted model compute what the HF model computes:
//   --qk-norm-block  append the per-layer q_norm / k_norm gains as the
//                    trailing "QKN1" block (v4 readers ignore it; this
//                    library loads it), with zero moments;
//   --rope-permute   reorder each head's rows of Wq and Wk (and the QK-norm
//                    gains) so that row 2i holds HF row i and row 2i+1 holds
//                    HF row i + hd/2: rotating interleaved pairs of the
//                    permuted projection is HF's rotate_half rotation, and
//                    q.k is unchanged because q and k move alike;
//   --hf-exact       both.
// to-hf applies the inverse permutation with --rope-permute and writes F32
// tensors under HF names (tied: model.embed_tokens.weight) plus a config.json
// (copied from --config, else a minimal one like export_hf.py's).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <dirent.h>

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace {

// ------------------------------------------------------------------ JSON
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonParser {
  const char* p;
  const char* end;
  std::string err;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool parse(Json& out) {
    ws();
    if (p >= end) return fail("unexpected end");
    const char c = *p;
    if (c == '{') return object(out);
    if (c == '[') return array(out);
    if (c == '"') {
      out.kind = Json::Str;
      return string(out.str);
    }
    if (c == 't' && end - p >= 4 && !std::strncmp(p, "true", 4)) {
      out.kind = Json::Bool, out.b = true, p += 4;
      return true;
    }
    if (c == 'f' && end - p >= 5 && !std::strncmp(p, "false", 5)) {
      out.kind = Json::Bool, out.b = false, p += 5;
      return true;
    }
    if (c == 'n' && end - p >= 4 && !std::strncmp(p, "null", 4)) {
      out.kind = Json::Null, p += 4;
      return true;
    }
    return number(out);
  }
  bool fail(const char* m) {
    err = m;
    return false;
  }
  bool string(std::string& s) {
    ++p;   // opening quote
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) return fail("bad escape");
        switch (*p) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u': {   // keep ASCII; anything else becomes '?'
            if (end - p < 5) return fail("bad \\u escape");
            const unsigned v = (unsigned)std::strtoul(std::string(p + 1, p + 5).c_str(), nullptr, 16);
            s += v < 128 ? (char)v : '?';
            p += 4;
            break;
          }
          default: s += *p;
        }
        ++p;
      } else {
        s += *p++;
      }
    }
    if (p >= end) return fail("unterminated string");
    ++p;
    return true;
  }
  bool number(Json& out) {
    char* e = nullptr;
    out.num = std::strtod(p, &e);
    if (e == p) return fail("bad value");
    out.kind = Json::Num;
    p = e;
    return true;
  }
  bool array(Json& out) {
    out.kind = Json::Arr;
    ++p;
    ws();
    if (p < end && *p == ']') {
      ++p;
      return true;
    }
    for (;;) {
      Json v;
      if (!parse(v)) return false;
      out.arr.push_back(std::move(v));
      ws();
      if (p < end && *p == ',') {
        ++p;
        continue;
      }
      if (p < end && *p == ']') {
        ++p;
        return true;
      }
      return fail("expected , or ]");
    }
  }
  bool object(Json& out) {
    out.kind = Json::Obj;
    ++p;
    ws();
    if (p < end && *p == '}') {
      ++p;
      return true;
    }
    for (;;) {
      ws();
      if (p >= end || *p != '"') return fail("expected key");
      std::string k;
      if (!string(k)) return false;
      ws();
      if (p >= end || *p != ':') return fail("expected :");
      ++p;
      Json v;
      if (!parse(v)) return false;
      out.obj.emplace_back(std::move(k), std::move(v));
      ws();
      if (p < end && *p == ',') {
        ++p;
        continue;
      }
      if (p < end && *p == '}') {
        ++p;
        return true;
      }
      return fail("expected , or }");
    }
  }
};

bool parse_json(const std::string& text, Json& out, std::string& err) {
  JsonParser jp{text.data(), text.data() + text.size(), {}};
  if (!jp.parse(out)) {
    err = jp.err;
    return false;
  }
  return true;
}

bool read_file(const std::string& path, std::string& out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[65536];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
  std::fclose(f);
  return true;
}

[[noreturn]] void die(const std::string& m) {
  std::fprintf(stderr, "ne_convert: %s\n", m.c_str());
  std::exit(1);
}

// ------------------------------------------------------------------ mapped files
struct Mapped {
  const uint8_t* data = nullptr;
  size_t size = 0;
  int fd = -1;
  ~Mapped() {
    if (data) munmap(const_cast<uint8_t*>(data), size);
    if (fd >= 0) close(fd);
  }
};

std::unique_ptr<Mapped> map_file(const std::string& path) {
  auto m = std::make_unique<Mapped>();
  m->fd = open(path.c_str(), O_RDONLY);
  if (m->fd < 0) die("cannot open " + path);
  struct stat st;
  if (fstat(m->fd, &st) != 0) die("cannot stat " + path);
  m->size = (size_t)st.st_size;
  if (m->size > 0) {
    void* p = mmap(nullptr, m->size, PROT_READ, MAP_PRIVATE, m->fd, 0);
    if (p == MAP_FAILED) die("cannot map " + path);
    m->data = static_cast<const uint8_t*>(p);
  }
  return m;
}

// ------------------------------------------------------------------ safetensors
struct TensorRef {
  std::string dtype;            // F32, BF16, F16
  std::vector<long long> shape;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
};

// One file: 8-byte little-endian header length, JSON header
// {name: {dtype, shape, data_offsets: [begin, end]}, "__metadata__": {...}},
// then the data block the offsets index.
void load_safetensors(const Mapped& m, const std::string& path,
                      std::map<std::string, TensorRef>& out) {
  if (m.size < 8) die(path + ": too short for safetensors");
  uint64_t hlen = 0;
  std::memcpy(&hlen, m.data, 8);
  if (hlen > m.size - 8) die(path + ": bad header length");
  std::string text(reinterpret_cast<const char*>(m.data + 8), (size_t)hlen);
  Json h;
  std::string err;
  if (!parse_json(text, h, err) || h.kind != Json::Obj) die(path + ": bad header JSON (" + err + ")");
  const uint8_t* base = m.data + 8 + hlen;
  const size_t avail = m.size - 8 - hlen;
  for (const auto& kv : h.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& t = kv.second;
    const Json* dt = t.get("dtype");
    const Json* sh = t.get("shape");
    const Json* off = t.get("data_offsets");
    if (!dt || !sh || !off || off->arr.size() != 2) die(path + ": bad entry " + kv.first);
    TensorRef r;
    r.dtype = dt->str;
    for (const auto& d : sh->arr) r.shape.push_back((long long)d.num);
    const size_t b0 = (size_t)off->arr[0].num, b1 = (size_t)off->arr[1].num;
    if (b1 < b0 || b1 > avail) die(path + ": offsets out of range for " + kv.first);
    r.data = base + b0;
    r.bytes = b1 - b0;
    out[kv.first] = r;
  }
}

float bf16_to_f32(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// IEEE binary16 -> binary32 by field arithmetic (normals, subnormals, inf, nan).
float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else {   // subnormal: normalise
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400));
      man &= 0x3ff;
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 0x1f) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

std::vector<float> to_f32(const TensorRef& r, const std::string& name) {
  long long n = 1;
  for (long long d : r.shape) n *= d;
  std::vector<float> v((size_t)n);
  if (r.dtype == "F32") {
    if (r.bytes != (size_t)n * 4) die(name + ": size does not match shape");
    std::memcpy(v.data(), r.data, r.bytes);
  } else if (r.dtype == "BF16" || r.dtype == "F16") {
    if (r.bytes != (size_t)n * 2) die(name + ": size does not match shape");
    const bool bf = r.dtype == "BF16";
    for (long long i = 0; i < n; ++i) {
      uint16_t h;
      std::memcpy(&h, r.data + 2 * i, 2);
      v[(size_t)i] = bf ? bf16_to_f32(h) : f16_to_f32(h);
    }
  } else {
    die(name + ": unsupported dtype " + r.dtype);
  }
  return v;
}

// ------------------------------------------------------------------ v4
#pragma pack(push, 1)
struct Hdr {
  int32_t magic, version, step, total_steps;
  int32_t n_layers, vocab_size, dim, hidden_dim, n_heads, seq_len;
  float lr, loss;
  double cum_compile, cum_train, cum_wall;
  int32_t cum_steps, cum_batches, adam_t;
  int32_t kv_heads, head_dim, q_dim;
};
#pragma pack(pop)
static_assert(sizeof(Hdr) == 96, "v4 header is 96 bytes");
constexpr int32_t kMagic = 0x424C5A54;

struct Dims {
  int dim, hidden, heads, kv_heads, hd, n_layers, vocab;
  int q_dim() const { return heads * hd; }
  int kv_dim() const { return kv_heads * hd; }
};

// Row permutation of one projection [n_heads * hd, cols]: to_interleaved moves
// HF row i (i < hd/2) to 2i and HF row i + hd/2 to 2i + 1; the reverse undoes it.
void permute_heads(std::vector<float>& w, int n_heads, int hd, int cols, bool to_interleaved) {
  std::vector<float> out(w.size());
  for (int h = 0; h < n_heads; ++h)
    for (int i = 0; i < hd / 2; ++i) {
      const int hf[2] = {i, i + hd / 2};
      for (int j = 0; j < 2; ++j) {
        const size_t a = ((size_t)h * hd + hf[j]) * cols;      // HF row
        const size_t b = ((size_t)h * hd + 2 * i + j) * cols;  // interleaved row
        if (to_interleaved)
          std::memcpy(&out[b], &w[a], (size_t)cols * 4);
        else
          std::memcpy(&out[a], &w[b], (size_t)cols * 4);
      }
    }
  w.swap(out);
}

void write_all(FILE* f, const void* p, size_t n, const std::string& path) {
  if (n && std::fwrite(p, 1, n, f) != n) die("write failed: " + path);
}
void write_zeros(FILE* f, size_t floats, const std::string& path) {
  static const std::vector<float> z(1 << 16, 0.f);
  while (floats) {
    const size_t k = floats < z.size() ? floats : z.size();
    write_all(f, z.data(), k * 4, path);
    floats -= k;
  }
}

int cfg_int(const Json& cfg, const char* key, int fallback, bool required) {
  const Json* v = cfg.get(key);
  if (!v || v->kind != Json::Num) {
    if (required) die(std::string("config.json has no ") + key);
    return fallback;
  }
  return (int)v->num;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = std::strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// ------------------------------------------------------------------ from-hf
int from_hf(const std::string& dir, std::string out, int steps, int seq, bool qk_block,
            bool permute) {
  std::string text;
  if (!read_file(dir + "/config.json", text)) die("no config.json in " + dir);
  Json cfg;
  std::string err;
  if (!parse_json(text, cfg, err) || cfg.kind != Json::Obj) die("bad config.json: " + err);
  Dims d;
  d.dim = cfg_int(cfg, "hidden_size", 0, true);
  d.hidden = cfg_int(cfg, "intermediate_size", 0, true);
  d.heads = cfg_int(cfg, "num_attention_heads", 0, true);
  d.kv_heads = cfg_int(cfg, "num_key_value_heads", d.heads, false);
  d.hd = cfg_int(cfg, "head_dim", d.dim / d.heads, false);
  d.n_layers = cfg_int(cfg, "num_hidden_layers", 0, true);
  d.vocab = cfg_int(cfg, "vocab_size", 0, true);
  if (permute && d.hd % 2) die("--rope-permute needs an even head_dim");

  std::vector<std::string> files;
  if (DIR* dp = opendir(dir.c_str())) {
    while (dirent* e = readdir(dp)) {
      const std::string n = e->d_name;
      if (ends_with(n, ".safetensors")) files.push_back(dir + "/" + n);
    }
    closedir(dp);
  }
  if (files.empty()) die("no *.safetensors in " + dir);
  std::vector<std::unique_ptr<Mapped>> maps;
  std::map<std::string, TensorRef> T;
  for (const auto& f : files) {
    maps.push_back(map_file(f));
    load_safetensors(*maps.back(), f, T);
  }
  auto get = [&](const std::string& name, size_t expect) {
    auto it = T.find(name);
    if (it == T.end()) die("missing weight: " + name);
    std::vector<float> v = to_f32(it->second, name);
    if (v.size() != expect)
      die(name + ": " + std::to_string(v.size()) + " elements, expected " + std::to_string(expect));
    return v;
  };
  const bool has_qk = T.count("model.layers.0.self_attn.q_norm.weight") > 0;
  if (out.empty()) {
    const Json* mt = cfg.get("model_type");
    out = std::string("ane_") + (mt && mt->kind == Json::Str ? mt->str : "model") + "_dyn_ckpt.bin";
  }
  FILE* f = std::fopen(out.c_str(), "wb");
  if (!f) die("cannot create " + out);
  Hdr h{};
  h.magic = kMagic;
  h.version = 4;
  h.total_steps = steps;
  h.n_layers = d.n_layers;
  h.vocab_size = d.vocab;
  h.dim = d.dim;
  h.hidden_dim = d.hidden;
  h.n_heads = d.heads;
  h.seq_len = seq;
  h.lr = 3e-4f;
  h.kv_heads = d.kv_heads;
  h.head_dim = d.hd;
  h.q_dim = d.q_dim();
  write_all(f, &h, sizeof h, out);
  const size_t D = d.dim, F = d.hidden, Q = d.q_dim(), KV = d.kv_dim();
  const size_t sizes[9] = {Q * D, KV * D, KV * D, D * Q, F * D, D * F, F * D, D, D};
  const char* names[9] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight",
                          "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                          "mlp.gate_proj.weight",    "mlp.down_proj.weight",
                          "mlp.up_proj.weight",      "input_layernorm.weight",
                          "post_attention_layernorm.weight"};
  for (int L = 0; L < d.n_layers; ++L) {
    for (int i = 0; i < 9; ++i) {
      std::vector<float> w = get("model.layers." + std::to_string(L) + "." + names[i], sizes[i]);
      if (permute && i == 0) permute_heads(w, d.heads, d.hd, d.dim, true);
      if (permute && i == 1) permute_heads(w, d.kv_heads, d.hd, d.dim, true);
      write_all(f, w.data(), w.size() * 4, out);
    }
    for (int i = 0; i < 9; ++i) write_zeros(f, 2 * sizes[i], out);   // m, v
  }
  std::vector<float> rf = get("model.norm.weight", D);
  write_all(f, rf.data(), D * 4, out);
  write_zeros(f, 2 * D, out);
  const char* ename = T.count("lm_head.weight") ? "lm_head.weight" : "model.embed_tokens.weight";
  std::vector<float> emb = get(ename, (size_t)d.vocab * D);
  write_all(f, emb.data(), emb.size() * 4, out);
  write_zeros(f, 2 * emb.size(), out);
  if (qk_block && has_qk) {
    write_all(f, "QKN1", 4, out);
    const int32_t ext[2] = {d.n_layers, d.hd};
    write_all(f, ext, sizeof ext, out);
    for (int L = 0; L < d.n_layers; ++L) {
      const std::string p = "model.layers." + std::to_string(L) + ".self_attn.";
      for (const char* nm : {"q_norm.weight", "k_norm.weight"}) {
        std::vector<float> g = get(p + nm, (size_t)d.hd);
        if (permute) permute_heads(g, 1, d.hd, 1, true);
        write_all(f, g.data(), g.size() * 4, out);
      }
      write_zeros(f, 4 * (size_t)d.hd, out);   // m, v of q_norm, then of k_norm
    }
  }
  if (std::fclose(f) != 0) die("write failed: " + out);
  std::printf("model: L=%d D=%d F=%d Hq=%d Hkv=%d hd=%d V=%d%s\n", d.n_layers, d.dim, d.hidden,
              d.heads, d.kv_heads, d.hd, d.vocab, has_qk ? " (QK-norm)" : "");
  if (has_qk && !qk_block)
    std::printf("note: q_norm / k_norm gains not written (--qk-norm-block keeps them)\n");
  std::printf("checkpoint: %s (embedding from %s%s)\n", out.c_str(), ename,
              permute ? ", q/k rows in interleaved-pair RoPE order" : "");
  return 0;
}

// ------------------------------------------------------------------ to-hf
struct OutTensor {
  std::string name;
  std::vector<long long> shape;
  std::vector<float> data;
};

void write_safetensors(const std::string& path, const std::vector<OutTensor>& ts) {
  std::string hdr = "{\"__metadata__\":{\"format\":\"pt\"}";
  size_t off = 0;
  for (const auto& t : ts) {
    const size_t nb = t.data.size() * 4;
    hdr += ",\"" + t.name + "\":{\"dtype\":\"F32\",\"shape\":[";
    for (size_t i = 0; i < t.shape.size(); ++i)
      hdr += (i ? "," : "") + std::to_string(t.shape[i]);
    hdr += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + nb) + "]}";
    off += nb;
  }
  hdr += "}";
  while ((8 + hdr.size()) % 8) hdr += ' ';   // data block 8-byte aligned
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) die("cannot create " + path);
  const uint64_t n = hdr.size();
  write_all(f, &n, 8, path);
  write_all(f, hdr.data(), hdr.size(), path);
  for (const auto& t : ts) write_all(f, t.data.data(), t.data.size() * 4, path);
  if (std::fclose(f) != 0) die("write failed: " + path);
}

// mkdir -p
void make_dirs(const std::string& dir) {
  for (size_t i = 1; i <= dir.size(); ++i) {
    if (i == dir.size() || dir[i] == '/') {
      const std::string p = dir.substr(0, i);
      if (mkdir(p.c_str(), 0755) != 0 && errno != EEXIST) die("cannot create " + p);
    }
  }
}

int to_hf(const std::string& ckpt, const std::string& dir, const std::string& cfg_path,
          bool permute) {
  auto m = map_file(ckpt);
  if (m->size < sizeof(Hdr)) die(ckpt + ": too short");
  Hdr h;
  std::memcpy(&h, m->data, sizeof h);
  if (h.magic != kMagic || h.version != 4) die(ckpt + ": not a v4 checkpoint");
  Dims d{h.dim, h.hidden_dim, h.n_heads, h.kv_heads, h.head_dim, h.n_layers, h.vocab_size};
  if (d.kv_heads <= 0 || d.hd <= 0 || h.q_dim != d.q_dim()) die(ckpt + ": bad GQA fields");
  const size_t D = d.dim, F = d.hidden, Q = d.q_dim(), KV = d.kv_dim();
  const size_t sizes[9] = {Q * D, KV * D, KV * D, D * Q, F * D, D * F, F * D, D, D};
  const long long shapes[9][2] = {{(long long)Q, (long long)D}, {(long long)KV, (long long)D},
                                  {(long long)KV, (long long)D}, {(long long)D, (long long)Q},
                                  {(long long)F, (long long)D},  {(long long)D, (long long)F},
                                  {(long long)F, (long long)D},  {(long long)D, 0},
                                  {(long long)D, 0}};
  const char* names[9] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight",
                          "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                          "mlp.gate_proj.weight",    "mlp.down_proj.weight",
                          "mlp.up_proj.weight",      "input_layernorm.weight",
                          "post_attention_layernorm.weight"};
  size_t pos = sizeof(Hdr);
  auto take = [&](size_t n) {
    if (pos + n * 4 > m->size) die(ckpt + ": truncated");
    std::vector<float> v(n);
    std::memcpy(v.data(), m->data + pos, n * 4);
    pos += n * 4;
    return v;
  };
  std::vector<OutTensor> ts;
  for (int L = 0; L < d.n_layers; ++L) {
    for (int i = 0; i < 9; ++i) {
      OutTensor t;
      t.name = "model.layers." + std::to_string(L) + "." + names[i];
      t.shape = {shapes[i][0]};
      if (shapes[i][1]) t.shape.push_back(shapes[i][1]);
      t.data = take(sizes[i]);
      if (permute && i == 0) permute_heads(t.data, d.heads, d.hd, d.dim, false);
      if (permute && i == 1) permute_heads(t.data, d.kv_heads, d.hd, d.dim, false);
      ts.push_back(std::move(t));
    }
    for (int i = 0; i < 9; ++i) pos += 2 * sizes[i] * 4;   // Adam moments
  }
  OutTensor rf{"model.norm.weight", {(long long)D}, take(D)};
  pos += 2 * D * 4;
  OutTensor emb{"model.embed_tokens.weight", {(long long)d.vocab, (long long)D},
                take((size_t)d.vocab * D)};
  pos += 2 * (size_t)d.vocab * D * 4;
  bool has_qk = false;
  if (pos + 12 <= m->size && !std::memcmp(m->data + pos, "QKN1", 4)) {
    int32_t ext[2];
    std::memcpy(ext, m->data + pos + 4, 8);
    if (ext[0] != d.n_layers || ext[1] != d.hd) die(ckpt + ": QKN1 block does not match header");
    pos += 12;
    has_qk = true;
    for (int L = 0; L < d.n_layers; ++L) {
      for (const char* nm : {"q_norm.weight", "k_norm.weight"}) {
        OutTensor t{"model.layers." + std::to_string(L) + ".self_attn." + nm, {(long long)d.hd},
                    take((size_t)d.hd)};
        if (permute) permute_heads(t.data, 1, d.hd, 1, false);
        ts.push_back(std::move(t));
      }
      pos += 4 * (size_t)d.hd * 4;
    }
  }
  ts.push_back(std::move(rf));
  ts.push_back(std::move(emb));
  make_dirs(dir);
  write_safetensors(dir + "/model.safetensors", ts);
  std::string cfg;
  if (!cfg_path.empty()) {
    if (!read_file(cfg_path, cfg)) die("cannot read " + cfg_path);
  } else {
    char buf[1024];
    std::snprintf(buf, sizeof buf,
                  "{\n  \"architectures\": [\"%s\"],\n  \"model_type\": \"%s\",\n"
                  "  \"hidden_size\": %d,\n  \"intermediate_size\": %d,\n"
                  "  \"num_attention_heads\": %d,\n  \"num_key_value_heads\": %d,\n"
                  "  \"head_dim\": %d,\n  \"num_hidden_layers\": %d,\n  \"vocab_size\": %d,\n"
                  "  \"max_position_embeddings\": 32768,\n  \"rms_norm_eps\": 1e-05,\n"
                  "  \"tie_word_embeddings\": true,\n  \"torch_dtype\": \"float32\"\n}\n",
                  "Qwen3ForCausalLM", "qwen3", d.dim, d.hidden, d.heads, d.kv_heads, d.hd,
                  d.n_layers, d.vocab);
    cfg = buf;
  }
  FILE* f = std::fopen((dir + "/config.json").c_str(), "wb");
  if (!f) die("cannot create " + dir + "/config.json");
  write_all(f, cfg.data(), cfg.size(), dir);
  std::fclose(f);
  std::printf("exported: %s/model.safetensors (%zu tensors%s%s)\n", dir.c_str(), ts.size(),
              has_qk ? ", QK-norm gains" : "", permute ? ", HF rotate_half row order" : "");
  return 0;
}

void usage(FILE* f) {
  std::fprintf(f,
               "usage: ne_convert from-hf <model_dir> [-o ckpt.bin] [--steps N] [--seq S]\n"
               "                  [--qk-norm-block] [--rope-permute] [--hf-exact]\n"
               "       ne_convert to-hf <ckpt.bin> -o <dir> [--config config.json]\n"
               "                  [--rope-permute] [--hf-exact]\n");
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2 || !std::strcmp(argv[1], "--help") || !std::strcmp(argv[1], "-h")) {
    usage(argc < 2 ? stderr : stdout);
    return argc < 2 ? 2 : 0;
  }
  const std::string mode = argv[1];
  std::string src, out, cfg;
  int steps = 10000, seq = 256;
  bool qk_block = false, permute = false;
  for (int i = 2; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) {
        usage(stderr);
        std::exit(2);
      }
      return argv[++i];
    };
    if (a == "-o" || a == "--output") out = next();
    else if (a == "--steps") steps = std::atoi(next().c_str());
    else if (a == "--seq") seq = std::atoi(next().c_str());
    else if (a == "--config") cfg = next();
    else if (a == "--qk-norm-block") qk_block = true;
    else if (a == "--rope-permute") permute = true;
    else if (a == "--hf-exact") qk_block = permute = true;
    else if (!a.empty() && a[0] == '-') {
      usage(stderr);
      return 2;
    } else if (src.empty()) src = a;
    else {
      usage(stderr);
      return 2;
    }
  }
  if (src.empty()) {
    usage(stderr);
    return 2;
  }
  if (mode == "from-hf") return from_hf(src, out, steps, seq, qk_block, permute);
  if (mode == "to-hf") {
    if (out.empty()) {
      usage(stderr);
      return 2;
    }
    return to_hf(src, out, cfg, permute);
  }
  usage(stderr);
  return 2;
}
