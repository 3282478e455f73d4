// Checkpoint loading and saving: MLX-format model directories (config.json
// plus model.safetensors, or shards listed by model.safetensors.index.json).
//
// Follows the reference's load path for Qwen3 / Llama:
//   load_llm_from_directory (src/llm/llm_factory.cpp:272-290) reads
//   config.json; load_safetensors_from_directory (src/common/safetensors.cpp:
//   23-75) picks the shard index first, then a single model.safetensors
//   larger than 1 KiB, then every *.safetensors in the directory, later
//   files replacing earlier names; parse_base_configuration
//   (src/common/base_config.cpp:9-73) reads the default quantization and the
//   per-layer overrides; register_quantized_weights
//   (src/common/quantize_utils.cpp:14-104) treats every prefix with
//   .weight + .scales as an affine-quantized linear layer with the override's
//   bits / group size (quantization_for, include/mlx-lm/common/base_config.h:
//   47-54); the model's sanitize drops lm_head.weight when the embeddings are
//   tied (qwen3.cpp:223-226) and the rotary inv_freq buffers (llama.cpp:
//   473-485); load_weights binds the names of the model's weight_map.
//
// The tensors go straight from the mapped file into the model's device
// arena (a tensor-parallel rank copies only its block).  Stricter than the
// reference where a silent fallback would run garbage: a weight the model
// needs and the checkpoint lacks, a shape that disagrees with config.json,
// or an unquantized linear layer (the kernels take MLX affine 4/8-bit group-64
// weights) is an error.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <set>

namespace lmx {
namespace ld {

// ---------------------------------------------------------------------------
// JSON (RFC 8259): enough for config.json, the shard index and safetensors
// headers.  Numbers are kept as doubles (exact for every integer below 2^53).
// ---------------------------------------------------------------------------
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double n = 0;
  std::string s;
  std::vector<Json> a;
  std::vector<std::pair<std::string, Json>> o;
  const Json* get(const std::string& k) const {
    if (kind != Obj) return nullptr;
    for (const auto& kv : o)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  bool is_int() const { return kind == Num && std::floor(n) == n && std::fabs(n) < 9.007199254740992e15; }
};

struct JsonParser {
  const char* p;
  const char* end;
  std::string err;
  int depth = 0;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail(const char* what) {
    if (err.empty()) err = what;
    return false;
  }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if ((size_t)(end - p) < n || std::memcmp(p, w, n)) return fail("bad literal");
    p += n;
    return true;
  }
  static void put_utf8(std::string& s, uint32_t c) {
    if (c < 0x80) {
      s += (char)c;
    } else if (c < 0x800) {
      s += (char)(0xC0 | (c >> 6));
      s += (char)(0x80 | (c & 63));
    } else if (c < 0x10000) {
      s += (char)(0xE0 | (c >> 12));
      s += (char)(0x80 | ((c >> 6) & 63));
      s += (char)(0x80 | (c & 63));
    } else {
      s += (char)(0xF0 | (c >> 18));
      s += (char)(0x80 | ((c >> 12) & 63));
      s += (char)(0x80 | ((c >> 6) & 63));
      s += (char)(0x80 | (c & 63));
    }
  }
  bool hex4(uint32_t& v) {
    if (end - p < 4) return fail("short \\u escape");
    v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    return true;
  }
  bool str(std::string& out) {
    if (p >= end || *p != '"') return fail("expected string");
    ++p;
    out.clear();
    while (p < end && *p != '"') {
      const char c = *p++;
      if ((unsigned char)c < 0x20) return fail("control character in string");
      if (c != '\\') {
        out += c;
        continue;
      }
      if (p >= end) return fail("bad escape");
      const char e = *p++;
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t c1;
          if (!hex4(c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00) {  // surrogate pair
            uint32_t c2;
            if (end - p < 2 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
            p += 2;
            if (!hex4(c2) || c2 < 0xDC00 || c2 >= 0xE000) return fail("bad surrogate pair");
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          }
          put_utf8(out, c1);
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p >= end) return fail("unterminated string");
    ++p;
    return true;
  }
  bool value(Json& v) {
    if (++depth > 64) return fail("nesting too deep");
    ws();
    if (p >= end) return fail("unexpected end");
    bool ok = true;
    const char c = *p;
    if (c == '{') {
      ++p;
      v.kind = Json::Obj;
      ws();
      if (p < end && *p == '}') {
        ++p;
      } else {
        for (;;) {
          ws();
          std::string k;
          if (!str(k)) return false;
          ws();
          if (p >= end || *p != ':') return fail("expected ':'");
          ++p;
          v.o.emplace_back(std::move(k), Json());
          if (!value(v.o.back().second)) return false;
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == '}') {
            ++p;
            break;
          }
          return fail("expected ',' or '}'");
        }
      }
    } else if (c == '[') {
      ++p;
      v.kind = Json::Arr;
      ws();
      if (p < end && *p == ']') {
        ++p;
      } else {
        for (;;) {
          v.a.emplace_back();
          if (!value(v.a.back())) return false;
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == ']') {
            ++p;
            break;
          }
          return fail("expected ',' or ']'");
        }
      }
    } else if (c == '"') {
      v.kind = Json::Str;
      ok = str(v.s);
    } else if (c == 't') {
      v.kind = Json::Bool;
      v.b = true;
      ok = lit("true");
    } else if (c == 'f') {
      v.kind = Json::Bool;
      ok = lit("false");
    } else if (c == 'n') {
      ok = lit("null");
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      // the grammar's number: -?(0|[1-9][0-9]*)(.[0-9]+)?([eE][+-]?[0-9]+)?
      const char* q = p;
      if (q < end && *q == '-') ++q;
      if (q < end && *q == '0') {
        ++q;
      } else {
        if (q >= end || *q < '1' || *q > '9') return fail("bad number");
        while (q < end && *q >= '0' && *q <= '9') ++q;
      }
      if (q < end && *q == '.') {
        ++q;
        if (q >= end || *q < '0' || *q > '9') return fail("bad number");
        while (q < end && *q >= '0' && *q <= '9') ++q;
      }
      if (q < end && (*q == 'e' || *q == 'E')) {
        ++q;
        if (q < end && (*q == '+' || *q == '-')) ++q;
        if (q >= end || *q < '0' || *q > '9') return fail("bad number");
        while (q < end && *q >= '0' && *q <= '9') ++q;
      }
      v.kind = Json::Num;
      v.n = std::strtod(std::string(p, q).c_str(), nullptr);
      p = q;
    } else {
      return fail("unexpected character");
    }
    --depth;
    return ok;
  }
};

static int parse_json(const char* text, size_t n, Json& out, const char* what) {
  JsonParser jp{text, text + n, std::string()};
  bool ok = jp.value(out);
  if (ok) {
    jp.ws();
    if (jp.p != jp.end) ok = jp.fail("trailing characters");
  }
  if (!ok)
    return set_error(LMX_ERR_IO, "%s: malformed JSON at byte %zu (%s)", what, (size_t)(jp.p - text), jp.err.c_str());
  return LMX_OK;
}

static int read_text(const std::string& path, std::string& out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return set_error(LMX_ERR_IO, "cannot open %s", path.c_str());
  char buf[65536];
  size_t n;
  out.clear();
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
  const bool bad = std::ferror(f);
  std::fclose(f);
  return bad ? set_error(LMX_ERR_IO, "read error on %s", path.c_str()) : LMX_OK;
}

static bool is_file(const std::string& p, int64_t* size = nullptr) {
  struct stat sb;
  if (stat(p.c_str(), &sb) || !S_ISREG(sb.st_mode)) return false;
  if (size) *size = (int64_t)sb.st_size;
  return true;
}

// ---------------------------------------------------------------------------
// safetensors: u64 little-endian header length N, N bytes of JSON
// {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__":
// {...}}, then the data; offsets count from the first byte after the header.
// ---------------------------------------------------------------------------
static int dtype_size(const std::string& d) {
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  return 0;
}

struct MappedFile {
  std::string path;
  const uint8_t* base = nullptr;
  size_t size = 0;
  size_t data0 = 0;  // first data byte
  MappedFile() = default;
  MappedFile(const MappedFile&) = delete;
  MappedFile& operator=(const MappedFile&) = delete;
  ~MappedFile() {
    if (base) munmap((void*)base, size);
  }
};

struct TensorRef {
  int file = -1;
  std::string dtype;
  std::vector<int64_t> shape;
  size_t off = 0, bytes = 0;  // absolute offset in the file
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
};

struct TensorSet {
  std::vector<std::unique_ptr<MappedFile>> files;
  std::map<std::string, TensorRef> t;
  const uint8_t* data(const TensorRef& r) const { return files[r.file]->base + r.off; }
};

// Map one file and add its tensors (a name already present is replaced).
static int st_open(const std::string& path, TensorSet& ts) {
  auto mf = std::make_unique<MappedFile>();
  mf->path = path;
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return set_error(LMX_ERR_IO, "cannot open %s", path.c_str());
  struct stat sb;
  if (fstat(fd, &sb) || sb.st_size < 8) {
    close(fd);
    return set_error(LMX_ERR_IO, "%s: not a safetensors file (size)", path.c_str());
  }
  mf->size = (size_t)sb.st_size;
  void* p = mmap(nullptr, mf->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return set_error(LMX_ERR_IO, "cannot map %s", path.c_str());
  mf->base = (const uint8_t*)p;
  uint64_t hn = 0;
  for (int i = 7; i >= 0; --i) hn = (hn << 8) | mf->base[i];
  if (hn > mf->size - 8 || hn > ((uint64_t)100 << 20))
    return set_error(LMX_ERR_IO, "%s: header length %llu out of range", path.c_str(), (unsigned long long)hn);
  mf->data0 = 8 + (size_t)hn;
  Json h;
  int rc = parse_json((const char*)mf->base + 8, (size_t)hn, h, path.c_str());
  if (rc) return rc;
  if (h.kind != Json::Obj) return set_error(LMX_ERR_IO, "%s: header is not an object", path.c_str());
  const int fi = (int)ts.files.size();
  const size_t avail = mf->size - mf->data0;
  for (const auto& kv : h.o) {
    if (kv.first == "__metadata__") continue;
    const Json& e = kv.second;
    const Json *dt = e.get("dtype"), *sh = e.get("shape"), *of = e.get("data_offsets");
    if (!dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !of || of->kind != Json::Arr ||
        of->a.size() != 2 || !of->a[0].is_int() || !of->a[1].is_int())
      return set_error(LMX_ERR_IO, "%s: bad entry for %s", path.c_str(), kv.first.c_str());
    TensorRef r;
    r.file = fi;
    r.dtype = dt->s;
    for (const Json& d : sh->a) {
      if (!d.is_int() || d.n < 0) return set_error(LMX_ERR_IO, "%s: bad shape of %s", path.c_str(), kv.first.c_str());
      r.shape.push_back((int64_t)d.n);
    }
    const int es = dtype_size(r.dtype);
    const double b0 = of->a[0].n, b1 = of->a[1].n;
    if (!es || b0 < 0 || b1 < b0 || b1 > (double)avail || (int64_t)(b1 - b0) != r.numel() * es)
      return set_error(LMX_ERR_IO, "%s: %s: dtype %s, offsets [%.0f, %.0f) do not fit the shape or the file",
                       path.c_str(), kv.first.c_str(), r.dtype.c_str(), b0, b1);
    r.off = mf->data0 + (size_t)b0;
    r.bytes = (size_t)(b1 - b0);
    ts.t[kv.first] = r;
  }
  ts.files.push_back(std::move(mf));
  return LMX_OK;
}

// load_safetensors_from_directory's file choice (safetensors.cpp:23-75).
static int st_open_dir(const std::string& dir, TensorSet& ts) {
  const std::string idx = dir + "/model.safetensors.index.json";
  if (is_file(idx)) {
    std::string text;
    int rc = read_text(idx, text);
    Json j;
    if (!rc) rc = parse_json(text.data(), text.size(), j, idx.c_str());
    if (rc) return rc;
    const Json* wm = j.get("weight_map");
    if (wm && wm->kind == Json::Obj) {
      std::set<std::string> shards;
      for (const auto& kv : wm->o) {
        if (kv.second.kind != Json::Str) return set_error(LMX_ERR_IO, "%s: bad weight_map entry", idx.c_str());
        shards.insert(kv.second.s);
      }
      for (const std::string& s : shards) {
        if (!is_file(dir + "/" + s)) return set_error(LMX_ERR_IO, "missing shard file: %s/%s", dir.c_str(), s.c_str());
        rc = st_open(dir + "/" + s, ts);
        if (rc) return rc;
      }
      return LMX_OK;
    }
  }
  int64_t sz = 0;
  if (is_file(dir + "/model.safetensors", &sz) && sz > 1024) return st_open(dir + "/model.safetensors", ts);
  std::vector<std::string> names;
  if (DIR* d = opendir(dir.c_str())) {
    while (dirent* e = readdir(d)) {
      const std::string n = e->d_name;
      if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) names.push_back(n);
    }
    closedir(d);
  } else {
    return set_error(LMX_ERR_IO, "cannot open directory %s", dir.c_str());
  }
  std::sort(names.begin(), names.end());
  for (const std::string& n : names) {
    int rc = st_open(dir + "/" + n, ts);
    if (rc) return rc;
  }
  if (ts.t.empty()) return set_error(LMX_ERR_IO, "no .safetensors files found in %s", dir.c_str());
  return LMX_OK;
}

// ---------------------------------------------------------------------------
// config.json
// ---------------------------------------------------------------------------
struct QuantCfg {
  int bits = 4, group = 64;
  bool present = false;                             // "quantization" in config.json
  std::map<std::string, std::pair<int, int>> over;  // prefix -> (bits, group)
  // quantization_for: the override for this exact prefix, else the default
  // (a `false` entry, "do not quantize", also falls back to the default)
  std::pair<int, int> for_prefix(const std::string& p) const {
    auto it = over.find(p);
    return it != over.end() ? it->second : std::make_pair(bits, group);
  }
};

struct LoadedConfig {
  lmx_model_config c{};
  QuantCfg q;
  std::string model_type;
  std::vector<int> eos;
};

static bool num(const Json& j, const char* k, double& out) {
  const Json* v = j.get(k);
  if (!v || v->kind != Json::Num) return false;
  out = v->n;
  return true;
}

static int req_int(const Json& j, const char* k, int& out, const char* path) {
  const Json* v = j.get(k);
  if (!v || !v->is_int()) return set_error(LMX_ERR_IO, "%s: missing integer \"%s\"", path, k);
  out = (int)v->n;
  return LMX_OK;
}

// Qwen3Configuration / LlamaConfiguration from_json (qwen3.cpp:13-35,
// llama.cpp:22-55) and parse_base_configuration (base_config.cpp:9-73).
static int parse_config(const Json& j, const char* path, LoadedConfig& out) {
  if (j.kind != Json::Obj) return set_error(LMX_ERR_IO, "%s: not a JSON object", path);
  const Json* mt = j.get("model_type");
  out.model_type = mt && mt->kind == Json::Str ? mt->s : "";
  const bool qwen3 = out.model_type == "qwen3";
  const bool llama = out.model_type == "llama" || out.model_type == "mistral";
  if (!qwen3 && !llama)
    return set_error(LMX_ERR_UNSUPPORTED, "%s: model_type \"%s\" (supported: qwen3, llama, mistral)", path,
                     out.model_type.c_str());
  lmx_model_config& c = out.c;
  std::memset(&c, 0, sizeof c);
  int rc = req_int(j, "hidden_size", c.hidden, path);
  if (!rc) rc = req_int(j, "num_hidden_layers", c.layers, path);
  if (!rc) rc = req_int(j, "intermediate_size", c.inter, path);
  if (!rc) rc = req_int(j, "num_attention_heads", c.heads, path);
  if (!rc) rc = req_int(j, "vocab_size", c.vocab, path);
  if (rc) return rc;
  double d;
  if (!num(j, "rms_norm_eps", d)) return set_error(LMX_ERR_IO, "%s: missing \"rms_norm_eps\"", path);
  c.eps = (float)d;
  if (qwen3) {
    rc = req_int(j, "num_key_value_heads", c.kv_heads, path);
    if (!rc) rc = req_int(j, "head_dim", c.head_dim, path);
    if (rc) return rc;
    c.rope_theta = num(j, "rope_theta", d) ? (float)d : 1000000.0f;
  } else {
    const Json* kvh = j.get("num_key_value_heads");
    c.kv_heads = kvh && kvh->is_int() ? (int)kvh->n : c.heads;
    const Json* hd = j.get("head_dim");
    c.head_dim = hd && hd->is_int() ? (int)hd->n : (c.heads ? c.hidden / c.heads : 0);
    c.rope_theta = num(j, "rope_theta", d) ? (float)d : 10000.0f;
    const Json* rt = j.get("rope_traditional");
    if (rt && rt->kind == Json::Bool && rt->b)
      return set_error(LMX_ERR_UNSUPPORTED, "%s: rope_traditional (the kernels rotate the half-split pairs)", path);
    for (const char* k : {"attention_bias", "mlp_bias"}) {
      const Json* v = j.get(k);
      if (v && v->kind == Json::Bool && v->b) return set_error(LMX_ERR_UNSUPPORTED, "%s: %s", path, k);
    }
  }
  c.qk_norm = qwen3 ? 1 : 0;
  const Json* tie = j.get("tie_word_embeddings");
  c.tied = tie && tie->kind == Json::Bool && tie->b ? 1 : 0;
  // Llama-3 frequency scaling (LlamaDynamicNTKScalingRoPE::compute_freqs,
  // llama.cpp:122-183): only for rope_type "llama3"; defaults factor 1,
  // low 1, high 4, original context 8192
  c.rope_factor = 0.0f;
  const Json* rs = j.get("rope_scaling");
  if (llama && rs && rs->kind == Json::Obj) {
    const Json* ty = rs->get("rope_type");
    if (!ty) ty = rs->get("type");
    if (ty && ty->kind == Json::Str && ty->s == "llama3") {
      c.rope_factor = num(*rs, "factor", d) ? (float)d : 1.0f;
      c.rope_low_freq = num(*rs, "low_freq_factor", d) ? (float)d : 1.0f;
      c.rope_high_freq = num(*rs, "high_freq_factor", d) ? (float)d : 4.0f;
      c.rope_orig_max_pos = num(*rs, "original_max_position_embeddings", d) ? (float)d : 8192.0f;
    } else if (ty && ty->kind == Json::Str && ty->s != "default") {
      return set_error(LMX_ERR_UNSUPPORTED, "%s: rope_scaling type \"%s\"", path, ty->s.c_str());
    }
  }
  // EOS: top level, else text_config (base_config.cpp:16-26)
  const Json* eos = j.get("eos_token_id");
  if (!eos) {
    const Json* tc = j.get("text_config");
    if (tc) eos = tc->get("eos_token_id");
  }
  if (eos && eos->is_int()) out.eos.push_back((int)eos->n);
  if (eos && eos->kind == Json::Arr)
    for (const Json& e : eos->a)
      if (e.is_int()) out.eos.push_back((int)e.n);
  // quantization: default + per-layer overrides; "language_model." stripped
  const Json* qj = j.get("quantization");
  if (!qj) qj = j.get("quantization_config");
  if (qj && qj->kind == Json::Obj) {
    QuantCfg& q = out.q;
    q.present = true;
    q.group = num(*qj, "group_size", d) ? (int)d : 64;
    q.bits = num(*qj, "bits", d) ? (int)d : 4;
    const Json* mode = qj->get("mode");
    if (mode && mode->kind == Json::Str && mode->s != "affine")
      return set_error(LMX_ERR_UNSUPPORTED, "%s: quantization mode \"%s\" (affine only)", path, mode->s.c_str());
    static const char* const skip[] = {"group_size", "bits", "mode", "quant_method", "linear_class",
                                       "quantization_mode"};
    for (const auto& kv : qj->o) {
      if (std::find_if(std::begin(skip), std::end(skip), [&](const char* s) { return kv.first == s; }) !=
          std::end(skip))
        continue;
      std::string key = kv.first;
      if (key.compare(0, 15, "language_model.") == 0) key = key.substr(15);
      if (kv.second.kind == Json::Obj) {
        const int b = num(kv.second, "bits", d) ? (int)d : q.bits;
        const int g = num(kv.second, "group_size", d) ? (int)d : q.group;
        q.over[key] = {b, g};
      }
    }
  }
  c.bits = out.q.bits;
  c.group_size = out.q.group;
  return LMX_OK;
}

static int load_config(const std::string& path_in, LoadedConfig& out) {
  std::string path = path_in;
  if (!is_file(path)) path += "/config.json";
  if (!is_file(path)) return set_error(LMX_ERR_IO, "config.json not found in %s", path_in.c_str());
  std::string text;
  int rc = read_text(path, text);
  Json j;
  if (!rc) rc = parse_json(text.data(), text.size(), j, path.c_str());
  if (!rc) rc = parse_config(j, path.c_str(), out);
  return rc;
}

// ---------------------------------------------------------------------------
// the checkpoint as a WeightSource
// ---------------------------------------------------------------------------
static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);  // NaN stays NaN
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u;
  uint32_t u;
  if (e == 31) {
    u = s | 0x7F800000u | (m << 13);
  } else if (e) {
    u = s | ((e + 112u) << 23) | (m << 13);
  } else if (m) {  // subnormal: value m * 2^-24
    const float v = std::ldexp((float)m, -24);
    std::memcpy(&u, &v, 4);
    u |= s;
  } else {
    u = s;
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// Element i of a floating tensor (BF16 / F16 / F32) as bf16 bits: BF16 as
// is, the others rounded to nearest even.
static inline uint16_t elem_bf16(const uint8_t* p, const std::string& dt, int64_t i) {
  if (dt == "BF16") {
    uint16_t v;
    std::memcpy(&v, p + 2 * i, 2);
    return v;
  }
  if (dt == "F16") {
    uint16_t v;
    std::memcpy(&v, p + 2 * i, 2);
    return f32_to_bf16_rne(f16_to_f32(v));
  }
  float f;
  std::memcpy(&f, p + 4 * i, 4);
  return f32_to_bf16_rne(f);
}

static bool float_dtype(const std::string& d) { return d == "BF16" || d == "F16" || d == "F32"; }

struct FileSource : WeightSource {
  const TensorSet& ts;
  const QuantCfg& q;
  std::set<std::string> used;
  FileSource(const TensorSet& t, const QuantCfg& qc) : ts(t), q(qc) {}

  const TensorRef* find(const std::string& n) const {
    auto it = ts.t.find(n);
    return it == ts.t.end() ? nullptr : &it->second;
  }

  // Rows [row0, row0+N) x columns [c0, c0+ncols) of a row-major 2-D tensor
  // (ld columns of esz bytes) into device memory, as bf16 when conv.
  int copy_block(const TensorRef& r, int esz, int64_t ld, int64_t row0, int64_t N, int64_t c0, int64_t ncols,
                 void* dst, bool conv, cudaStream_t st) {
    const uint8_t* base = ts.data(r);
    if (!conv) {
      return cuda_check(cudaMemcpy2DAsync(dst, (size_t)(ncols * esz), base + (row0 * ld + c0) * esz,
                                          (size_t)(ld * esz), (size_t)(ncols * esz), (size_t)N,
                                          cudaMemcpyHostToDevice, st),
                        "load: copy tensor");
    }
    std::vector<uint16_t> tmp((size_t)(N * ncols));
    for (int64_t i = 0; i < N; ++i)
      for (int64_t j = 0; j < ncols; ++j) tmp[(size_t)(i * ncols + j)] = elem_bf16(base, r.dtype, (row0 + i) * ld + c0 + j);
    int rc = cuda_check(cudaMemcpyAsync(dst, tmp.data(), tmp.size() * 2, cudaMemcpyHostToDevice, st), "load: copy");
    if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "load: copy");  // tmp goes out of scope
    return rc;
  }

  int qweight(Arena& ar, QWeight& w, uint32_t, const std::string& name, int N, int K, int64_t row0, int64_t col0,
              int64_t Nfull, int64_t Kfull, cudaStream_t st) override {
    const TensorRef* tw = find(name + ".weight");
    if (!tw) return set_error(LMX_ERR_IO, "checkpoint lacks %s.weight", name.c_str());
    const TensorRef* ts_ = find(name + ".scales");
    const TensorRef* tb = find(name + ".biases");
    if (!ts_)
      return set_error(LMX_ERR_UNSUPPORTED,
                       "%s is not quantized (the kernels take MLX affine 4/8-bit group-64 weights)", name.c_str());
    if (!tb) return set_error(LMX_ERR_UNSUPPORTED, "%s: quantized without biases (affine mode only)", name.c_str());
    const std::pair<int, int> bg = q.for_prefix(name);
    const int bits = bg.first, group = bg.second;
    if ((bits != 4 && bits != 8) || group != 64)
      return set_error(LMX_ERR_UNSUPPORTED, "%s: %d-bit group-%d quantization (4 or 8 bits, group 64)", name.c_str(),
                       bits, group);
    const int64_t wpr = Kfull * bits / 32, gpr = Kfull / 64;
    if (tw->dtype != "U32" || tw->shape.size() != 2 || tw->shape[0] != Nfull || tw->shape[1] != wpr)
      return set_error(LMX_ERR_IO, "%s.weight: %s [%lld, %lld], expected U32 [%lld, %lld] (%d-bit, %lld columns)",
                       name.c_str(), tw->dtype.c_str(), (long long)(tw->shape.size() > 0 ? tw->shape[0] : -1),
                       (long long)(tw->shape.size() > 1 ? tw->shape[1] : -1), (long long)Nfull, (long long)wpr, bits,
                       (long long)Kfull);
    for (const TensorRef* t : {ts_, tb})
      if (!float_dtype(t->dtype) || t->shape.size() != 2 || t->shape[0] != Nfull || t->shape[1] != gpr)
        return set_error(LMX_ERR_IO, "%s: scales / biases must be floating [%lld, %lld]", name.c_str(),
                         (long long)Nfull, (long long)gpr);
    w.N = N;
    w.K = K;
    w.bits = bits;
    int rc = ar.alloc(&w.w, (size_t)N * K * bits / 32, false);
    if (!rc) rc = ar.alloc(&w.s, (size_t)N * (K / 64), false);
    if (!rc) rc = ar.alloc(&w.b, (size_t)N * (K / 64), false);
    if (!rc) rc = copy_block(*tw, 4, wpr, row0, N, col0 * bits / 32, (int64_t)K * bits / 32, w.w, false, st);
    if (!rc) rc = copy_block(*ts_, 2, gpr, row0, N, col0 / 64, K / 64, w.s, ts_->dtype != "BF16", st);
    if (!rc) rc = copy_block(*tb, 2, gpr, row0, N, col0 / 64, K / 64, w.b, tb->dtype != "BF16", st);
    used.insert(name + ".weight");
    used.insert(name + ".scales");
    used.insert(name + ".biases");
    return rc;
  }

  int norm(Arena& ar, bf16_t** p, const std::string& name, int n, cudaStream_t st) override {
    const TensorRef* t = find(name);
    if (!t) return set_error(LMX_ERR_IO, "checkpoint lacks %s", name.c_str());
    if (!float_dtype(t->dtype) || t->shape.size() != 1 || t->shape[0] != n)
      return set_error(LMX_ERR_IO, "%s: expected a floating [%d] vector", name.c_str(), n);
    int rc = ar.alloc(p, (size_t)n, false);
    if (!rc) rc = copy_block(*t, t->dtype == "F32" ? 4 : 2, n, 0, 1, 0, n, *p, t->dtype != "BF16", st);
    used.insert(name);
    return rc;
  }
};

static int load_model(const std::string& dir, TpComm* comm, Model** out) {
  LoadedConfig lc;
  int rc = load_config(dir, lc);
  if (rc) return rc;
  if (!lc.q.present)
    return set_error(LMX_ERR_UNSUPPORTED, "%s: no \"quantization\" in config.json (the kernels take quantized weights)",
                     dir.c_str());
  TensorSet ts;
  rc = st_open_dir(dir, ts);
  if (rc) return rc;
  FileSource src(ts, lc.q);
  rc = model_build(lc.c, src, comm, out);
  if (rc) return rc;
  return cuda_check(cudaDeviceSynchronize(), "load: finish copies");
}

// ---------------------------------------------------------------------------
// saving (tensor-parallel size 1): config.json + one model.safetensors with
// the names, dtypes and shapes an MLX checkpoint of the same model has
// ---------------------------------------------------------------------------
static void json_num(std::string& s, const char* k, double v, bool is_int) {
  char b[64];
  if (is_int) std::snprintf(b, sizeof b, "\"%s\": %lld", k, (long long)v);
  else std::snprintf(b, sizeof b, "\"%s\": %.9g", k, v);
  s += b;
}

struct SaveItem {
  std::string name, dtype;
  std::vector<int64_t> shape;
  const void* dev = nullptr;
  size_t bytes = 0;
};

static int save_model(const Model& m, const std::string& dir) {
  if (m.tp > 1) return set_error(LMX_ERR_UNSUPPORTED, "save: a tensor-parallel shard (save the tp 1 model)");
  if (m.n_layers != m.c.layers) return set_error(LMX_ERR_UNSUPPORTED, "save: a layer view (save its model)");
  const lmx_model_config& c = m.c;
  std::vector<SaveItem> items;
  auto add_q = [&](const std::string& name, const QWeight& q) {
    const int64_t wpr = (int64_t)q.K * q.bits / 32, gpr = q.K / 64;
    items.push_back({name + ".weight", "U32", {q.N, wpr}, q.w, (size_t)(q.N * wpr * 4)});
    items.push_back({name + ".scales", "BF16", {q.N, gpr}, q.s, (size_t)(q.N * gpr * 2)});
    items.push_back({name + ".biases", "BF16", {q.N, gpr}, q.b, (size_t)(q.N * gpr * 2)});
  };
  auto add_v = [&](const std::string& name, const bf16_t* p, int n) {
    items.push_back({name, "BF16", {n}, p, (size_t)n * 2});
  };
  static const char* const kProj[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                       "mlp.gate_proj",    "mlp.up_proj",      "mlp.down_proj"};
  std::string over;  // per-layer quantization overrides for weights not at c.bits
  auto note = [&](const std::string& name, const QWeight& q) {
    if (q.bits == c.bits) return;
    char b[160];
    std::snprintf(b, sizeof b, ",\n    \"%s\": {\"group_size\": 64, \"bits\": %d}", name.c_str(), q.bits);
    over += b;
  };
  add_q("model.embed_tokens", m.embed);
  note("model.embed_tokens", m.embed);
  for (int l = 0; l < c.layers; ++l) {
    const std::string pre = "model.layers." + std::to_string(l) + ".";
    for (int k = 0; k < 7; ++k) {
      add_q(pre + kProj[k], m.L[l].w[k]);
      note(pre + kProj[k], m.L[l].w[k]);
    }
    add_v(pre + "input_layernorm.weight", m.L[l].in_norm, c.hidden);
    add_v(pre + "post_attention_layernorm.weight", m.L[l].post_norm, c.hidden);
    if (c.qk_norm) {
      add_v(pre + "self_attn.q_norm.weight", m.L[l].q_norm, c.head_dim);
      add_v(pre + "self_attn.k_norm.weight", m.L[l].k_norm, c.head_dim);
    }
  }
  add_v("model.norm.weight", m.final_norm, c.hidden);
  if (!c.tied) {
    add_q("lm_head", m.lm_head);
    note("lm_head", m.lm_head);
  }
  // header (names sorted, data in the same order, 8-byte aligned header)
  std::sort(items.begin(), items.end(), [](const SaveItem& a, const SaveItem& b) { return a.name < b.name; });
  std::string h = "{\"__metadata__\":{\"format\":\"mlx\"}";
  size_t off = 0;
  for (const SaveItem& it : items) {
    h += ",\"" + it.name + "\":{\"dtype\":\"" + it.dtype + "\",\"shape\":[";
    for (size_t i = 0; i < it.shape.size(); ++i) h += (i ? "," : "") + std::to_string(it.shape[i]);
    h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + it.bytes) + "]}";
    off += it.bytes;
  }
  h += "}";
  while (h.size() % 8) h += ' ';
  mkdir(dir.c_str(), 0755);
  const std::string st_path = dir + "/model.safetensors";
  FILE* f = std::fopen(st_path.c_str(), "wb");
  if (!f) return set_error(LMX_ERR_IO, "cannot create %s", st_path.c_str());
  uint8_t len[8];
  for (int i = 0; i < 8; ++i) len[i] = (uint8_t)((uint64_t)h.size() >> (8 * i));
  bool ok = std::fwrite(len, 1, 8, f) == 8 && std::fwrite(h.data(), 1, h.size(), f) == h.size();
  std::vector<uint8_t> buf;
  for (const SaveItem& it : items) {
    if (!ok) break;
    buf.resize(it.bytes);
    if (cudaMemcpy(buf.data(), it.dev, it.bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
      std::fclose(f);
      return cuda_check(cudaGetLastError(), "save: copy tensor");
    }
    ok = std::fwrite(buf.data(), 1, it.bytes, f) == it.bytes;
  }
  ok = std::fclose(f) == 0 && ok;
  if (!ok) return set_error(LMX_ERR_IO, "write error on %s", st_path.c_str());
  // config.json in the Hugging Face / MLX field names
  std::string j = "{\n  \"model_type\": \"";
  j += c.qk_norm ? "qwen3" : "llama";
  j += "\",\n  ";
  json_num(j, "hidden_size", c.hidden, true);
  j += ",\n  ";
  json_num(j, "num_hidden_layers", c.layers, true);
  j += ",\n  ";
  json_num(j, "intermediate_size", c.inter, true);
  j += ",\n  ";
  json_num(j, "num_attention_heads", c.heads, true);
  j += ",\n  ";
  json_num(j, "num_key_value_heads", c.kv_heads, true);
  j += ",\n  ";
  json_num(j, "head_dim", c.head_dim, true);
  j += ",\n  ";
  json_num(j, "vocab_size", c.vocab, true);
  j += ",\n  ";
  json_num(j, "rope_theta", c.rope_theta, false);
  j += ",\n  ";
  json_num(j, "rms_norm_eps", c.eps, false);
  j += ",\n  \"tie_word_embeddings\": ";
  j += c.tied ? "true" : "false";
  if (!c.qk_norm && c.rope_factor > 1.0f) {
    j += ",\n  \"rope_scaling\": {\"rope_type\": \"llama3\", ";
    json_num(j, "factor", c.rope_factor, false);
    j += ", ";
    json_num(j, "low_freq_factor", c.rope_low_freq, false);
    j += ", ";
    json_num(j, "high_freq_factor", c.rope_high_freq, false);
    j += ", ";
    json_num(j, "original_max_position_embeddings", c.rope_orig_max_pos, false);
    j += "}";
  }
  j += ",\n  \"quantization\": {\n    \"group_size\": 64,\n    ";
  json_num(j, "bits", c.bits, true);
  j += over + "\n  }\n}\n";
  const std::string cfg_path = dir + "/config.json";
  f = std::fopen(cfg_path.c_str(), "wb");
  if (!f) return set_error(LMX_ERR_IO, "cannot create %s", cfg_path.c_str());
  ok = std::fwrite(j.data(), 1, j.size(), f) == j.size();
  ok = std::fclose(f) == 0 && ok;
  return ok ? LMX_OK : set_error(LMX_ERR_IO, "write error on %s", cfg_path.c_str());
}

}  // namespace ld
}  // namespace lmx

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" int lmx_model_config_load(const char* path, lmx_model_config* cfg, int32_t* eos_ids, int max_eos,
                                     int* n_eos) {
  if (!path || !cfg) return set_error(LMX_ERR_INVALID, "model_config_load: null argument");
  lmx::ld::LoadedConfig lc;
  int rc = lmx::ld::load_config(path, lc);
  if (rc) return rc;
  *cfg = lc.c;
  if (n_eos) *n_eos = (int)lc.eos.size();
  for (int i = 0; eos_ids && i < max_eos && i < (int)lc.eos.size(); ++i) eos_ids[i] = lc.eos[i];
  return LMX_OK;
}

extern "C" int lmx_model_quant_for(const char* path, const char* prefix, int* bits, int* group_size) {
  if (!path || !prefix || !bits || !group_size) return set_error(LMX_ERR_INVALID, "model_quant_for: null argument");
  lmx::ld::LoadedConfig lc;
  int rc = lmx::ld::load_config(path, lc);
  if (rc) return rc;
  const auto bg = lc.q.for_prefix(prefix);
  *bits = bg.first;
  *group_size = bg.second;
  return LMX_OK;
}

extern "C" int lmx_safetensors_tensor(const char* file, const char* name, char* dtype, int64_t* shape, int max_dims,
                                      int* ndim, uint64_t* data_offset) {
  if (!file || !name) return set_error(LMX_ERR_INVALID, "safetensors_tensor: null argument");
  lmx::ld::TensorSet ts;
  int rc = lmx::ld::st_open(file, ts);
  if (rc) return rc;
  auto it = ts.t.find(name);
  if (it == ts.t.end()) return set_error(LMX_ERR_INVALID, "%s: no tensor %s", file, name);
  const auto& r = it->second;
  if (dtype) std::snprintf(dtype, 16, "%s", r.dtype.c_str());
  if (ndim) *ndim = (int)r.shape.size();
  for (int i = 0; shape && i < max_dims && i < (int)r.shape.size(); ++i) shape[i] = r.shape[i];
  if (data_offset) *data_offset = r.off;
  return LMX_OK;
}

extern "C" int lmx_model_load(const char* dir, void** model) {
  if (!dir || !model) return set_error(LMX_ERR_INVALID, "model_load: null argument");
  lmx::Model* m = nullptr;
  int rc = lmx::ld::load_model(dir, nullptr, &m);
  if (!rc) *model = m;
  return rc;
}

extern "C" int lmx_model_load_tp(const char* dir, void* comm, void** model) {
  if (!dir || !model) return set_error(LMX_ERR_INVALID, "model_load_tp: null argument");
  lmx::Model* m = nullptr;
  int rc = lmx::ld::load_model(dir, (lmx::TpComm*)comm, &m);
  if (!rc) *model = m;
  return rc;
}

extern "C" int lmx_model_save(void* model, const char* dir) {
  if (!model || !dir) return set_error(LMX_ERR_INVALID, "model_save: null argument");
  return lmx::ld::save_model(*(const lmx::Model*)model, dir);
}
