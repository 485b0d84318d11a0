// Host-side parsing: a small JSON reader, ModelConfig (src/config.rs:39-172)
// and the safetensors header (src/safetensors_loader.rs:83-147).
#include "loader.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>

namespace tmg {

// ---------------------------------------------------------------------------
// JSON
// ---------------------------------------------------------------------------
namespace {

struct Parser {
  const char* p;
  const char* e;
  std::string err;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool fail(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  bool lit(const char* s) {
    size_t n = std::strlen(s);
    if (size_t(e - p) < n || std::strncmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  static void put_utf8(std::string& o, uint32_t c) {
    if (c < 0x80) o += char(c);
    else if (c < 0x800) { o += char(0xC0 | (c >> 6)); o += char(0x80 | (c & 63)); }
    else if (c < 0x10000) { o += char(0xE0 | (c >> 12)); o += char(0x80 | ((c >> 6) & 63)); o += char(0x80 | (c & 63)); }
    else { o += char(0xF0 | (c >> 18)); o += char(0x80 | ((c >> 12) & 63)); o += char(0x80 | ((c >> 6) & 63)); o += char(0x80 | (c & 63)); }
  }
  bool hex4(uint32_t* out) {
    if (e - p < 4) return false;
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else return false;
    }
    *out = v;
    return true;
  }
  bool str(std::string& o) {
    if (p >= e || *p != '"') return fail("expected string");
    ++p;
    while (p < e && *p != '"') {
      char c = *p++;
      if (c != '\\') { o += c; continue; }
      if (p >= e) return fail("bad escape");
      char x = *p++;
      switch (x) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t c1;
          if (!hex4(&c1)) return fail("bad \\u escape");
          if (c1 >= 0xD800 && c1 < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            p += 2;
            uint32_t c2;
            if (!hex4(&c2)) return fail("bad \\u escape");
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          }
          put_utf8(o, c1);
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p >= e) return fail("unterminated string");
    ++p;
    return true;
  }
  bool num(Json& j) {
    const char* s = p;
    bool is_int = true;
    if (p < e && *p == '-') ++p;
    while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' ||
                     *p == '+' || *p == '-')) {
      if (*p == '.' || *p == 'e' || *p == 'E') is_int = false;
      ++p;
    }
    std::string t(s, p);
    if (t.empty() || t == "-") return fail("bad number");
    char* endp = nullptr;
    j.type = Json::Num;
    j.num = std::strtod(t.c_str(), &endp);
    if (endp == t.c_str()) return fail("bad number");
    j.is_uint = false;
    if (is_int && t[0] != '-') {
      errno = 0;
      unsigned long long u = std::strtoull(t.c_str(), nullptr, 10);
      if (errno == 0) {
        j.is_uint = true;
        j.u = u;
      }
    }
    return true;
  }
  bool value(Json& j, int depth) {
    if (depth > 64) return fail("nesting too deep");
    ws();
    if (p >= e) return fail("unexpected end");
    char c = *p;
    if (c == '{') {
      ++p;
      j.type = Json::Obj;
      ws();
      if (p < e && *p == '}') { ++p; return true; }
      for (;;) {
        ws();
        std::string k;
        if (!str(k)) return false;
        ws();
        if (p >= e || *p != ':') return fail("expected ':'");
        ++p;
        Json v;
        if (!value(v, depth + 1)) return false;
        j.obj.emplace_back(std::move(k), std::move(v));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p;
      j.type = Json::Arr;
      ws();
      if (p < e && *p == ']') { ++p; return true; }
      for (;;) {
        Json v;
        if (!value(v, depth + 1)) return false;
        j.arr.push_back(std::move(v));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') { j.type = Json::Str; return str(j.str); }
    if (lit("true")) { j.type = Json::Bool; j.b = true; return true; }
    if (lit("false")) { j.type = Json::Bool; j.b = false; return true; }
    if (lit("null")) { j.type = Json::Null; return true; }
    return num(j);
  }
};

}  // namespace

const Json* Json::get(const std::string& k) const {
  if (type != Obj) return nullptr;
  for (auto& kv : obj)
    if (kv.first == k) return &kv.second;
  return nullptr;
}

bool json_parse(const char* text, size_t n, Json& out, std::string& err) {
  Parser ps{text, text + n, {}};
  if (!ps.value(out, 0)) {
    err = "invalid JSON: " + ps.err;
    return false;
  }
  ps.ws();
  if (ps.p != ps.e) {
    err = "invalid JSON: trailing characters";
    return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// ModelConfig::from_json, src/config.rs:39-93
// ---------------------------------------------------------------------------
static bool get_uint(const Json& cfg, const char* key, uint64_t* out) {
  const Json* v = cfg.get(key);
  if (!v || v->type != Json::Num || !v->is_uint) return false;
  *out = v->u;
  return true;
}

bool config_from_json(const Json& cfg, tmg_config* out, std::string& err) {
  std::memset(out, 0, sizeof(*out));
  if (cfg.type != Json::Obj) {
    err = "config is not a JSON object";
    return false;
  }
  auto need = [&](const char* k, uint64_t* v) {
    if (!get_uint(cfg, k, v)) {
      err = std::string("config missing integer field `") + k + "`";
      return false;
    }
    return true;
  };
  uint64_t hidden, heads, layers, inter, vocab, kv, hd, bos;
  if (!need("hidden_size", &hidden) || !need("num_attention_heads", &heads)) return false;
  if (!get_uint(cfg, "num_key_value_heads", &kv)) kv = heads;
  if (!get_uint(cfg, "head_dim", &hd)) hd = heads ? hidden / heads : 0;
  double theta = 10000.0;
  const Json* rt = cfg.get("rope_theta");
  if (rt && rt->type == Json::Num) theta = rt->num;
  else if (const Json* rp = cfg.get("rope_parameters")) {
    const Json* r2 = rp->get("rope_theta");
    if (r2 && r2->type == Json::Num) theta = r2->num;
  }
  out->n_eos = 0;
  if (const Json* e = cfg.get("eos_token_id")) {
    if (e->type == Json::Num) {
      if (!e->is_uint) {
        err = "bad eos_token_id";
        return false;
      }
      out->eos_token_ids[out->n_eos++] = uint32_t(e->u);
    } else if (e->type == Json::Arr) {
      for (auto& v : e->arr) {
        if (v.type == Json::Num && v.is_uint) {
          if (out->n_eos >= TMG_MAX_EOS) {
            err = "more than 8 eos_token_id values";
            return false;
          }
          out->eos_token_ids[out->n_eos++] = uint32_t(v.u);
        }
      }
    }
  }
  if (!need("num_hidden_layers", &layers) || !need("intermediate_size", &inter) ||
      !need("vocab_size", &vocab))
    return false;
  double eps = 1e-5;
  if (const Json* ev = cfg.get("rms_norm_eps"))
    if (ev->type == Json::Num) eps = ev->num;
  if (!get_uint(cfg, "bos_token_id", &bos)) bos = 0;
  const uint64_t lim = 0x7fffffffull;
  if (hidden > lim || heads > lim || kv > lim || hd > lim || layers > lim || inter > lim ||
      vocab > lim) {
    err = "config value out of range";
    return false;
  }
  out->hidden_size = int32_t(hidden);
  out->num_hidden_layers = int32_t(layers);
  out->num_attention_heads = int32_t(heads);
  out->num_key_value_heads = int32_t(kv);
  out->head_dim = int32_t(hd);
  out->intermediate_size = int32_t(inter);
  out->vocab_size = int32_t(vocab);
  out->rms_norm_eps = float(eps);
  out->rope_theta = float(theta);
  out->bos_token_id = uint32_t(bos);
  return true;
}

bool read_file(const std::string& path, std::string& out, std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    err = "reading config " + path + ": cannot open";
    return false;
  }
  std::ostringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return true;
}

// ---------------------------------------------------------------------------
// Safetensors, src/safetensors_loader.rs:83-147
// ---------------------------------------------------------------------------
MappedFile::~MappedFile() {
  if (base && base != MAP_FAILED) munmap(base, size);
  if (fd >= 0) close(fd);
}

bool MappedFile::open(const std::string& path, std::string& err) {
  fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    err = "opening " + path + ": " + std::strerror(errno);
    return false;
  }
  struct stat st;
  if (fstat(fd, &st) != 0) {
    err = "stat " + path + ": " + std::strerror(errno);
    return false;
  }
  size = size_t(st.st_size);
  if (size == 0) {
    err = "safetensors file too small: " + path;
    return false;
  }
  base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE | MAP_POPULATE, fd, 0);
  if (base == MAP_FAILED) {
    base = nullptr;
    err = "mmapping " + path + ": " + std::strerror(errno);
    return false;
  }
  return true;
}

bool safetensors_parse(const uint8_t* bytes, size_t n, std::vector<StTensor>& out,
                       std::string& err) {
  out.clear();
  if (n < 8) {
    err = "safetensors file too small";
    return false;
  }
  uint64_t hl = 0;
  for (int i = 7; i >= 0; --i) hl = (hl << 8) | bytes[i];
  if (hl > n - 8) {
    err = "safetensors header truncated";
    return false;
  }
  Json h;
  if (!json_parse(reinterpret_cast<const char*>(bytes + 8), size_t(hl), h, err)) {
    err = "invalid safetensors header JSON (" + err + ")";
    return false;
  }
  if (h.type != Json::Obj) {
    err = "safetensors header is not an object";
    return false;
  }
  const uint64_t data0 = 8 + hl, dsize = n - data0;
  for (auto& kv : h.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& t = kv.second;
    const Json* dt = t.get("dtype");
    const Json* sh = t.get("shape");
    const Json* off = t.get("data_offsets");
    if (!dt || dt->type != Json::Str || !sh || sh->type != Json::Arr || !off ||
        off->type != Json::Arr || off->arr.size() != 2) {
      err = "malformed safetensors entry `" + kv.first + "`";
      return false;
    }
    StTensor st;
    st.name = kv.first;
    int esz;
    if (dt->str == "F32") { st.dtype = 0; esz = 4; }
    else if (dt->str == "BF16") { st.dtype = 1; esz = 2; }
    else if (dt->str == "F16") { st.dtype = 2; esz = 2; }
    else {
      err = "unsupported dtype " + dt->str + " for tensor " + kv.first;
      return false;
    }
    uint64_t numel = 1;
    for (auto& d : sh->arr) {
      if (d.type != Json::Num || !d.is_uint) {
        err = "bad shape for tensor " + kv.first;
        return false;
      }
      st.shape.push_back(int64_t(d.u));
      numel *= d.u;
    }
    if (!off->arr[0].is_uint || !off->arr[1].is_uint || off->arr[0].u > off->arr[1].u ||
        off->arr[1].u > dsize) {
      err = "bad data_offsets for tensor " + kv.first;
      return false;
    }
    st.offset = int64_t(data0 + off->arr[0].u);
    st.nbytes = int64_t(off->arr[1].u - off->arr[0].u);
    if (uint64_t(st.nbytes) != numel * uint64_t(esz)) {
      err = "tensor " + kv.first + ": byte length does not match its shape";
      return false;
    }
    out.push_back(std::move(st));
  }
  return true;
}

namespace {
uint64_t le_u64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
  return v;
}
uint32_t le_u32(const uint8_t* p) {
  return uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24;
}
}  // namespace

bool tmb_parse(const uint8_t* bytes, size_t n, tmg_config* cfg, std::vector<TmbTensor>& out,
               std::string& err) {
  out.clear();
  if (n < 16) {
    err = "TMB file too small";
    return false;
  }
  if (std::memcmp(bytes, "TMB1", 4) != 0) {
    err = "not a TMB1 file (wrong magic)";
    return false;
  }
  const uint64_t cfg_len = le_u64(bytes + 4);
  const uint32_t count = le_u32(bytes + 12);
  // every step checks the bytes it reads against what is left of the file
  uint64_t pos = 16;
  auto need = [&](uint64_t k, const char* what) {
    if (k > n - pos) {
      err = std::string("TMB file truncated in the ") + what;
      return false;
    }
    return true;
  };
  if (!need(cfg_len, "config")) return false;
  Json cj;
  if (!json_parse(reinterpret_cast<const char*>(bytes + pos), size_t(cfg_len), cj, err)) {
    err = "TMB config JSON (" + err + ")";
    return false;
  }
  tmg_config c{};
  if (!config_from_json(cj, &c, err)) return false;
  pos += cfg_len;
  if (!need(8, "weights length")) return false;
  const uint64_t weights_len = le_u64(bytes + pos);
  const uint64_t weights_off = (pos + 8 + 7) & ~uint64_t(7);  // TENSOR_ALIGN = 8
  if (weights_off > n || weights_len > n - weights_off) {
    err = "TMB weights section runs past the end of the file";
    return false;
  }
  pos = weights_off + weights_len;
  out.reserve(count);
  for (uint32_t i = 0; i < count; ++i) {
    if (!need(4, "index")) return false;
    const uint32_t name_len = le_u32(bytes + pos);
    pos += 4;
    if (!need(uint64_t(name_len) + 16, "index")) return false;
    TmbTensor t;
    t.name.assign(reinterpret_cast<const char*>(bytes + pos), name_len);
    pos += name_len;
    const uint64_t off = le_u64(bytes + pos), len = le_u64(bytes + pos + 8);
    pos += 16;
    if (off > n || len > n - off) {
      err = "TMB tensor range out of bounds: " + t.name;
      return false;
    }
    t.offset = int64_t(off);
    t.nbytes = int64_t(len);
    out.push_back(std::move(t));
  }
  if (cfg) *cfg = c;
  return true;
}

// f16_to_f32, src/safetensors_loader.rs:149-173
float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000) << 16;
  uint32_t ex = (h >> 10) & 0x1f;
  uint32_t frac = h & 0x3ff;
  uint32_t bits;
  if (ex == 0) {
    if (frac == 0) {
      bits = sign;
    } else {
      uint32_t e2 = 127 - 1;
      uint32_t f = frac;
      while ((f & 0x400) == 0) {
        f <<= 1;
        e2 -= 1;
      }
      f &= 0x3ff;
      bits = sign | (e2 << 23) | (f << 13);
    }
  } else if (ex == 0x1f) {
    bits = sign | 0x7f800000u | (frac << 13);
  } else {
    bits = sign | ((ex + 127 - 15) << 23) | (frac << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

}  // namespace tmg
