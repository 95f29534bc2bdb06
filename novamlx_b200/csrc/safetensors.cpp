// safetensors files on the host side of the C ABI:
//   * a reader/writer of the format (8-byte little-endian header length, a
//     JSON header mapping tensor names to {dtype, shape, data_offsets} plus an
//     optional "__metadata__" string map, then the raw data), with the
//     header checks of Sources/NovaMLXPrefixCache/SafetensorsHeader.swift:12-31
//     (length > 0 and < 16 MiB);
//   * nmx_model_load_safetensors: an MLX checkpoint (pre-quantized u32
//     `weight` with `scales` / `biases`, PATCHES.md:21-40, names unchanged)
//     straight into the model, optionally as one tensor-parallel rank's
//     shard (rows of q/k/v/gate/up, K columns of o/down);
//   * nmx_ssd_save_block / nmx_ssd_load_block: the SSD prefix-block store's
//     file format (SSDCacheStore.saveBlock / loadBlock,
//     Sources/NovaMLXPrefixCache/SSDCacheStore.swift:132-135,194-269): one
//     file per block at <dir>/<first hex digit>/<hex SHA-1>.safetensors,
//     tensors "i.j" (layer i, state j: 0 keys, 1 values, shape
//     [1, kv heads, block tokens, head dim]), metadata block_hash,
//     token_count, num_layers, model_name, created_at, layer_cache_types;
//     written to a .tmp.safetensors file and renamed. Pages move between the
//     file and the device pool without a detour through any array library.
#include <sys/stat.h>

#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "model.h"

namespace {

using nmx::set_error;

// ------------------------------------------------------------------ JSON
struct JVal {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  double num = 0;
  long long inum = 0;
  bool b = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* e;
  bool ok = true;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if (size_t(e - p) < n || strncmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  static void utf8(std::string& o, unsigned cp) {
    if (cp < 0x80) {
      o += char(cp);
    } else if (cp < 0x800) {
      o += char(0xC0 | (cp >> 6));
      o += char(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += char(0xE0 | (cp >> 12));
      o += char(0x80 | ((cp >> 6) & 0x3F));
      o += char(0x80 | (cp & 0x3F));
    } else {
      o += char(0xF0 | (cp >> 18));
      o += char(0x80 | ((cp >> 12) & 0x3F));
      o += char(0x80 | ((cp >> 6) & 0x3F));
      o += char(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(unsigned& v) {
    if (e - p < 4) return false;
    v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= unsigned(c - '0');
      else if (c >= 'a' && c <= 'f') v |= unsigned(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= unsigned(c - 'A' + 10);
      else return false;
    }
    return true;
  }
  bool string(std::string& o) {
    if (p >= e || *p != '"') return false;
    ++p;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= e) return false;
        const char c = *p++;
        switch (c) {
          case '"': o += '"'; break;
          case '\\': o += '\\'; break;
          case '/': o += '/'; break;
          case 'b': o += '\b'; break;
          case 'f': o += '\f'; break;
          case 'n': o += '\n'; break;
          case 'r': o += '\r'; break;
          case 't': o += '\t'; break;
          case 'u': {
            unsigned cp;
            if (!hex4(cp)) return false;
            if (cp >= 0xD800 && cp < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
              p += 2;
              unsigned lo;
              if (!hex4(lo)) return false;
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            }
            utf8(o, cp);
            break;
          }
          default: return false;
        }
      } else {
        o += *p++;
      }
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool value(JVal& v, int depth) {
    if (depth > 64) return false;
    ws();
    if (p >= e) return false;
    if (*p == '{') {
      v.kind = JVal::OBJ;
      ++p;
      ws();
      if (p < e && *p == '}') {
        ++p;
        return true;
      }
      for (;;) {
        ws();
        std::string k;
        if (!string(k)) return false;
        ws();
        if (p >= e || *p != ':') return false;
        ++p;
        JVal c;
        if (!value(c, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(c));
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == '}') {
          ++p;
          return true;
        }
        return false;
      }
    }
    if (*p == '[') {
      v.kind = JVal::ARR;
      ++p;
      ws();
      if (p < e && *p == ']') {
        ++p;
        return true;
      }
      for (;;) {
        JVal c;
        if (!value(c, depth + 1)) return false;
        v.arr.push_back(std::move(c));
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == ']') {
          ++p;
          return true;
        }
        return false;
      }
    }
    if (*p == '"') {
      v.kind = JVal::STR;
      return string(v.str);
    }
    if (lit("true")) {
      v.kind = JVal::BOOL;
      v.b = true;
      return true;
    }
    if (lit("false")) {
      v.kind = JVal::BOOL;
      return true;
    }
    if (lit("null")) return true;
    // number
    const char* s = p;
    if (p < e && (*p == '-' || *p == '+')) ++p;
    bool frac = false;
    while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+')) {
      if (*p == '.' || *p == 'e' || *p == 'E') frac = true;
      ++p;
    }
    if (p == s) return false;
    const std::string t(s, p);
    v.kind = JVal::NUM;
    v.num = strtod(t.c_str(), nullptr);
    v.inum = frac ? (long long)v.num : strtoll(t.c_str(), nullptr, 10);
    return true;
  }
};

void json_escape(std::string& o, const std::string& s) {
  o += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (c < 0x20) {
          char b[8];
          snprintf(b, sizeof b, "\\u%04x", c);
          o += b;
        } else {
          o += char(c);
        }
    }
  }
  o += '"';
}

// ------------------------------------------------------------ the format
struct TensorInfo {
  std::string name, dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // within the data section
};

constexpr uint64_t kMaxHeader = 16ull << 20;

size_t dtype_bytes(const std::string& d) {
  if (d == "U8" || d == "I8" || d == "BOOL") return 1;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  return 0;
}

}  // namespace

struct nmx_safetensors_s {
  FILE* f = nullptr;
  uint64_t data_off = 0, file_size = 0;
  std::vector<TensorInfo> tensors;
  std::map<std::string, std::string> meta;
  ~nmx_safetensors_s() {
    if (f) fclose(f);
  }
};

namespace {

nmx_status_t st_open(const char* path, std::unique_ptr<nmx_safetensors_s>& out) {
  auto s = std::make_unique<nmx_safetensors_s>();
  s->f = fopen(path, "rb");
  NMX_CHECK(s->f != nullptr, NMX_ERR_NOT_FOUND, std::string("safetensors: cannot open ") + path);
  fseek(s->f, 0, SEEK_END);
  s->file_size = uint64_t(ftell(s->f));
  fseek(s->f, 0, SEEK_SET);
  unsigned char lenb[8];
  NMX_CHECK(fread(lenb, 1, 8, s->f) == 8, NMX_ERR_INVALID, "safetensors: short read of the header length");
  uint64_t hl = 0;
  for (int i = 7; i >= 0; --i) hl = (hl << 8) | lenb[i];
  NMX_CHECK(hl > 0 && hl < kMaxHeader && 8 + hl <= s->file_size, NMX_ERR_INVALID,
            "safetensors: header length out of range");
  std::string hdr(size_t(hl), '\0');
  NMX_CHECK(fread(&hdr[0], 1, size_t(hl), s->f) == size_t(hl), NMX_ERR_INVALID, "safetensors: short header");
  JParser jp{hdr.data(), hdr.data() + hdr.size()};
  JVal root;
  NMX_CHECK(jp.value(root, 0) && root.kind == JVal::OBJ, NMX_ERR_INVALID, "safetensors: header is not a JSON object");
  s->data_off = 8 + hl;
  const uint64_t data_size = s->file_size - s->data_off;
  for (const auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      NMX_CHECK(kv.second.kind == JVal::OBJ, NMX_ERR_INVALID, "safetensors: __metadata__ must be an object");
      for (const auto& m : kv.second.obj)
        if (m.second.kind == JVal::STR) s->meta[m.first] = m.second.str;
      continue;
    }
    const JVal& t = kv.second;
    const JVal* dt = t.get("dtype");
    const JVal* sh = t.get("shape");
    const JVal* off = t.get("data_offsets");
    NMX_CHECK(t.kind == JVal::OBJ && dt && dt->kind == JVal::STR && sh && sh->kind == JVal::ARR && off &&
                  off->kind == JVal::ARR && off->arr.size() == 2,
              NMX_ERR_INVALID, "safetensors: malformed entry " + kv.first);
    TensorInfo ti;
    ti.name = kv.first;
    ti.dtype = dt->str;
    uint64_t n = 1;
    for (const auto& d : sh->arr) {
      NMX_CHECK(d.kind == JVal::NUM && d.inum >= 0, NMX_ERR_INVALID, "safetensors: bad shape of " + kv.first);
      ti.shape.push_back(d.inum);
      n *= uint64_t(d.inum);
    }
    ti.begin = uint64_t(off->arr[0].inum);
    ti.end = uint64_t(off->arr[1].inum);
    const size_t eb = dtype_bytes(ti.dtype);
    NMX_CHECK(eb > 0, NMX_ERR_UNSUPPORTED, "safetensors: unsupported dtype " + ti.dtype);
    NMX_CHECK(ti.begin <= ti.end && ti.end <= data_size && ti.end - ti.begin == n * eb, NMX_ERR_INVALID,
              "safetensors: data offsets of " + kv.first + " do not match its shape");
    s->tensors.push_back(std::move(ti));
  }
  out = std::move(s);
  return NMX_OK;
}

nmx_status_t st_read(nmx_safetensors_s* s, const TensorInfo& t, void* dst) {
  NMX_CHECK(fseek(s->f, long(s->data_off + t.begin), SEEK_SET) == 0, NMX_ERR_INVALID, "safetensors: seek failed");
  const size_t n = size_t(t.end - t.begin);
  NMX_CHECK(fread(dst, 1, n, s->f) == n, NMX_ERR_INVALID, "safetensors: short read of " + t.name);
  return NMX_OK;
}

struct WTensor {
  std::string name, dtype;
  std::vector<int64_t> shape;
  const void* data;
  size_t bytes;
};

nmx_status_t st_write(const std::string& path, const std::vector<WTensor>& ts,
                      const std::vector<std::pair<std::string, std::string>>& meta) {
  std::string h = "{";
  bool first = true;
  if (!meta.empty()) {
    h += "\"__metadata__\":{";
    for (size_t i = 0; i < meta.size(); ++i) {
      if (i) h += ',';
      json_escape(h, meta[i].first);
      h += ':';
      json_escape(h, meta[i].second);
    }
    h += '}';
    first = false;
  }
  uint64_t off = 0;
  for (const auto& t : ts) {
    if (!first) h += ',';
    first = false;
    json_escape(h, t.name);
    h += ":{\"dtype\":";
    json_escape(h, t.dtype);
    h += ",\"shape\":[";
    for (size_t i = 0; i < t.shape.size(); ++i) {
      if (i) h += ',';
      h += std::to_string(t.shape[i]);
    }
    h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + t.bytes) + "]}";
    off += t.bytes;
  }
  h += '}';
  while (h.size() % 8) h += ' ';  // data starts 8-byte aligned
  FILE* f = fopen(path.c_str(), "wb");
  NMX_CHECK(f != nullptr, NMX_ERR_INVALID, "safetensors: cannot write " + path);
  unsigned char lenb[8];
  uint64_t hl = h.size();
  for (int i = 0; i < 8; ++i) lenb[i] = (unsigned char)((hl >> (8 * i)) & 0xFF);
  bool ok = fwrite(lenb, 1, 8, f) == 8 && fwrite(h.data(), 1, h.size(), f) == h.size();
  for (const auto& t : ts) ok = ok && fwrite(t.data, 1, t.bytes, f) == t.bytes;
  ok = (fclose(f) == 0) && ok;
  NMX_CHECK(ok, NMX_ERR_INVALID, "safetensors: write failed for " + path);
  return NMX_OK;
}

nmx_dtype_t nmx_dtype_of(const std::string& d, bool* ok) {
  *ok = true;
  if (d == "U32") return NMX_U32;
  if (d == "F16") return NMX_F16;
  if (d == "BF16") return NMX_BF16;
  if (d == "F32") return NMX_F32;
  *ok = false;
  return NMX_F16;
}

// tensor-parallel slice of one checkpoint tensor (rows of q/k/v/gate/up and
// their biases, K columns of o/down), or the whole tensor
struct Slice {
  bool rows = false, cols = false;
  int64_t len = 0;  // rows, or columns in storage units
};

Slice tp_slice(const std::string& name, const nmx_model_cfg& local, int tp, int bits, int gs) {
  Slice s;
  if (tp <= 1) return s;
  const size_t dot = name.rfind('.');
  if (dot == std::string::npos) return s;
  const std::string kind = name.substr(dot + 1);
  const size_t d2 = name.rfind('.', dot - 1);
  const std::string mod = name.substr(d2 == std::string::npos ? 0 : d2 + 1, dot - (d2 == std::string::npos ? 0 : d2 + 1));
  const int64_t nq = int64_t(local.n_heads) * local.head_dim, nkv = int64_t(local.n_kv_heads) * local.head_dim;
  const int64_t f = local.ffn;
  if (mod == "q_proj") s.len = nq;
  else if (mod == "k_proj" || mod == "v_proj") s.len = nkv;
  else if (mod == "gate_proj" || mod == "up_proj") s.len = f;
  if (s.len) {
    s.rows = true;
    return s;
  }
  int64_t k = 0;
  if (mod == "o_proj") k = nq;
  else if (mod == "down_proj") k = f;
  if (!k) return s;
  if (kind == "weight") s.len = k * bits / 32;
  else if (kind == "scales" || kind == "biases") s.len = k / gs;
  else return s;  // an o/down bias (none in Llama/Qwen2) is replicated
  s.cols = true;
  return s;
}

std::string hex20(const uint8_t* h) {
  static const char* d = "0123456789abcdef";
  std::string s;
  for (int i = 0; i < 20; ++i) {
    s += d[h[i] >> 4];
    s += d[h[i] & 15];
  }
  return s;
}

bool mkdir_p(const std::string& dir) {
  std::string cur;
  for (size_t i = 0; i <= dir.size(); ++i) {
    if (i == dir.size() || dir[i] == '/') {
      if (!cur.empty() && mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST) return false;
    }
    if (i < dir.size()) cur += dir[i];
  }
  return true;
}

}  // namespace

extern "C" {

NMX_API nmx_status_t nmx_safetensors_open(const char* path, nmx_safetensors_t* out) {
  nmx::clear_error();
  NMX_CHECK(path && out, NMX_ERR_INVALID, "nmx_safetensors_open: null argument");
  std::unique_ptr<nmx_safetensors_s> s;
  NMX_TRY(st_open(path, s));
  *out = s.release();
  return NMX_OK;
}

NMX_API void nmx_safetensors_close(nmx_safetensors_t s) { delete s; }

NMX_API int nmx_safetensors_count(nmx_safetensors_t s) { return s ? int(s->tensors.size()) : 0; }

NMX_API nmx_status_t nmx_safetensors_info(nmx_safetensors_t s, int i, char* name, int name_cap, char* dtype,
                                          int64_t* shape, int* ndim, uint64_t* nbytes) {
  nmx::clear_error();
  NMX_CHECK(s && i >= 0 && i < int(s->tensors.size()), NMX_ERR_INVALID, "nmx_safetensors_info: index out of range");
  const TensorInfo& t = s->tensors[size_t(i)];
  if (name && name_cap > 0) {
    NMX_CHECK(int(t.name.size()) < name_cap, NMX_ERR_INVALID, "nmx_safetensors_info: name buffer too small");
    memcpy(name, t.name.c_str(), t.name.size() + 1);
  }
  if (dtype) {
    strncpy(dtype, t.dtype.c_str(), 7);
    dtype[7] = '\0';
  }
  if (ndim) *ndim = int(t.shape.size());
  if (shape)
    for (size_t d = 0; d < t.shape.size() && d < 8; ++d) shape[d] = t.shape[d];
  if (nbytes) *nbytes = t.end - t.begin;
  return NMX_OK;
}

NMX_API int nmx_safetensors_metadata(nmx_safetensors_t s, const char* key, char* out, int cap) {
  if (!s || !key) return -1;
  auto it = s->meta.find(key);
  if (it == s->meta.end()) return -1;
  if (out && cap > 0) {
    const size_t n = std::min(it->second.size(), size_t(cap - 1));
    memcpy(out, it->second.data(), n);
    out[n] = '\0';
  }
  return int(it->second.size());
}

NMX_API nmx_status_t nmx_safetensors_read(nmx_safetensors_t s, const char* name, void* host, uint64_t host_bytes) {
  nmx::clear_error();
  NMX_CHECK(s && name && host, NMX_ERR_INVALID, "nmx_safetensors_read: null argument");
  for (const auto& t : s->tensors)
    if (t.name == name) {
      NMX_CHECK(host_bytes >= t.end - t.begin, NMX_ERR_INVALID, "nmx_safetensors_read: buffer too small");
      return st_read(s, t, host);
    }
  NMX_CHECK(false, NMX_ERR_NOT_FOUND, std::string("nmx_safetensors_read: no tensor ") + name);
}

NMX_API nmx_status_t nmx_safetensors_write(const char* path, int n, const char* const* names,
                                           const char* const* dtypes, const int64_t* const* shapes, const int* ndims,
                                           const void* const* data, int n_meta, const char* const* meta_keys,
                                           const char* const* meta_values) {
  nmx::clear_error();
  NMX_CHECK(path && n >= 0 && (n == 0 || (names && dtypes && shapes && ndims && data)), NMX_ERR_INVALID,
            "nmx_safetensors_write: null argument");
  std::vector<WTensor> ts;
  for (int i = 0; i < n; ++i) {
    WTensor t;
    t.name = names[i];
    t.dtype = dtypes[i];
    const size_t eb = dtype_bytes(t.dtype);
    NMX_CHECK(eb > 0, NMX_ERR_UNSUPPORTED, "nmx_safetensors_write: unsupported dtype " + t.dtype);
    size_t cnt = 1;
    for (int d = 0; d < ndims[i]; ++d) {
      t.shape.push_back(shapes[i][d]);
      cnt *= size_t(shapes[i][d]);
    }
    t.data = data[i];
    t.bytes = cnt * eb;
    ts.push_back(std::move(t));
  }
  std::vector<std::pair<std::string, std::string>> meta;
  for (int i = 0; i < n_meta; ++i) meta.emplace_back(meta_keys[i], meta_values[i]);
  return st_write(path, ts, meta);
}

NMX_API nmx_status_t nmx_model_load_safetensors(nmx_model_t model, const char* path, int tp_rank, int tp_size,
                                                int* n_loaded, int* n_skipped) {
  nmx::clear_error();
  NMX_CHECK(model && path, NMX_ERR_INVALID, "nmx_model_load_safetensors: null argument");
  NMX_CHECK(tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size, NMX_ERR_INVALID,
            "nmx_model_load_safetensors: tensor-parallel rank out of range");
  std::unique_ptr<nmx_safetensors_s> s;
  NMX_TRY(st_open(path, s));
  const nmx_model_cfg& local = model->m->cfg;
  int loaded = 0, skipped = 0;
  std::vector<unsigned char> buf, part;
  for (const auto& t : s->tensors) {
    bool ok = false;
    const nmx_dtype_t dt = nmx_dtype_of(t.dtype, &ok);
    if (!ok) {
      ++skipped;
      continue;
    }
    buf.resize(size_t(t.end - t.begin));
    NMX_TRY(st_read(s.get(), t, buf.data()));
    const Slice sl = tp_slice(t.name, local, tp_size, local.bits, local.group_size);
    const size_t eb = dtype_bytes(t.dtype);
    std::vector<int64_t> shape = t.shape;
    const void* src = buf.data();
    if (sl.rows) {
      NMX_CHECK(!shape.empty() && shape[0] == sl.len * tp_size, NMX_ERR_INVALID,
                "nmx_model_load_safetensors: " + t.name + " does not split into the ranks' rows");
      size_t row_bytes = eb;
      for (size_t d = 1; d < shape.size(); ++d) row_bytes *= size_t(shape[d]);
      src = buf.data() + size_t(tp_rank) * size_t(sl.len) * row_bytes;
      shape[0] = sl.len;
    } else if (sl.cols) {
      NMX_CHECK(shape.size() == 2 && shape[1] == sl.len * tp_size, NMX_ERR_INVALID,
                "nmx_model_load_safetensors: " + t.name + " does not split into the ranks' columns");
      part.resize(size_t(shape[0]) * size_t(sl.len) * eb);
      for (int64_t r = 0; r < shape[0]; ++r)
        memcpy(part.data() + size_t(r) * size_t(sl.len) * eb,
               buf.data() + (size_t(r) * size_t(shape[1]) + size_t(tp_rank) * size_t(sl.len)) * eb,
               size_t(sl.len) * eb);
      src = part.data();
      shape[1] = sl.len;
    }
    const nmx_status_t st = nmx_model_load_tensor(model, t.name.c_str(), src, dt, shape.data(), int(shape.size()));
    if (st == NMX_ERR_NOT_FOUND) {
      nmx::clear_error();
      ++skipped;  // a tensor the model has no slot for (e.g. rotary tables)
      continue;
    }
    NMX_TRY(st);
    ++loaded;
  }
  if (n_loaded) *n_loaded = loaded;
  if (n_skipped) *n_skipped = skipped;
  return NMX_OK;
}

NMX_API nmx_status_t nmx_ssd_save_block(nmx_kv_pool_t pool, int block_id, const uint8_t hash20[20], int token_count,
                                        const char* model_name, const char* cache_dir) {
  nmx::clear_error();
  NMX_CHECK(pool && hash20 && cache_dir, NMX_ERR_INVALID, "nmx_ssd_save_block: null argument");
  nmx::KvPool* p = pool->p;
  NMX_CHECK(p->kv_bits == 0, NMX_ERR_UNSUPPORTED, "nmx_ssd_save_block: the SSD store holds f16 blocks");
  const nmx_model_cfg& cf = p->model->cfg;
  const int L = cf.n_layers, bt = int(p->block_bytes / (size_t(cf.n_kv_heads) * cf.head_dim * 2));
  std::vector<unsigned char> host(size_t(L) * 2 * p->block_bytes);
  const int32_t id = block_id;
  NMX_TRY(nmx_kv_read_blocks(pool, &id, 1, host.data()));
  const std::string hex = hex20(hash20);
  const std::string dir = std::string(cache_dir) + "/" + hex.substr(0, 1);
  NMX_CHECK(mkdir_p(dir), NMX_ERR_INVALID, "nmx_ssd_save_block: cannot create " + dir);
  std::vector<WTensor> ts;
  for (int l = 0; l < L; ++l)
    for (int j = 0; j < 2; ++j) {
      WTensor t;
      t.name = std::to_string(l) + "." + std::to_string(j);
      t.dtype = cf.dtype == NMX_BF16 ? "BF16" : "F16";
      t.shape = {1, cf.n_kv_heads, bt, cf.head_dim};
      t.data = host.data() + (size_t(l) * 2 + j) * p->block_bytes;
      t.bytes = p->block_bytes;
      ts.push_back(std::move(t));
    }
  std::string types = "[";
  for (int l = 0; l < L; ++l) types += std::string(l ? "," : "") + "\"KVCacheSimple\"";
  types += "]";
  const double now =
      std::chrono::duration<double>(std::chrono::system_clock::now().time_since_epoch()).count();
  std::vector<std::pair<std::string, std::string>> meta = {
      {"block_hash", hex},
      {"token_count", std::to_string(token_count)},
      {"num_layers", std::to_string(L)},
      {"model_name", model_name ? model_name : ""},
      {"created_at", std::to_string(now)},
      {"layer_cache_types", types},
  };
  const std::string path = dir + "/" + hex + ".safetensors";
  const std::string tmp = dir + "/" + hex + ".tmp.safetensors";
  NMX_TRY(st_write(tmp, ts, meta));
  NMX_CHECK(rename(tmp.c_str(), path.c_str()) == 0, NMX_ERR_INVALID, "nmx_ssd_save_block: rename failed");
  return NMX_OK;
}

NMX_API nmx_status_t nmx_ssd_load_block(nmx_kv_pool_t pool, const uint8_t hash20[20], const char* cache_dir,
                                        int block_id, int* token_count) {
  nmx::clear_error();
  NMX_CHECK(pool && hash20 && cache_dir, NMX_ERR_INVALID, "nmx_ssd_load_block: null argument");
  nmx::KvPool* p = pool->p;
  NMX_CHECK(p->kv_bits == 0, NMX_ERR_UNSUPPORTED, "nmx_ssd_load_block: the SSD store holds f16 blocks");
  const nmx_model_cfg& cf = p->model->cfg;
  const int L = cf.n_layers;
  const std::string hex = hex20(hash20);
  const std::string path = std::string(cache_dir) + "/" + hex.substr(0, 1) + "/" + hex + ".safetensors";
  std::unique_ptr<nmx_safetensors_s> s;
  NMX_TRY(st_open(path.c_str(), s));
  auto nl = s->meta.find("num_layers");
  NMX_CHECK(nl != s->meta.end() && atoi(nl->second.c_str()) == L, NMX_ERR_INVALID,
            "nmx_ssd_load_block: the block was saved for another layer count");
  auto bh = s->meta.find("block_hash");
  NMX_CHECK(bh == s->meta.end() || bh->second == hex, NMX_ERR_INVALID, "nmx_ssd_load_block: hash mismatch");
  std::vector<unsigned char> host(size_t(L) * 2 * p->block_bytes);
  std::map<std::string, const TensorInfo*> by;
  for (const auto& t : s->tensors) by[t.name] = &t;
  for (int l = 0; l < L; ++l)
    for (int j = 0; j < 2; ++j) {
      auto it = by.find(std::to_string(l) + "." + std::to_string(j));
      NMX_CHECK(it != by.end(), NMX_ERR_INVALID, "nmx_ssd_load_block: missing layer state");
      NMX_CHECK(it->second->end - it->second->begin == p->block_bytes, NMX_ERR_INVALID,
                "nmx_ssd_load_block: block shape does not match the pool");
      NMX_TRY(st_read(s.get(), *it->second, host.data() + (size_t(l) * 2 + j) * p->block_bytes));
    }
  const int32_t id = block_id;
  NMX_TRY(nmx_kv_write_blocks(pool, &id, 1, host.data()));
  if (token_count) {
    auto tc = s->meta.find("token_count");
    *token_count = tc == s->meta.end() ? 0 : atoi(tc->second.c_str());
  }
  return NMX_OK;
}

}  // extern "C"
