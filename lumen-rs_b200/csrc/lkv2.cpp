// LKV2 file format (crates/lumen-mlx/src/kv_disk.rs), host side: CRC-32,
// the manifest's JSON, records, reader checks.
#include "lkv2.h"

#include <cctype>
#include <cstdio>
#include <cstring>

#include "common.h"

namespace lc {

int lkv2_elem_size(uint8_t d) {
  switch (d) {  // stored_elem_size (kv_disk.rs:70-78)
    case kLkvBool: case kLkvU8: case kLkvI8: return 1;
    case kLkvU16: case kLkvI16: case kLkvF16: case kLkvBF16: return 2;
    case kLkvF32: case kLkvU32: case kLkvI32: return 4;
    case kLkvU64: case kLkvI64: case kLkvF64: return 8;
    default: return -1;
  }
}

int64_t Lkv2Record::elems() const {
  if (shape.empty()) return 0;  // elem_count (kv_disk.rs:134-140)
  int64_t n = 1;
  for (int32_t d : shape) n *= d < 0 ? 0 : d;
  return n;
}

// CRC-32/IEEE, reflected polynomial 0xEDB88320, init and final xor ~0.
uint32_t crc32_ieee(const uint8_t* p, size_t n, uint32_t crc) {
  static uint32_t table[256];
  static bool ready = false;
  if (!ready) {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      table[i] = c;
    }
    ready = true;
  }
  crc = ~crc;
  for (size_t i = 0; i < n; ++i) crc = table[(crc ^ p[i]) & 0xFF] ^ (crc >> 8);
  return ~crc;
}

// ---- JSON ------------------------------------------------------------------

namespace {

void json_str(std::string& o, const std::string& s) {
  static const char* hex = "0123456789abcdef";
  o += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\b': o += "\\b"; break;
      case '\f': o += "\\f"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (c < 0x20) {
          o += "\\u00";
          o += hex[c >> 4];
          o += hex[c & 15];
        } else {
          o += (char)c;
        }
    }
  }
  o += '"';
}

void json_opt(std::string& o, const char* key, int64_t v) {
  if (v < 0) return;
  o += ",\"";
  o += key;
  o += "\":" + std::to_string(v);
}

// A JSON value: enough of the grammar for manifests (numbers kept as text).
struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  std::string s;  // number text or string
  std::vector<JVal> a;
  std::vector<std::pair<std::string, JVal>> o;
  const JVal* get(const char* k) const {
    for (auto& kv : o)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const std::string& t;
  size_t i = 0;
  int depth = 0;
  explicit JParser(const std::string& s) : t(s) {}
  [[noreturn]] void fail(const char* what) {
    LC_THROW(LC_ERR_IO, std::string("LKV2 manifest: ") + what + " at byte " + std::to_string(i));
  }
  void ws() {
    while (i < t.size() && (t[i] == ' ' || t[i] == '\n' || t[i] == '\r' || t[i] == '\t')) ++i;
  }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if (t.compare(i, n, w) == 0) {
      i += n;
      return true;
    }
    return false;
  }
  static void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o += (char)cp;
    } else if (cp < 0x800) {
      o += (char)(0xC0 | (cp >> 6));
      o += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += (char)(0xE0 | (cp >> 12));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    } else {
      o += (char)(0xF0 | (cp >> 18));
      o += (char)(0x80 | ((cp >> 12) & 0x3F));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (i + 4 > t.size()) fail("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = t[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string str() {
    if (i >= t.size() || t[i] != '"') fail("expected a string");
    ++i;
    std::string o;
    while (true) {
      if (i >= t.size()) fail("unterminated string");
      const char c = t[i++];
      if (c == '"') break;
      if ((unsigned char)c < 0x20) fail("control character in string");
      if (c != '\\') {
        o += c;
        continue;
      }
      if (i >= t.size()) fail("unterminated escape");
      const char e = t[i++];
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            if (!(i + 1 < t.size() && t[i] == '\\' && t[i + 1] == 'u')) fail("lone surrogate");
            i += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(o, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return o;
  }
  JVal val() {
    if (++depth > 64) fail("nesting too deep");
    ws();
    if (i >= t.size()) fail("unexpected end");
    JVal v;
    const char c = t[i];
    if (c == '{') {
      v.kind = JVal::Obj;
      ++i;
      ws();
      if (i < t.size() && t[i] == '}') {
        ++i;
      } else {
        while (true) {
          ws();
          std::string k = str();
          ws();
          if (i >= t.size() || t[i] != ':') fail("expected ':'");
          ++i;
          v.o.emplace_back(std::move(k), val());
          ws();
          if (i < t.size() && t[i] == ',') { ++i; continue; }
          if (i < t.size() && t[i] == '}') { ++i; break; }
          fail("expected ',' or '}'");
        }
      }
    } else if (c == '[') {
      v.kind = JVal::Arr;
      ++i;
      ws();
      if (i < t.size() && t[i] == ']') {
        ++i;
      } else {
        while (true) {
          v.a.push_back(val());
          ws();
          if (i < t.size() && t[i] == ',') { ++i; continue; }
          if (i < t.size() && t[i] == ']') { ++i; break; }
          fail("expected ',' or ']'");
        }
      }
    } else if (c == '"') {
      v.kind = JVal::Str;
      v.s = str();
    } else if (lit("null")) {
      v.kind = JVal::Null;
    } else if (lit("true")) {
      v.kind = JVal::Bool;
      v.b = true;
    } else if (lit("false")) {
      v.kind = JVal::Bool;
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      v.kind = JVal::Num;
      const size_t b = i;
      if (t[i] == '-') ++i;
      while (i < t.size() && (std::isdigit((unsigned char)t[i]) || t[i] == '.' || t[i] == 'e' || t[i] == 'E' ||
                              t[i] == '+' || t[i] == '-'))
        ++i;
      v.s = t.substr(b, i - b);
    } else {
      fail("unexpected character");
    }
    --depth;
    return v;
  }
};

// Non-negative integers as the reference's usize / u32 / u64 fields.
uint64_t as_uint(const JVal& v, const char* what, uint64_t max) {
  if (v.kind != JVal::Num || v.s.empty() || v.s[0] == '-')
    LC_THROW(LC_ERR_IO, std::string("LKV2 manifest: ") + what + " is not a non-negative integer");
  uint64_t r = 0;
  for (char c : v.s) {
    if (c < '0' || c > '9') LC_THROW(LC_ERR_IO, std::string("LKV2 manifest: ") + what + " is not an integer");
    const uint64_t d = (uint64_t)(c - '0');
    if (r > (max - d) / 10) LC_THROW(LC_ERR_IO, std::string("LKV2 manifest: ") + what + " out of range");
    r = r * 10 + d;
  }
  return r;
}

int64_t opt_uint(const JVal& o, const char* key, uint64_t max) {
  const JVal* v = o.get(key);
  if (!v || v->kind == JVal::Null) return -1;
  return (int64_t)as_uint(*v, key, max);
}

const JVal& need(const JVal& o, const char* key) {
  const JVal* v = o.get(key);
  if (!v) LC_THROW(LC_ERR_IO, std::string("LKV2 manifest: missing field ") + key);
  return *v;
}

constexpr uint64_t kUsizeMax = (uint64_t)INT64_MAX;  // kept representable as int64 here

}  // namespace

std::string lkv2_manifest_json(const Lkv2Manifest& m) {
  std::string o = "{\"model_fingerprint\":";
  json_str(o, m.model_fingerprint);
  o += ",\"created_at_unix\":" + std::to_string(m.created_at_unix);
  o += ",\"position\":" + std::to_string(m.position);
  o += ",\"prefix_tokens\":[";
  for (size_t k = 0; k < m.prefix_tokens.size(); ++k) {
    if (k) o += ',';
    o += std::to_string(m.prefix_tokens[k]);
  }
  o += ']';
  if (m.last_token >= 0) o += ",\"last_token\":" + std::to_string(m.last_token);
  o += ",\"is_deep\":";
  o += m.is_deep ? "true" : "false";
  o += ",\"layers\":[";
  for (size_t k = 0; k < m.layers.size(); ++k) {
    const Lkv2Layer& L = m.layers[k];
    if (k) o += ',';
    o += "{\"kind\":";
    json_str(o, L.kind);
    o += ",\"offset\":" + std::to_string(L.offset);
    o += ",\"base_offset\":" + std::to_string(L.base_offset);
    o += ",\"arrays\":[";
    for (size_t j = 0; j < L.arrays.size(); ++j) {
      if (j) o += ',';
      o += L.arrays[j] < 0 ? std::string("null") : std::to_string(L.arrays[j]);
    }
    o += ']';
    json_opt(o, "lengths_id", L.lengths_id);
    json_opt(o, "left_padding_id", L.left_padding_id);
    json_opt(o, "max_size", L.max_size);
    json_opt(o, "keep", L.keep);
    json_opt(o, "idx", L.idx);
    json_opt(o, "bits", L.bits);
    json_opt(o, "qjl_m", L.qjl_m);
    json_opt(o, "group_size", L.group_size);
    json_opt(o, "v_bits", L.v_bits);
    o += '}';
  }
  o += "]}";
  return o;
}

Lkv2Manifest lkv2_parse_manifest(const std::string& json) {
  JParser p(json);
  const JVal root = p.val();
  p.ws();
  if (p.i != json.size()) p.fail("trailing characters");
  if (root.kind != JVal::Obj) LC_THROW(LC_ERR_IO, "LKV2 manifest: not a JSON object");
  Lkv2Manifest m;
  const JVal& fp = need(root, "model_fingerprint");
  if (fp.kind != JVal::Str) LC_THROW(LC_ERR_IO, "LKV2 manifest: model_fingerprint is not a string");
  m.model_fingerprint = fp.s;
  m.created_at_unix = as_uint(need(root, "created_at_unix"), "created_at_unix", UINT64_MAX);
  m.position = as_uint(need(root, "position"), "position", kUsizeMax);
  const JVal& pt = need(root, "prefix_tokens");
  if (pt.kind != JVal::Arr) LC_THROW(LC_ERR_IO, "LKV2 manifest: prefix_tokens is not an array");
  for (const JVal& v : pt.a) m.prefix_tokens.push_back((uint32_t)as_uint(v, "prefix_tokens", UINT32_MAX));
  m.last_token = opt_uint(root, "last_token", UINT32_MAX);
  if (const JVal* d = root.get("is_deep")) {
    if (d->kind != JVal::Bool) LC_THROW(LC_ERR_IO, "LKV2 manifest: is_deep is not a bool");
    m.is_deep = d->b;
  }
  const JVal& ls = need(root, "layers");
  if (ls.kind != JVal::Arr) LC_THROW(LC_ERR_IO, "LKV2 manifest: layers is not an array");
  for (const JVal& lv : ls.a) {
    if (lv.kind != JVal::Obj) LC_THROW(LC_ERR_IO, "LKV2 manifest: a layer is not an object");
    Lkv2Layer L;
    const JVal& k = need(lv, "kind");
    if (k.kind != JVal::Str) LC_THROW(LC_ERR_IO, "LKV2 manifest: layer kind is not a string");
    L.kind = k.s;
    L.offset = as_uint(need(lv, "offset"), "offset", kUsizeMax);
    if (const JVal* b = lv.get("base_offset")) L.base_offset = as_uint(*b, "base_offset", kUsizeMax);
    if (const JVal* a = lv.get("arrays")) {
      if (a->kind != JVal::Arr) LC_THROW(LC_ERR_IO, "LKV2 manifest: arrays is not an array");
      for (const JVal& e : a->a)
        L.arrays.push_back(e.kind == JVal::Null ? -1 : (int64_t)as_uint(e, "arrays", kUsizeMax));
    }
    L.lengths_id = opt_uint(lv, "lengths_id", kUsizeMax);
    L.left_padding_id = opt_uint(lv, "left_padding_id", kUsizeMax);
    L.max_size = opt_uint(lv, "max_size", kUsizeMax);
    L.keep = opt_uint(lv, "keep", kUsizeMax);
    L.idx = opt_uint(lv, "idx", kUsizeMax);
    L.bits = opt_uint(lv, "bits", UINT32_MAX);
    L.qjl_m = opt_uint(lv, "qjl_m", kUsizeMax);
    if (const JVal* g = lv.get("group_size"); g && g->kind != JVal::Null) {
      if (g->kind != JVal::Num) LC_THROW(LC_ERR_IO, "LKV2 manifest: group_size is not a number");
      L.group_size = std::stoll(g->s);  // i32 in the reference
    }
    L.v_bits = opt_uint(lv, "v_bits", UINT32_MAX);
    m.layers.push_back(std::move(L));
  }
  return m;
}

// ---- file ------------------------------------------------------------------

namespace {

struct File {
  FILE* f = nullptr;
  std::string path;
  File(const std::string& p, const char* mode) : path(p) {
    f = std::fopen(p.c_str(), mode);
    if (!f) LC_THROW(LC_ERR_IO, "cannot open " + p);
  }
  ~File() {
    if (f) std::fclose(f);
  }
  void write(const void* p, size_t n) {
    if (n && std::fwrite(p, 1, n, f) != n) LC_THROW(LC_ERR_IO, "write failed: " + path);
  }
  void read(void* p, size_t n, const char* what) {
    if (n && std::fread(p, 1, n, f) != n) LC_THROW(LC_ERR_IO, std::string("LKV2: file ends inside the ") + what);
  }
};

template <class T>
void put_le(std::vector<uint8_t>& b, T v) {
  for (size_t k = 0; k < sizeof(T); ++k) b.push_back((uint8_t)((uint64_t)v >> (8 * k)));
}

template <class T>
T get_le(const uint8_t* p) {
  uint64_t v = 0;
  for (size_t k = 0; k < sizeof(T); ++k) v |= (uint64_t)p[k] << (8 * k);
  return (T)v;
}

}  // namespace

void lkv2_write(const std::string& path, const Lkv2Manifest& m, const std::vector<Lkv2Record>& recs) {
  // checked before anything is written (validate_len, kv_disk.rs:143-155)
  for (const Lkv2Record& r : recs) {
    const int es = lkv2_elem_size(r.dtype);
    LC_REQUIRE(es > 0 && r.shape.size() <= 8, LC_ERR_INVALID, "LKV2: bad record dtype or rank");
    LC_REQUIRE((int64_t)r.data.size() == r.elems() * es, LC_ERR_INVALID, "LKV2: record length != shape x dtype");
  }
  const std::string tmp = path + ".tmp";
  {
    File f(tmp, "wb");
    std::vector<uint8_t> h;
    h.insert(h.end(), {'L', 'K', 'V', '2'});
    put_le<uint32_t>(h, 2);
    const std::string json = lkv2_manifest_json(m);
    put_le<uint32_t>(h, (uint32_t)json.size());
    f.write(h.data(), h.size());
    f.write(json.data(), json.size());
    h.clear();
    put_le<uint32_t>(h, crc32_ieee(reinterpret_cast<const uint8_t*>(json.data()), json.size()));
    put_le<uint32_t>(h, (uint32_t)recs.size());
    f.write(h.data(), h.size());
    for (const Lkv2Record& r : recs) {
      h.clear();
      h.push_back(r.dtype);
      put_le<uint32_t>(h, (uint32_t)r.shape.size());
      for (int32_t d : r.shape) put_le<int32_t>(h, d);
      put_le<uint64_t>(h, (uint64_t)r.data.size());
      uint32_t crc = crc32_ieee(h.data(), h.size());
      crc = crc32_ieee(r.data.data(), r.data.size(), crc);
      f.write(h.data(), h.size());
      f.write(r.data.data(), r.data.size());
      h.clear();
      put_le<uint32_t>(h, crc);
      f.write(h.data(), h.size());
    }
    if (std::fflush(f.f) != 0) LC_THROW(LC_ERR_IO, "write failed: " + tmp);
  }
  if (std::rename(tmp.c_str(), path.c_str()) != 0) {
    std::remove(tmp.c_str());
    LC_THROW(LC_ERR_IO, "cannot rename " + tmp + " to " + path);
  }
}

void lkv2_read(const std::string& path, Lkv2Manifest& m, std::vector<Lkv2Record>& recs) {
  File f(path, "rb");
  std::fseek(f.f, 0, SEEK_END);
  const int64_t size = (int64_t)std::ftell(f.f);
  std::fseek(f.f, 0, SEEK_SET);
  uint8_t h[4];
  f.read(h, 4, "magic");
  if (std::memcmp(h, "LKV2", 4) != 0) LC_THROW(LC_ERR_MAGIC, "LKV2: bad magic in " + path);
  f.read(h, 4, "version");
  const uint32_t ver = get_le<uint32_t>(h);
  if (ver != 2) LC_THROW(LC_ERR_MAGIC, "LKV2: unsupported version " + std::to_string(ver));
  f.read(h, 4, "manifest length");
  const uint32_t jl = get_le<uint32_t>(h);
  // the file must hold what a length field declares before it is allocated
  if ((int64_t)jl > size - (int64_t)std::ftell(f.f)) LC_THROW(LC_ERR_IO, "LKV2: manifest length exceeds the file");
  std::string json(jl, '\0');
  f.read(json.data(), jl, "manifest");
  f.read(h, 4, "manifest CRC");
  if (get_le<uint32_t>(h) != crc32_ieee(reinterpret_cast<const uint8_t*>(json.data()), json.size()))
    LC_THROW(LC_ERR_IO, "LKV2: manifest CRC mismatch (corrupt file)");
  m = lkv2_parse_manifest(json);
  f.read(h, 4, "record count");
  const uint32_t n = get_le<uint32_t>(h);
  recs.clear();
  for (uint32_t k = 0; k < n; ++k) {
    Lkv2Record r;
    std::vector<uint8_t> hdr(5);
    f.read(hdr.data(), 5, "record header");
    r.dtype = hdr[0];
    const int es = lkv2_elem_size(r.dtype);
    if (es < 0) LC_THROW(LC_ERR_IO, "LKV2: unknown dtype tag " + std::to_string(r.dtype));
    const uint32_t ndim = get_le<uint32_t>(hdr.data() + 1);
    if (ndim > 8) LC_THROW(LC_ERR_IO, "LKV2: implausible ndim " + std::to_string(ndim));
    hdr.resize(5 + 4 * ndim + 8);
    f.read(hdr.data() + 5, 4 * ndim + 8, "record header");
    uint64_t expect = ndim ? 1 : 0;
    bool overflow = false;
    for (uint32_t d = 0; d < ndim; ++d) {
      const int32_t v = get_le<int32_t>(hdr.data() + 5 + 4 * d);
      if (v < 0) LC_THROW(LC_ERR_IO, "LKV2: negative dimension");
      r.shape.push_back(v);
      if (v && expect > UINT64_MAX / (uint64_t)v) overflow = true;
      expect *= (uint64_t)v;
    }
    if (!overflow && expect > UINT64_MAX / (uint64_t)es) overflow = true;
    expect *= (uint64_t)es;
    const uint64_t len = get_le<uint64_t>(hdr.data() + 5 + 4 * ndim);
    // kv_disk.rs:199-247: the stored length must be the one shape x dtype implies
    if (overflow || len != expect)
      LC_THROW(LC_ERR_IO, "LKV2: record payload length disagrees with its shape and dtype (corrupt record)");
    if ((int64_t)len > size - (int64_t)std::ftell(f.f)) LC_THROW(LC_ERR_IO, "LKV2: record payload exceeds the file");
    r.data.resize(len);
    f.read(r.data.data(), len, "record payload");
    uint32_t crc = crc32_ieee(hdr.data(), hdr.size());
    crc = crc32_ieee(r.data.data(), r.data.size(), crc);
    f.read(h, 4, "record CRC");
    if (get_le<uint32_t>(h) != crc) LC_THROW(LC_ERR_IO, "LKV2: record CRC mismatch (corrupt file)");
    recs.push_back(std::move(r));
  }
  uint8_t extra;
  if (std::fread(&extra, 1, 1, f.f) != 0)
    LC_THROW(LC_ERR_IO, "LKV2: trailing bytes after " + std::to_string(n) + " records (corrupt record count)");
}

}  // namespace lc
