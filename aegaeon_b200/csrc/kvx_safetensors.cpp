// Safetensors header reader (host only): the metadata step before weights are
// cached and uploaded during a model switch.
//
// Replaces the reference's Rust extension `read_safetensors_meta_as_json`
// (quick_model_loader/rsrc/lib.rs:19-51), which maps the file and calls the
// `safetensors` crate (0.4.3, Cargo.toml) `SafeTensors::read_metadata`.  The
// published format and the crate's checks are restated here:
//   * bytes [0, 8): n = header length, little-endian u64; file >= 8 bytes,
//     n <= 100,000,000, 8 + n <= file size;
//   * bytes [8, 8 + n): UTF-8 JSON object; key "__metadata__" (optional) is a
//     string -> string map; every other key is a tensor
//     {"dtype": D, "shape": [u64...], "data_offsets": [begin, end]};
//   * tensors sorted by data_offsets must tile [0, end) without gaps, each
//     (end - begin) == prod(shape) * size(dtype), and 8 + n + end == file size.
// The result is the JSON the reference returns: file_path, size (file bytes),
// offset (8 + n) and tensor_info_map (name -> dtype, shape, data_offsets).
#include <sys/stat.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/kvx.h"

namespace kvx {
void record_error(const std::string& msg);  // kvx_runtime.cu

namespace {

constexpr uint64_t kMaxHeader = 100000000ull;

struct Json {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  bool b = false;
  bool is_uint = false;  // a non-negative integer literal
  uint64_t u = 0;
  std::string s;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;  // in order; duplicates kept
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), end_(p + n) {}
  bool parse(Json* out) {
    ws();
    if (!value(out, 0)) return false;
    ws();
    return p_ == end_;
  }

 private:
  const char* p_;
  const char* end_;

  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if (size_t(end_ - p_) < n || std::memcmp(p_, w, n)) return false;
    p_ += n;
    return true;
  }
  static void put_utf8(std::string* s, uint32_t c) {
    if (c < 0x80) {
      s->push_back(char(c));
    } else if (c < 0x800) {
      s->push_back(char(0xC0 | (c >> 6)));
      s->push_back(char(0x80 | (c & 0x3F)));
    } else if (c < 0x10000) {
      s->push_back(char(0xE0 | (c >> 12)));
      s->push_back(char(0x80 | ((c >> 6) & 0x3F)));
      s->push_back(char(0x80 | (c & 0x3F)));
    } else {
      s->push_back(char(0xF0 | (c >> 18)));
      s->push_back(char(0x80 | ((c >> 12) & 0x3F)));
      s->push_back(char(0x80 | ((c >> 6) & 0x3F)));
      s->push_back(char(0x80 | (c & 0x3F)));
    }
  }
  bool hex4(uint32_t* v) {
    if (end_ - p_ < 4) return false;
    uint32_t x = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      x <<= 4;
      if (c >= '0' && c <= '9') x |= uint32_t(c - '0');
      else if (c >= 'a' && c <= 'f') x |= uint32_t(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') x |= uint32_t(c - 'A' + 10);
      else return false;
    }
    *v = x;
    return true;
  }
  bool string(std::string* s) {
    if (p_ >= end_ || *p_ != '"') return false;
    ++p_;
    while (p_ < end_) {
      const unsigned char c = static_cast<unsigned char>(*p_++);
      if (c == '"') return true;
      if (c < 0x20) return false;
      if (c != '\\') {
        s->push_back(char(c));
        continue;
      }
      if (p_ >= end_) return false;
      const char e = *p_++;
      switch (e) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t c1;
          if (!hex4(&c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00) {  // surrogate pair
            uint32_t c2;
            if (!lit("\\u") || !hex4(&c2) || c2 < 0xDC00 || c2 >= 0xE000) return false;
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          } else if (c1 >= 0xDC00 && c1 < 0xE000) {
            return false;
          }
          put_utf8(s, c1);
          break;
        }
        default:
          return false;
      }
    }
    return false;
  }
  bool number(Json* out) {
    const char* b = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
    if (*p_ == '0') {
      ++p_;
    } else {
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    bool integer = true;
    if (p_ < end_ && *p_ == '.') {
      integer = false;
      ++p_;
      if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      integer = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    out->kind = Json::kNum;
    if (integer && *b != '-') {
      uint64_t v = 0;
      bool ok = true;
      for (const char* q = b; q < p_; ++q) {
        const uint64_t d = uint64_t(*q - '0');
        if (v > (~0ull - d) / 10) { ok = false; break; }
        v = v * 10 + d;
      }
      out->is_uint = ok;
      out->u = v;
    }
    return true;
  }
  bool value(Json* out, int depth) {
    if (depth > 64 || p_ >= end_) return false;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      out->kind = Json::kObj;
      ws();
      if (p_ < end_ && *p_ == '}') { ++p_; return true; }
      for (;;) {
        ws();
        std::string key;
        if (!string(&key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return false;
        ++p_;
        ws();
        Json v;
        if (!value(&v, depth + 1)) return false;
        out->obj.emplace_back(std::move(key), std::move(v));
        ws();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == '}') { ++p_; return true; }
        return false;
      }
    }
    if (c == '[') {
      ++p_;
      out->kind = Json::kArr;
      ws();
      if (p_ < end_ && *p_ == ']') { ++p_; return true; }
      for (;;) {
        ws();
        Json v;
        if (!value(&v, depth + 1)) return false;
        out->arr.push_back(std::move(v));
        ws();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == ']') { ++p_; return true; }
        return false;
      }
    }
    if (c == '"') {
      out->kind = Json::kStr;
      return string(&out->s);
    }
    if (lit("true")) { out->kind = Json::kBool; out->b = true; return true; }
    if (lit("false")) { out->kind = Json::kBool; out->b = false; return true; }
    if (lit("null")) { out->kind = Json::kNull; return true; }
    return number(out);
  }
};

bool valid_utf8(const unsigned char* s, size_t n) {
  size_t i = 0;
  while (i < n) {
    const unsigned char c = s[i];
    size_t k;
    uint32_t cp;
    if (c < 0x80) { ++i; continue; }
    if ((c & 0xE0) == 0xC0) { k = 1; cp = c & 0x1F; }
    else if ((c & 0xF0) == 0xE0) { k = 2; cp = c & 0x0F; }
    else if ((c & 0xF8) == 0xF0) { k = 3; cp = c & 0x07; }
    else return false;
    if (i + k >= n) return false;  // continuation bytes past the end
    for (size_t j = 1; j <= k; ++j) {
      if ((s[i + j] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (s[i + j] & 0x3F);
    }
    if ((k == 1 && cp < 0x80) || (k == 2 && cp < 0x800) || (k == 3 && cp < 0x10000) ||
        cp > 0x10FFFF || (cp >= 0xD800 && cp < 0xE000))
      return false;
    i += k + 1;
  }
  return true;
}

int dtype_size(const std::string& d) {
  static const std::map<std::string, int> sizes = {
      {"BOOL", 1}, {"U8", 1},  {"I8", 1},  {"F8_E5M2", 1}, {"F8_E4M3", 1},
      {"I16", 2},  {"U16", 2}, {"F16", 2}, {"BF16", 2},    {"I32", 4},
      {"U32", 4},  {"F32", 4}, {"F64", 8}, {"I64", 8},     {"U64", 8}};
  auto it = sizes.find(d);
  return it == sizes.end() ? 0 : it->second;
}

struct Tensor {
  std::string name, dtype;
  std::vector<uint64_t> shape;
  uint64_t begin = 0, end = 0;
};

void json_escape(const std::string& s, std::string* out) {
  out->push_back('"');
  for (unsigned char c : s) {
    switch (c) {
      case '"': *out += "\\\""; break;
      case '\\': *out += "\\\\"; break;
      case '\n': *out += "\\n"; break;
      case '\r': *out += "\\r"; break;
      case '\t': *out += "\\t"; break;
      case '\b': *out += "\\b"; break;
      case '\f': *out += "\\f"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", c);
          *out += buf;
        } else {
          out->push_back(char(c));
        }
    }
  }
  out->push_back('"');
}

constexpr int kIo = KVX_ERR_IO, kFormat = KVX_ERR_FORMAT;

int fmt_error(const std::string& why) {
  record_error("Fail to read the metadata from the given buffer: " + why);
  return kFormat;
}

int read_meta(const char* path, std::string* json) {
  FILE* f = std::fopen(path, "rb");
  if (!f) {
    record_error(std::string("cannot open ") + path + ": " + std::strerror(errno));
    return kIo;
  }
  struct stat stt;
  if (fstat(fileno(f), &stt) != 0) {
    std::fclose(f);
    record_error(std::string("cannot stat ") + path);
    return kIo;
  }
  const uint64_t size = uint64_t(stt.st_size);
  std::string header;
  uint64_t n = 0;
  int rc = 0;
  do {
    if (size < 8) { rc = fmt_error("header too small"); break; }
    unsigned char lenb[8];
    if (std::fread(lenb, 1, 8, f) != 8) { rc = fmt_error("short read"); break; }
    for (int i = 7; i >= 0; --i) n = (n << 8) | lenb[i];
    if (n > kMaxHeader) { rc = fmt_error("header too large"); break; }
    if (8 + n > size) { rc = fmt_error("invalid header length"); break; }
    header.resize(size_t(n));
    if (n && std::fread(&header[0], 1, size_t(n), f) != size_t(n)) { rc = fmt_error("short read"); break; }
  } while (false);
  std::fclose(f);
  if (rc) return rc;
  if (!valid_utf8(reinterpret_cast<const unsigned char*>(header.data()), header.size()))
    return fmt_error("header is not UTF-8");
  Json root;
  if (!Parser(header.data(), header.size()).parse(&root) || root.kind != Json::kObj)
    return fmt_error("header is not a JSON object");
  // Later duplicates replace earlier ones, as when deserializing into a map.
  std::map<std::string, const Json*> fields;
  for (const auto& kv : root.obj) fields[kv.first] = &kv.second;
  std::vector<Tensor> tensors;
  for (const auto& kv : fields) {
    const Json& v = *kv.second;
    if (kv.first == "__metadata__") {
      if (v.kind == Json::kNull) continue;
      if (v.kind != Json::kObj) return fmt_error("__metadata__ is not a map");
      for (const auto& m : v.obj)
        if (m.second.kind != Json::kStr) return fmt_error("__metadata__ values must be strings");
      continue;
    }
    if (v.kind != Json::kObj) return fmt_error("tensor entry is not an object");
    const Json *dt = nullptr, *sh = nullptr, *off = nullptr;
    for (const auto& m : v.obj) {
      if (m.first == "dtype") dt = &m.second;
      else if (m.first == "shape") sh = &m.second;
      else if (m.first == "data_offsets") off = &m.second;
    }
    if (!dt || !sh || !off) return fmt_error("tensor entry misses dtype, shape or data_offsets");
    if (dt->kind != Json::kStr || !dtype_size(dt->s)) return fmt_error("unknown dtype");
    if (sh->kind != Json::kArr) return fmt_error("shape is not an array");
    if (off->kind != Json::kArr || off->arr.size() != 2) return fmt_error("bad data_offsets");
    Tensor t;
    t.name = kv.first;
    t.dtype = dt->s;
    for (const Json& d : sh->arr) {
      if (d.kind != Json::kNum || !d.is_uint) return fmt_error("bad shape entry");
      t.shape.push_back(d.u);
    }
    for (int i = 0; i < 2; ++i)
      if (off->arr[i].kind != Json::kNum || !off->arr[i].is_uint) return fmt_error("bad data_offsets");
    t.begin = off->arr[0].u;
    t.end = off->arr[1].u;
    tensors.push_back(std::move(t));
  }
  // validate(): contiguous tiling from 0, sizes consistent with shape x dtype.
  std::vector<const Tensor*> order;
  for (const Tensor& t : tensors) order.push_back(&t);
  std::stable_sort(order.begin(), order.end(), [](const Tensor* a, const Tensor* b) {
    return a->begin != b->begin ? a->begin < b->begin : a->end < b->end;
  });
  uint64_t start = 0;
  for (const Tensor* t : order) {
    if (t->begin != start || t->end < t->begin) return fmt_error("invalid offset for " + t->name);
    start = t->end;
    unsigned __int128 nel = 1;
    for (uint64_t d : t->shape) {
      nel *= d;
      if (nel >> 64) return fmt_error("validation overflow");
    }
    const unsigned __int128 nbytes = nel * unsigned(dtype_size(t->dtype));
    if (nbytes >> 64) return fmt_error("validation overflow");
    if (uint64_t(nbytes) != t->end - t->begin) return fmt_error("tensor info invalid: " + t->name);
  }
  if (start + 8 + n != size) return fmt_error("metadata incomplete buffer");
  // Pretty JSON (2-space indent), tensors in file order.
  std::string& o = *json;
  o = "{\n  \"file_path\": ";
  json_escape(path, &o);
  o += ",\n  \"size\": " + std::to_string(size);
  o += ",\n  \"offset\": " + std::to_string(8 + n);
  o += ",\n  \"tensor_info_map\": {";
  bool first = true;
  for (const Tensor* t : order) {
    o += first ? "\n    " : ",\n    ";
    first = false;
    json_escape(t->name, &o);
    o += ": {\n      \"dtype\": ";
    json_escape(t->dtype, &o);
    o += ",\n      \"shape\": [";
    for (size_t i = 0; i < t->shape.size(); ++i)
      o += (i ? ", " : "") + std::to_string(t->shape[i]);
    o += "],\n      \"data_offsets\": [" + std::to_string(t->begin) + ", " +
         std::to_string(t->end) + "]\n    }";
  }
  o += first ? "}\n}" : "\n  }\n}";
  return 0;
}

}  // namespace
}  // namespace kvx

extern "C" int kvx_safetensors_meta_json(const char* file_path, char* out, uint64_t capacity,
                                         uint64_t* length_out) {
  kvx::record_error("");
  if (!file_path || !length_out) {
    kvx::record_error("null argument");
    return KVX_ERR_INVALID_ARGUMENT;
  }
  std::string json;
  const int rc = kvx::read_meta(file_path, &json);
  if (rc) return rc;
  *length_out = json.size();
  if (out && capacity > json.size()) std::memcpy(out, json.c_str(), json.size() + 1);
  return KVX_OK;
}
