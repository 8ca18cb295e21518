// .ponni weight files: the PONNI profile of Safetensors.
//
// Byte-compatible with the reference reader/writer
// (src/utils/ponni_safetensors.h:175-407, strict JSON src/utils/ponni_json.h):
//   [u64 little-endian header length][JSON header, space-padded to 8 bytes][payload]
// Header: "__metadata__" with ponni.profile_version "1", ponni.model_fingerprint,
// ponni.schema_fingerprint (FNV-1a-64 of "ponni-tensor-schema-v1\n" + one
// "name\tdtype\tdims\n" line per tensor, name-sorted), ponni.payload_checksum_fnv1a64
// (FNV-1a-64 of the payload), ponni.source_framework, ponni.target; then one
// descriptor {dtype, shape, data_offsets} per tensor.  A template model stores
// one tensor "parameters" (F32, or F64 for double models).
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "model.h"

namespace ponni_b200 {
namespace {

uint64_t fnv1a64(const unsigned char* p, size_t n) {
  uint64_t h = UINT64_C(14695981039346656037);
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= UINT64_C(1099511628211);
  }
  return h;
}

std::string fnv_string(uint64_t h) {
  char b[32];
  snprintf(b, sizeof b, "fnv1a64:%016llx", (unsigned long long)h);
  return b;
}

// ----------------------------------------------------------------- JSON ---
// Complete JSON value grammar; duplicate object keys and nesting deeper than
// 64 are errors, as in the reference parser.
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  std::string text;  // string value, or the number's literal text
  std::vector<Json> array;
  std::map<std::string, Json> object;
};

class JsonReader {
 public:
  JsonReader(const char* b, size_t n) : p_(b), end_(b + n) {}
  bool parse(Json& out, std::string& err) {
    ws();
    if (!value(out, 0)) {
      err = err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      err = "trailing characters after JSON value";
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* end_;
  std::string err_;
  bool fail(const std::string& m) {
    if (err_.empty()) err_ = m;
    return false;
  }
  void ws() {
    while (p_ != end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* s) {
    for (; *s; ++s, ++p_)
      if (p_ == end_ || *p_ != *s) return fail("invalid literal");
    return true;
  }
  static int hex(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
  }
  bool u4(unsigned& cp) {
    if (end_ - p_ < 4) return fail("incomplete Unicode escape");
    cp = 0;
    for (int i = 0; i < 4; ++i) {
      int d = hex(p_[i]);
      if (d < 0) return fail("invalid Unicode escape");
      cp = cp * 16 + (unsigned)d;
    }
    p_ += 4;
    return true;
  }
  static void utf8(std::string& o, unsigned cp) {
    if (cp <= 0x7f) {
      o.push_back((char)cp);
    } else if (cp <= 0x7ff) {
      o.push_back((char)(0xc0 | (cp >> 6)));
      o.push_back((char)(0x80 | (cp & 0x3f)));
    } else if (cp <= 0xffff) {
      o.push_back((char)(0xe0 | (cp >> 12)));
      o.push_back((char)(0x80 | ((cp >> 6) & 0x3f)));
      o.push_back((char)(0x80 | (cp & 0x3f)));
    } else {
      o.push_back((char)(0xf0 | (cp >> 18)));
      o.push_back((char)(0x80 | ((cp >> 12) & 0x3f)));
      o.push_back((char)(0x80 | ((cp >> 6) & 0x3f)));
      o.push_back((char)(0x80 | (cp & 0x3f)));
    }
  }
  bool str(std::string& o) {
    if (p_ == end_ || *p_ != '"') return fail("expected string");
    ++p_;
    while (p_ != end_) {
      unsigned char c = (unsigned char)*p_++;
      if (c == '"') return true;
      if (c < 0x20) return fail("unescaped control character in string");
      if (c != '\\') {
        o.push_back((char)c);
        continue;
      }
      if (p_ == end_) return fail("incomplete string escape");
      char e = *p_++;
      switch (e) {
        case '"': o.push_back('"'); break;
        case '\\': o.push_back('\\'); break;
        case '/': o.push_back('/'); break;
        case 'b': o.push_back('\b'); break;
        case 'f': o.push_back('\f'); break;
        case 'n': o.push_back('\n'); break;
        case 'r': o.push_back('\r'); break;
        case 't': o.push_back('\t'); break;
        case 'u': {
          unsigned cp;
          if (!u4(cp)) return false;
          if (cp >= 0xd800 && cp <= 0xdbff) {
            if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') return fail("missing low Unicode surrogate");
            p_ += 2;
            unsigned lo;
            if (!u4(lo)) return false;
            if (lo < 0xdc00 || lo > 0xdfff) return fail("invalid low Unicode surrogate");
            cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00);
          } else if (cp >= 0xdc00 && cp <= 0xdfff) {
            return fail("unpaired low Unicode surrogate");
          }
          utf8(o, cp);
          break;
        }
        default: return fail("invalid string escape");
      }
    }
    return fail("unterminated string");
  }
  bool digits() {
    if (p_ == end_ || *p_ < '0' || *p_ > '9') return false;
    while (p_ != end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    return true;
  }
  bool number(Json& v) {
    const char* b = p_;
    if (*p_ == '-') ++p_;
    if (p_ == end_) return fail("incomplete number");
    if (*p_ == '0') ++p_;
    else if (!digits()) return fail("invalid number");
    if (p_ != end_ && *p_ == '.') {
      ++p_;
      if (!digits()) return fail("invalid fractional number");
    }
    if (p_ != end_ && (*p_ == 'e' || *p_ == 'E')) {
      ++p_;
      if (p_ != end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (!digits()) return fail("invalid exponent");
    }
    v.kind = Json::Number;
    v.text.assign(b, p_);
    return true;
  }
  bool value(Json& v, int depth) {
    if (depth >= 64) return fail("JSON nesting limit exceeded");
    if (p_ == end_) return fail("expected JSON value");
    char c = *p_;
    if (c == '{') {
      v.kind = Json::Object;
      ++p_;
      ws();
      if (p_ != end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      while (p_ != end_) {
        std::string key;
        ws();
        if (!str(key)) return false;
        ws();
        if (p_ == end_ || *p_ != ':') return fail("expected ':'");
        ++p_;
        ws();
        Json child;
        if (!value(child, depth + 1)) return false;
        if (!v.object.emplace(key, std::move(child)).second) return fail("duplicate object key " + key);
        ws();
        if (p_ != end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        if (p_ == end_ || *p_ != ',') return fail("expected ','");
        ++p_;
      }
      return fail("unterminated object");
    }
    if (c == '[') {
      v.kind = Json::Array;
      ++p_;
      ws();
      if (p_ != end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      while (p_ != end_) {
        ws();
        Json child;
        if (!value(child, depth + 1)) return false;
        v.array.push_back(std::move(child));
        ws();
        if (p_ != end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        if (p_ == end_ || *p_ != ',') return fail("expected ','");
        ++p_;
      }
      return fail("unterminated array");
    }
    if (c == '"') {
      v.kind = Json::String;
      return str(v.text);
    }
    if (c == 't') { v.kind = Json::Bool; v.text = "true"; return lit("true"); }
    if (c == 'f') { v.kind = Json::Bool; v.text = "false"; return lit("false"); }
    if (c == 'n') { v.kind = Json::Null; return lit("null"); }
    if (c == '-' || (c >= '0' && c <= '9')) return number(v);
    return fail("unexpected character in JSON");
  }
};

// ------------------------------------------------------------ PONNI file ---
struct Descriptor {
  std::string name, dtype;
  std::vector<size_t> shape;
  size_t begin = 0, end = 0;
};

bool parse_size(const Json& v, size_t& out) {
  if (v.kind != Json::Number || v.text.empty()) return false;
  size_t r = 0;
  for (char c : v.text) {
    if (c < '0' || c > '9') return false;
    size_t d = (size_t)(c - '0');
    if (r > (SIZE_MAX - d) / 10) return false;
    r = r * 10 + d;
  }
  out = r;
  return true;
}

size_t dtype_size(const std::string& t) {
  if (t == "BOOL" || t == "I8" || t == "U8") return 1;
  if (t == "F16" || t == "BF16" || t == "I16" || t == "U16") return 2;
  if (t == "F32" || t == "I32" || t == "U32") return 4;
  if (t == "F64" || t == "I64" || t == "U64") return 8;
  return 0;
}

bool elements_of(const std::vector<size_t>& shape, size_t& n) {
  n = 1;
  for (size_t d : shape) {
    if (d != 0 && n > SIZE_MAX / d) return false;
    n *= d;
  }
  return true;
}

std::string schema_fingerprint(std::vector<Descriptor> ds) {
  std::sort(ds.begin(), ds.end(), [](const Descriptor& a, const Descriptor& b) { return a.name < b.name; });
  std::ostringstream s;
  s << "ponni-tensor-schema-v1\n";
  for (const auto& d : ds) {
    s << d.name << '\t' << d.dtype << '\t';
    for (size_t i = 0; i < d.shape.size(); ++i) s << (i ? "," : "") << d.shape[i];
    s << '\n';
  }
  const std::string t = s.str();
  return fnv_string(fnv1a64(reinterpret_cast<const unsigned char*>(t.data()), t.size()));
}

std::string json_escape(const std::string& v) {
  std::string o = "\"";
  for (unsigned char c : v) {
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
          char b[8];
          snprintf(b, sizeof b, "\\u%04x", c);
          o += b;
        } else {
          o.push_back((char)c);
        }
    }
  }
  return o + "\"";
}

// Structural checks of PonniFile::load (src/utils/ponni_safetensors.h:187-309).
struct PonniFile {
  std::vector<unsigned char> bytes;
  size_t data_offset = 0;
  std::map<std::string, std::string> metadata;
  std::map<std::string, Descriptor> tensors;

  bool load(const std::string& path, std::string& err) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) { err = "cannot open PONNI file: " + path; return false; }
    std::streamsize size = f.tellg();
    if (size < 0) { err = "cannot determine PONNI file size: " + path; return false; }
    f.seekg(0);
    bytes.resize((size_t)size);
    if (size > 0 && !f.read(reinterpret_cast<char*>(bytes.data()), size)) {
      err = "cannot read PONNI file: " + path;
      return false;
    }
    if (bytes.size() < 10) { err = "PONNI file is shorter than a Safetensors header"; return false; }
    uint64_t hs = 0;
    for (int i = 0; i < 8; ++i) hs |= (uint64_t)bytes[i] << (8 * i);
    if (hs < 2 || hs > 100u * 1024 * 1024 || hs > bytes.size() - 8) {
      err = "PONNI file has an invalid Safetensors header size";
      return false;
    }
    data_offset = 8 + (size_t)hs;
    Json root;
    std::string perr;
    JsonReader reader(reinterpret_cast<const char*>(bytes.data() + 8), (size_t)hs);
    if (!reader.parse(root, perr)) { err = "invalid Safetensors JSON: " + perr; return false; }
    if (root.kind != Json::Object) { err = "Safetensors header root must be an object"; return false; }
    for (const auto& kv : root.object) {
      const std::string& name = kv.first;
      const Json& v = kv.second;
      if (name == "__metadata__") {
        if (v.kind != Json::Object) { err = "Safetensors metadata must be an object"; return false; }
        for (const auto& m : v.object) {
          if (m.second.kind != Json::String) { err = "Safetensors metadata values must be strings"; return false; }
          metadata.emplace(m.first, m.second.text);
        }
        continue;
      }
      if (v.kind != Json::Object) {
        err = "Safetensors tensor descriptor for " + name + " must be an object";
        return false;
      }
      auto it_d = v.object.find("dtype"), it_s = v.object.find("shape"), it_o = v.object.find("data_offsets");
      if (it_d == v.object.end() || it_s == v.object.end() || it_o == v.object.end() ||
          it_d->second.kind != Json::String || it_s->second.kind != Json::Array ||
          it_o->second.kind != Json::Array || it_o->second.array.size() != 2) {
        err = "incomplete Safetensors descriptor for " + name;
        return false;
      }
      Descriptor d;
      d.name = name;
      d.dtype = it_d->second.text;
      for (const auto& dim : it_s->second.array) {
        size_t x;
        if (!parse_size(dim, x)) { err = "invalid Safetensors shape for " + name; return false; }
        d.shape.push_back(x);
      }
      if (!parse_size(it_o->second.array[0], d.begin) || !parse_size(it_o->second.array[1], d.end)) {
        err = "invalid Safetensors offsets for " + name;
        return false;
      }
      size_t sb = dtype_size(d.dtype), n = 0;
      if (sb == 0 || !elements_of(d.shape, n) || n > SIZE_MAX / sb || d.begin > d.end ||
          d.end > bytes.size() - data_offset || d.end - d.begin != n * sb) {
        err = "Safetensors dtype, shape, and byte length disagree for " + name;
        return false;
      }
      tensors.emplace(name, d);
    }
    if (metadata.empty()) { err = "PONNI file has no Safetensors metadata"; return false; }
    const char* keys[] = {"ponni.profile_version", "ponni.model_fingerprint", "ponni.schema_fingerprint",
                          "ponni.payload_checksum_fnv1a64"};
    for (const char* k : keys)
      if (!metadata.count(k)) { err = "PONNI Safetensors metadata is incomplete"; return false; }
    if (metadata["ponni.profile_version"] != "1") {
      err = "unsupported PONNI profile version " + metadata["ponni.profile_version"];
      return false;
    }
    std::vector<Descriptor> phys;
    for (const auto& kv : tensors) phys.push_back(kv.second);
    std::sort(phys.begin(), phys.end(), [](const Descriptor& a, const Descriptor& b) {
      return a.begin != b.begin ? a.begin < b.begin : a.end < b.end;
    });
    size_t cursor = 0;
    for (const auto& d : phys) {
      if (d.begin != cursor) { err = "Safetensors payload has a hole or overlap before " + d.name; return false; }
      cursor = d.end;
    }
    if (cursor != bytes.size() - data_offset) {
      err = "Safetensors payload contains unindexed trailing bytes";
      return false;
    }
    if (metadata["ponni.schema_fingerprint"] != schema_fingerprint(phys)) {
      err = "PONNI tensor-schema fingerprint does not match the Safetensors descriptors";
      return false;
    }
    const std::string sum = fnv_string(fnv1a64(bytes.data() + data_offset, bytes.size() - data_offset));
    if (metadata["ponni.payload_checksum_fnv1a64"] != sum) { err = "PONNI payload checksum mismatch"; return false; }
    return true;
  }
};

}  // namespace
}  // namespace ponni_b200

using namespace ponni_b200;

extern "C" {

// Reference Inference::save_weights (src/ponni_Inference.h:320-333) with
// write_ponni_file (src/utils/ponni_safetensors.h:351-407), target "template".
ponni_b200_status ponni_b200_model_save_weights(ponni_b200_model* m, const char* path) {
  if (!m || !path) return PONNI_B200_ERR_INVALID_ARGUMENT;
  const int64_t n = ponni_b200_num_trainable_parameters(m);
  if (n == 0) return pb_fail(m, PONNI_B200_ERR_IO, "cannot save weights from a model with no trainable parameters");
  const size_t esz = dtype_bytes(m->dtype);
  std::vector<unsigned char> host((size_t)n * esz);
  ponni_b200_get_trainable_parameters(m, host.data(), n);
  const bool f64 = m->dtype == PONNI_B200_F64;
  std::vector<unsigned char> payload;
  payload.reserve((size_t)n * (f64 ? 8 : 4));
  for (int64_t i = 0; i < n; ++i) {
    double v = load_scalar(m->dtype, host.data() + (size_t)i * esz);
    unsigned char b[8];
    if (f64) {
      memcpy(b, &v, 8);
    } else {
      float f = (float)v;
      memcpy(b, &f, 4);
    }
    payload.insert(payload.end(), b, b + (f64 ? 8 : 4));
  }
  Descriptor d{"parameters", f64 ? "F64" : "F32", {(size_t)n}, 0, payload.size()};
  const std::string checksum = fnv_string(fnv1a64(payload.data(), payload.size()));
  const std::string schema = schema_fingerprint({d});
  std::ostringstream h;
  h << "{\"__metadata__\":{\"ponni.profile_version\":\"1\","
    << "\"ponni.model_fingerprint\":" << json_escape(pb_schema_fingerprint(m)) << ','
    << "\"ponni.schema_fingerprint\":" << json_escape(schema) << ','
    << "\"ponni.payload_checksum_fnv1a64\":" << json_escape(checksum) << ','
    << "\"ponni.source_framework\":\"ponni-cpp\","
    << "\"ponni.target\":" << json_escape("template") << '}';
  h << ',' << json_escape(d.name) << ":{\"dtype\":" << json_escape(d.dtype) << ",\"shape\":[" << n
    << "],\"data_offsets\":[0," << payload.size() << "]}}";
  std::string header = h.str();
  header.append((8 - header.size() % 8) % 8, ' ');
  std::vector<unsigned char> bytes;
  for (int i = 0; i < 8; ++i) bytes.push_back((unsigned char)(((uint64_t)header.size() >> (8 * i)) & 0xff));
  bytes.insert(bytes.end(), header.begin(), header.end());
  bytes.insert(bytes.end(), payload.begin(), payload.end());
  std::ofstream f(path, std::ios::binary | std::ios::trunc);
  if (!f) return pb_fail(m, PONNI_B200_ERR_IO, std::string("cannot open PONNI output file: ") + path);
  f.write(reinterpret_cast<const char*>(bytes.data()), (std::streamsize)bytes.size());
  if (!f) return pb_fail(m, PONNI_B200_ERR_IO, std::string("cannot write PONNI output file: ") + path);
  return PONNI_B200_OK;
}

// Reference Inference::load_weights (src/ponni_Inference.h:295-316) with
// PonniFile::validate (src/utils/ponni_safetensors.h:327-347).
ponni_b200_status ponni_b200_model_load_weights(ponni_b200_model* m, const char* path) {
  if (!m || !path) return PONNI_B200_ERR_INVALID_ARGUMENT;
  const int64_t n = ponni_b200_num_trainable_parameters(m);
  if (n == 0) return pb_fail(m, PONNI_B200_ERR_IO, "cannot load weights into a model with no trainable parameters");
  PonniFile file;
  std::string err;
  if (!file.load(path, err)) return pb_fail(m, PONNI_B200_ERR_IO, err);
  const bool f64 = m->dtype == PONNI_B200_F64;
  auto mf = file.metadata.find("ponni.model_fingerprint");
  if (mf == file.metadata.end() || mf->second != pb_schema_fingerprint(m))
    return pb_fail(m, PONNI_B200_ERR_MISMATCH, "PONNI model fingerprint does not match this model");
  if (file.tensors.size() != 1)
    return pb_fail(m, PONNI_B200_ERR_MISMATCH, "PONNI tensor count does not match this model");
  auto it = file.tensors.find("parameters");
  if (it == file.tensors.end())
    return pb_fail(m, PONNI_B200_ERR_MISMATCH, "PONNI file is missing tensor parameters");
  if (it->second.dtype != (f64 ? "F64" : "F32"))
    return pb_fail(m, PONNI_B200_ERR_MISMATCH, "PONNI tensor dtype mismatch for parameters");
  if (it->second.shape != std::vector<size_t>{(size_t)n})
    return pb_fail(m, PONNI_B200_ERR_MISMATCH, "PONNI tensor shape mismatch for parameters");
  const unsigned char* src = file.bytes.data() + file.data_offset + it->second.begin;
  const size_t esz = dtype_bytes(m->dtype);
  std::vector<unsigned char> host((size_t)n * esz);
  for (int64_t i = 0; i < n; ++i) {
    double v;
    if (f64) {
      memcpy(&v, src + 8 * i, 8);
    } else {
      float fv;
      memcpy(&fv, src + 4 * i, 4);
      v = fv;
    }
    store_scalar(m->dtype, host.data() + (size_t)i * esz, v);
  }
  return ponni_b200_set_trainable_parameters(m, host.data(), n);
}

// Reference load_ponni_tensor<N> (src/utils/ponni_safetensors.h:409-444).
ponni_b200_status ponni_b200_read_ponni_tensor(const char* path, const char* name, float* out, size_t capacity,
                                               int64_t* shape, int* rank, char* err, size_t err_len) {
  auto fail = [&](ponni_b200_status s, const std::string& msg) {
    if (err && err_len) {
      size_t n = std::min(err_len - 1, msg.size());
      memcpy(err, msg.data(), n);
      err[n] = 0;
    }
    return s;
  };
  if (!path || !name || !shape || !rank) return fail(PONNI_B200_ERR_INVALID_ARGUMENT, "NULL argument");
  PonniFile file;
  std::string e;
  if (!file.load(path, e)) return fail(PONNI_B200_ERR_IO, e);
  auto it = file.tensors.find(name);
  if (it == file.tensors.end())
    return fail(PONNI_B200_ERR_MISMATCH, std::string("PONNI file is missing tensor ") + name);
  const Descriptor& d = it->second;
  if (d.shape.empty() || d.shape.size() > 4)
    return fail(PONNI_B200_ERR_MISMATCH, std::string("PONNI tensor rank mismatch for ") + name);
  if (d.dtype != "F32" && d.dtype != "F64")
    return fail(PONNI_B200_ERR_MISMATCH, std::string("PONNI tensor must use F32 or F64: ") + name);
  *rank = (int)d.shape.size();
  size_t n = 1;
  for (size_t i = 0; i < d.shape.size(); ++i) {
    shape[i] = (int64_t)d.shape[i];
    n *= d.shape[i];
  }
  if (!out) return PONNI_B200_OK;
  if (capacity < n) return fail(PONNI_B200_ERR_INVALID_ARGUMENT, "output capacity too small");
  const unsigned char* src = file.bytes.data() + file.data_offset + d.begin;
  for (size_t i = 0; i < n; ++i) {
    if (d.dtype == "F32") {
      memcpy(&out[i], src + 4 * i, 4);
    } else {
      double v;
      memcpy(&v, src + 8 * i, 8);
      out[i] = (float)v;
    }
  }
  return PONNI_B200_OK;
}

}  // extern "C"
