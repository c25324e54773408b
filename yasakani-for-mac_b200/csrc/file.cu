// Loader of `.yskn` containers: open, validate, enumerate, and create matrix handles
// straight from a file (host code only; the kernels are untouched).
//
// Replaces the reference's readers: src/format.hpp:26-61 (Container::open) with
// src/loader.cpp:19-60 (Model::upload_linear) on the CUDA side, and
// crates/yskn-format/src/lib.rs:97-172 (Container::new) with
// crates/yskn-format/src/tensor.rs:31-63,83-196,212-236 (rotation, tensor and vector
// descriptors) on the Rust side. Layout of the file: docs/FORMAT.md:33-107.
//
// The file is memory-mapped read-only. Opening checks everything the reference reader
// checks, with its messages, and touches no GPU, so a host without one can inspect a
// file. Loading a tensor copies its code stream to the device through a pinned
// staging buffer (two 16 MiB halves, so the host copy of one chunk overlaps the
// transfer of the other), builds the sign streams its rotations name, and hands
// everything to yskn_b200_matrix_create[_shard], which packs the codes into the
// streaming layout; the staging memory and the unpacked device copy are freed before
// the call returns.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <climits>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_set>
#include <utility>
#include <vector>

#include "common.cuh"

namespace yskn {
namespace {

// ------------------------------------------------------------------ JSON
// A small reader for the header: objects, arrays, strings (with escapes), numbers,
// true/false/null. Numbers written as non-negative integers that fit 64 bits are
// kept exactly (`is_uint`); the format's sizes and offsets must be of that kind.
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  bool is_uint = false;
  uint64_t u = 0;
  std::string s;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  size_t begin = 0, end = 0;  // byte span of the value in the header text

  // A key given twice keeps its last value.
  const Json* get(const char* key) const {
    for (auto it = obj.rbegin(); it != obj.rend(); ++it)
      if (it->first == key) return &it->second;
    return nullptr;
  }
};

class JsonReader {
 public:
  JsonReader(const char* text, size_t n) : t_(text), n_(n) {}
  bool read(Json& out, std::string& err) {
    skip();
    if (!value(out, 0)) {
      err = err_;
      return false;
    }
    skip();
    if (i_ != n_) {
      err = "trailing characters after the header object";
      return false;
    }
    return true;
  }

 private:
  const char* t_;
  size_t n_, i_ = 0;
  std::string err_;

  bool bad(const char* what) {
    err_ = std::string("header is not valid JSON: ") + what + " at byte " + std::to_string(i_);
    return false;
  }
  void skip() {
    while (i_ < n_ && (t_[i_] == ' ' || t_[i_] == '\t' || t_[i_] == '\n' || t_[i_] == '\r')) ++i_;
  }
  bool literal(const char* word) {
    const size_t k = std::strlen(word);
    if (n_ - i_ < k || std::memcmp(t_ + i_, word, k) != 0) return bad("unknown literal");
    i_ += k;
    return true;
  }
  bool value(Json& v, int depth) {
    if (depth > 128) return bad("nesting too deep");
    if (i_ >= n_) return bad("unexpected end");
    v.begin = i_;
    bool ok;
    switch (t_[i_]) {
      case '{': ok = object(v, depth); break;
      case '[': ok = array(v, depth); break;
      case '"': v.kind = Json::Str; ok = string(v.s); break;
      case 't': v.kind = Json::Bool; v.b = true; ok = literal("true"); break;
      case 'f': v.kind = Json::Bool; v.b = false; ok = literal("false"); break;
      case 'n': v.kind = Json::Null; ok = literal("null"); break;
      default: ok = number(v);
    }
    v.end = i_;
    return ok;
  }
  bool object(Json& v, int depth) {
    v.kind = Json::Obj;
    ++i_;
    skip();
    if (i_ < n_ && t_[i_] == '}') return ++i_, true;
    for (;;) {
      skip();
      if (i_ >= n_ || t_[i_] != '"') return bad("expected a member name");
      std::string key;
      if (!string(key)) return false;
      skip();
      if (i_ >= n_ || t_[i_] != ':') return bad("expected ':'");
      ++i_;
      skip();
      Json member;
      if (!value(member, depth + 1)) return false;
      v.obj.emplace_back(std::move(key), std::move(member));
      skip();
      if (i_ < n_ && t_[i_] == ',') {
        ++i_;
        continue;
      }
      if (i_ < n_ && t_[i_] == '}') return ++i_, true;
      return bad("expected ',' or '}'");
    }
  }
  bool array(Json& v, int depth) {
    v.kind = Json::Arr;
    ++i_;
    skip();
    if (i_ < n_ && t_[i_] == ']') return ++i_, true;
    for (;;) {
      skip();
      Json item;
      if (!value(item, depth + 1)) return false;
      v.arr.push_back(std::move(item));
      skip();
      if (i_ < n_ && t_[i_] == ',') {
        ++i_;
        continue;
      }
      if (i_ < n_ && t_[i_] == ']') return ++i_, true;
      return bad("expected ',' or ']'");
    }
  }
  static void put_utf8(std::string& s, uint32_t c) {
    if (c < 0x80) {
      s += (char)c;
    } else if (c < 0x800) {
      s += (char)(0xc0 | (c >> 6));
      s += (char)(0x80 | (c & 0x3f));
    } else if (c < 0x10000) {
      s += (char)(0xe0 | (c >> 12));
      s += (char)(0x80 | ((c >> 6) & 0x3f));
      s += (char)(0x80 | (c & 0x3f));
    } else {
      s += (char)(0xf0 | (c >> 18));
      s += (char)(0x80 | ((c >> 12) & 0x3f));
      s += (char)(0x80 | ((c >> 6) & 0x3f));
      s += (char)(0x80 | (c & 0x3f));
    }
  }
  bool hex4(uint32_t& c) {
    if (n_ - i_ < 4) return bad("short \\u escape");
    c = 0;
    for (int k = 0; k < 4; ++k) {
      const char h = t_[i_++];
      c <<= 4;
      if (h >= '0' && h <= '9') c |= h - '0';
      else if (h >= 'a' && h <= 'f') c |= h - 'a' + 10;
      else if (h >= 'A' && h <= 'F') c |= h - 'A' + 10;
      else return bad("bad \\u escape");
    }
    return true;
  }
  bool string(std::string& s) {
    ++i_;  // opening quote
    for (;;) {
      if (i_ >= n_) return bad("unterminated string");
      const unsigned char ch = (unsigned char)t_[i_++];
      if (ch == '"') return true;
      if (ch < 0x20) return bad("control character in a string");
      if (ch != '\\') {
        s += (char)ch;
        continue;
      }
      if (i_ >= n_) return bad("unterminated escape");
      const char e = t_[i_++];
      switch (e) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t c;
          if (!hex4(c)) return false;
          if (c >= 0xd800 && c < 0xdc00) {  // high surrogate: a low one must follow
            uint32_t lo;
            if (n_ - i_ < 2 || t_[i_] != '\\' || t_[i_ + 1] != 'u') return bad("unpaired surrogate");
            i_ += 2;
            if (!hex4(lo) || lo < 0xdc00 || lo >= 0xe000) return bad("unpaired surrogate");
            c = 0x10000 + ((c - 0xd800) << 10) + (lo - 0xdc00);
          } else if (c >= 0xdc00 && c < 0xe000) {
            return bad("unpaired surrogate");
          }
          put_utf8(s, c);
          break;
        }
        default: return bad("unknown escape");
      }
    }
  }
  bool number(Json& v) {
    v.kind = Json::Num;
    const size_t start = i_;
    bool neg = false, integral = true;
    if (i_ < n_ && t_[i_] == '-') neg = true, ++i_;
    if (i_ >= n_ || t_[i_] < '0' || t_[i_] > '9') return bad("expected a value");
    if (t_[i_] == '0') {
      ++i_;
    } else {
      while (i_ < n_ && t_[i_] >= '0' && t_[i_] <= '9') ++i_;
    }
    const size_t int_end = i_;
    if (i_ < n_ && t_[i_] == '.') {
      integral = false;
      ++i_;
      if (i_ >= n_ || t_[i_] < '0' || t_[i_] > '9') return bad("bad fraction");
      while (i_ < n_ && t_[i_] >= '0' && t_[i_] <= '9') ++i_;
    }
    if (i_ < n_ && (t_[i_] == 'e' || t_[i_] == 'E')) {
      integral = false;
      ++i_;
      if (i_ < n_ && (t_[i_] == '+' || t_[i_] == '-')) ++i_;
      if (i_ >= n_ || t_[i_] < '0' || t_[i_] > '9') return bad("bad exponent");
      while (i_ < n_ && t_[i_] >= '0' && t_[i_] <= '9') ++i_;
    }
    if (integral && !neg) {
      uint64_t u = 0;
      bool fits = true;
      for (size_t k = start; k < int_end; ++k) {
        const uint64_t digit = (uint64_t)(t_[k] - '0');
        if (u > (UINT64_MAX - digit) / 10) fits = false;
        u = u * 10 + digit;
      }
      v.is_uint = fits;
      v.u = u;
    }
    return true;
  }
};

// Well-formed UTF-8 (no overlong forms, no surrogates, at most U+10FFFF).
bool valid_utf8(const unsigned char* p, size_t n) {
  size_t i = 0;
  while (i < n) {
    const unsigned char c = p[i];
    int extra;
    uint32_t cp;
    if (c < 0x80) {
      ++i;
      continue;
    } else if ((c & 0xe0) == 0xc0) {
      extra = 1, cp = c & 0x1f;
    } else if ((c & 0xf0) == 0xe0) {
      extra = 2, cp = c & 0x0f;
    } else if ((c & 0xf8) == 0xf0) {
      extra = 3, cp = c & 0x07;
    } else {
      return false;
    }
    if (n - i <= (size_t)extra) return false;
    for (int k = 1; k <= extra; ++k) {
      if ((p[i + k] & 0xc0) != 0x80) return false;
      cp = (cp << 6) | (p[i + k] & 0x3f);
    }
    if ((extra == 1 && cp < 0x80) || (extra == 2 && cp < 0x800) || (extra == 3 && cp < 0x10000) || cp > 0x10ffff ||
        (cp >= 0xd800 && cp < 0xe000))
      return false;
    i += extra + 1;
  }
  return true;
}

// ------------------------------------------------------------- descriptors
struct Rotation {
  int rule;
  uint64_t seed, offset;
};

struct TensorDesc {
  std::string name;
  int role;  // YSKN_ROLE_*
  uint64_t rows, cols, phys, bits;
  int layout;
  uint64_t stream_off, stream_bytes, lut_off, scale_off;
  Rotation rot_in;
  bool has_rot_out;
  Rotation rot_out;
};

struct VectorDesc {
  std::string name;
  uint64_t off, n;
  int dtype;  // YSKN_VECTOR_*
};

// Field access with the reference reader's messages (crates/yskn-format/src/lib.rs:277-340).
struct Check {
  std::string err;
  bool invalid(const std::string& m) {
    if (err.empty()) err = m;
    return false;
  }
  bool unsupported(const std::string& m) { return invalid("unsupported: " + m); }
  const Json* required(const Json& o, const char* key) {
    const Json* v = o.get(key);
    if (!v) invalid(std::string("missing ") + key);
    return v;
  }
  bool number(const Json& o, const char* key, uint64_t& out) {
    const Json* v = required(o, key);
    if (!v) return false;
    if (v->kind != Json::Num || !v->is_uint) return invalid(std::string(key) + " must be an unsigned integer");
    out = v->u;
    return true;
  }
  bool number_or(const Json& o, const char* key, uint64_t dflt, uint64_t& out) {
    if (!o.get(key)) return out = dflt, true;
    return number(o, key, out);
  }
  bool text(const Json& o, const char* key, std::string& out) {
    const Json* v = required(o, key);
    if (!v) return false;
    if (v->kind != Json::Str) return invalid(std::string(key) + " must be a string");
    out = v->s;
    return true;
  }
  bool text_or(const Json& o, const char* key, const char* dflt, std::string& out) {
    if (!o.get(key)) return out = dflt, true;
    return text(o, key, out);
  }
  bool region(uint64_t off, uint64_t len, uint64_t first, uint64_t end) {
    if (off > UINT64_MAX - len) return invalid("data offset plus length overflow");
    if (off < first || off + len > end)
      return invalid("data region " + std::to_string(off) + "+" + std::to_string(len) + " lies outside payload");
    return true;
  }

  // tensor.rs:31-63: H512 with its sign stream, or (output side only) none/null.
  bool rotation(const Json& v, uint64_t blocks, bool allow_none, bool& present, Rotation& r) {
    present = false;
    if (allow_none && v.kind == Json::Null) return true;
    if (v.kind != Json::Obj) return invalid("rotation must be an object");
    std::string kind;
    if (!text(v, "kind", kind)) return false;
    if (kind == "H512" || kind == "none") {
      uint64_t qm = 0;
      if (!number_or(v, "qm_off", 0, qm)) return false;
      if (qm != 0) return invalid("rotation " + kind + " must have qm_off=0");
    }
    if (kind == "none" && allow_none) return true;
    if (kind != "H512") return unsupported("rotation " + kind);
    uint64_t m;
    if (!number(v, "m", m)) return false;
    if (m != blocks) return invalid("rotation block count differs from tensor dimensions");
    std::string rule;
    if (!text_or(v, "rule", "splitmix64", rule)) return false;
    if (rule == "splitmix64") r.rule = YSKN_SIGNS_SPLITMIX64;
    else if (rule == "mulberry32_7919_13") r.rule = YSKN_SIGNS_MULBERRY32;
    else return unsupported("sign rule " + rule);
    if (!number(v, "sign_seed", r.seed) || !number(v, "sign_offset", r.offset)) return false;
    present = true;
    return true;
  }

  // tensor.rs:83-196.
  bool tensor(const Json& v, uint64_t first, uint64_t end, TensorDesc& t) {
    if (v.kind != Json::Obj) return invalid("tensor must be an object");
    if (!text(v, "name", t.name)) return false;
    if (t.name.empty()) return invalid("empty tensor name");
    std::string role;
    if (!text(v, "role", role)) return false;
    if (role == "body") t.role = YSKN_ROLE_BODY;
    else if (role == "head") t.role = YSKN_ROLE_HEAD;
    else if (role == "embedding") t.role = YSKN_ROLE_EMBEDDING;
    else if (role == "draft") t.role = YSKN_ROLE_DRAFT;
    else return unsupported("tensor role " + role);
    if (!number(v, "rows", t.rows) || !number(v, "cols", t.cols) ||
        !number_or(v, "physical_rows", t.rows, t.phys))
      return false;
    if (t.rows == 0 || t.cols == 0 || t.cols % 512 || t.phys < t.rows)
      return invalid("invalid matrix dimensions for " + t.name);
    const std::pair<const char*, uint64_t> fixed[3] = {{"l", 12}, {"d", 2}, {"t", 256}};
    for (const auto& f : fixed) {
      uint64_t x;
      if (!number_or(v, f.first, f.second, x)) return false;
      if (x != f.second) return unsupported(t.name + ": " + f.first + " must be " + std::to_string(f.second));
    }
    if (!number(v, "bits", t.bits)) return false;
    if (t.bits < 4 || t.bits > 8) return unsupported(t.name + ": bits must be 4..8");
    std::string start;
    if (!text_or(v, "start", "zero", start)) return false;
    if (start != "zero") return unsupported(t.name + ": start=" + start);
    const Json* rar = v.get("rar");
    if (rar && rar->kind != Json::Null) return unsupported(t.name + ": rar is unspecified");
    uint64_t bias = 0;
    if (!number_or(v, "bias_off", 0, bias)) return false;
    if (bias != 0) return unsupported(t.name + ": bias_off must be zero");
    std::string layout;
    if (!text_or(v, "layout", "warp", layout)) return false;
    if (layout == "row") t.layout = YSKN_LAYOUT_ROW;
    else if (layout == "warp") t.layout = YSKN_LAYOUT_WARP;
    else return unsupported("layout " + layout);
    const uint64_t per_row = t.cols / 256;
    if (t.phys > UINT64_MAX / per_row) return invalid("sequence count overflow");
    const uint64_t seqs = t.phys * per_row;
    if (t.layout == YSKN_LAYOUT_WARP && seqs % 32) return invalid("warp layout requires a multiple of 32 sequences");
    if (seqs > UINT64_MAX / (t.bits * 16)) return invalid("code stream length overflow");
    if (!number(v, "stream_off", t.stream_off) || !number(v, "stream_bytes", t.stream_bytes)) return false;
    if (t.stream_bytes != seqs * t.bits * 16) return invalid(t.name + ": stream_bytes differs from matrix shape");
    if (!number(v, "lut_off", t.lut_off) || !number(v, "scale_off", t.scale_off)) return false;
    if (t.phys > UINT64_MAX / 2) return invalid("scale length overflow");
    if (!region(t.stream_off, t.stream_bytes, first, end) || !region(t.lut_off, 16384, first, end) ||
        !region(t.scale_off, 2 * t.phys, first, end))
      return false;
    if (const Json* ri = v.get("rot_in")) {
      bool present;
      if (!rotation(*ri, t.cols / 512, false, present, t.rot_in)) return false;
      if (!present) return invalid("input rotation is required");
    } else {
      t.rot_in = {YSKN_SIGNS_MULBERRY32, 7, 0};
    }
    if (const Json* ro = v.get("rot_out")) {
      if (!rotation(*ro, t.rows / 512, true, t.has_rot_out, t.rot_out)) return false;
    } else if (t.role == YSKN_ROLE_HEAD || t.role == YSKN_ROLE_EMBEDDING) {
      t.has_rot_out = false;
    } else {
      t.has_rot_out = true;
      t.rot_out = {YSKN_SIGNS_MULBERRY32, 7, t.cols};
    }
    if (t.has_rot_out && (t.rows % 512 || t.phys % 512))
      return invalid("output rotation requires whole 512-row blocks");
    return true;
  }

  // tensor.rs:212-236.
  bool vector(const Json& v, uint64_t first, uint64_t end, VectorDesc& d) {
    if (v.kind != Json::Obj) return invalid("vector must be an object");
    if (!text(v, "name", d.name)) return false;
    if (d.name.empty()) return invalid("empty vector name");
    if (!number(v, "off", d.off) || !number(v, "n", d.n)) return false;
    if (d.n > UINT64_MAX / 2) return invalid("vector length overflow");
    if (!region(d.off, 2 * d.n, first, end)) return false;
    std::string dtype;
    if (!text_or(v, "dtype", "f16", dtype)) return false;
    if (dtype == "f16") d.dtype = YSKN_VECTOR_F16;
    else if (dtype == "bf16") d.dtype = YSKN_VECTOR_BF16;
    else return unsupported("vector dtype " + dtype);
    return true;
  }
};

}  // namespace
}  // namespace yskn

using namespace yskn;

struct yskn_b200_file {
  const unsigned char* map = nullptr;
  size_t bytes = 0;
  uint32_t version = 0;
  uint64_t header_bytes = 0, data_offset = 0;
  std::string model_json;
  std::vector<TensorDesc> tensors;
  std::vector<VectorDesc> vectors;
};

static yskn_b200_file* open_fail(yskn_b200_file* f, const std::string& msg) {
  if (f) {
    if (f->map) munmap(const_cast<unsigned char*>(f->map), f->bytes);
    delete f;
  }
  fail(YSKN_EINVAL, "file_open: " + msg);
  return nullptr;
}

extern "C" YSKN_B200_API yskn_b200_file* yskn_b200_file_open(const char* path) {
  if (!path) return open_fail(nullptr, "null path");
  const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return open_fail(nullptr, std::string("cannot open ") + path + ": " + std::strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 0) {
    const std::string m = std::string("cannot stat ") + path + ": " + std::strerror(errno);
    ::close(fd);
    return open_fail(nullptr, m);
  }
  std::unique_ptr<yskn_b200_file> f(new yskn_b200_file);
  f->bytes = (size_t)st.st_size;
  if (f->bytes < 32) {
    ::close(fd);
    return open_fail(nullptr, "magic must be YSKN");
  }
  void* m = mmap(nullptr, f->bytes, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);  // the mapping keeps the file
  if (m == MAP_FAILED) return open_fail(nullptr, std::string("cannot map ") + path + ": " + std::strerror(errno));
  f->map = static_cast<const unsigned char*>(m);
  yskn_b200_file* F = f.release();
  const unsigned char* p = F->map;
  // lib.rs:97-120: prefix, version, declared lengths.
  if (std::memcmp(p, "YSKN", 4) != 0) return open_fail(F, "magic must be YSKN");
  std::memcpy(&F->version, p + 4, 4);
  if (F->version != 1) return open_fail(F, "unsupported: version " + std::to_string(F->version));
  uint64_t file_bytes;
  std::memcpy(&F->header_bytes, p + 8, 8);
  std::memcpy(&F->data_offset, p + 16, 8);
  std::memcpy(&file_bytes, p + 24, 8);
  if (file_bytes != (uint64_t)F->bytes) return open_fail(F, "declared file length differs from actual length");
  if (F->header_bytes > UINT64_MAX - 32) return open_fail(F, "header length overflow");
  const uint64_t header_end = 32 + F->header_bytes;
  if (header_end > F->data_offset || F->data_offset > file_bytes)
    return open_fail(F, "header or first data offset lies outside the file");
  // lib.rs:121-147: the header object and its descriptors.
  const char* text = reinterpret_cast<const char*>(p + 32);
  if (!valid_utf8(p + 32, (size_t)F->header_bytes)) return open_fail(F, "header is not valid UTF-8");
  Json root;
  std::string err;
  if (!JsonReader(text, (size_t)F->header_bytes).read(root, err)) return open_fail(F, err);
  Check c;
  if (root.kind != Json::Obj) return open_fail(F, "header must be an object");
  const Json* model = c.required(root, "model");
  if (!model) return open_fail(F, c.err);
  if (model->kind != Json::Obj) return open_fail(F, "model must be an object");
  F->model_json.assign(text + model->begin, model->end - model->begin);
  const Json* tensors = c.required(root, "tensors");
  if (!tensors) return open_fail(F, c.err);
  if (tensors->kind != Json::Arr) return open_fail(F, "tensors must be an array");
  std::unordered_set<std::string> names;
  auto unique = [&](const std::string& n) { return names.insert(n).second; };
  for (const Json& e : tensors->arr) {
    TensorDesc t{};
    if (!c.tensor(e, F->data_offset, file_bytes, t)) return open_fail(F, c.err);
    if (!unique(t.name)) return open_fail(F, "duplicate parameter " + t.name);
    F->tensors.push_back(std::move(t));
  }
  const Json* vectors = c.required(root, "vectors");
  if (!vectors) return open_fail(F, c.err);
  if (vectors->kind != Json::Arr) return open_fail(F, "vectors must be an array");
  for (const Json& e : vectors->arr) {
    VectorDesc v{};
    if (!c.vector(e, F->data_offset, file_bytes, v)) return open_fail(F, c.err);
    if (!unique(v.name)) return open_fail(F, "duplicate parameter " + v.name);
    F->vectors.push_back(std::move(v));
  }
  // lib.rs:149-161: zeros between the header and the first data block.
  for (uint64_t k = header_end; k < F->data_offset; ++k)
    if (p[k]) return open_fail(F, "nonzero bytes between header and first data block");
  return F;
}

extern "C" YSKN_B200_API void yskn_b200_file_close(yskn_b200_file* f) {
  if (!f) return;
  if (f->map) munmap(const_cast<unsigned char*>(f->map), f->bytes);
  delete f;
}

extern "C" YSKN_B200_API int yskn_b200_file_tensor_count(const yskn_b200_file* f) {
  return f ? (int)f->tensors.size() : fail(YSKN_EINVAL, "file: null handle");
}

extern "C" YSKN_B200_API int yskn_b200_file_vector_count(const yskn_b200_file* f) {
  return f ? (int)f->vectors.size() : fail(YSKN_EINVAL, "file: null handle");
}

extern "C" YSKN_B200_API const char* yskn_b200_file_model_json(const yskn_b200_file* f) {
  return f ? f->model_json.c_str() : nullptr;
}

extern "C" YSKN_B200_API int yskn_b200_file_find(const yskn_b200_file* f, const char* name, int* is_vector) {
  if (!f || !name) return fail(YSKN_EINVAL, "file_find: null argument");
  for (size_t i = 0; i < f->tensors.size(); ++i)
    if (f->tensors[i].name == name) {
      if (is_vector) *is_vector = 0;
      return (int)i;
    }
  for (size_t i = 0; i < f->vectors.size(); ++i)
    if (f->vectors[i].name == name) {
      if (is_vector) *is_vector = 1;
      return (int)i;
    }
  return fail(YSKN_EINVAL, std::string("file_find: no parameter named ") + name);
}

extern "C" YSKN_B200_API const char* yskn_b200_file_tensor_name(const yskn_b200_file* f, int i) {
  return f && i >= 0 && i < (int)f->tensors.size() ? f->tensors[i].name.c_str() : nullptr;
}

extern "C" YSKN_B200_API int yskn_b200_file_tensor_info(const yskn_b200_file* f, int i, int64_t* out) {
  if (!f || !out || i < 0 || i >= (int)f->tensors.size()) return fail(YSKN_EINVAL, "file_tensor_info: bad argument");
  const TensorDesc& t = f->tensors[i];
  const int64_t v[YSKN_TENSOR_INFO_FIELDS] = {t.role,
                                              (int64_t)t.rows,
                                              (int64_t)t.cols,
                                              (int64_t)t.phys,
                                              (int64_t)t.bits,
                                              t.layout,
                                              (int64_t)t.stream_off,
                                              (int64_t)t.stream_bytes,
                                              (int64_t)t.lut_off,
                                              (int64_t)t.scale_off,
                                              t.rot_in.rule,
                                              (int64_t)t.rot_in.seed,
                                              (int64_t)t.rot_in.offset,
                                              t.has_rot_out ? 1 : 0,
                                              t.has_rot_out ? t.rot_out.rule : -1,
                                              t.has_rot_out ? (int64_t)t.rot_out.seed : 0,
                                              t.has_rot_out ? (int64_t)t.rot_out.offset : 0};
  std::memcpy(out, v, sizeof v);
  return YSKN_OK;
}

extern "C" YSKN_B200_API const char* yskn_b200_file_vector_name(const yskn_b200_file* f, int i) {
  return f && i >= 0 && i < (int)f->vectors.size() ? f->vectors[i].name.c_str() : nullptr;
}

extern "C" YSKN_B200_API int yskn_b200_file_vector_info(const yskn_b200_file* f, int i, int64_t* out3) {
  if (!f || !out3 || i < 0 || i >= (int)f->vectors.size()) return fail(YSKN_EINVAL, "file_vector_info: bad argument");
  const VectorDesc& v = f->vectors[i];
  out3[0] = (int64_t)v.off;
  out3[1] = (int64_t)v.n;
  out3[2] = v.dtype;
  return YSKN_OK;
}

extern "C" YSKN_B200_API int yskn_b200_file_vector_read(const yskn_b200_file* f, int i, float* h_out, int64_t n) {
  if (!f || !h_out || i < 0 || i >= (int)f->vectors.size()) return fail(YSKN_EINVAL, "file_vector_read: bad argument");
  const VectorDesc& v = f->vectors[i];
  if ((uint64_t)n != v.n) return fail(YSKN_EINVAL, "file_vector_read: n differs from the vector's length");
  const unsigned char* src = f->map + v.off;
  for (int64_t k = 0; k < n; ++k) {
    uint16_t h;
    std::memcpy(&h, src + 2 * k, 2);  // no alignment is promised
    if (v.dtype == YSKN_VECTOR_BF16) {
      const uint32_t bits = (uint32_t)h << 16;
      std::memcpy(h_out + k, &bits, 4);
    } else {
      h_out[k] = half_bits_to_float(h);
    }
  }
  return YSKN_OK;
}

// Code stream of tensor t into fresh device memory, through a pinned staging buffer
// (two halves: the host copy of one chunk overlaps the transfer of the other).
static int upload_codes(const yskn_b200_file* f, const TensorDesc& t, uint32_t** d_out) {
  constexpr size_t HALF = 16u << 20;
  *d_out = nullptr;
  uint32_t* d = nullptr;
  unsigned char* pinned = nullptr;
  cudaStream_t st = nullptr;
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaError_t e = cudaMalloc(&d, t.stream_bytes);
  if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&pinned), 2 * HALF, cudaHostAllocDefault);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming);
  const unsigned char* src = f->map + t.stream_off;
  for (uint64_t pos = 0, k = 0; e == cudaSuccess && pos < t.stream_bytes; pos += HALF, ++k) {
    const size_t n = (size_t)std::min<uint64_t>(HALF, t.stream_bytes - pos);
    unsigned char* buf = pinned + (k & 1) * HALF;
    if (k >= 2) e = cudaEventSynchronize(done[k & 1]);  // this half's previous transfer
    if (e != cudaSuccess) break;
    std::memcpy(buf, src + pos, n);
    e = cudaMemcpyAsync(reinterpret_cast<unsigned char*>(d) + pos, buf, n, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaEventRecord(done[k & 1], st);
  }
  if (st) {
    const cudaError_t s = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = s;
  }
  for (cudaEvent_t ev : done)
    if (ev) cudaEventDestroy(ev);
  if (st) cudaStreamDestroy(st);
  if (pinned) cudaFreeHost(pinned);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "file_load_matrix: code stream upload");
  }
  *d_out = d;
  return YSKN_OK;
}

static yskn_b200_matrix* load_matrix(const yskn_b200_file* f, int i, bool shard, int r0, int r1, int c0, int c1) {
  if (!f || i < 0 || i >= (int)f->tensors.size()) {
    fail(YSKN_EINVAL, "file_load_matrix: bad handle or tensor index");
    return nullptr;
  }
  const TensorDesc& t = f->tensors[i];
  if (t.role == YSKN_ROLE_EMBEDDING) {
    fail(YSKN_EINVAL, "file_load_matrix: " + t.name +
                          " is an embedding (decoded row by row with its 16-bit table, not a linear operator)");
    return nullptr;
  }
  if (t.rows > (uint64_t)INT_MAX || t.phys > (uint64_t)INT_MAX || t.cols > (uint64_t)INT_MAX) {
    fail(YSKN_EINVAL, "file_load_matrix: " + t.name + " is larger than this library's int shapes");
    return nullptr;
  }
  std::vector<uint16_t> lut16(8192), scale16((size_t)t.phys);
  std::memcpy(lut16.data(), f->map + t.lut_off, 16384);  // no alignment is promised
  std::memcpy(scale16.data(), f->map + t.scale_off, 2 * (size_t)t.phys);
  std::vector<int8_t> s_in((size_t)t.cols), s_out;
  if (int rc = yskn_b200_signs(t.rot_in.rule, t.rot_in.seed, t.rot_in.offset, (int64_t)t.cols, s_in.data())) {
    (void)rc;
    return nullptr;
  }
  if (t.has_rot_out) {
    s_out.resize((size_t)t.phys);
    if (yskn_b200_signs(t.rot_out.rule, t.rot_out.seed, t.rot_out.offset, (int64_t)t.phys, s_out.data()))
      return nullptr;
  }
  uint32_t* d_codes = nullptr;
  if (upload_codes(f, t, &d_codes)) return nullptr;
  const int8_t* so = t.has_rot_out ? s_out.data() : nullptr;
  yskn_b200_matrix* m =
      shard ? yskn_b200_matrix_create_shard(d_codes, t.layout, (int)t.rows, (int)t.phys, (int)t.cols, (int)t.bits,
                                            lut16.data(), scale16.data(), s_in.data(), so, r0, r1, c0, c1)
            : yskn_b200_matrix_create(d_codes, t.layout, (int)t.rows, (int)t.phys, (int)t.cols, (int)t.bits,
                                      lut16.data(), scale16.data(), s_in.data(), so);
  const cudaError_t e = cudaFree(d_codes);  // the handle holds its own packed copy
  if (m && e != cudaSuccess) {
    yskn_b200_matrix_destroy(m);
    cuda_fail(e, "file_load_matrix: freeing the staged code stream");
    return nullptr;
  }
  return m;
}

extern "C" YSKN_B200_API yskn_b200_matrix* yskn_b200_file_load_matrix(const yskn_b200_file* f, int i) {
  return load_matrix(f, i, false, 0, 0, 0, 0);
}

extern "C" YSKN_B200_API yskn_b200_matrix* yskn_b200_file_load_matrix_shard(const yskn_b200_file* f, int i,
                                                                           int row_begin, int row_end,
                                                                           int col_begin, int col_end) {
  return load_matrix(f, i, true, row_begin, row_end, col_begin, col_end);
}

// Coded embedding: the main table and up to two residual tables, checked as the
// reference engine checks them before use (src/engine35.cpp:272-299): role embedding, row
// layout, no padding rows, no output rotation, the residuals of the main table's shape
// and input-rotation offset (their own seed and rule are not compared, and the main
// table's signs are used, as there: docs/spec/02_COMPRESSED_LINEAR.md:305-312), and a
// second residual only with a first.
extern "C" YSKN_B200_API yskn_b200_embedding* yskn_b200_file_load_embedding(const yskn_b200_file* f, int main_i,
                                                                         int res_i, int res2_i) {
  auto bad = [](const std::string& m) -> yskn_b200_embedding* {
    fail(YSKN_EINVAL, "file_load_embedding: " + m);
    return nullptr;
  };
  const int n_tensors = f ? (int)f->tensors.size() : 0;
  if (!f || main_i < 0 || main_i >= n_tensors || res_i >= n_tensors || res2_i >= n_tensors)
    return bad("bad handle or tensor index");
  if (res2_i >= 0 && res_i < 0) return bad("a second residual table needs the first");
  const int idx[3] = {main_i, res_i, res2_i};
  const TensorDesc& m = f->tensors[main_i];
  int n = 0;
  const TensorDesc* parts[3];
  for (int k = 0; k < 3; ++k) {
    if (idx[k] < 0) continue;
    const TensorDesc& t = f->tensors[idx[k]];
    if (t.role != YSKN_ROLE_EMBEDDING || t.layout != YSKN_LAYOUT_ROW || t.phys != t.rows || t.has_rot_out)
      return bad(t.name + ": an embedding table must have role embedding, row layout, no padding rows and no "
                          "output rotation");
    if (t.rows != m.rows || t.cols != m.cols || t.rot_in.offset != m.rot_in.offset)
      return bad(t.name + ": a residual table must have the main table's shape and input-rotation offset");
    if (t.rows > (uint64_t)INT_MAX || t.cols > (uint64_t)INT_MAX) return bad(t.name + ": too large");
    parts[n++] = &t;
  }
  std::vector<std::vector<uint16_t>> lut(n, std::vector<uint16_t>(8192)), scale(n);
  std::vector<int8_t> s_in((size_t)m.cols);
  if (yskn_b200_signs(m.rot_in.rule, m.rot_in.seed, m.rot_in.offset, (int64_t)m.cols, s_in.data())) return nullptr;
  uint32_t* d_codes[3] = {nullptr, nullptr, nullptr};
  const uint16_t* luts[3];
  const uint16_t* scales[3];
  int bits[3];
  for (int k = 0; k < n; ++k) {
    const TensorDesc& t = *parts[k];
    std::memcpy(lut[k].data(), f->map + t.lut_off, 16384);  // no alignment is promised
    scale[k].resize((size_t)t.rows);
    std::memcpy(scale[k].data(), f->map + t.scale_off, 2 * (size_t)t.rows);
    luts[k] = lut[k].data();
    scales[k] = scale[k].data();
    bits[k] = (int)t.bits;
  }
  yskn_b200_embedding* e = nullptr;
  int rc = YSKN_OK;
  for (int k = 0; k < n && rc == YSKN_OK; ++k) rc = upload_codes(f, *parts[k], &d_codes[k]);
  if (rc == YSKN_OK)
    e = yskn_b200_embedding_create(n, d_codes, bits, (int)m.rows, (int)m.cols, luts, scales, s_in.data());
  for (uint32_t* d : d_codes)
    if (d) cudaFree(d);  // the handle holds its own copies
  return e;
}
