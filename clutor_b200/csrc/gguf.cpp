// GGUF parsing (see gguf.h). Bounds-checked throughout: a truncated or corrupt image is an error, never a read past its end.
#include "gguf.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>

namespace clb {

namespace {

enum : uint32_t { V_U8, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64 };

struct Cursor {
  const uint8_t *p;
  size_t n, pos = 0;
  bool bad = false;
  bool need(size_t k) {
    if (bad || k > n - pos) { bad = true; return false; }
    return true;
  }
  template <class T>
  T rd() {
    T v{};
    if (need(sizeof(T))) { std::memcpy(&v, p + pos, sizeof(T)); pos += sizeof(T); }
    return v;
  }
  std::string str() {
    const uint64_t len = rd<uint64_t>();
    if (len > (1u << 24) || !need(static_cast<size_t>(len))) { bad = true; return {}; }
    std::string s(reinterpret_cast<const char *>(p + pos), static_cast<size_t>(len));
    pos += static_cast<size_t>(len);
    return s;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case V_U8: case V_I8: case V_BOOL: return 1;
    case V_U16: case V_I16: return 2;
    case V_U32: case V_I32: case V_F32: return 4;
    case V_U64: case V_I64: case V_F64: return 8;
    default: return 0;
  }
}

void fail(char *err, size_t errlen, const char *fmt, ...) {
  if (!err || !errlen) return;
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(err, errlen, fmt, ap);
  va_end(ap);
}

// ggml block sizes (elements, bytes) for the types a model of this library may hold
bool block_of(uint32_t type, uint64_t &elems, uint64_t &bytes) {
  switch (type) {
    case 0: elems = 1; bytes = 4; return true;      // F32
    case 1: elems = 1; bytes = 2; return true;      // F16
    case 8: elems = 32; bytes = 34; return true;    // Q8_0
    case 12: elems = 256; bytes = 144; return true; // Q4_K
    case 14: elems = 256; bytes = 210; return true; // Q6_K
    case 30: elems = 1; bytes = 2; return true;     // BF16
    default: return false;
  }
}

}  // namespace

uint64_t gguf_row_bytes(uint32_t type, uint64_t n) {
  uint64_t e = 0, b = 0;
  if (!block_of(type, e, b) || n % e) return 0;
  return n / e * b;
}

int Gguf::parse(const uint8_t *image, size_t n, char *err, size_t errlen) {
  base = image;
  size = n;
  Cursor c{image, n};
  if (n < 4 || std::memcmp(image, "GGUF", 4)) { fail(err, errlen, "not a GGUF file (bad magic)"); return 1; }
  c.pos = 4;
  version = c.rd<uint32_t>();
  const uint64_t nt = c.rd<uint64_t>(), nkv = c.rd<uint64_t>();
  if (c.bad) { fail(err, errlen, "truncated GGUF header"); return 1; }
  if (version != 2 && version != 3) { fail(err, errlen, "unsupported GGUF version %u", version); return 1; }
  if (nt > 1000000 || nkv > 1000000) { fail(err, errlen, "implausible tensor or metadata count"); return 1; }
  for (uint64_t i = 0; i < nkv; ++i) {
    const std::string key = c.str();
    GgufValue v;
    v.type = c.rd<uint32_t>();
    if (c.bad) { fail(err, errlen, "corrupt metadata"); return 1; }
    if (v.type == V_STR) {
      v.s = c.str();
    } else if (v.type == V_ARR) {
      v.arr_type = c.rd<uint32_t>();
      v.arr_count = c.rd<uint64_t>();
      if (v.arr_type == V_STR) {
        for (uint64_t j = 0; j < v.arr_count && !c.bad; ++j) c.str();
      } else {
        const size_t es = scalar_size(v.arr_type);
        if (!es || v.arr_count > (n / es) || !c.need(static_cast<size_t>(v.arr_count * es))) { fail(err, errlen, "corrupt metadata array \"%s\"", key.c_str()); return 1; }
        c.pos += static_cast<size_t>(v.arr_count * es);
      }
    } else {
      const size_t es = scalar_size(v.type);
      if (!es || !c.need(es)) { fail(err, errlen, "corrupt metadata value \"%s\"", key.c_str()); return 1; }
      const uint8_t *q = image + c.pos;
      switch (v.type) {
        case V_U8: v.u = q[0]; break;
        case V_I8: v.u = static_cast<uint64_t>(static_cast<int64_t>(static_cast<int8_t>(q[0]))); break;
        case V_BOOL: v.u = q[0] != 0; break;
        case V_U16: { uint16_t t; std::memcpy(&t, q, 2); v.u = t; break; }
        case V_I16: { int16_t t; std::memcpy(&t, q, 2); v.u = static_cast<uint64_t>(static_cast<int64_t>(t)); break; }
        case V_U32: { uint32_t t; std::memcpy(&t, q, 4); v.u = t; break; }
        case V_I32: { int32_t t; std::memcpy(&t, q, 4); v.u = static_cast<uint64_t>(static_cast<int64_t>(t)); break; }
        case V_U64: case V_I64: std::memcpy(&v.u, q, 8); break;
        case V_F32: { float t; std::memcpy(&t, q, 4); v.f = t; break; }
        case V_F64: std::memcpy(&v.f, q, 8); break;
      }
      c.pos += es;
    }
    if (c.bad) { fail(err, errlen, "corrupt metadata value \"%s\"", key.c_str()); return 1; }
    kv[key] = std::move(v);
  }
  uint64_t align = 32;
  uint64_t a = 0;
  if (get_u64("general.alignment", a) && a > 0 && a <= (1u << 20)) align = a;
  tensors.resize(static_cast<size_t>(nt));
  for (uint64_t i = 0; i < nt; ++i) {
    GgufTensor &t = tensors[static_cast<size_t>(i)];
    t.name = c.str();
    t.n_dims = c.rd<uint32_t>();
    if (c.bad || t.n_dims == 0 || t.n_dims > 4) { fail(err, errlen, "tensor %llu: bad directory entry", static_cast<unsigned long long>(i)); return 1; }
    for (uint32_t d = 0; d < t.n_dims; ++d) t.dims[d] = c.rd<uint64_t>();
    t.type = c.rd<uint32_t>();
    t.offset = c.rd<uint64_t>();
    if (c.bad) { fail(err, errlen, "truncated tensor directory"); return 1; }
  }
  const uint64_t data = (c.pos + align - 1) / align * align;
  for (size_t i = 0; i < tensors.size(); ++i) {
    GgufTensor &t = tensors[i];
    uint64_t be = 0, bb = 0;
    if (!block_of(t.type, be, bb)) { t.nbytes = 0; by_name[t.name] = i; continue; }   // a type no kernel here reads
    uint64_t elems = 1;
    for (uint32_t d = 0; d < t.n_dims; ++d) {
      if (t.dims[d] == 0 || elems > (~0ull) / t.dims[d]) { fail(err, errlen, "tensor \"%s\": bad dims", t.name.c_str()); return 1; }
      elems *= t.dims[d];
    }
    if (t.dims[0] % be) { fail(err, errlen, "tensor \"%s\": rows of %llu elements are not whole blocks", t.name.c_str(), static_cast<unsigned long long>(t.dims[0])); return 1; }
    t.nbytes = elems / be * bb;
    t.offset += data;
    if (t.offset > n || t.nbytes > n - t.offset) { fail(err, errlen, "tensor \"%s\" points outside the file (truncated?)", t.name.c_str()); return 1; }
    by_name[t.name] = i;
  }
  return 0;
}

const GgufTensor *Gguf::find(const std::string &name) const {
  auto it = by_name.find(name);
  return it == by_name.end() ? nullptr : &tensors[it->second];
}

bool Gguf::get_u64(const std::string &key, uint64_t &out) const {
  auto it = kv.find(key);
  if (it == kv.end()) return false;
  const uint32_t t = it->second.type;
  if (t == V_F32 || t == V_F64 || t == V_STR || t == V_ARR) return false;
  out = it->second.u;
  return true;
}

bool Gguf::get_f64(const std::string &key, double &out) const {
  auto it = kv.find(key);
  if (it == kv.end()) return false;
  const uint32_t t = it->second.type;
  if (t == V_F32 || t == V_F64) { out = it->second.f; return true; }
  if (t == V_STR || t == V_ARR) return false;
  out = static_cast<double>(it->second.u);
  return true;
}

bool Gguf::get_str(const std::string &key, std::string &out) const {
  auto it = kv.find(key);
  if (it == kv.end() || it->second.type != V_STR) return false;
  out = it->second.s;
  return true;
}

}  // namespace clb
