// GGUF model files: the header, metadata and tensor directory of a GGUF image in host memory (the format the reference reads
// in c/src/gguf.c:113-166 and c/src/meta.c). Host code only; tensor data stays where it is.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace clb {

struct GgufTensor {
  std::string name;
  uint32_t n_dims = 0;
  uint64_t dims[4] = {1, 1, 1, 1};   // innermost first: a matrix is [cols, rows], fused experts [cols, rows, n_expert]
  uint32_t type = 0;                 // ggml type id
  uint64_t offset = 0;               // from the start of the image
  uint64_t nbytes = 0;
};

struct GgufValue {
  uint32_t type = 0;                 // gguf value type; arrays keep only their element type and count
  uint64_t u = 0;                    // integer and bool values
  double f = 0;                      // float values
  std::string s;                     // string values
  uint32_t arr_type = 0;
  uint64_t arr_count = 0;
};

struct Gguf {
  const uint8_t *base = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  std::unordered_map<std::string, GgufValue> kv;
  std::vector<GgufTensor> tensors;
  std::unordered_map<std::string, size_t> by_name;

  // Parses the image; returns 0, or 1 with err set (truncated or malformed image, tensor outside it, unknown type).
  int parse(const uint8_t *image, size_t n, char *err, size_t errlen);
  const GgufTensor *find(const std::string &name) const;
  bool get_u64(const std::string &key, uint64_t &out) const;   // any integer type
  bool get_f64(const std::string &key, double &out) const;     // any float or integer type
  bool get_str(const std::string &key, std::string &out) const;
};

// Bytes of one row of n elements of a ggml type, 0 for a type this library does not read.
uint64_t gguf_row_bytes(uint32_t type, uint64_t n);

}  // namespace clb
