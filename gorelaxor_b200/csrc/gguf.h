// GGUF reader for the token loops: the subset internal/gguf reads
// (versions 2 and 3; F32, F16, BF16 and Q8_0 tensors), with the same
// hostile-input checks (internal/gguf/gguf.go:121-354): every length,
// count, dimension and offset is checked against the bytes present before
// it is used, and a failure is an error, never a crash.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <variant>
#include <vector>

namespace grx {

enum GType { G_F32 = 0, G_F16 = 1, G_Q8_0 = 8, G_BF16 = 30 };

struct GTensor {
  std::string name;
  std::vector<int64_t> dims;  // dims[0] is the row length
  int type = 0;
  uint64_t offset = 0;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
  int64_t elems() const {
    int64_t n = 1;
    for (int64_t d : dims) n *= d;
    return n;
  }
};

// A key's value: integers (any width, and bools) as int64, floats as
// double, strings, or an array of those.
struct GValue {
  enum Kind { INT, FLOAT, STR, ARR } kind = INT;
  int64_t i = 0;
  double f = 0;
  std::string s;
  std::vector<GValue> a;
};

class GGUF {
 public:
  // Parses bytes (copied). Returns false with err set on any problem.
  bool parse(const void* bytes, size_t len);
  std::string err;
  int version = 0;
  std::map<std::string, GValue> kv;
  std::map<std::string, GTensor> tensors;

  bool has(const std::string& name) const { return tensors.count(name) != 0; }
  int64_t get_int(const std::string& key, int64_t def) const;
  double get_float(const std::string& key, double def) const;
  std::string get_string(const std::string& key, const std::string& def) const;
  // The tensor as float32 (F16/BF16/Q8_0 widened); false if absent.
  bool float32(const std::string& name, std::vector<float>& out) const;
  // Weight shape (gguf.go:544-560): cols = first dim > 1, rows = the rest.
  bool matrix_shape(const std::string& name, int64_t* rows, int64_t* cols) const;

 private:
  std::vector<uint8_t> buf_;
};

float f16_to_f32(uint16_t h);
uint16_t f32_to_f16(float f);

}  // namespace grx
