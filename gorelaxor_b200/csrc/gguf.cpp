// GGUF parsing, internal/gguf/gguf.go restated in C++ (see gguf.h).
#include "gguf.h"

#include <cmath>
#include <cstring>

namespace grx {

namespace {

struct Reader {
  const uint8_t* b;
  size_t n, off = 0;
  std::string err;
  Reader(const uint8_t* p, size_t len) : b(p), n(len) {}
  // gguf.go:121-133: a read past the end sets the error once.
  const uint8_t* take(size_t k) {
    if (!err.empty()) return nullptr;
    if (k > n - off) {
      err = "gguf: file is cut short";
      return nullptr;
    }
    const uint8_t* p = b + off;
    off += k;
    return p;
  }
  uint64_t uint(size_t k) {
    const uint8_t* p = take(k);
    uint64_t v = 0;
    if (p)
      for (size_t i = 0; i < k; i++) v |= uint64_t(p[i]) << (8 * i);
    return v;
  }
  std::string str() {
    uint64_t k = uint(8);
    if (k > (1u << 30)) {
      if (err.empty()) err = "gguf: string too long";
      return "";
    }
    const uint8_t* p = take(size_t(k));
    return p ? std::string((const char*)p, size_t(k)) : std::string();
  }
  // gguf.go:160-213.
  GValue value(uint32_t t, int depth) {
    GValue v;
    switch (t) {
      case 0: v.i = int64_t(uint(1)); break;
      case 1: v.i = int8_t(uint(1)); break;
      case 2: v.i = int64_t(uint(2)); break;
      case 3: v.i = int16_t(uint(2)); break;
      case 4: v.i = int64_t(uint(4)); break;
      case 5: v.i = int32_t(uint(4)); break;
      case 6: {
        uint32_t u = uint32_t(uint(4));
        float f;
        std::memcpy(&f, &u, 4);
        v.kind = GValue::FLOAT;
        v.f = f;
        break;
      }
      case 7: v.i = uint(1) != 0; break;
      case 8: v.kind = GValue::STR; v.s = str(); break;
      case 9: {
        if (depth > 2) {
          if (err.empty()) err = "gguf: arrays nested too deep";
          return v;
        }
        uint32_t et = uint32_t(uint(4));
        uint64_t cnt = uint(8);
        // Every element takes at least one byte: a count can't pass the
        // bytes left, so a lying count allocates nothing (gguf.go:187-192).
        if (cnt > n - off || cnt > (1u << 24)) {
          if (err.empty()) err = "gguf: array too long";
          return v;
        }
        v.kind = GValue::ARR;
        for (uint64_t i = 0; i < cnt && err.empty(); i++) v.a.push_back(value(et, depth + 1));
        break;
      }
      case 10: v.i = int64_t(uint(8)); break;
      case 11: v.i = int64_t(uint(8)); break;
      case 12: {
        uint64_t u = uint(8);
        double d;
        std::memcpy(&d, &u, 8);
        v.kind = GValue::FLOAT;
        v.f = d;
        break;
      }
      default:
        if (err.empty()) err = "gguf: unknown value type " + std::to_string(t);
    }
    return v;
  }
};

// byteSize, gguf.go:356-371.
bool byte_size(const GTensor& t, size_t* out, std::string* err) {
  uint64_t n = uint64_t(t.elems());
  switch (t.type) {
    case G_F32: *out = size_t(n * 4); return true;
    case G_F16:
    case G_BF16: *out = size_t(n * 2); return true;
    case G_Q8_0:
      if (t.dims.empty() || t.dims[0] % 32 != 0) {
        *err = "gguf: Q8_0 tensor " + t.name + " rows are not a multiple of 32";
        return false;
      }
      *out = size_t(n / 32 * 34);
      return true;
  }
  *err = "gguf: tensor " + t.name + " has type " + std::to_string(t.type) + ", which this reader doesn't handle";
  return false;
}

}  // namespace

float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h >> 15) << 31, exp = (uint32_t(h) >> 10) & 0x1f, man = uint32_t(h) & 0x3ff, bits;
  if (exp == 0 && man == 0) {
    bits = sign;
  } else if (exp == 0) {
    uint32_t e = 127 - 15 + 1;
    while ((man & 0x400) == 0) {
      man <<= 1;
      e--;
    }
    bits = sign | e << 23 | (man & 0x3ff) << 13;
  } else if (exp == 0x1f) {
    bits = sign | 0xffu << 23 | man << 13;
  } else {
    bits = sign | (exp + 127 - 15) << 23 | man << 13;
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_f16(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  uint16_t sign = uint16_t(b >> 16) & 0x8000;
  int32_t exp = int32_t(b >> 23) & 0xff;
  uint32_t man = b & 0x7fffff;
  if (exp == 0xff) return man ? (sign | 0x7e00) : (sign | 0x7c00);
  int32_t e = exp - 127 + 15;
  if (e >= 0x1f) return sign | 0x7c00;
  if (e <= 0) {
    if (e < -10) return sign;
    man |= 0x800000;
    uint32_t shift = uint32_t(14 - e), h = man >> shift, rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1))) h++;
    return sign | uint16_t(h);
  }
  uint32_t h = uint32_t(e) << 10 | man >> 13, rem = man & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
  return sign | uint16_t(h);
}

// parseHeader + Parse, gguf.go:262-354.
bool GGUF::parse(const void* bytes, size_t len) {
  buf_.assign((const uint8_t*)bytes, (const uint8_t*)bytes + len);
  Reader r(buf_.data(), buf_.size());
  const uint8_t* magic = r.take(4);
  if (!magic || std::memcmp(magic, "GGUF", 4) != 0) {
    err = "gguf: not a GGUF file";
    return false;
  }
  version = int(r.uint(4));
  if (version < 2 || version > 3) {
    err = "gguf: version " + std::to_string(version) + " is not supported";
    return false;
  }
  uint64_t nt = r.uint(8), nkv = r.uint(8);
  if (!r.err.empty()) {
    err = r.err;
    return false;
  }
  if (nt > (1u << 20) || nkv > (1u << 20)) {
    err = "gguf: header counts out of range";
    return false;
  }
  for (uint64_t i = 0; i < nkv && r.err.empty(); i++) {
    std::string k = r.str();
    uint32_t t = uint32_t(r.uint(4));
    kv[k] = r.value(t, 0);
  }
  uint64_t size = len;
  std::vector<std::string> order;
  for (uint64_t i = 0; i < nt && r.err.empty(); i++) {
    GTensor t;
    t.name = r.str();
    uint32_t nd = uint32_t(r.uint(4));
    if (nd > 4) {
      err = "gguf: tensor " + t.name + " has " + std::to_string(nd) + " dimensions";
      return false;
    }
    uint64_t elems = 1;
    for (uint32_t d = 0; d < nd; d++) {
      uint64_t v = r.uint(8);
      // Each dimension and the product must fit in the file (gguf.go:317-325).
      if (v == 0 || v > size || (elems *= v) > size) {
        err = "gguf: tensor " + t.name + " has an impossible size";
        return false;
      }
      t.dims.push_back(int64_t(v));
    }
    t.type = int(r.uint(4));
    t.offset = r.uint(8);
    if (r.err.empty()) {
      order.push_back(t.name);
      tensors[t.name] = t;
    }
  }
  if (!r.err.empty()) {
    err = r.err;
    return false;
  }
  uint64_t align = 32;
  auto a = kv.find("general.alignment");
  if (a != kv.end()) {
    uint64_t v = uint64_t(a->second.i);
    if (a->second.kind != GValue::INT || v < 8 || v > 4096 || (v & (v - 1)) != 0) {
      err = "gguf: general.alignment must be a power of two from 8 to 4096";
      return false;
    }
    align = v;
  }
  uint64_t base = (r.off + align - 1) / align * align;
  uint64_t total = 0;
  for (auto& kvp : tensors) {
    GTensor& t = kvp.second;
    size_t nb;
    if (!byte_size(t, &nb, &err)) return false;
    // In this order, so no sum can wrap around (gguf.go:345-350).
    if (base > size || t.offset > size - base || uint64_t(nb) > size - base - t.offset) {
      err = "gguf: tensor " + t.name + " runs past the end of the file";
      return false;
    }
    t.data = buf_.data() + base + t.offset;
    t.bytes = nb;
    total += nb;
  }
  // Tensors that overlap would each cost their full size (gguf.go:92-101).
  if (total > size) {
    err = "gguf: the tensors overlap";
    return false;
  }
  return true;
}

int64_t GGUF::get_int(const std::string& key, int64_t def) const {
  auto it = kv.find(key);
  if (it == kv.end() || it->second.kind != GValue::INT) return def;
  return it->second.i;
}

double GGUF::get_float(const std::string& key, double def) const {
  auto it = kv.find(key);
  if (it == kv.end()) return def;
  if (it->second.kind == GValue::FLOAT) return it->second.f;
  if (it->second.kind == GValue::INT) return double(it->second.i);
  return def;
}

std::string GGUF::get_string(const std::string& key, const std::string& def) const {
  auto it = kv.find(key);
  if (it == kv.end() || it->second.kind != GValue::STR) return def;
  return it->second.s;
}

bool GGUF::float32(const std::string& name, std::vector<float>& out) const {
  auto it = tensors.find(name);
  if (it == tensors.end()) return false;
  const GTensor& t = it->second;
  int64_t n = t.elems();
  out.resize(size_t(n));
  const uint8_t* p = t.data;
  switch (t.type) {
    case G_F32:
      std::memcpy(out.data(), p, size_t(n) * 4);
      return true;
    case G_F16:
      for (int64_t i = 0; i < n; i++) out[size_t(i)] = f16_to_f32(uint16_t(p[2 * i] | p[2 * i + 1] << 8));
      return true;
    case G_BF16:
      for (int64_t i = 0; i < n; i++) {
        uint32_t u = uint32_t(p[2 * i] | p[2 * i + 1] << 8) << 16;
        std::memcpy(&out[size_t(i)], &u, 4);
      }
      return true;
    case G_Q8_0:
      for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t* blk = p + b * 34;
        float d = f16_to_f32(uint16_t(blk[0] | blk[1] << 8));
        for (int i = 0; i < 32; i++) out[size_t(b * 32 + i)] = d * float(int8_t(blk[2 + i]));
      }
      return true;
  }
  return false;
}

bool GGUF::matrix_shape(const std::string& name, int64_t* rows, int64_t* cols) const {
  auto it = tensors.find(name);
  if (it == tensors.end()) return false;
  const GTensor& t = it->second;
  int64_t c = 1;
  for (int64_t d : t.dims) {
    c = d;
    if (d > 1) break;
  }
  if (t.type == G_Q8_0 && c != t.dims[0]) return false;
  *cols = c;
  *rows = t.elems() / std::max<int64_t>(c, 1);
  return true;
}

}  // namespace grx
