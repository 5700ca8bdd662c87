// TEST INFRASTRUCTURE ONLY: the CPU oracle. Nothing in the product links,
// loads or calls this code; tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline leg use it as the checker.
//
// A C++ restatement of gorelaxor's shared kernels (internal/kern), order-
// faithful to the amd64 path the reference runs on processors with AVX2,
// FMA, F16C and AVX512-VNNI (the fastest path it has, and the one its
// benchmarks quote). Every function names the reference lines it follows.
// Built with -ffp-contract=off so that no multiply-add is fused unless the
// reference's assembly fuses it (written here as std::fma). Go itself never
// fuses on amd64 at its default GOAMD64=v1, so Go lines are unfused here.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>

namespace orc {

constexpr int QK = 32;       // internal/kern/kern.go:34
constexpr int Q8BYTES = 34;  // internal/kern/kern.go:35

// ---------------------------------------------------------------- f16 ---

// f16toF32, internal/kern/f16.go:14-33 (the f16tab entries).
inline float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h >> 15) << 31;
  uint32_t exp = (uint32_t(h) >> 10) & 0x1f;
  uint32_t man = uint32_t(h) & 0x3ff;
  uint32_t bits;
  if (exp == 0 && man == 0) {
    bits = sign;
  } else if (exp == 0) {
    uint32_t e = 127 - 15 + 1;
    while ((man & 0x400) == 0) {
      man <<= 1;
      e--;
    }
    man &= 0x3ff;
    bits = sign | e << 23 | man << 13;
  } else if (exp == 0x1f) {
    bits = sign | 0xffu << 23 | man << 13;
  } else {
    bits = sign | (exp + 127 - 15) << 23 | man << 13;
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// f32toF16, internal/kern/f16.go:36-71 (round to nearest, ties to even).
inline uint16_t f32_to_f16(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  uint16_t sign = uint16_t(b >> 16) & 0x8000;
  int32_t exp = int32_t(b >> 23) & 0xff;
  uint32_t man = b & 0x7fffff;
  if (exp == 0xff) return man != 0 ? (sign | 0x7e00) : (sign | 0x7c00);
  int32_t e = exp - 127 + 15;
  if (e >= 0x1f) return sign | 0x7c00;
  if (e <= 0) {
    if (e < -10) return sign;
    man |= 0x800000;
    uint32_t shift = uint32_t(14 - e);
    uint32_t h = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1) == 1)) h++;
    return sign | uint16_t(h);
  }
  uint32_t h = uint32_t(e) << 10 | man >> 13;
  uint32_t rem = man & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1) == 1)) h++;
  return sign | uint16_t(h);
}

inline float bits_f32(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// ---------------------------------------------------------------- exp ---

// expf, internal/kern/mathx.go:7-33 (scalar Go; the tails of the vector
// helpers and every scalar caller use it).
inline float expf_go(float x) {
  if (x < -87.f) return 0.f;
  if (x > 88.f) return INFINITY;
  float t = x * 1.4426950408889634f + 0.5f;
  int32_t ni = int32_t(t);
  if (float(ni) > t) ni--;
  float n = float(ni);
  float r = x - n * 0.693145751953125f - n * 1.428606765330187e-06f;
  float p = float(1.0 / 720) * r + float(1.0 / 120);
  p = p * r + float(1.0 / 24);
  p = p * r + float(1.0 / 6);
  p = p * r + 0.5f;
  p = p * r + 1.f;
  p = p * r + 1.f;
  if (ni < -126) return p * bits_f32(uint32_t(ni + 127 + 64) << 23) * 5.421010862427522e-20f;
  return p * bits_f32(uint32_t(ni + 127) << 23);
}

// EXP8, internal/kern/kernels_amd64.s:238-257 with the constants of
// :217-233: clamp to [-87, 88], n = round-to-even(x·log2e), fused
// reduction by the split ln2, fused Horner steps, scale by 2^n.
inline float exp_avx(float x) {
  const float log2e = bits_f32(0x3fb8aa3b), ln2hi = bits_f32(0x3f317200), ln2lo = bits_f32(0x35bfbe8e);
  const float c720 = bits_f32(0x3ab60b61), c120 = bits_f32(0x3c088889), c24 = bits_f32(0x3d2aaaab);
  const float c6 = bits_f32(0x3e2aaaab), c2 = 0.5f, one = 1.f;
  x = std::fmax(x, -87.f);  // VMAXPS: x is the first source, NaN-free inputs
  x = std::fmin(x, 88.f);
  float n = std::nearbyint(x * log2e);
  float r = std::fma(-n, ln2hi, x);
  r = std::fma(-n, ln2lo, r);
  float p = std::fma(c720, r, c120);
  p = std::fma(r, p, c24);
  p = std::fma(r, p, c6);
  p = std::fma(r, p, c2);
  p = std::fma(r, p, one);
  p = std::fma(r, p, one);
  int32_t ni = int32_t(n);
  return p * bits_f32(uint32_t(ni + 127) << 23);
}

// expSub, internal/kern/kernels_amd64.go:107-117 + expSubAVX
// kernels_amd64.s:261-283 (8 lane sums, then VEXTRACTF128/VHADDPS) and
// expSubGo mathx.go:92-101 for the tail.
inline float expsub_vec(float* x, int len, float mx) {
  int n = len & ~7;
  float s = 0.f;
  if (n > 0) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < n; c += 8)
      for (int l = 0; l < 8; l++) {
        float e = exp_avx(x[c + l] - mx);
        x[c + l] = e;
        acc[l] = acc[l] + e;
      }
    float h0 = acc[0] + acc[4], h1 = acc[1] + acc[5], h2 = acc[2] + acc[6], h3 = acc[3] + acc[7];
    s = (h0 + h1) + (h2 + h3);
  }
  float t = 0.f;
  for (int i = n; i < len; i++) {
    float e = expf_go(x[i] - mx);
    x[i] = e;
    t += e;
  }
  return s + t;
}

// ------------------------------------------------- GELU, SiLU, ReLU ---

// gelu, internal/kern/mathx.go:36-52.
inline float gelu_go(float v) {
  const float c = float(0.7978845608028654);
  float u = c * v * (1.f + 0.044715f * v * v);
  float t;
  if (u > 9.f)
    t = 1.f;
  else if (u < -9.f)
    t = -1.f;
  else
    t = 1.f - 2.f / (expf_go(2.f * u) + 1.f);
  return 0.5f * v * (1.f + t);
}

// geluAVX, internal/kern/kernels_amd64.s:301-339.
inline float gelu_avx(float v) {
  float u = v * v;
  u = std::fma(bits_f32(0x3d372713), u, 1.f);
  u = v * u;
  u = bits_f32(0x3f4c422a) * u;
  u = std::fmin(u, 9.f);
  u = std::fmax(u, -9.f);
  float e = exp_avx(u + u);
  e = e + 1.f;
  e = 2.f / e;
  e = 1.f - e;
  e = e + 1.f;
  e = e * v;
  return e * 0.5f;
}

inline bool fast_on();
inline bool gelu_vec_fast(float* x, int len);
inline bool silu_vec_fast(float* x, int len);

// geluVec, internal/kern/kernels_amd64.go:119-129.
inline void gelu_vec(float* x, int len) {
  if (fast_on() && gelu_vec_fast(x, len)) return;
  int n = len & ~7;
  for (int i = 0; i < n; i++) x[i] = gelu_avx(x[i]);
  for (int i = n; i < len; i++) x[i] = gelu_go(x[i]);
}

// siluGo, internal/kern/mathx.go:115-119.
inline float silu_go(float v) { return v / (1.f + expf_go(-v)); }

// siluAVX, internal/kern/kernels_amd64.s:441-459.
inline float silu_avx(float v) {
  float e = exp_avx(0.f - v);
  return v / (e + 1.f);
}

// siluVec, internal/kern/kernels_amd64.go:241-250.
inline void silu_vec(float* x, int len) {
  if (fast_on() && silu_vec_fast(x, len)) return;
  int n = len & ~7;
  for (int i = 0; i < n; i++) x[i] = silu_avx(x[i]);
  for (int i = n; i < len; i++) x[i] = silu_go(x[i]);
}

// sigmoid, conformer/encoder.go:13 (scalar expf).
inline float sigmoid_go(float v) { return 1.f / (1.f + expf_go(-v)); }

// --------------------------------------------------------------- dots ---

// dotF32Go, internal/kern/gemm.go:294-308.
inline float dot_f32_go(const float* x, const float* y, int len) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  int i = 0;
  for (; i + 4 <= len; i += 4) {
    s0 += x[i] * y[i];
    s1 += x[i + 1] * y[i + 1];
    s2 += x[i + 2] * y[i + 2];
    s3 += x[i + 3] * y[i + 3];
  }
  for (; i < len; i++) s0 += x[i] * y[i];
  return s0 + s1 + s2 + s3;
}

// HSUM, internal/kern/kernels_amd64.s:92-97: high half onto low, then two
// horizontal adds.
inline float hsum8(const float a[8]) {
  float h0 = a[0] + a[4], h1 = a[1] + a[5], h2 = a[2] + a[6], h3 = a[3] + a[7];
  return (h0 + h1) + (h2 + h3);
}

// dot4f32avx, internal/kern/kernels_amd64.s:157-204: per row two 8-lane
// FMA accumulators (elements 16c..16c+7 and 16c+8..16c+15), added, then
// HSUM. k is a multiple of 16.
inline void dot4_f32_avx(const float* x, const float* w, long ld, int k, float out[4]) {
  for (int r = 0; r < 4; r++) {
    const float* wr = w + r * ld;
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0}, b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < k; c += 16)
      for (int l = 0; l < 8; l++) {
        a[l] = std::fma(x[c + l], wr[c + l], a[l]);
        b[l] = std::fma(x[c + 8 + l], wr[c + 8 + l], b[l]);
      }
    for (int l = 0; l < 8; l++) a[l] = a[l] + b[l];
    out[r] = hsum8(a);
  }
}

// dotF32x4, internal/kern/kernels_amd64.go:75-95.
inline void dot_f32x4(const float* x, const float* w, long ld, int k, float out[4]) {
  int kk = k & ~15;
  if (kk > 0)
    dot4_f32_avx(x, w, ld, kk, out);
  else
    out[0] = out[1] = out[2] = out[3] = 0;
  if (kk < k)
    for (int r = 0; r < 4; r++) out[r] += dot_f32_go(x + kk, w + r * ld + kk, k - kk);
}

// dotF16Go, internal/kern/gemm.go:310-325.
inline float dot_f16_go(const float* x, const uint16_t* y, int len) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  int i = 0;
  for (; i + 4 <= len; i += 4) {
    s0 += x[i] * f16_to_f32(y[i]);
    s1 += x[i + 1] * f16_to_f32(y[i + 1]);
    s2 += x[i + 2] * f16_to_f32(y[i + 2]);
    s3 += x[i + 3] * f16_to_f32(y[i + 3]);
  }
  for (; i < len; i++) s0 += x[i] * f16_to_f32(y[i]);
  return s0 + s1 + s2 + s3;
}

// dot4f16avx, internal/kern/kernels_amd64.s:99-155 (same lane structure
// as dot4f32avx, halves widened by VCVTPH2PS, which is exact).
inline void dot4_f16_avx(const float* x, const uint16_t* w, long ld, int k, float out[4]) {
  for (int r = 0; r < 4; r++) {
    const uint16_t* wr = w + r * ld;
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0}, b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < k; c += 16)
      for (int l = 0; l < 8; l++) {
        a[l] = std::fma(x[c + l], f16_to_f32(wr[c + l]), a[l]);
        b[l] = std::fma(x[c + 8 + l], f16_to_f32(wr[c + 8 + l]), b[l]);
      }
    for (int l = 0; l < 8; l++) a[l] = a[l] + b[l];
    out[r] = hsum8(a);
  }
}

// dotF16x4, internal/kern/kernels_amd64.go:53-73 (whisper/kernels_amd64.go
// has the same code).
inline void dot_f16x4(const float* x, const uint16_t* w, long ld, int k, float out[4]) {
  int kk = k & ~15;
  if (kk > 0)
    dot4_f16_avx(x, w, ld, kk, out);
  else
    out[0] = out[1] = out[2] = out[3] = 0;
  if (kk < k)
    for (int r = 0; r < 4; r++) out[r] += dot_f16_go(x + kk, w + r * ld + kk, k - kk);
}

// dotQ8Go, internal/kern/kern.go:249-266.
inline float dot_q8_go(const float* x, const uint8_t* q, int k) {
  float s = 0;
  for (int b = 0; b * QK < k; b++) {
    const uint8_t* blk = q + b * Q8BYTES;
    float d = f16_to_f32(uint16_t(blk[0] | blk[1] << 8));
    const float* xs = x + b * QK;
    const int8_t* qs = (const int8_t*)(blk + 2);
    float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    for (int i = 0; i < QK; i += 4) {
      a0 += xs[i] * float(qs[i]);
      a1 += xs[i + 1] * float(qs[i + 1]);
      a2 += xs[i + 2] * float(qs[i + 2]);
      a3 += xs[i + 3] * float(qs[i + 3]);
    }
    s += d * (a0 + a1 + a2 + a3);
  }
  return s;
}

// dot4q8avx, internal/kern/kernels_amd64.s:343-399: per block, lane l
// holds q[l]·x[l] then three fused steps over q[8+l], q[16+l], q[24+l];
// the block's 8 lanes are then fused into the row accumulator by the
// block's f16 scale; HSUM at the end.
inline float dot_q8_avx_row(const float* x, const uint8_t* q, int nb) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int b = 0; b < nb; b++) {
    const uint8_t* blk = q + b * Q8BYTES;
    const int8_t* qs = (const int8_t*)(blk + 2);
    const float* xs = x + b * QK;
    float d = f16_to_f32(uint16_t(blk[0] | blk[1] << 8));
    for (int l = 0; l < 8; l++) {
      float y = float(qs[l]) * xs[l];
      y = std::fma(float(qs[8 + l]), xs[8 + l], y);
      y = std::fma(float(qs[16 + l]), xs[16 + l], y);
      y = std::fma(float(qs[24 + l]), xs[24 + l], y);
      acc[l] = std::fma(y, d, acc[l]);
    }
  }
  return hsum8(acc);
}

// dotQ8x4, internal/kern/kernels_amd64.go:131-140.
inline void dot_q8x4(const float* x, const uint8_t* q, long ld, int k, float out[4]) {
  int nb = k / QK;
  for (int r = 0; r < 4; r++) out[r] = dot_q8_avx_row(x, q + r * ld, nb);
}

// ----------------------------------------------------------- weights ---

enum WType { F32 = 0, F16 = 1, Q8_0 = 2 };

struct PanelSlot;  // fast.h: a Q8_0 weight's panels for the fast mode

// Weight, internal/kern/kern.go:41-50. `dropped` is DropRows (kern.go:99):
// a packed Q8_0 weight whose products all take the int8 kernel. `slot`
// (shared by every copy of a model's weight) keeps the fast mode's panels,
// packed on first use, as Weight.panels does (kern.go:48-49).
struct Weight {
  int rows = 0, cols = 0;
  WType type = F32;
  const float* f = nullptr;
  const uint16_t* h = nullptr;
  const uint8_t* q = nullptr;
  bool dropped = false;
  std::shared_ptr<PanelSlot> slot;
};

inline bool fast_on();
inline bool gemv_rows_fast_ok(float* y, const float* x, const Weight& w, const float* bias);

// gemvRows for one row of A, internal/kern/gemm.go:195-259 (m=1, so no
// Q8_0 widening; whisper/gemm.go:187-218 gemv is the same for F16/F32).
inline void gemv_rows(float* y, const float* x, const Weight& w, const float* bias) {
  if (fast_on() && gemv_rows_fast_ok(y, x, w, bias)) return;
  int n = w.rows, k = w.cols;
  for (int j = 0; j < n; j += 4) {
    if (j + 4 <= n) {
      float out[4];
      switch (w.type) {
        case F16:
          dot_f16x4(x, w.h + long(j) * k, k, k, out);
          break;
        case Q8_0:
          dot_q8x4(x, w.q + long(j) * (k / QK) * Q8BYTES, (k / QK) * Q8BYTES, k, out);
          break;
        default:
          dot_f32x4(x, w.f + long(j) * k, k, k, out);
      }
      for (int r = 0; r < 4; r++) y[j + r] = out[r];
    } else {
      for (int jj = j; jj < n; jj++) {
        switch (w.type) {
          case F16:
            y[jj] = dot_f16_go(x, w.h + long(jj) * k, k);
            break;
          case Q8_0:
            y[jj] = dot_q8_go(x, w.q + long(jj) * (k / QK) * Q8BYTES, k);
            break;
          default:
            y[jj] = dot_f32_go(x, w.f + long(jj) * k, k);
        }
      }
    }
    if (bias)
      for (int jj = j; jj < std::min(j + 4, n); jj++) y[jj] += bias[jj];
  }
}

// quantU8Go, internal/kern/q8int.go:88-105 (bit-identical to quantU8avx,
// vnni_amd64.s:197-256, as q8int_test.go:9-35 checks). The byte kept here
// is the signed value q; the reference stores q+128 and subtracts 128·Σw
// per block (vnni_amd64.s:58-60), which gives the same integer sums.
inline void quant_q8_act(int8_t* q, float* sc, const float* x, int nb) {
  const float inv127 = bits_f32(0x3c010204);
  for (int b = 0; b < nb; b++) {
    const float* xs = x + b * QK;
    float amax = 0;
    for (int i = 0; i < QK; i++) amax = std::max(amax, std::fabs(xs[i]));
    sc[b] = amax * inv127;
    float id = amax != 0 ? 127.f / amax : 0.f;
    for (int i = 0; i < QK; i++) {
      double r = std::nearbyint(double(xs[i] * id));
      int32_t v = int32_t(r);
      q[b * QK + i] = int8_t(std::min(127, std::max(-128, v)));
    }
  }
}

// matmulQ8Int, internal/kern/q8int.go:148-223, with the tile arithmetic of
// q8tileEVEX (vnni_amd64.s:58-69, 103-123): per output, c starts at the
// bias (or 0) and each block b in order adds fma(float(s_b)·dw, da, c),
// where s_b is the exact int32 block dot. Rows are independent, so the
// reference's tiling and threading do not change any value.
inline void matmul_q8_int(float* c, int ldc, const float* a, int lda, int m, const Weight& w, const float* bias) {
  int n = w.rows, k = w.cols, nb = k / QK;
  std::vector<int8_t> qa((size_t)(k));
  std::vector<float> sa((size_t)(nb));
  long ldw = long(nb) * Q8BYTES;
  for (int i = 0; i < m; i++) {
    quant_q8_act(qa.data(), sa.data(), a + long(i) * lda, nb);
    for (int j = 0; j < n; j++) {
      const uint8_t* wr = w.q + j * ldw;
      float cv = bias ? bias[j] : 0.f;
      for (int b = 0; b < nb; b++) {
        const uint8_t* blk = wr + b * Q8BYTES;
        const int8_t* qs = (const int8_t*)(blk + 2);
        int32_t s = 0;
        for (int t = 0; t < QK; t++) s += int32_t(qa[b * QK + t]) * int32_t(qs[t]);
        float dw = f16_to_f32(uint16_t(blk[0] | blk[1] << 8));
        float t = float(s) * dw;
        cv = std::fma(t, sa[b], cv);
      }
      c[long(i) * ldc + j] = cv;
    }
  }
}

// Weight.ToQ8, internal/kern/kern.go:139-170: each block of 32 values
// scaled by its largest magnitude over 127 (float32 division), rounded half
// away from zero, the scale stored as f16 (the converter's rule,
// tools/convert_nemo.py:154-167).
inline void to_q8(uint8_t* out, const float* v, int rows, int cols) {
  int nb = cols / QK;
  for (int j = 0; j < rows; j++)
    for (int b = 0; b < nb; b++) {
      const float* xs = v + long(j) * cols + b * QK;
      uint8_t* blk = out + (long(j) * nb + b) * Q8BYTES;
      float amax = 0;
      for (int i = 0; i < QK; i++) amax = std::max(amax, std::fabs(xs[i]));
      float d = amax / 127.f;
      float id = d != 0 ? 1.f / d : 0.f;
      uint16_t h = f32_to_f16(d);
      blk[0] = uint8_t(h & 0xff);
      blk[1] = uint8_t(h >> 8);
      for (int i = 0; i < QK; i++) blk[2 + i] = uint8_t(int8_t(std::round(double(xs[i] * id))));
    }
}

// The fast mode (fast.h): the same values from SIMD kernels; false when
// this processor lacks them.
inline bool fast_on();
inline bool linear_fast(float* dst, const float* x, int m, const Weight& w, const float* bias);

// MatMul / Linear dispatch, internal/kern/kern.go:185-201 (the useInt
// case, intMinM = 2, q8int.go:137; m ≤ smallM always on the token loop).
inline void linear(float* dst, const float* x, int m, const Weight& w, const float* bias) {
  if (fast_on() && linear_fast(dst, x, m, w, bias)) return;
  if (m == 0 || w.rows == 0) return;
  if (w.type == Q8_0 && (w.dropped || m >= 2)) {
    matmul_q8_int(dst, w.rows, x, w.cols, m, w, bias);
    return;
  }
  for (int i = 0; i < m; i++) gemv_rows(dst + long(i) * w.rows, x + long(i) * w.cols, w, bias);
}

// kern.Add / addTo, internal/kern/mathx.go:104-109.
inline void add_to(float* dst, const float* src, int n) {
  for (int i = 0; i < n; i++) dst[i] += src[i];
}

// Argmax with a strict '>' from index 0 (conformer/rnnt.go:70-78,
// whisper/transcribe.go:462-466).
inline int argmax(const float* v, int n) {
  int best = 0;
  for (int i = 0; i < n; i++)
    if (v[i] > v[best]) best = i;
  return best;
}

}  // namespace orc
