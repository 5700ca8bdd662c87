// Device arithmetic shared by the token-loop kernels.
//
// Every kernel file is compiled with --fmad=false, so a multiply followed
// by an add stays two roundings unless the code asks for __fmaf_rn. That is
// how the reference's arithmetic is reproduced bit for bit: its Go code
// never fuses on amd64 (GOAMD64=v1), and its assembly fuses exactly where
// the helpers below call __fmaf_rn. Division and square root are the IEEE
// operations (nvcc's default -prec-div/-prec-sqrt).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace grx {

constexpr int QK = 32;  // values per Q8_0 block (internal/kern/kern.go:34)

__device__ __forceinline__ float bits_f(uint32_t u) { return __uint_as_float(u); }

// f16tab widening (internal/kern/f16.go:14-33): exact for every half,
// subnormals included, which is what cvt.f32.f16 does.
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// int32 → float32 for |s| < 2^22 in two full-rate operations: the integer
// is placed in the mantissa of 1.5·2^23 and the bias subtracted. Exact
// (the value is an integer below 2^22), so it equals the conversion
// VCVTDQ2PS does in the reference's tile (vnni_amd64.s:61-62). A Q8_0 block
// dot is at most 32·128·128 = 2^19 in magnitude.
__device__ __forceinline__ float i2f_small(int32_t s) {
  return __fsub_rn(__int_as_float(s + 0x4B400000), 12582912.0f);
}

// Packed float32 pairs in one 64-bit register (sm_100 .f32x2 operations):
// each half is the IEEE operation rounded once, so a pair operation gives
// exactly two scalar results. Values stay packed between operations so no
// moves are spent repacking them.
typedef uint64_t f2;
__device__ __forceinline__ f2 f2fma(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f2 f2mul(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 f2add(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 f2dup(float x) {
  f2 d;
  asm("mov.b64 %0, {%1, %1};" : "=l"(d) : "f"(x));
  return d;
}
__device__ __forceinline__ f2 f2make(float lo, float hi) {
  f2 d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ float f2lo(f2 v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float f2hi(f2 v) { return __uint_as_float(uint32_t(v >> 32)); }

// The float whose bits are 1.5·2^23: an int32 s with |s| < 2^22 added to its
// bit pattern gives the float 1.5·2^23 + s exactly.
constexpr int32_t MAGIC_BITS = 0x4B400000;
constexpr float MAGIC = 12582912.0f;

// EXP8, internal/kern/kernels_amd64.s:238-257 (constants :217-233): the
// reference's vector e^x, lane by lane.
__device__ __forceinline__ float exp_avx(float x) {
  x = fmaxf(x, -87.f);
  x = fminf(x, 88.f);
  float n = rintf(__fmul_rn(x, bits_f(0x3fb8aa3b)));
  float r = __fmaf_rn(-n, bits_f(0x3f317200), x);
  r = __fmaf_rn(-n, bits_f(0x35bfbe8e), r);
  float p = __fmaf_rn(bits_f(0x3ab60b61), r, bits_f(0x3c088889));
  p = __fmaf_rn(r, p, bits_f(0x3d2aaaab));
  p = __fmaf_rn(r, p, bits_f(0x3e2aaaab));
  p = __fmaf_rn(r, p, 0.5f);
  p = __fmaf_rn(r, p, 1.f);
  p = __fmaf_rn(r, p, 1.f);
  int ni = __float2int_rn(n);
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

// expf, internal/kern/mathx.go:7-33: the reference's scalar e^x (used for
// the tails of its vector helpers and by its scalar callers).
__device__ __forceinline__ float expf_go(float x) {
  if (x < -87.f) return 0.f;
  if (x > 88.f) return __int_as_float(0x7f800000);
  float t = __fadd_rn(__fmul_rn(x, 1.4426950408889634f), 0.5f);
  int ni = __float2int_rz(t);
  if (float(ni) > t) ni--;
  float n = float(ni);
  float r = __fsub_rn(__fsub_rn(x, __fmul_rn(n, 0.693145751953125f)), __fmul_rn(n, 1.428606765330187e-06f));
  float p = __fadd_rn(__fmul_rn(float(1.0 / 720), r), float(1.0 / 120));
  p = __fadd_rn(__fmul_rn(p, r), float(1.0 / 24));
  p = __fadd_rn(__fmul_rn(p, r), float(1.0 / 6));
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.f);
  p = __fadd_rn(__fmul_rn(p, r), 1.f);
  if (ni < -126) return __fmul_rn(__fmul_rn(p, __int_as_float((ni + 127 + 64) << 23)), 5.421010862427522e-20f);
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

// geluAVX, internal/kern/kernels_amd64.s:301-339.
__device__ __forceinline__ float gelu_avx(float v) {
  float u = __fmul_rn(v, v);
  u = __fmaf_rn(bits_f(0x3d372713), u, 1.f);
  u = __fmul_rn(v, u);
  u = __fmul_rn(bits_f(0x3f4c422a), u);
  u = fminf(u, 9.f);
  u = fmaxf(u, -9.f);
  float e = exp_avx(__fadd_rn(u, u));
  e = __fadd_rn(e, 1.f);
  e = __fdiv_rn(2.f, e);
  e = __fsub_rn(1.f, e);
  e = __fadd_rn(e, 1.f);
  e = __fmul_rn(e, v);
  return __fmul_rn(e, 0.5f);
}

// gelu, internal/kern/mathx.go:36-52.
__device__ __forceinline__ float gelu_go(float v) {
  const float c = float(0.7978845608028654);
  float u = __fmul_rn(__fmul_rn(c, v), __fadd_rn(1.f, __fmul_rn(__fmul_rn(0.044715f, v), v)));
  float t;
  if (u > 9.f)
    t = 1.f;
  else if (u < -9.f)
    t = -1.f;
  else
    t = __fsub_rn(1.f, __fdiv_rn(2.f, __fadd_rn(expf_go(__fmul_rn(2.f, u)), 1.f)));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.f, t));
}

// siluAVX, internal/kern/kernels_amd64.s:441-459.
__device__ __forceinline__ float silu_avx(float v) {
  float e = exp_avx(__fsub_rn(0.f, v));
  return __fdiv_rn(v, __fadd_rn(e, 1.f));
}

// siluGo, internal/kern/mathx.go:115-119.
__device__ __forceinline__ float silu_go(float v) { return __fdiv_rn(v, __fadd_rn(1.f, expf_go(-v))); }

// sigmoid, conformer/encoder.go:13.
__device__ __forceinline__ float sigmoid_go(float v) { return __fdiv_rn(1.f, __fadd_rn(1.f, expf_go(-v))); }

// HSUM (internal/kern/kernels_amd64.s:92-97) over an 8-lane group held by
// lanes g..g+7 of a warp (g a multiple of 8): the result lands in lane g.
__device__ __forceinline__ float hsum8_lanes(float a) {
  float x = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 4));   // lanes 0-3: a_l + a_{l+4}
  float y = __fadd_rn(x, __shfl_down_sync(0xffffffffu, x, 1));   // lanes 0, 2: (x0+x1), (x2+x3)
  return __fadd_rn(y, __shfl_down_sync(0xffffffffu, y, 2));      // lane 0
}

// Q8_0 rounding of one 32-value block held one value per lane of a warp
// (quantU8, internal/kern/q8int.go:88-105; the kept byte is the signed
// value, see the tile comment in vnni_amd64.s:5-13). Returns the lane's
// int8 and writes the block scale through *sc in every lane.
__device__ __forceinline__ int8_t quant_lane(float v, float* sc) {
  float a = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  *sc = __fmul_rn(a, bits_f(0x3c010204));
  float id = a != 0.f ? __fdiv_rn(127.f, a) : 0.f;
  int q = __float2int_rn(__fmul_rn(v, id));
  q = min(127, max(-128, q));
  return int8_t(q);
}

// The same rounding for a value whose block is spread over `width` lanes
// holding `per` values each (amax already reduced by the caller).
__device__ __forceinline__ int8_t quant_val(float v, float amax) {
  float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
  int q = __float2int_rn(__fmul_rn(v, id));
  q = min(127, max(-128, q));
  return int8_t(q);
}

__device__ __forceinline__ float quant_scale(float amax) { return __fmul_rn(amax, bits_f(0x3c010204)); }

}  // namespace grx
