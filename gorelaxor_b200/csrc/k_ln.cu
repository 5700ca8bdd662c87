// LayerNorm (pockettts/nn.go:27-49) fused with what consumes it: Q8_0
// rounding for the next int8 product (LN_Q8), a plain float32 row
// (out_norm, LN_F32), or the flow head's adaLN modulation
// n·(1+scale)+shift (pockettts/lm.go:140-143, 153-156; LN_MOD).
//
// One CTA per row, four values per thread. The mean and variance are
// float64 sums as in the reference; the reduction order differs from its
// sequential loop, which changes a float64 sum of float32 inputs by at most
// a few float64 ulps, far below what reaches a float32 output.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

__device__ __forceinline__ double block_sum(double v, double* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  double t = 0;
  for (int i = 0; i < nw; i++) t += sh[i];
  return t;
}

__global__ void k_ln(LnArgs a, int D) {
  __shared__ double sh[32];
  int m = blockIdx.x, t = threadIdx.x;
  const float4 v4 = reinterpret_cast<const float4*>(a.x + (size_t)m * D)[t];
  float v[4] = {v4.x, v4.y, v4.z, v4.w};
  double s = ((double(v[0]) + double(v[1])) + double(v[2])) + double(v[3]);
  double mean = block_sum(s, sh) / double(D);
  double q = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    double dd = double(v[i]) - mean;
    q += dd * dd;
  }
  double var = block_sum(q, sh);
  double inv = 1.0 / sqrt(var / double(D) + a.eps);
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    o[i] = float((double(v[i]) - mean) * inv);
    if (a.w) o[i] = __fadd_rn(__fmul_rn(o[i], a.w[4 * t + i]), a.b[4 * t + i]);
  }
  if (a.mode == LN_F32) {
    reinterpret_cast<float4*>(a.y + (size_t)m * D)[t] = make_float4(o[0], o[1], o[2], o[3]);
    if (!a.eosw) return;
    // eos = dotF32Go(y, w) + b: four strided unfused sums over the row
    // (gemm.go:294-308), the row and the weight staged on chip.
    __shared__ float srow[4096], sw[4096];
    reinterpret_cast<float4*>(srow)[t] = make_float4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<float4*>(sw)[t] = reinterpret_cast<const float4*>(a.eosw)[t];
    __syncthreads();
    if (t < 32) {
      const int D4 = D & ~3;
      float s = 0.f;
      if (t < 4)
        for (int i = t; i < D4; i += 4) s = __fadd_rn(s, __fmul_rn(srow[i], sw[i]));
      const float s1 = __shfl_sync(0xffffffffu, s, 1), s2 = __shfl_sync(0xffffffffu, s, 2),
                  s3 = __shfl_sync(0xffffffffu, s, 3);
      if (t == 0) {
        for (int i = D4; i < D; i++) s = __fadd_rn(s, __fmul_rn(srow[i], sw[i]));
        const float e = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3), a.eosb);
        if (a.eos) a.eos[m] = e;
        if (a.io && a.io->eos) a.io->eos[(size_t)a.io->frame * a.io->rows + a.io->row0 + m] = e;
        if (a.pos) a.pos[m] += 1;
      }
    }
    return;
  }
  if (a.mode == LN_MOD) {
    const float* sh_ = a.mod + (size_t)m * a.ldmod + a.shift;
    const float* sc_ = a.mod + (size_t)m * a.ldmod + a.scale;
#pragma unroll
    for (int i = 0; i < 4; i++) o[i] = __fadd_rn(__fmul_rn(o[i], __fadd_rn(1.f, sc_[4 * t + i])), sh_[4 * t + i]);
    reinterpret_cast<float4*>(a.y + (size_t)m * D)[t] = make_float4(o[0], o[1], o[2], o[3]);
    return;
  }
  // LN_Q8: a 32-value block is eight consecutive threads of one warp.
  float amax = fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])), fmaxf(fabsf(o[2]), fabsf(o[3])));
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) packed |= uint32_t(uint8_t(quant_val(o[i], amax))) << (8 * i);
  reinterpret_cast<uint32_t*>(a.q8 + (size_t)m * D)[t] = packed;
  if ((t & 7) == 0) {
    const float sc = quant_scale(amax);
    a.q8s[(size_t)m * (D / QK) + t / 8] = make_float2(sc, sc);
  }
}

// Plain Q8_0 rounding of float rows (the int8 path's quantU8 step alone).
__global__ void k_quant(const float* x, int K, int8_t* q, float2* s) {
  int m = blockIdx.x;  // rows on x: up to 2^31 − 1 of them
  int i = blockIdx.y * blockDim.x + threadIdx.x;  // one value per thread
  if (i >= K) return;
  float v = x[(size_t)m * K + i];
  float sc;
  int8_t qq = quant_lane(v, &sc);
  q[(size_t)m * K + i] = qq;
  if ((threadIdx.x & 31) == 0) s[(size_t)m * (K / QK) + i / QK] = make_float2(sc, sc);
}

}  // namespace

void launch_ln(const LnArgs& a, int M, int D, cudaStream_t st) { k_ln<<<M, D / 4, 0, st>>>(a, D); }

void launch_quant(const float* x, int M, int K, int8_t* q, float2* s, cudaStream_t st) {
  dim3 g(M, (K + 255) / 256);
  k_quant<<<g, 256, 0, st>>>(x, K, q, s);
}

}  // namespace grx
