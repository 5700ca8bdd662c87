// Single-query attention over the KV cache, one CTA per (stream, head):
// transformer.attend for one query, pockettts/nn.go:200-243, with the
// reference's arithmetic kept value for value:
//  * scores: dot4f32avx order for keys in whole groups of four
//    (kernels_amd64.s:157-204 — lane l of a 16-lane half warp runs the
//    fused chain over elements 16c+l, then the AVX lane pairs and HSUM are
//    replayed with shuffles), dotF32Go order for the last nk%4 keys
//    (gemm.go:294-308), then ·1/√64;
//  * softmax: max, expSub (EXP8 with 8 running lane sums and HSUM for the
//    first nk&~7 scores, scalar expf for the rest, kernels_amd64.go:107-117),
//    scores times 1/Σ;
//  * values: o = fma(w_j, v_j, o) for j in order, skipping w_j == 0
//    (AddScaled/axpyAVX, nn.go:232-236) — one thread per output value runs
//    that chain, the warp reading each value row coalesced.
// The output is also rounded to Q8_0 blocks here (a head's 64 values are
// two whole blocks) for the attn_out product that follows.
//
// The cache is laid out per head, [stream][layer][k|v][head][pos][64]
// float32, so a head's keys are one contiguous run that the CTA streams
// from HBM once: the kernel is bound by those bytes.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

constexpr int HD = 64;
constexpr uint32_t FULL = 0xffffffffu;

__global__ void __launch_bounds__(64) k_attn(AttnArgs a) {
  extern __shared__ float sc[];  // [cap] scores, then weights
  __shared__ float red[4];
  const int h = blockIdx.x, m = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = a.pos[m] + 1;
  const size_t kbase = ((((size_t)m * a.layers + a.layer) * 2 + 0) * a.heads + h) * (size_t)a.cap * HD;
  const size_t vbase = ((((size_t)m * a.layers + a.layer) * 2 + 1) * a.heads + h) * (size_t)a.cap * HD;
  const float* K = a.kv + kbase;
  const float* V = a.kv + vbase;
  const float* q = a.q + (size_t)m * a.d + h * HD;
  unsigned long long* ts = nullptr;
  if (a.io && a.io->attn_ts)
    ts = a.io->attn_ts + (((size_t)a.io->frame * a.layers + a.layer) * a.io->parts + a.io->part) * 2;
  if (ts && tid == 0) {
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    atomicMin(ts, t0);
  }

  // --- scores, keys in groups of four (two keys per warp pass) ---
  const int half = lane >> 4, l = lane & 15;
  const float q0 = q[l], q1 = q[16 + l], q2 = q[32 + l], q3 = q[48 + l];
  const int nk4 = nk & ~3;
  constexpr int U = 8;  // key pairs in flight per warp
  for (int p0 = warp * U; 2 * p0 < nk4; p0 += 2 * U) {
    float k[U][4];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = 2 * (p0 + u) + half;
      if (j < nk4) {
        const float* kr = K + (size_t)j * HD + l;
        k[u][0] = kr[0];
        k[u][1] = kr[16];
        k[u][2] = kr[32];
        k[u][3] = kr[48];
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = 2 * (p0 + u) + half;
      float acc = __fmaf_rn(q0, k[u][0], 0.f);
      acc = __fmaf_rn(q1, k[u][1], acc);
      acc = __fmaf_rn(q2, k[u][2], acc);
      acc = __fmaf_rn(q3, k[u][3], acc);
      // lanes 0-7 of each half: A_l + B_l (VADDPS Y8, Y4, Y4), then HSUM.
      const float p = __fadd_rn(acc, __shfl_down_sync(FULL, acc, 8));
      const float s = hsum8_lanes(p);
      if (l == 0 && j < nk4) sc[j] = __fmul_rn(s, 0.125f);
    }
  }
  // --- the last nk%4 keys: dotF32Go (four strided unfused sums) ---
  if (warp == 0) {
    for (int j = nk4; j < nk; j++) {
      float s = 0.f;
      if (lane < 4)
        for (int i = lane; i < HD; i += 4) s = __fadd_rn(s, __fmul_rn(q[i], K[(size_t)j * HD + i]));
      const float s1 = __shfl_sync(FULL, s, 1), s2 = __shfl_sync(FULL, s, 2), s3 = __shfl_sync(FULL, s, 3);
      if (lane == 0) sc[j] = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3), 0.125f);
    }
  }
  __syncthreads();

  // --- softmax ---
  float mx = -__int_as_float(0x7f800000);
  for (int j = tid; j < nk; j += 64) mx = fmaxf(mx, sc[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = fmaxf(red[0], red[1]);
  const int n8 = nk & ~7;
  for (int j = tid; j < nk; j += 64) {
    const float x = __fsub_rn(sc[j], mx);
    sc[j] = j < n8 ? exp_avx(x) : expf_go(x);
  }
  __syncthreads();
  if (warp == 0) {
    float part = 0.f;
    if (lane < 8)
      for (int c = lane; c < n8; c += 8) part = __fadd_rn(part, sc[c]);
    const float savx = hsum8_lanes(part);
    if (lane == 0) {
      float tail = 0.f;
      for (int j = n8; j < nk; j++) tail = __fadd_rn(tail, sc[j]);
      red[2] = __fdiv_rn(1.f, __fadd_rn(savx, tail));
    }
  }
  __syncthreads();
  const float inv = red[2];
  for (int j = tid; j < nk; j += 64) sc[j] = __fmul_rn(sc[j], inv);
  __syncthreads();

  // --- values: thread tid owns output value tid, chain over j in order ---
  float o = 0.f;
  const float* vp = V + tid;
  constexpr int UV = 16;
  int j = 0;
  for (; j + UV <= nk; j += UV) {
    float v[UV];
#pragma unroll
    for (int u = 0; u < UV; u++) v[u] = vp[(size_t)(j + u) * HD];
#pragma unroll
    for (int u = 0; u < UV; u++) {
      const float w = sc[j + u];
      if (w != 0.f) o = __fmaf_rn(w, v[u], o);
    }
  }
  for (; j < nk; j++) {
    const float w = sc[j];
    if (w != 0.f) o = __fmaf_rn(w, vp[(size_t)j * HD], o);
  }
  if (a.out) a.out[(size_t)m * a.d + h * HD + tid] = o;
  float s;
  const int8_t qv = quant_lane(o, &s);
  a.q8[(size_t)m * a.d + h * HD + tid] = qv;
  if (lane == 0) a.q8s[(size_t)m * (a.d / QK) + h * 2 + warp] = make_float2(s, s);
  if (ts) {
    __syncthreads();
    if (tid == 0) {
      unsigned long long t1;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
      atomicMax(ts + 1, t1);
    }
  }
}

}  // namespace

void launch_attn(const AttnArgs& a, int M, cudaStream_t st) {
  dim3 grid(a.heads, M);
  k_attn<<<grid, 64, size_t(a.cap) * sizeof(float), st>>>(a);
}

}  // namespace grx
