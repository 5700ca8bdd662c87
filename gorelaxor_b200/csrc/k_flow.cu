// The float path of products with one row of activations per stream
// (internal/kern/gemm.go:195-259, kern.go:189 false branch): what the flow
// head, the input and end-of-speech projections take in the reference.
//
// Eight lanes compute one output exactly as one AVX row accumulator does:
//  * Q8_0 weight with rows kept (dot4q8avx, kernels_amd64.s:343-399): per
//    block, lane l forms q[l]·x[l] and three fused steps over q[8+l],
//    q[16+l], q[24+l], then fuses that into its accumulator by the block's
//    f16 scale; HSUM at the end;
//  * F32 weight (dot4f32avx, kernels_amd64.s:157-204): lane l keeps the two
//    8-lane accumulators for elements 16c+l and 16c+8+l, adds them, HSUM.
// The bias is added after the dot (gemm.go:251-255), then the epilogue the
// flow head applies to that output (FEpi).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

__global__ void k_tick(FrameIO* io) { io->frame += 1; }

// timeEmbed.embed's normalization and timeConds' mean (lm.go:75-103), one
// CTA per decode step, one thread per value; float64 sums reduced in a
// fixed order (see k_ln for why the order does not reach the output).
__global__ void k_time_norm(const float* y0, const float* y1, const float* a0, const float* a1, int N, float* tc) {
  __shared__ double sh[32];
  const int s = blockIdx.x, i = threadIdx.x, w = i >> 5, l = i & 31, nw = blockDim.x >> 5;
  float out[2];
  for (int k = 0; k < 2; k++) {
    const float* y = (k == 0 ? y0 : y1) + (size_t)s * N;
    const float v = i < N ? y[i] : 0.f;
    double t = i < N ? double(v) : 0.0;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    __syncthreads();
    if (l == 0) sh[w] = t;
    __syncthreads();
    double sum = 0;
    for (int j = 0; j < nw; j++) sum += sh[j];
    const double mean = sum / double(N);
    double q = i < N ? (double(v) - mean) * (double(v) - mean) : 0.0;
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    __syncthreads();
    if (l == 0) sh[w] = q;
    __syncthreads();
    double qs = 0;
    for (int j = 0; j < nw; j++) qs += sh[j];
    const float inv = float(1.0 / sqrt(qs / double(N - 1) + 1e-5));
    const float* al = k == 0 ? a0 : a1;
    out[k] = i < N ? __fmul_rn(v, __fmul_rn(al[i], inv)) : 0.f;
  }
  if (i < N) tc[(size_t)s * N + i] = __fdiv_rn(__fadd_rn(out[0], out[1]), 2.f);
}

__global__ void k_cond_step(const float* y0, const float* tc, float* sy, int N) {
  const int m = blockIdx.y, n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n < N) sy[(size_t)m * N + n] = silu_avx(__fadd_rn(y0[(size_t)m * N + n], tc[n]));
}

}  // namespace

void flow_kernels_init() { flin_kernels_init(); }

void launch_tick(FrameIO* io, cudaStream_t st) { k_tick<<<1, 1, 0, st>>>(io); }

void launch_time_norm(const float* y0, const float* y1, const float* a0, const float* a1, int N, int steps,
                      float* tc, cudaStream_t st) {
  k_time_norm<<<steps, ((N + 31) / 32) * 32, 0, st>>>(y0, y1, a0, a1, N, tc);
}

void launch_cond_step(const float* y0, const float* tc, float* sy, int M, int N, cudaStream_t st) {
  dim3 grid((N + 127) / 128, M);
  k_cond_step<<<grid, 128, 0, st>>>(y0, tc, sy, N);
}

}  // namespace grx
