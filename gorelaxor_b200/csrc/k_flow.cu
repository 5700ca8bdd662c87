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

// Rows past the last whole group of four take the scalar Go dots in the
// reference (gemm.go:239-249): dotQ8Go (kern.go:249-266) or dotF32Go
// (gemm.go:294-308). Run serially by the row's first lane.
__device__ float tail_row(const FArgs& a, const float* x, int n) {
  if (a.wq) {
    const int nb = a.K / QK;
    const int8_t* q = a.wq + (size_t)n * a.K;
    float s = 0.f;
    for (int b = 0; b < nb; b++) {
      const float d = h2f(a.wd[(size_t)n * nb + b]);
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int i = 0; i < QK; i += 4) {
        a0 = __fadd_rn(a0, __fmul_rn(x[b * QK + i], float(q[b * QK + i])));
        a1 = __fadd_rn(a1, __fmul_rn(x[b * QK + i + 1], float(q[b * QK + i + 1])));
        a2 = __fadd_rn(a2, __fmul_rn(x[b * QK + i + 2], float(q[b * QK + i + 2])));
        a3 = __fadd_rn(a3, __fmul_rn(x[b * QK + i + 3], float(q[b * QK + i + 3])));
      }
      s = __fadd_rn(s, __fmul_rn(d, __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3)));
    }
    return s;
  }
  const float* w = a.wf + (size_t)n * a.K;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int i = 0;
  for (; i + 4 <= a.K; i += 4) {
    s0 = __fadd_rn(s0, __fmul_rn(x[i], w[i]));
    s1 = __fadd_rn(s1, __fmul_rn(x[i + 1], w[i + 1]));
    s2 = __fadd_rn(s2, __fmul_rn(x[i + 2], w[i + 2]));
    s3 = __fadd_rn(s3, __fmul_rn(x[i + 3], w[i + 3]));
  }
  for (; i < a.K; i++) s0 = __fadd_rn(s0, __fmul_rn(x[i], w[i]));
  return __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
}

__global__ void __launch_bounds__(256) k_flin(FArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = lane >> 3, l = lane & 7;
  const int n = blockIdx.x * 32 + warp * 4 + grp;
  const int m = blockIdx.y;
  const bool valid = n < a.N;
  const int nn = valid ? n : 0;
  const float* x = a.x_noise ? a.io->noise + ((size_t)a.io->frame * gridDim.y + m) * a.ldx : a.x + (size_t)m * a.ldx;
  float r;
  if (a.wq) {
    const int nb = a.K / QK;
    const int8_t* wr = a.wq + (size_t)nn * a.K;
    const uint16_t* dr = a.wd + (size_t)nn * nb;
    float acc = 0.f;
    for (int b = 0; b < nb; b++) {
      const int8_t* qb = wr + b * QK + l;
      const float* xb = x + b * QK + l;
      float y = __fmul_rn(float(qb[0]), xb[0]);
      y = __fmaf_rn(float(qb[8]), xb[8], y);
      y = __fmaf_rn(float(qb[16]), xb[16], y);
      y = __fmaf_rn(float(qb[24]), xb[24], y);
      acc = __fmaf_rn(y, h2f(dr[b]), acc);
    }
    r = hsum8_lanes(acc);
  } else {
    const float* wr = a.wf + (size_t)nn * a.K;
    float s = 0.f, t = 0.f;
    for (int c = 0; c < a.K; c += 16) {
      s = __fmaf_rn(x[c + l], wr[c + l], s);
      t = __fmaf_rn(x[c + 8 + l], wr[c + 8 + l], t);
    }
    r = hsum8_lanes(__fadd_rn(s, t));
  }
  if (l != 0 || !valid) return;
  if (n >= (a.N & ~3)) r = tail_row(a, x, n);
  float v = a.bias ? __fadd_rn(r, a.bias[n]) : r;
  float* yp = a.y + (size_t)m * a.ldy + n;
  switch (a.epi) {
    case FE_COND:
      *yp = silu_avx(__fadd_rn(v, a.aux[n]));
      break;
    case FE_SILU:
      *yp = silu_avx(v);
      break;
    case FE_GATE:
      *yp = __fadd_rn(*yp, __fmul_rn(a.aux[(size_t)m * a.ldaux + n], v));
      break;
    case FE_LATENT: {
      const float* aux = a.aux_noise ? a.io->noise + (size_t)a.io->frame * gridDim.y * a.ldaux : a.aux;
      const float cur = __fadd_rn(aux[(size_t)m * a.ldaux + n], __fdiv_rn(v, a.steps));
      *yp = cur;
      const float sc = __fadd_rn(__fmul_rn(cur, a.stdv[n]), a.mean[n]);
      if (a.out2) a.out2[(size_t)m * a.ldy + n] = cur;
      if (a.out3) a.out3[(size_t)m * a.ldy + n] = sc;
      if (a.io_out) {
        const size_t o = ((size_t)a.io->frame * gridDim.y + m) * a.ldy + n;
        if (a.io->latent) a.io->latent[o] = cur;
        if (a.io->scaled) a.io->scaled[o] = sc;
      }
      break;
    }
    default:
      *yp = v;
  }
}

// eos: gemvRows with one weight row takes the scalar tail, dotF32Go
// (four strided unfused sums, gemm.go:294-308), then + eos bias (lm.go:193-
// 194). Also moves the stream's position on by the frame just made.
__global__ void k_eos(const float* x, const float* w, float b, int K, const FrameIO* io, float* eos, int* pos) {
  const int m = blockIdx.x, lane = threadIdx.x;
  const float* xr = x + (size_t)m * K;
  const int K4 = K & ~3;
  float s = 0.f;
  if (lane < 4)
    for (int i = lane; i < K4; i += 4) s = __fadd_rn(s, __fmul_rn(xr[i], w[i]));
  const float s1 = __shfl_sync(0xffffffffu, s, 1), s2 = __shfl_sync(0xffffffffu, s, 2),
              s3 = __shfl_sync(0xffffffffu, s, 3);
  if (lane == 0) {
    for (int i = K4; i < K; i++) s = __fadd_rn(s, __fmul_rn(xr[i], w[i]));
    const float e = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3), b);
    if (eos) eos[m] = e;
    if (io && io->eos) io->eos[(size_t)io->frame * gridDim.x + m] = e;
    pos[m] += 1;
  }
}

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

void launch_flin(const FArgs& a, int M, cudaStream_t st) {
  dim3 grid((a.N + 31) / 32, M);
  k_flin<<<grid, 256, 0, st>>>(a);
}

void launch_eos(const float* x, const float* w, float b, int K, const FrameIO* io, float* eos, int* pos, int M,
                cudaStream_t st) {
  k_eos<<<M, 32, 0, st>>>(x, w, b, K, io, eos, pos);
}

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
