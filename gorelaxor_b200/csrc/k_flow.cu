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

constexpr int MT = 16;  // streams per CTA: each weight byte is loaded once for all of them

// The CTA's activations in shared memory, stream-minor so that one 16-byte
// load gives four streams' values of element k: x[m][k] sits at
// k·MT + 4·((m/4) ^ (k mod 4)) + m mod 4 (the XOR spreads the stores of
// consecutive k over the banks).
__device__ __forceinline__ int sx_at(int k, int m) { return k * MT + 4 * ((m >> 2) ^ (k & 3)) + (m & 3); }

// Rows past the last whole group of four take the scalar Go dots in the
// reference (gemm.go:239-249): dotQ8Go (kern.go:249-266) or dotF32Go
// (gemm.go:294-308). Run serially by the row's first lane.
__device__ float tail_row(const FArgs& a, const float* sx, int m, int n) {
  if (a.wq) {
    const int nb = a.K / QK;
    const int8_t* q = a.wq + (size_t)n * a.K;
    float s = 0.f;
    for (int b = 0; b < nb; b++) {
      const float d = h2f(a.wd[(size_t)n * nb + b]);
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int i = 0; i < QK; i += 4) {
        const int k = b * QK + i;
        a0 = __fadd_rn(a0, __fmul_rn(sx[sx_at(k, m)], float(q[k])));
        a1 = __fadd_rn(a1, __fmul_rn(sx[sx_at(k + 1, m)], float(q[k + 1])));
        a2 = __fadd_rn(a2, __fmul_rn(sx[sx_at(k + 2, m)], float(q[k + 2])));
        a3 = __fadd_rn(a3, __fmul_rn(sx[sx_at(k + 3, m)], float(q[k + 3])));
      }
      s = __fadd_rn(s, __fmul_rn(d, __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3)));
    }
    return s;
  }
  const float* w = a.wf + (size_t)n * a.K;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int i = 0;
  for (; i + 4 <= a.K; i += 4) {
    s0 = __fadd_rn(s0, __fmul_rn(sx[sx_at(i, m)], w[i]));
    s1 = __fadd_rn(s1, __fmul_rn(sx[sx_at(i + 1, m)], w[i + 1]));
    s2 = __fadd_rn(s2, __fmul_rn(sx[sx_at(i + 2, m)], w[i + 2]));
    s3 = __fadd_rn(s3, __fmul_rn(sx[sx_at(i + 3, m)], w[i + 3]));
  }
  for (; i < a.K; i++) s0 = __fadd_rn(s0, __fmul_rn(sx[sx_at(i, m)], w[i]));
  return __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
}

__device__ __forceinline__ void flin_out(const FArgs& a, int m, int n, float r) {
  const float v = a.bias ? __fadd_rn(r, a.bias[n]) : r;
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
      const int M = a.M;
      const float* aux = a.aux_noise ? a.io->noise + (size_t)a.io->frame * M * a.ldaux : a.aux;
      const float cur = __fadd_rn(aux[(size_t)m * a.ldaux + n], __fdiv_rn(v, a.steps));
      *yp = cur;
      const float sc = __fadd_rn(__fmul_rn(cur, a.stdv[n]), a.mean[n]);
      if (a.out2) a.out2[(size_t)m * a.ldy + n] = cur;
      if (a.out3) a.out3[(size_t)m * a.ldy + n] = sc;
      if (a.io_out) {
        const size_t o = ((size_t)a.io->frame * M + m) * a.ldy + n;
        if (a.io->latent) a.io->latent[o] = cur;
        if (a.io->scaled) a.io->scaled[o] = sc;
      }
      break;
    }
    default:
      *yp = v;
  }
}

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(uint32_t(__cvta_generic_to_shared(dst))), "l"(src));
}

// Shared memory of k_flin: the MT streams' activations (see sx_at), then the
// CTA's 64 weight rows (row stride padded by 16 bytes so the row groups of a
// warp read different banks), then their Q8_0 block scales.
constexpr int FR = 1;               // weight rows per 8-lane group
constexpr int FROWS = 32 * FR;     // weight rows per CTA: 8 warps × 4 groups × FR rows
__host__ __device__ constexpr int flin_wstride(int K, bool q8) { return (q8 ? K : 4 * K) + 16; }
__host__ __device__ constexpr size_t flin_smem(int K, bool q8) {
  return size_t(MT) * K * 4 + size_t(FROWS) * flin_wstride(K, q8) + (q8 ? size_t(FROWS) * (K / QK) * 2 : 0);
}

// Tile: 32·FR output rows (8 warps × 4 groups of 8 lanes × FR rows) × MT
// streams. A lane keeps its accumulators for its rows and all MT streams as
// packed float pairs and steps them with f32x2 operations (each half is the
// scalar IEEE operation).
__global__ void __launch_bounds__(256) k_flin(FArgs a) {
  extern __shared__ __align__(16) uint8_t fsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = lane >> 3, l = lane & 7;
  const int row0 = (warp * 4 + grp) * FR, n0 = blockIdx.x * FROWS;
  const int m0 = blockIdx.y * MT, mt = min(MT, a.M - m0);
  const int K = a.K;
  const bool q8 = a.wq != nullptr;
  float* sx = reinterpret_cast<float*>(fsm);
  uint8_t* sw = fsm + size_t(MT) * K * 4;
  const int ws = flin_wstride(K, q8);
  uint16_t* sd = reinterpret_cast<uint16_t*>(sw + size_t(FROWS) * ws);
  const int nrows = min(FROWS, a.N - n0);
  {  // weight rows (and scales) by async copies, overlapping the x staging
    const int rb = q8 ? K : 4 * K, cpr = rb / 16;
    const uint8_t* src = q8 ? reinterpret_cast<const uint8_t*>(a.wq + (size_t)n0 * K)
                            : reinterpret_cast<const uint8_t*>(a.wf + (size_t)n0 * K);
    for (int i = threadIdx.x; i < nrows * cpr; i += blockDim.x) {
      const int r = i / cpr, c = i - r * cpr;
      cp16(sw + r * ws + c * 16, src + (size_t)r * rb + c * 16);
    }
    if (q8) {
      const int nb = K / QK, bytes = nrows * nb * 2;
      const uint8_t* ds = reinterpret_cast<const uint8_t*>(a.wd + (size_t)n0 * nb);
      for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x)
        cp16(reinterpret_cast<uint8_t*>(sd) + i * 16, ds + i * 16);
      for (int i = (bytes / 16) * 16 + threadIdx.x; i < bytes; i += blockDim.x)
        reinterpret_cast<uint8_t*>(sd)[i] = ds[i];
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }
  const float* xsrc = a.x_noise ? a.io->noise + (size_t)a.io->frame * a.M * a.ldx : a.x;
  // x: a thread reads four streams' value of one k (coalesced along k) and
  // stores them as one 16-byte group.
  for (int i = threadIdx.x; i < K * (MT / 4); i += blockDim.x) {
    const int k = i % K, q4 = i / K;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int m = 4 * q4 + j;
      v[j] = m < mt ? xsrc[(size_t)(m0 + m) * a.ldx + k] : 0.f;
    }
    *reinterpret_cast<float4*>(&sx[sx_at(k, 4 * q4)]) = make_float4(v[0], v[1], v[2], v[3]);
  }
  asm volatile("cp.async.wait_all;\n" ::);
  __syncthreads();
  f2 acc[FR][MT / 2];
#pragma unroll
  for (int r = 0; r < FR; r++)
#pragma unroll
    for (int p = 0; p < MT / 2; p++) acc[r][p] = 0;
  if (q8) {
    const int nb = K / QK;
    for (int b = 0; b < nb; b++) {
      const int k = b * QK + l;
      f2 Q[FR][4], D[FR];
#pragma unroll
      for (int r = 0; r < FR; r++) {
        const int8_t* wr = reinterpret_cast<const int8_t*>(sw + (row0 + r) * ws);
#pragma unroll
        for (int i = 0; i < 4; i++) Q[r][i] = f2dup(float(wr[k + 8 * i]));
        D[r] = f2dup(h2f(sd[(row0 + r) * nb + b]));
      }
#pragma unroll
      for (int g4 = 0; g4 < MT / 4; g4++) {
        f2 X[4][2];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const f2* xp = reinterpret_cast<const f2*>(&sx[sx_at(k + 8 * i, 4 * g4)]);
          X[i][0] = xp[0];
          X[i][1] = xp[1];
        }
#pragma unroll
        for (int r = 0; r < FR; r++)
#pragma unroll
          for (int h = 0; h < 2; h++) {
            f2 y = f2mul(Q[r][0], X[0][h]);
            y = f2fma(Q[r][1], X[1][h], y);
            y = f2fma(Q[r][2], X[2][h], y);
            y = f2fma(Q[r][3], X[3][h], y);
            acc[r][2 * g4 + h] = f2fma(y, D[r], acc[r][2 * g4 + h]);
          }
      }
    }
  } else {
    f2 t[FR][MT / 2];
#pragma unroll
    for (int r = 0; r < FR; r++)
#pragma unroll
      for (int p = 0; p < MT / 2; p++) t[r][p] = 0;
    for (int c = 0; c < K; c += 16) {
      f2 W[FR][2];
#pragma unroll
      for (int r = 0; r < FR; r++) {
        const float* wr = reinterpret_cast<const float*>(sw + (row0 + r) * ws);
        W[r][0] = f2dup(wr[c + l]);
        W[r][1] = f2dup(wr[c + 8 + l]);
      }
#pragma unroll
      for (int g4 = 0; g4 < MT / 4; g4++) {
        const f2* x0 = reinterpret_cast<const f2*>(&sx[sx_at(c + l, 4 * g4)]);
        const f2* x1 = reinterpret_cast<const f2*>(&sx[sx_at(c + 8 + l, 4 * g4)]);
        const f2 X0[2] = {x0[0], x0[1]}, X1[2] = {x1[0], x1[1]};
#pragma unroll
        for (int r = 0; r < FR; r++)
#pragma unroll
          for (int h = 0; h < 2; h++) {
            acc[r][2 * g4 + h] = f2fma(X0[h], W[r][0], acc[r][2 * g4 + h]);
            t[r][2 * g4 + h] = f2fma(X1[h], W[r][1], t[r][2 * g4 + h]);
          }
      }
    }
#pragma unroll
    for (int r = 0; r < FR; r++)
#pragma unroll
      for (int p = 0; p < MT / 2; p++) acc[r][p] = f2add(acc[r][p], t[r][p]);
  }
#pragma unroll
  for (int r = 0; r < FR; r++) {
    float v[MT];
#pragma unroll
    for (int p = 0; p < MT / 2; p++) {
      v[2 * p] = hsum8_lanes(f2lo(acc[r][p]));
      v[2 * p + 1] = hsum8_lanes(f2hi(acc[r][p]));
    }
    const int n = n0 + row0 + r;
    if (l != 0 || row0 + r >= nrows) continue;
    const bool tail = n >= (a.N & ~3);
#pragma unroll
    for (int m = 0; m < MT; m++)
      if (m < mt) flin_out(a, m0 + m, n, tail ? tail_row(a, sx, m, n) : v[m]);
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

void launch_flin(const FArgs& a0, int M, cudaStream_t st) {
  FArgs a = a0;
  a.M = M;
  dim3 grid((a.N + FROWS - 1) / FROWS, (M + MT - 1) / MT);
  k_flin<<<grid, 256, flin_smem(a.K, a.wq != nullptr), st>>>(a);
}

// The float path stages MT rows of K activations and 32·FR weight rows:
// with F32 weights K up to 1024 fits the 227 KB a CTA may opt into.
constexpr int FLIN_MAX_K = 1024;

void flow_kernels_init() {
  const size_t a = flin_smem(FLIN_MAX_K, false), b = flin_smem(2048, true);
  cudaFuncSetAttribute(k_flin, cudaFuncAttributeMaxDynamicSharedMemorySize, int(a > b ? a : b));
}

// Q8_0 weights take less shared memory per K: up to 2048 fits (~200 KB).
int flin_max_k_q8() { return 2048; }

int flin_max_k() { return FLIN_MAX_K; }

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
