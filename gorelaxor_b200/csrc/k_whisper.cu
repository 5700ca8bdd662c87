// The Whisper text decoder's token loop on the device (whisper/decoder.go,
// encoder.go:120-140, transcribe.go:370-520): the embedding, the layer
// norm, self- and cross-attention, the packed-order product used for the
// cross K/V prep, and process + sample at temperature 0. The per-token
// products are k_flin's F16 path (Q8_0 widened as f16(q·d)).
//
// Every reduction follows the reference's order: dotF32Go (four strided
// unfused sums), dot4f32avx (16 lanes of fused chains, then HSUM), expSub
// (EXP8 lanes over len&~7 with eight running lane sums, then Go expf for the
// rest), softmax's ·(1/Σ), the unfused value sum of self-attention. The only
// sums the GPU reorders are the three float32 sums over the vocabulary in
// process/sample; they reach a token only through comparisons, which are
// checked against a safe margin and, when closer, recomputed in the
// reference's sequential order.
#include <algorithm>
#include <cuda_fp16.h>
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace grx {

namespace {

#define NINF (-__int_as_float(0x7f800000))

__device__ __forceinline__ float q8h(int8_t q, float d) { return __half2float(__float2half_rn(__fmul_rn(float(q), d))); }

__device__ __forceinline__ float wmat_at(const WMat& w, int row, int col) {
  if (w.f) return w.f[(size_t)row * w.cols + col];
  if (w.h) return __half2float(__ushort_as_half(w.h[(size_t)row * w.cols + col]));
  return q8h(w.q[(size_t)row * w.cols + col], h2f(w.d[(size_t)row * (w.cols / QK) + col / QK]));
}

template <class T>
__device__ __forceinline__ T warp_max(T v) {
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block max over blockDim.x threads (multiple of 32), result to all.
__device__ float block_max(float v, float* sh) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  float r = sh[0];
  for (int i = 1; i < nw; i++) r = fmaxf(r, sh[i]);
  return r;
}

__device__ float block_sum(float v, float* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; i++) r += sh[i];
  return r;
}

__device__ double block_sum_d(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  double r = 0;
  for (int i = 0; i < nw; i++) r += sh[i];
  return r;
}

// ---------------------------------------------------------------- embed

__global__ void k_wembed(WRows r, WMat emb, const float* pos, float* x) {
  const int row = blockIdx.x, tok = r.row_tok[row], p = r.row_pos[row];
  for (int j = threadIdx.x; j < r.st; j += blockDim.x)
    x[(size_t)row * r.st + j] = __fadd_rn(wmat_at(emb, tok, j), pos[(size_t)p * r.st + j]);
}

// ------------------------------------------------------------ layerNorm
// whisper/mathx.go:55-75: float64 sums (their order does not reach the
// float32 results but in a last-ulp tie), mean and 1/sd as float32, then
// ((v − mean)·inv)·w + b.
__global__ void k_wln(const float* x, float* y, const float* w, const float* b, int n) {
  __shared__ double sh[32];
  const float* xr = x + (size_t)blockIdx.x * n;
  float* yr = y + (size_t)blockIdx.x * n;
  double s = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += double(xr[i]);
  s = block_sum_d(s, sh);
  const float mean = float(s / double(n));
  double vs = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double d = double(__fsub_rn(xr[i], mean));
    vs += d * d;
  }
  vs = block_sum_d(vs, sh);
  const float inv = float(1.0 / sqrt(vs / double(n) + 1e-5));
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    yr[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[i], mean), inv), w[i]), b[i]);
}

// expSub of e[0, n) in place (kernels_amd64.go expSub + expSubAVX): EXP8 for
// the first n&~7 with eight lane sums in order, HSUM, then Go expf for the
// rest summed in order. Threads 0..7 of the block do the sums. Returns Σ to
// every thread.
__device__ float exp_sub(float* e, int n, float mx, float* sh) {
  const int n8 = n & ~7;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float d = __fsub_rn(e[j], mx);
    e[j] = j < n8 ? exp_avx(d) : expf_go(d);
  }
  __syncthreads();
  if (threadIdx.x < 8) {
    float a = 0.f;
#pragma unroll 8
    for (int c = threadIdx.x; c < n8; c += 8) a = __fadd_rn(a, e[c]);
    sh[threadIdx.x] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    if (n8 > 0)
      s = __fadd_rn(__fadd_rn(__fadd_rn(sh[0], sh[4]), __fadd_rn(sh[1], sh[5])),
                    __fadd_rn(__fadd_rn(sh[2], sh[6]), __fadd_rn(sh[3], sh[7])));
    float t = 0.f;
    for (int j = n8; j < n; j++) t = __fadd_rn(t, e[j]);
    sh[8] = __fadd_rn(s, t);
  }
  __syncthreads();
  return sh[8];
}

// -------------------------------------------------------- self-attention
// decoder.go:70-87 for (row, head): s_j = dotF32Go(q, k_j)·(1/√hd) over the
// stream's cache rows 0..pos, softmax, o[d] = Σ_j p_j·v_j[d] (unfused, in j
// order). 128 threads; hd = 64.
__global__ void __launch_bounds__(128) k_wself(WRows r, const float* q, const float* sk, const float* sv, float* att) {
  extern __shared__ float wsm[];  // [text_ctx] scores, [64] q
  __shared__ float sh[40];
  const int row = blockIdx.x, h = blockIdx.y, hd = 64, st = r.st;
  const int s = r.row_stream[row], n = r.row_pos[row] + 1;
  float* sc = wsm;
  float* qh = wsm + r.text_ctx;
  if (threadIdx.x < hd) qh[threadIdx.x] = q[(size_t)row * st + h * hd + threadIdx.x];
  __syncthreads();
  const float scale = float(1.0 / sqrt(double(hd)));
  const float* kb = sk + (size_t)s * r.text_ctx * st + h * hd;
  float mx = NINF;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float* kj = kb + (size_t)j * st;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int i = 0; i < 64; i += 4) {
      const float4 k4 = *reinterpret_cast<const float4*>(kj + i);
      s0 = __fadd_rn(s0, __fmul_rn(qh[i], k4.x));
      s1 = __fadd_rn(s1, __fmul_rn(qh[i + 1], k4.y));
      s2 = __fadd_rn(s2, __fmul_rn(qh[i + 2], k4.z));
      s3 = __fadd_rn(s3, __fmul_rn(qh[i + 3], k4.w));
    }
    const float v = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3), scale);
    sc[j] = v;
    mx = fmaxf(mx, v);
  }
  mx = block_max(mx, sh);
  const float sum = exp_sub(sc, n, mx, sh);
  const float inv = __fdiv_rn(1.f, sum);
  for (int j = threadIdx.x; j < n; j += blockDim.x) sc[j] = __fmul_rn(sc[j], inv);
  __syncthreads();
  if (threadIdx.x < hd) {
    const float* vb = sv + (size_t)s * r.text_ctx * st + h * hd + threadIdx.x;
    float o = 0.f;
    for (int j = 0; j < n; j++) o = __fadd_rn(o, __fmul_rn(sc[j], vb[(size_t)j * st]));
    att[(size_t)row * st + h * hd + threadIdx.x] = o;
  }
}

// ------------------------------------------------- bulk copies to shared --
// A CTA stages rows it streams into shared memory with cp.async.bulk (this
// CTA's own shared memory; no cluster-wide forms), completing on one
// mbarrier. Every wait is bounded by about a second of %globaltimer; a CTA
// whose copies do not arrive computes from global memory instead and waits
// again (bounded) before leaving, so its shared memory is never released
// under a copy in flight.
constexpr unsigned long long kBulkWaitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long wtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool wbar_try(uint32_t bar) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar)
      : "memory");
  return ok != 0;
}
// Thread 0: arms the barrier for `bytes` and starts n copies of `each` bytes
// (16-byte multiples, 16-byte aligned), source i at src + i·src_stride floats.
__device__ void wbulk_start(uint64_t* mbar, float* dst, const float* src, size_t src_stride, int n, uint32_t each) {
  const uint32_t bar = uint32_t(__cvta_generic_to_shared(mbar));
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(uint32_t(n) * each) : "memory");
  for (int i = 0; i < n; i++)
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            uint32_t(__cvta_generic_to_shared(dst)) + uint32_t(i) * each),
        "l"(src + i * src_stride), "r"(each), "r"(bar)
        : "memory");
}
// Every thread: true once the copies have landed (thread 0 waits, bounded).
__device__ bool wbulk_wait(uint64_t* mbar, int* ok) {
  const uint32_t bar = uint32_t(__cvta_generic_to_shared(mbar));
  if (threadIdx.x == 0) {
    const unsigned long long t0 = wtime();
    bool got = wbar_try(bar);
    while (!got && wtime() - t0 < kBulkWaitNs) got = wbar_try(bar);
    *ok = got;
  }
  __syncthreads();
  if (!*ok) return false;
  wbar_try(bar);  // every thread observes the completed phase itself
  return true;
}
// Before leaving after a wait that gave up: wait once more, bounded.
__device__ void wbulk_drain(uint64_t* mbar, int ok) {
  if (threadIdx.x == 0 && !ok) {
    const uint32_t bar = uint32_t(__cvta_generic_to_shared(mbar));
    const unsigned long long t0 = wtime();
    while (!wbar_try(bar) && wtime() - t0 < kBulkWaitNs) {
    }
  }
  __syncthreads();
}

// ------------------------------------------------------- cross-attention
// decoder.go:93-119 for (row, head): scores by dot4f32avx over the stream's
// pre-scaled keys (16 lanes per key: lane l16 chains element 16c + l16,
// then lanes l and l+8 add, HSUM), softmax, and o[d] = dot4f32avx(p, Vᵀ[d])
// over ctx&~15 plus dotF32Go of the rest. hd = 64. Every key's score, and
// every o[d], is a computation of its own; only the softmax's sum runs over
// all keys. So the work splits two ways without changing a bit: k_wcross
// does a (row, head) in one CTA; at few rows, k_wcross_sc spreads a head's
// keys over KS CTAs (scores and a maximum per chunk into scratch) and
// k_wcross_o spreads its 64 outputs over DS CTAs, each forming the softmax
// from the stored scores.

// Scores of keys [j0, j1) (j1 ≤ ctx&~3) into sc[j], groups of 16 lanes per
// key, from kb (or, given, ks = those keys' rows staged in shared memory);
// with `tail`, also the keys past the last group of four (dotF32Go, from
// kb). Returns the thread's maximum.
__device__ __forceinline__ float wcross_scores(const float* qh, const float* kb, int j0, int j1, bool tail, int ctx, float* sc,
                               const float* ks = nullptr) {
  const int l16 = threadIdx.x & 15, grp = threadIdx.x >> 4, ng = blockDim.x >> 4;
  float mx = NINF;
  // UK keys' rows are loaded before the first of them is used (bytes in
  // flight for the HBM stream); each key's dot is unchanged.
  constexpr int UK = 8;
  for (int jb = j0; jb < j1; jb += ng * UK) {
    float kv[UK][4];
#pragma unroll
    for (int u = 0; u < UK; u++) {
      const int j = jb + ng * u + grp;
      if (j < j1) {
        const float* kj = ks ? ks + (size_t)(j - j0) * 64 : kb + (size_t)j * 64;
#pragma unroll
        for (int c = 0; c < 4; c++) kv[u][c] = kj[16 * c + l16];
      }
    }
#pragma unroll
    for (int u = 0; u < UK; u++) {
      const int j = jb + ng * u + grp;
      float a = 0.f;
      if (j < j1) {
#pragma unroll
        for (int c = 0; c < 4; c++) a = __fmaf_rn(qh[16 * c + l16], kv[u][c], a);
      }
      a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 8));  // lanes l < 8: acc0_l + acc1_l
      float x = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 4));
      float y = __fadd_rn(x, __shfl_down_sync(0xffffffffu, x, 1));
      const float z = __fadd_rn(y, __shfl_down_sync(0xffffffffu, y, 2));
      if (l16 == 0 && j < j1) {
        sc[j] = z;
        mx = fmaxf(mx, z);
      }
    }
  }
  if (tail)
    for (int j = (ctx & ~3) + threadIdx.x; j < ctx; j += blockDim.x) {  // keys past the last group of four: dotF32Go
      const float* kj = kb + (size_t)j * 64;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
      for (int i = 0; i < 64; i += 4) {
        s0 = __fadd_rn(s0, __fmul_rn(qh[i], kj[i]));
        s1 = __fadd_rn(s1, __fmul_rn(qh[i + 1], kj[i + 1]));
        s2 = __fadd_rn(s2, __fmul_rn(qh[i + 2], kj[i + 2]));
        s3 = __fadd_rn(s3, __fmul_rn(qh[i + 3], kj[i + 3]));
      }
      sc[j] = __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
      mx = fmaxf(mx, sc[j]);
    }
  return mx;
}

// Scores to probabilities in place: expSub against mx, then · (1/Σ).
__device__ __forceinline__ void wcross_softmax(float* sc, int ctx, float mx, float* sh) {
  const float sum = exp_sub(sc, ctx, mx, sh);
  const float inv = __fdiv_rn(1.f, sum);
  for (int j = threadIdx.x; j < ctx; j += blockDim.x) sc[j] = __fmul_rn(sc[j], inv);
  __syncthreads();
}

// o[d] for d = d0 + grp + ng·i, i < ND (ng groups of 16 lanes, or only the
// first ngrp groups when given): the 16 lanes chain over ctx&~15 in steps of
// 16, then the HSUM and dotF32Go of the rest; p = probabilities in shared
// memory, V row d at vb + (d − vd0)·ctx.
template <int ND>
__device__ __forceinline__ void wcross_out(const float* p, const float* vb, int ctx, int d0, float* att, int vd0 = 0, int ngrp = 0) {
  const int l16 = threadIdx.x & 15, grp = threadIdx.x >> 4, ng = blockDim.x >> 4;
  if (ngrp && grp >= ngrp) return;  // whole warps (ngrp even)
  const int cf = ctx & ~15;
  float acc[ND];
#pragma unroll
  for (int i = 0; i < ND; i++) acc[i] = 0.f;
  constexpr int UV = 8;
  for (int c0 = 0; c0 < cf; c0 += 16 * UV) {
    float vv[UV][ND];
#pragma unroll
    for (int u = 0; u < UV; u++) {
      const int c = c0 + 16 * u;
      if (c < cf)
#pragma unroll
        for (int i = 0; i < ND; i++) vv[u][i] = vb[(size_t)(d0 - vd0 + grp + ng * i) * ctx + c + l16];
    }
#pragma unroll
    for (int u = 0; u < UV; u++) {
      const int c = c0 + 16 * u;
      if (c < cf) {
        const float pc = p[c + l16];
#pragma unroll
        for (int i = 0; i < ND; i++) acc[i] = __fmaf_rn(pc, vv[u][i], acc[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < ND; i++) {
    float a = __fadd_rn(acc[i], __shfl_down_sync(0xffffffffu, acc[i], 8));
    float x = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 4));
    float y = __fadd_rn(x, __shfl_down_sync(0xffffffffu, x, 1));
    float z = __fadd_rn(y, __shfl_down_sync(0xffffffffu, y, 2));
    if (l16 == 0) {
      const int d = d0 + grp + ng * i;
      if (cf < ctx) {  // + dotF32Go of the tail (kernels_amd64.go dotF32x4)
        const float* vd = vb + (size_t)(d - vd0) * ctx;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        int t = cf;
        for (; t + 4 <= ctx; t += 4) {
          s0 = __fadd_rn(s0, __fmul_rn(p[t], vd[t]));
          s1 = __fadd_rn(s1, __fmul_rn(p[t + 1], vd[t + 1]));
          s2 = __fadd_rn(s2, __fmul_rn(p[t + 2], vd[t + 2]));
          s3 = __fadd_rn(s3, __fmul_rn(p[t + 3], vd[t + 3]));
        }
        for (; t < ctx; t++) s0 = __fadd_rn(s0, __fmul_rn(p[t], vd[t]));
        z = __fadd_rn(z, __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3));
      }
      att[d] = z;
    }
  }
}

// One CTA per (row, head), 256 threads.
__global__ void __launch_bounds__(256) k_wcross(WRows r, const float* q, const float* ck, const float* cvt, float* att) {
  extern __shared__ float wsm[];  // [audio_ctx] scores, [64] q
  __shared__ float sh[40];
  const int row = blockIdx.x, h = blockIdx.y, hd = 64, st = r.st, ctx = r.audio_ctx;
  const int s = r.row_stream[row];
  float* sc = wsm;
  float* qh = wsm + ctx;
  if (threadIdx.x < hd) qh[threadIdx.x] = q[(size_t)row * st + h * hd + threadIdx.x];
  __syncthreads();
  const float* kb = ck + ((size_t)s * r.nh + h) * ctx * hd;
  const float* vb = cvt + ((size_t)s * r.nh + h) * hd * ctx;
  float mx = wcross_scores(qh, kb, 0, ctx & ~3, true, ctx, sc);
  mx = block_max(mx, sh);
  wcross_softmax(sc, ctx, mx, sh);
  wcross_out<4>(sc, vb, ctx, 0, att + (size_t)row * st + h * hd);
}

// Scores of the keys of chunk blockIdx.z (ch keys, a multiple of 16; the
// last chunk also takes the keys past ctx&~3) into sg[row][h][ctx], the
// chunk's maximum into mg[row][h][chunk]. The chunk's key rows (contiguous)
// are staged in shared memory by one bulk copy. 128 threads.
__global__ void __launch_bounds__(128) k_wcross_sc(WRows r, const float* q, const float* ck, int ch, float* sg,
                                                   float* mg) {
  extern __shared__ __align__(128) float ksm[];  // [ch][64]
  __shared__ float qh[64];
  __shared__ float sh[40];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int ok;
  const int row = blockIdx.x, h = blockIdx.y, kc = blockIdx.z, nks = gridDim.z, hd = 64, ctx = r.audio_ctx;
  const int s = r.row_stream[row], ctx4 = ctx & ~3;
  const float* kb = ck + ((size_t)s * r.nh + h) * ctx * hd;
  const int j0 = kc * ch, j1 = min(ctx4, j0 + ch);
  if (threadIdx.x == 0) wbulk_start(&mbar, ksm, kb + (size_t)j0 * hd, 0, 1, uint32_t(j1 - j0) * hd * 4);
  if (threadIdx.x < hd) qh[threadIdx.x] = q[(size_t)row * r.st + h * hd + threadIdx.x];
  const bool staged = wbulk_wait(&mbar, &ok);
  const size_t rh = (size_t)row * r.nh + h;
  float mx = wcross_scores(qh, kb, j0, j1, kc == nks - 1, ctx, sg + rh * ctx, staged ? ksm : nullptr);
  mx = block_max(mx, sh);
  if (threadIdx.x == 0) mg[rh * nks + kc] = mx;
  wbulk_drain(&mbar, ok);
}

// The softmax of (row, head) from the stored scores and maxima, then the
// DW outputs of slice blockIdx.z: 16 lanes per output, 16·DW threads. With
// STAGE the slice's V rows (DW rows of ctx floats) are staged in shared
// memory by bulk copies started first, so they land while the softmax is
// formed; without, they stream from global memory.
template <int DW, bool STAGE>
__global__ void __launch_bounds__(16 * DW) k_wcross_o(WRows r, const float* cvt, int nks, const float* sg,
                                                     const float* mg, float* att) {
  extern __shared__ __align__(128) float wsm[];  // [ctx] probabilities (16-byte padded), [DW][ctx] V rows
  __shared__ float sh[40];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int ok;
  const int row = blockIdx.x, h = blockIdx.y, hd = 64, ctx = r.audio_ctx, d0 = blockIdx.z * DW;
  const int s = r.row_stream[row];
  const float* vb = cvt + ((size_t)s * r.nh + h) * hd * ctx;
  float* vsm = wsm + ((ctx + 3) & ~3);
  if (STAGE && threadIdx.x == 0) wbulk_start(&mbar, vsm, vb + (size_t)d0 * ctx, ctx, DW, uint32_t(ctx) * 4);
  const size_t rh = (size_t)row * r.nh + h;
  float mx = NINF;
  for (int i = 0; i < nks; i++) mx = fmaxf(mx, mg[rh * nks + i]);
  for (int j = threadIdx.x; j < ctx; j += blockDim.x) wsm[j] = sg[rh * ctx + j];
  __syncthreads();
  wcross_softmax(wsm, ctx, mx, sh);
  float* out = att + (size_t)row * r.st + h * hd;
  if constexpr (STAGE) {
    if (wbulk_wait(&mbar, &ok))
      wcross_out<1>(wsm, vsm, ctx, d0, out, d0);
    else
      wcross_out<1>(wsm, vb, ctx, d0, out);
    wbulk_drain(&mbar, ok);
  } else {
    wcross_out<1>(wsm, vb, ctx, d0, out);
  }
}

// --------------------------------------------------- packed-order product
// whisper/gemm.go:150-186 + k6x16avx: every output starts at its bias (or
// 0) and gets += the fused chain of each 256-deep pass. Tile 64 × 64, 256
// threads of 4 × 4 outputs, 32-deep slices staged in shared memory.
// Output (i, j) of group str of a packed-order product: the epilogue.
__device__ __forceinline__ void wmm_out(const WmmArgs& p, int str, int m, int n, int i, int j, float val) {
  float* cz = p.c + str * p.c_zs;
  const int hd = n / max(p.nh, 1);
  switch (p.mode) {
    case WM_CROSSK: {
      const int hh = j / hd, d = j % hd;
      p.c[((size_t)str * p.nh + hh) * (size_t)m * hd + (size_t)i * hd + d] = __fmul_rn(val, p.tsc);
      break;
    }
    case WM_CROSSV: {
      const int hh = j / hd, d = j % hd;
      p.c[((size_t)str * p.nh + hh) * (size_t)m * hd + (size_t)d * m + i] = val;
      break;
    }
    case WM_RESID:
      cz[(size_t)i * p.ldc + j] = __fadd_rn(cz[(size_t)i * p.ldc + j], val);
      break;
    case WM_GELU:
      cz[(size_t)i * p.ldc + j] = gelu_avx(val);
      break;
    case WM_GELU_ADD:
      cz[(size_t)i * p.ldc + j] = __fadd_rn(gelu_avx(val), p.aux[(size_t)i * p.ldc + j]);
      break;
    case WM_ROWPOS:
      p.c[(size_t)p.dst_row[i * p.rs_i + str] * p.ldc + j] = val;
      break;
    default:
      cz[(size_t)i * p.ldc + j] = val;
  }
}

constexpr int MM_T = 64, MM_S = 32, MM_LD = MM_T + 4;

__global__ void __launch_bounds__(256) k_wmm(WmmArgs p) {
  __shared__ __align__(16) float As[MM_S][MM_LD];
  __shared__ __align__(16) float Bs[MM_S][MM_LD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int i0 = blockIdx.y * MM_T, j0 = blockIdx.x * MM_T, str = blockIdx.z;
  WMat w = p.w;
  if (w.f) w.f += str * p.w_zs;  // a float32 weight per group (attention's keys and values)
  const int n = w.rows, k = w.cols, m = p.m, lda = p.lda;
  const float* A = p.a + str * p.a_zs;
  float cv[4][4], ch[4][4];
#pragma unroll
  for (int u = 0; u < 4; u++)
#pragma unroll
    for (int v = 0; v < 4; v++) {
      const int j = j0 + tx * 4 + v;
      cv[u][v] = p.bias && j < n ? p.bias[j] : 0.f;
    }
  const int sr = tid >> 2, sk8 = (tid & 3) * 8;  // staging: row/col sr, 8 values from sk8
  for (int p0 = 0; p0 < k; p0 += 256) {
    const int pn = min(256, k - p0);
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int v = 0; v < 4; v++) ch[u][v] = 0.f;
    for (int s0 = 0; s0 < pn; s0 += MM_S) {
      const int kk0 = p0 + s0;
      {
        const int i = i0 + sr;
        float va[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int kk = kk0 + sk8 + e;
          va[e] = i < m && kk < p0 + pn ? A[(size_t)i * lda + kk] : 0.f;
        }
        const int j = j0 + sr;
        float vbv[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int kk = kk0 + sk8 + e;
          vbv[e] = j < n && kk < p0 + pn ? wmat_at(w, j, kk) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int e = 0; e < 8; e++) {
          As[sk8 + e][sr] = va[e];
          Bs[sk8 + e][sr] = vbv[e];
        }
        __syncthreads();
      }
      const int sn = min(MM_S, pn - s0);
      for (int kk = 0; kk < sn; kk++) {
        const float4 a4 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
        const float4 b4 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
        const float av[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
          for (int v = 0; v < 4; v++) ch[u][v] = __fmaf_rn(av[u], bv[v], ch[u][v]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int v = 0; v < 4; v++) cv[u][v] = __fadd_rn(cv[u][v], ch[u][v]);
  }
#pragma unroll
  for (int u = 0; u < 4; u++)
#pragma unroll
    for (int v = 0; v < 4; v++) {
      const int i = i0 + ty * 4 + u, j = j0 + tx * 4 + v;
      if (i < m && j < n) wmm_out(p, str, m, n, i, j, cv[u][v]);
    }
}

// The packed order again, for the larger products: a 128 × 128 tile per CTA,
// 256 threads of 8 × 8 outputs (rows ty·4 + {0..3, 64..67}, columns likewise,
// so that each thread's float4 reads of the staged slices are
// conflict-free), 16-deep slices double-buffered through registers into
// shared memory (k-major). Each output still runs its own fused chain over
// k in order, folded into C at every 256-deep boundary; slices past K are
// zeros, and fma(0, 0, acc) leaves acc as it is (acc never becomes −0 from
// +0 by round-to-nearest sums). Needs K % 4 == 0, lda % 4 == 0 and 16-byte
// aligned A rows; WT selects the weight: 0 float32, 1 float16, 2 Q8_0
// widened to f16(q·d).
constexpr int G_BM = 128, G_BK = 16, G_LD = G_BM + 4;

template <int WT>
__device__ __forceinline__ float4 wmm2_wload(const WMat& w, int row, int k) {
  const size_t o = (size_t)row * w.cols + k;
  if (WT == 0) return *reinterpret_cast<const float4*>(w.f + o);
  if (WT == 1) {
    const uint2 h = *reinterpret_cast<const uint2*>(w.h + o);
    const __half2 lo = *reinterpret_cast<const __half2*>(&h.x), hi = *reinterpret_cast<const __half2*>(&h.y);
    return make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
  }
  const int q4 = *reinterpret_cast<const int*>(w.q + o);
  const float d = h2f(w.d[(size_t)row * (w.cols / QK) + k / QK]);
  return make_float4(q8h(int8_t(q4), d), q8h(int8_t(q4 >> 8), d), q8h(int8_t(q4 >> 16), d), q8h(int8_t(q4 >> 24), d));
}

template <int WT>
__global__ void __launch_bounds__(256) k_wmm2(WmmArgs p) {
  __shared__ __align__(16) float As[2][G_BK][G_LD];
  __shared__ __align__(16) float Bs[2][G_BK][G_LD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int i0 = blockIdx.y * G_BM, j0 = blockIdx.x * G_BM, str = blockIdx.z;
  WMat w = p.w;
  if (w.f) w.f += str * p.w_zs;
  const int n = w.rows, K = w.cols, m = p.m, lda = p.lda;
  const float* A = p.a + str * p.a_zs;
  // loads: rows lr and lr + 64 of A and of W, four k from lk
  const int lr = tid >> 2, lk = (tid & 3) * 4;
  float4 ra[2], rb[2];
  auto gload = [&](int k0) {
    const int k = k0 + lk;
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int r = i0 + lr + 64 * u, c = j0 + lr + 64 * u;
      ra[u] = r < m && k < K ? *reinterpret_cast<const float4*>(A + (size_t)r * lda + k) : make_float4(0, 0, 0, 0);
      rb[u] = c < n && k < K ? wmm2_wload<WT>(w, c, k) : make_float4(0, 0, 0, 0);
    }
  };
  auto sstore = [&](int b) {
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int r = lr + 64 * u;
      As[b][lk][r] = ra[u].x, As[b][lk + 1][r] = ra[u].y, As[b][lk + 2][r] = ra[u].z, As[b][lk + 3][r] = ra[u].w;
      Bs[b][lk][r] = rb[u].x, Bs[b][lk + 1][r] = rb[u].y, Bs[b][lk + 2][r] = rb[u].z, Bs[b][lk + 3][r] = rb[u].w;
    }
  };
  float cv[8][8], acc[8][8];
#pragma unroll
  for (int v = 0; v < 8; v++) {
    const int j = j0 + tx * 4 + (v & 3) + (v >> 2) * 64;
    const float b = p.bias && j < n ? p.bias[j] : 0.f;
#pragma unroll
    for (int u = 0; u < 8; u++) cv[u][v] = b;
  }
  const int ns = (K + G_BK - 1) / G_BK;
  gload(0);
  sstore(0);
  __syncthreads();
  for (int s = 0; s < ns; s++) {
    const int k0 = s * G_BK, b = s & 1;
    if ((k0 & 255) == 0) {
#pragma unroll
      for (int u = 0; u < 8; u++)
#pragma unroll
        for (int v = 0; v < 8; v++) acc[u][v] = 0.f;
    }
    if (s + 1 < ns) gload(k0 + G_BK);
#pragma unroll
    for (int kk = 0; kk < G_BK; kk++) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[b][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[b][kk][ty * 4 + 64]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[b][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[b][kk][tx * 4 + 64]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int u = 0; u < 8; u++)
#pragma unroll
        for (int v = 0; v < 8; v++) acc[u][v] = __fmaf_rn(av[u], bv[v], acc[u][v]);
    }
    if (((k0 + G_BK) & 255) == 0 || s + 1 == ns) {
#pragma unroll
      for (int u = 0; u < 8; u++)
#pragma unroll
        for (int v = 0; v < 8; v++) cv[u][v] = __fadd_rn(cv[u][v], acc[u][v]);
    }
    if (s + 1 < ns) {
      sstore(b ^ 1);
      __syncthreads();
    }
  }
  // plain row-major outputs leave as float4s (four columns of one row)
  const bool vec = (p.mode == WM_STORE || p.mode == WM_RESID || p.mode == WM_GELU || p.mode == WM_GELU_ADD) &&
                   p.ldc % 4 == 0 && p.c_zs % 4 == 0 && (reinterpret_cast<uintptr_t>(p.c) & 15) == 0;
#pragma unroll
  for (int u = 0; u < 8; u++) {
    const int i = i0 + ty * 4 + (u & 3) + (u >> 2) * 64;
    if (i >= m) continue;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int jb = j0 + tx * 4 + h * 64;
      if (vec && jb + 3 < n) {
        float* cp = p.c + str * p.c_zs + (size_t)i * p.ldc + jb;
        float4 o = make_float4(cv[u][4 * h], cv[u][4 * h + 1], cv[u][4 * h + 2], cv[u][4 * h + 3]);
        if (p.mode == WM_RESID) {
          const float4 y = *reinterpret_cast<const float4*>(cp);
          o = make_float4(__fadd_rn(y.x, o.x), __fadd_rn(y.y, o.y), __fadd_rn(y.z, o.z), __fadd_rn(y.w, o.w));
        } else if (p.mode == WM_GELU || p.mode == WM_GELU_ADD) {
          o = make_float4(gelu_avx(o.x), gelu_avx(o.y), gelu_avx(o.z), gelu_avx(o.w));
          if (p.mode == WM_GELU_ADD) {
            const float4 a = *reinterpret_cast<const float4*>(p.aux + (size_t)i * p.ldc + jb);
            o = make_float4(__fadd_rn(o.x, a.x), __fadd_rn(o.y, a.y), __fadd_rn(o.z, a.z), __fadd_rn(o.w, a.w));
          }
        }
        *reinterpret_cast<float4*>(cp) = o;
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (jb + e < n) wmm_out(p, str, m, n, i, jb + e, cv[u][4 * h + e]);
      }
    }
  }
}

// ------------------------------------------------------- audio encoder
// encode (encoder.go:10-118), per stream (grid y): the convolutions' window
// rows, the per-head split of q/k/v and the rows' softmax; the products are
// k_wmm's packed order.

// conv1's rows from a channel-major log-mel: x1[t][c·3 + k] = mel[c][t + k − 1]
// (0 outside the 3000 frames).
__global__ void k_wenc_conv1(const float* mel, float* x1, int nmel) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x, cols = nmel * 3;
  if (i >= 3000 * cols) return;
  const int t = i / cols, r = i - t * cols, c = r / 3, src = t + r - c * 3 - 1;
  x1[(size_t)s * 3000 * cols + i] = src >= 0 && src < 3000 ? mel[((size_t)s * nmel + c) * 3000 + src] : 0.f;
}

// conv2's (stride 2): x2[t][c·3 + k] = h1[2t + k − 1][c] (0 outside).
__global__ void k_wenc_conv2(const float* h1, float* x2, int st, int ctx) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x, cols = st * 3;
  if (i >= ctx * cols) return;
  const int t = i / cols, r = i - t * cols, c = r / 3, src = 2 * t + r - c * 3 - 1;
  x2[(size_t)s * ctx * cols + i] = src >= 0 && src < 3000 ? h1[((size_t)s * 3000 + src) * st + c] : 0.f;
}

// Per (stream, head) z: qh[z][t][d] = q·sc (copy, then scale), kh[z][t][d],
// vt[z][d][t].
__global__ void k_wenc_heads(const float* q, const float* k, const float* v, float* qh, float* kh, float* vt, int ctx,
                             int st, int nh, float sc) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ctx * st) return;
  const int hd = st / nh, t = i / st, j = i - t * st, h = j / hd, d = j - h * hd;
  const size_t src = (size_t)s * ctx * st + i, z = (size_t)s * nh + h;
  qh[(z * ctx + t) * hd + d] = __fmul_rn(q[src], sc);
  kh[(z * ctx + t) * hd + d] = k[src];
  vt[(z * hd + d) * ctx + t] = v[src];
}

// softmax (mathx.go:78-90) of rows of len values, a warp per row: the max,
// expSub (EXP8 lanes for the first len&~7 with eight running sums and HSUM,
// Go's expf and a sequential sum for the rest, added after), then × 1/Σ.
__global__ void k_wenc_softmax(float* x, int len, long rows) {
  const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float* r = x + row * len;
  float mx = NINF;
  for (int j = lane; j < len; j += 32) mx = fmaxf(mx, r[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int n8 = len & ~7;
  for (int j = lane; j < len; j += 32) {
    const float e = __fsub_rn(r[j], mx);
    r[j] = j < n8 ? exp_avx(e) : expf_go(e);
  }
  __syncwarp();
  float part = 0.f;
  if (lane < 8)
    for (int c = lane; c < n8; c += 8) part = __fadd_rn(part, r[c]);
  float sum = hsum8_lanes(part);
  if (lane == 0) {
    float tail = 0.f;
    for (int j = n8; j < len; j++) tail = __fadd_rn(tail, r[j]);
    sum = __fdiv_rn(1.f, __fadd_rn(sum, tail));
  }
  const float inv = __shfl_sync(0xffffffffu, sum, 0);
  __syncwarp();
  for (int j = lane; j < len; j += 32) r[j] = __fmul_rn(r[j], inv);
}

// The same softmax for rows of up to kSmRow values in one pass: a warp per
// row holds it in registers (lane l: values l + 32c), the exponentials go
// through shared memory for the eight lane sums.
constexpr int kSmRow = 1536, kSmPer = kSmRow / 32;

__global__ void __launch_bounds__(256) k_wenc_softmax_reg(float* x, int len, long rows) {
  __shared__ float es[8][kSmRow];
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * 8 + wid;
  if (row >= rows) return;
  float* r = x + row * len;
  float v[kSmPer];
  float mx = NINF;
#pragma unroll
  for (int c = 0; c < kSmPer; c++) {
    const int j = lane + 32 * c;
    v[c] = j < len ? r[j] : NINF;
    mx = fmaxf(mx, v[c]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int n8 = len & ~7;
#pragma unroll
  for (int c = 0; c < kSmPer; c++) {
    const int j = lane + 32 * c;
    if (j < len) {
      const float e = __fsub_rn(v[c], mx);
      v[c] = j < n8 ? exp_avx(e) : expf_go(e);
      es[wid][j] = v[c];
    }
  }
  __syncwarp();
  float part = 0.f;
  if (lane < 8)
    for (int c = lane; c < n8; c += 8) part = __fadd_rn(part, es[wid][c]);
  float sum = hsum8_lanes(part);
  if (lane == 0) {
    float tail = 0.f;
    for (int j = n8; j < len; j++) tail = __fadd_rn(tail, es[wid][j]);
    sum = __fdiv_rn(1.f, __fadd_rn(sum, tail));
  }
  const float inv = __shfl_sync(0xffffffffu, sum, 0);
#pragma unroll
  for (int c = 0; c < kSmPer; c++) {
    const int j = lane + 32 * c;
    if (j < len) r[j] = __fmul_rn(v[c], inv);
  }
}

// ------------------------------------------------------ process + sample

__device__ float expf_go_d(float x) { return expf_go(x); }

// The reference's sequential process + sample (transcribe.go:409-494) from
// logits already masked by the rules; one thread. The slow path for rows
// whose parallel decisions fall within the margin.
__device__ void proc_exact(const float* lg, int n, int beg, int* out) {
  float mx = NINF;
  for (int i = 0; i < n; i++) mx = fmaxf(mx, lg[i]);
  float s = 0.f;
  for (int i = 0; i < n; i++)
    if (lg[i] > NINF) s = __fadd_rn(s, expf_go_d(__fsub_rn(lg[i], mx)));
  const float ls = __fadd_rn(float(log(double(s))), mx);
  auto lp = [&](int i) { return lg[i] > NINF ? __fsub_rn(lg[i], ls) : NINF; };
  float ts_max = NINF;
  for (int i = beg; i < n; i++) ts_max = fmaxf(ts_max, lp(i));
  bool mask_text = false;
  if (ts_max > NINF) {
    float sum = 0.f;
    for (int i = beg; i < n; i++)
      if (lp(i) > NINF) sum = __fadd_rn(sum, expf_go_d(__fsub_rn(lp(i), ts_max)));
    const float ts_lp = __fadd_rn(float(log(double(sum))), ts_max);
    float text_max = NINF;
    for (int i = 0; i < beg; i++) text_max = fmaxf(text_max, lp(i));
    mask_text = ts_lp > text_max;
  }
  auto eff = [&](int i) { return mask_text && i < beg ? NINF : lg[i]; };
  float mx2 = NINF;
  for (int i = 0; i < n; i++) mx2 = fmaxf(mx2, eff(i));
  float s2 = 0.f;
  for (int i = 0; i < n; i++)
    if (eff(i) > NINF) s2 = __fadd_rn(s2, expf_go_d(__fsub_rn(eff(i), mx2)));
  auto prob = [&](int i) { return eff(i) > NINF ? __fdiv_rn(expf_go_d(__fsub_rn(eff(i), mx2)), s2) : 0.f; };
  int id = 0;
  float pid = prob(0);
  for (int i = 1; i < n; i++) {
    const float p = prob(i);
    if (p > pid) id = i, pid = p;
  }
  int tid = beg;
  float pt = prob(beg);
  for (int i = beg + 1; i < n; i++) {
    const float p = prob(i);
    if (p > pt) tid = i, pt = p;
  }
  if (id >= beg) tid = id;
  const float plog = mask_text && id < beg ? NINF : lp(id);
  out[0] = id;
  out[1] = tid;
  out[2] = __float_as_int(pid);
  out[3] = __float_as_int(plog);
}

// (value, index) with the larger value, the smaller index on a tie.
struct VI {
  float v;
  int i;
};
__device__ __forceinline__ VI vi_max(VI a, VI b) { return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a; }

__device__ VI block_vi_max(VI x, VI* sh) {
  for (int o = 16; o > 0; o >>= 1) {
    VI y{__shfl_xor_sync(0xffffffffu, x.v, o), __shfl_xor_sync(0xffffffffu, x.i, o)};
    x = vi_max(x, y);
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = x;
  __syncthreads();
  VI r = sh[0];
  for (int i = 1; i < nw; i++) r = vi_max(r, sh[i]);
  return r;
}

// One CTA per row. The rules mask in place (transcribe.go:378-408); the
// three float32 sums of logSoftmax, the timestamp rule and softmaxInf are
// taken in parallel, and every decision they feed is checked: the
// timestamp rule must clear a relative margin of 2e-4, and the winning
// probability must beat every earlier index's by a factor 1 − 2^-20 (the
// division by the sum can then not tie them). A row that misses a margin is
// recomputed by one thread in the reference's order.
//
// One pass takes e_i = expf(lg_i − max) for the whole row into scratch;
// without the timestamp rule's masking softmaxInf's terms are those same
// e_i (and so is its sum), so only the timestamps are taken again.
// Reductions of a row spread over a cluster of CL CTAs: each CTA's block
// result goes to its own slot, and after the cluster barrier every thread
// combines the CL slots in rank order (so every CTA holds the same value).
template <int CL>
__device__ float cl_max(float v, float* sh, float* slot) {
  v = block_max(v, sh);
  if constexpr (CL == 1) {
    return v;
  } else {
    cg::cluster_group c = cg::this_cluster();
    if (threadIdx.x == 0) *slot = v;
    c.sync();
    float r = NINF;
    for (int k = 0; k < CL; k++) r = fmaxf(r, *c.map_shared_rank(slot, k));
    return r;
  }
}
template <int CL>
__device__ float cl_sum(float v, float* sh, float* slot) {
  v = block_sum(v, sh);
  if constexpr (CL == 1) {
    return v;
  } else {
    cg::cluster_group c = cg::this_cluster();
    if (threadIdx.x == 0) *slot = v;
    c.sync();
    float r = 0.f;
    for (int k = 0; k < CL; k++) r = __fadd_rn(r, *c.map_shared_rank(slot, k));
    return r;
  }
}
template <int CL>
__device__ VI cl_vi_max(VI v, VI* sh, VI* slot) {
  v = block_vi_max(v, sh);
  if constexpr (CL == 1) {
    return v;
  } else {
    cg::cluster_group c = cg::this_cluster();
    if (threadIdx.x == 0) *slot = v;
    c.sync();
    VI r = *c.map_shared_rank(slot, 0);
    for (int k = 1; k < CL; k++) r = vi_max(r, *c.map_shared_rank(slot, k));
    return r;
  }
}

// The reductions process/sample makes over a row spread over several CTAs,
// through a cluster's distributed shared memory: each CTA's block result in
// its own slot, combined in rank order after the cluster barrier. Slots 0-7
// take floats, 0-1 the (value, index) pairs.
template <int CL>
struct ClusterRed {
  float* shf;
  VI* shv;
  float* clf;
  VI* clv;
  __device__ void max3(float& a, float& b, float& c) {
    a = cl_max<CL>(a, shf, &clf[0]);
    b = cl_max<CL>(b, shf, &clf[1]);
    c = cl_max<CL>(c, shf, &clf[2]);
  }
  __device__ float sum(float v, int slot) { return cl_sum<CL>(v, shf, &clf[3 + slot]); }
  __device__ void sum2(float& a, float& b) {
    a = cl_sum<CL>(a, shf, &clf[3]);
    b = cl_sum<CL>(b, shf, &clf[4]);
  }
  __device__ void vimax2(VI& a, VI& b) {
    a = cl_vi_max<CL>(a, shv, &clv[0]);
    b = cl_vi_max<CL>(b, shv, &clv[1]);
  }
  __device__ void max2(float& a, float& b) {
    a = cl_max<CL>(a, shf, &clf[6]);
    b = cl_max<CL>(b, shf, &clf[7]);
  }
  __device__ void done() {
    if constexpr (CL > 1) cg::this_cluster().sync();  // no CTA leaves while its slots may be read
  }
};

// process + sample of one row (transcribe.go:370-494) by the CTAs that share
// it: this CTA takes vocabulary entries [a0, a1), applies the rules that
// fall there and keeps its e_i; the sums combine partials in a fixed order,
// which the margins below make safe. `writer` marks the one CTA that writes
// the outputs: out[0..3] (id, tid, p, plog), the stream's sampling state
// and the next token.
//
// The float32 sums of logSoftmax, the timestamp rule and softmaxInf are taken
// in parallel, and every decision they feed is checked: the timestamp rule
// must clear a relative margin of 2e-4, and the winning probability must
// beat every earlier index's by a factor 1 − 2^-20 (the division by the sum
// can then not tie them). A row that misses a margin is recomputed by one
// thread in the reference's order. One pass takes e_i = expf(lg_i − max)
// for the whole row into scratch and, in the same reduction, the
// timestamps' Σ expf(lg_i − max_ts): the timestamp rule's logsumexp of
// logprobs[beg:] is log of that plus (max_ts − ls) (the reference sums
// expf((lg_i − ls) − (max_ts − ls)); the two differ by a few ulps of the
// exponents, far inside the margin), and with text masked it is softmaxInf's
// sum too, whose terms are then taken again into scratch.
//
// proc_prep is the first part: the rules on this CTA's entries and their
// maxima (all, timestamps, text), per thread; proc_finish the rest from the
// row's maxima.
__device__ __forceinline__ void proc_prep(float* lg, const WVocabDev& v, const WSample& q, int a0, int a1, int* amb,
                                          float& mx, float& mts, float& mtx) {
  const int beg = v.beg;
  const bool initial = q.nt == 0;
  auto setinf = [&](int i) {
    if (i >= a0 && i < a1) lg[i] = NINF;
  };
  if (threadIdx.x == 0) {
    *amb = 0;
    if (initial) {
      setinf(v.eot);
      if (v.space >= 0) setinf(v.space);
    }
    setinf(v.not_);
    setinf(v.sot), setinf(v.nosp), setinf(v.solm);
    setinf(v.translate), setinf(v.transcribe), setinf(v.prev);
  }
  for (int i = threadIdx.x; i < v.n_lang; i += blockDim.x) setinf(v.sot + 1 + i);
  for (int i = threadIdx.x; i < v.n_suppress; i += blockDim.x) setinf(v.suppress[i]);
  __syncthreads();
  const bool last = q.nt > 0 && q.last >= beg, penult = q.nt < 2 || q.penult >= beg;
  const int tid0 = int(round(1.0 / (30.0 / double(v.audio_ctx))));
  mx = NINF, mts = NINF, mtx = NINF;
  for (int i = a0 + threadIdx.x; i < a1; i += blockDim.x) {
    bool m = false;
    if (last) m = penult ? i >= beg : i < v.eot;
    if (initial && i >= beg + tid0 + 1) m = true;
    if (q.has_ts && i >= beg && i < beg + q.seek_delta / 2) m = true;
    float x = lg[i];
    if (m) lg[i] = x = NINF;
    mx = fmaxf(mx, x);
    if (i >= beg) mts = fmaxf(mts, x);
    else mtx = fmaxf(mtx, x);
  }
}

template <class Red>
__device__ __forceinline__ void proc_finish(Red& red, float* lg, float* e, const WVocabDev& v, WSample* sp,
                                            const WSample& q, int* orow, int* next_tok, int a0, int a1, bool writer,
                                            int* amb, float mx, float mts, float mtx) {
  const int n = v.n, beg = v.beg;
  // ---- logSoftmax's sum with e_i kept, and the timestamps' sum
  float s1 = 0.f, sts = 0.f;
  for (int i = a0 + threadIdx.x; i < a1; i += blockDim.x) {
    const float x = lg[i];
    const float ei = x > NINF ? expf_go(__fsub_rn(x, mx)) : 0.f;
    e[i] = ei;
    s1 = __fadd_rn(s1, ei);
    if (i >= beg && x > NINF) sts = __fadd_rn(sts, expf_go(__fsub_rn(x, mts)));
  }
  red.sum2(s1, sts);
  const float ls = __fadd_rn(float(log(double(s1))), mx);
  // ---- the timestamp rule
  const float ts_max = mts > NINF ? __fsub_rn(mts, ls) : NINF;  // the largest of logprobs[beg:]
  bool mask_text = false;
  if (ts_max > NINF) {
    const float ts_lp = __fadd_rn(float(log(double(sts))), ts_max);
    const float text_max = mtx > NINF ? __fsub_rn(mtx, ls) : NINF;
    mask_text = ts_lp > text_max;
    if (text_max > NINF && fabsf(ts_lp - text_max) <= 2e-4f * (1.f + fabsf(text_max))) *amb = 1;
  }
  // ---- softmaxInf's terms: the same e_i, or, with text masked, the
  // timestamps' against their own maximum (their sum is sts)
  const int lo = mask_text ? beg : 0;
  float s2 = s1;
  if (mask_text) {
    s2 = sts;
    for (int i = max(beg, a0) + threadIdx.x; i < a1; i += blockDim.x) {
      const float x = lg[i];
      e[i] = x > NINF ? expf_go(__fsub_rn(x, mts)) : 0.f;
    }
  }
  __syncthreads();
  VI best{-1.f, n}, bts{-1.f, n};
  for (int i = max(lo, a0) + threadIdx.x; i < a1; i += blockDim.x) {
    const float ei = e[i];
    best = vi_max(best, VI{ei, i});
    if (i >= beg) bts = vi_max(bts, VI{ei, i});
  }
  red.vimax2(best, bts);
  if (mask_text && lo > 0 && best.v < 0.f) best = VI{-1.f, n};
  // masked text has probability 0: it only wins if nothing else is positive
  if (mask_text && !(best.v > 0.f)) best = VI{0.f, 0};
  // the largest e before each winner that is smaller than it
  float near = 0.f, near_t = 0.f;
  for (int i = max(lo, a0) + threadIdx.x; i < a1; i += blockDim.x) {
    const float ei = e[i];
    if (i < best.i && ei < best.v) near = fmaxf(near, ei);
    if (i >= beg && i < bts.i && ei < bts.v) near_t = fmaxf(near_t, ei);
  }
  red.max2(near, near_t);
  const float margin = 1.f - 9.5367431640625e-07f;  // 1 − 2^-20
  if ((best.v > 0.f && near >= best.v * margin) || (bts.v > 0.f && near_t >= bts.v * margin)) *amb = 1;
  __syncthreads();
  if (threadIdx.x == 0 && writer) {
    int o[4];
    if (*amb) {
      proc_exact(lg, n, beg, o);
      if (v.exact_rows) atomicAdd(v.exact_rows, 1ull);
    } else {
      const int id = best.i;
      const int tid = id >= beg ? id : bts.i;
      o[0] = id;
      o[1] = tid;
      o[2] = __float_as_int(__fdiv_rn(best.v, s2));
      o[3] = __float_as_int(mask_text && id < beg ? NINF : __fsub_rn(lg[id], ls));
    }
    for (int i = 0; i < 4; i++) orow[i] = o[i];
    // the window loop's bookkeeping that process depends on (transcribe.go:218-224)
    WSample ns = q;
    ns.penult = q.last;
    ns.last = o[0];
    ns.nt = q.nt + 1;
    if (o[0] > beg) {
      ns.seek_delta = 2 * (o[0] - beg);
      ns.has_ts = 1;
    }
    *sp = ns;
    if (next_tok) *next_tok = o[0];
  }
  red.done();
}

template <class Red>
__device__ void proc_row(Red& red, float* lg, float* e, const WVocabDev& v, WSample* sp, int* orow, int* next_tok,
                         int a0, int a1, bool writer) {
  __shared__ int amb;
  const WSample q = *sp;
  float mx, mts, mtx;
  proc_prep(lg, v, q, a0, a1, &amb, mx, mts, mtx);
  red.max3(mx, mts, mtx);
  proc_finish(red, lg, e, v, sp, q, orow, next_tok, a0, a1, writer, &amb, mx, mts, mtx);
}

// Rows spread over clusters of CL CTAs (CL = 1: one CTA per row); CTA k of a
// row's cluster takes vocabulary entries [n·k/CL, n·(k+1)/CL).
template <int CL>
__global__ void __launch_bounds__(1024, 1) k_wproc(WRows r, float* logits, float* scratch, WVocabDev v, WSample* state,
                                                int* out, const int* step, int* next_tok) {
  __shared__ float shf[40];
  __shared__ VI shv[32];
  __shared__ float clf[8];
  __shared__ VI clv[2];
  const int row = blockIdx.x / CL, rank = blockIdx.x % CL, s = r.row_stream[row], n = v.n;
  const int a0 = int((long long)n * rank / CL), a1 = int((long long)n * (rank + 1) / CL);
  ClusterRed<CL> red{shf, shv, clf, clv};
  proc_row(red, logits + (size_t)row * n, scratch + (size_t)row * n, v, state + s,
           out + ((size_t)(step ? *step : 0) * r.rows + row) * 4, next_tok ? next_tok + row : nullptr, a0, a1,
           rank == 0);
}

// softmax(row)[nosp] (mathx.go:78-90): EXP8 lanes over n&~7 summed in order
// per lane, HSUM, Go expf over the rest; one CTA per row.
__global__ void k_wnospeech(const float* logits, int n, int nosp, float* scratch, float* out) {
  __shared__ float sh[40];
  const float* lg = logits + (size_t)blockIdx.x * n;
  float* e = scratch + (size_t)blockIdx.x * n;
  float mx = NINF;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    e[i] = lg[i];
    mx = fmaxf(mx, lg[i]);
  }
  mx = block_max(mx, sh);
  const float s = exp_sub(e, n, mx, sh);
  if (threadIdx.x == 0) out[blockIdx.x] = __fmul_rn(e[nosp], __fdiv_rn(1.f, s));
}

// Every row's position moves on by `advance` and its cache row for the next
// decode is set; the run's step counter, when given, moves on by one.
__global__ void k_wtick(int rows, int* row_pos, int* dst_row, int text_ctx, int advance, int* step) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r == 0 && step) *step += 1;
  if (r >= rows) return;
  const int p = row_pos[r] + advance;
  row_pos[r] = p;
  dst_row[r] = r * text_ctx + p;
}

// -------------------------------------- one stream's token loop, persistent
//
// k_wstep1 runs `steps` rounds of grx_whisper_run's step for a batch of one
// stream — process/sample of the last logits, then the decode of the sampled
// token — in one cooperative launch of one 256-thread CTA per SM, with a
// grid barrier where a step needs every CTA's results. Per layer: the q/k/v
// rows, self-attention (a few CTAs a head, each with some of its outputs),
// o with the residual, LayerNorm and xq, the cross scores (key chunks over
// the CTAs, their K rows staged ahead), the softmax and values (a slice of a
// head's outputs a CTA, its Vᵀ rows staged ahead), xo with the residual, LayerNorm and fc1,
// fc2 with the residual; then the final LayerNorm and the logits rows. Every
// CTA keeps a copy of the residual row and forms the LayerNorms itself.
//
// Each CTA's weight rows reach shared memory ahead of use: a ring of two
// buffers, the next layer's rows of all eight matrices (or the next chunk of
// logits rows) brought by bulk copies (a row each, on the buffer's mbarrier)
// while the current one is computed, so the products run on staged rows and
// only the barriers wait on memory. The cross K and V rows a CTA needs come
// the same way a few phases ahead.
//
// The arithmetic is the per-kernel path's: the products in k_flin's
// float-path lane order (one 8-lane group per output row, dot4f16avx with
// Q8_0 widened as f16(q·d)), the attention and process/sample code shared
// with those kernels; process/sample's sums combine the CTAs' partials in one
// fixed order on every CTA (the margins make the order safe, as for the
// cluster form). Every wait is bounded (about a second); one that runs out
// sets the error word and every CTA leaves.
constexpr int WS_NT = 256;
constexpr unsigned long long kWsWaitNs = 1000000000ull;

struct WsCtl {
  unsigned bar_k;
  int fail;
};

__device__ bool ws_sync(const WStep1Args& A, WsCtl& ctl) {
  __syncthreads();
  if (threadIdx.x == 0 && !ctl.fail) {
    ctl.bar_k += 1;
    const unsigned target = A.stall ? 0xffffffffu : ctl.bar_k * gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(A.bar) : "memory");
    const unsigned long long t0 = wtime();
    for (int it = 0;; it++) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(A.bar) : "memory");
      if (v >= target) break;
      if ((it & 63) == 63) {
        if (*(volatile int*)A.err) {
          ctl.fail = 1;
          break;
        }
        if (wtime() - t0 > kWsWaitNs) {
          atomicCAS(A.err, 0, 1);
          ctl.fail = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  return !ctl.fail;
}

// process/sample's reductions over the whole grid: each CTA's block result
// to its column of the partials, the grid barrier, then every CTA loads the
// columns into shared memory at once and combines them in one fixed order —
// lane l of a warp takes CTAs l, l+32, ... in sequence, then an xor tree over
// the lanes. Float slots: 0-2 the maxima, 3-5 the sums, 6-7 the "near"
// maxima; (value, index) slots 0-1.
struct GridRed {
  const WStep1Args& A;
  WsCtl& ctl;
  float* shf;
  VI* shv;
  float* gcol;  // [3][WS1_MAX_GRID] gathered columns
  VI* gvi;      // [2][WS1_MAX_GRID]
  float* res;   // [3] combined results
  VI* resv;     // [2]
  __device__ void put(int slot, float v) const {
    if (threadIdx.x == 0) A.part[size_t(slot) * gridDim.x + blockIdx.x] = v;
  }
  __device__ void gather(int s0, int ns) const {
    const int G = gridDim.x;
    for (int t = threadIdx.x; t < ns * G; t += blockDim.x) gcol[t] = A.part[size_t(s0) * G + t];
    __syncthreads();
  }
  // warp j < ns: slot j's maximum (sum = false) or sum into res[j]
  __device__ void combine(int ns, bool sum) const {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, G = gridDim.x;
    if (w < ns) {
      float a = sum ? 0.f : NINF;
      for (int k = l; k < G; k += 32) a = sum ? __fadd_rn(a, gcol[w * G + k]) : fmaxf(a, gcol[w * G + k]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float b = __shfl_xor_sync(0xffffffffu, a, o);
        a = sum ? __fadd_rn(a, b) : fmaxf(a, b);
      }
      if (l == 0) res[w] = a;
    }
    __syncthreads();
  }
  __device__ void max3(float& a, float& b, float& c) {
    a = block_max(a, shf);
    b = block_max(b, shf);
    c = block_max(c, shf);
    put(0, a), put(1, b), put(2, c);
    ws_sync(A, ctl);
    gather(0, 3);
    combine(3, false);
    a = res[0], b = res[1], c = res[2];
  }
  __device__ void sum2(float& a, float& b) {
    a = block_sum(a, shf);
    b = block_sum(b, shf);
    put(3, a), put(4, b);
    ws_sync(A, ctl);
    gather(3, 2);
    combine(2, true);
    a = res[0], b = res[1];
  }
  // the row's maxima whose partials the logits phase left in slots 0-2
  __device__ void maxima(float& a, float& b, float& c) {
    gather(0, 3);
    combine(3, false);
    a = res[0], b = res[1], c = res[2];
  }
  __device__ void vimax2(VI& a, VI& b) {
    a = block_vi_max(a, shv);
    b = block_vi_max(b, shv);
    VI* pv = reinterpret_cast<VI*>(A.partv);
    const int G = gridDim.x;
    if (threadIdx.x == 0) pv[blockIdx.x] = a, pv[G + blockIdx.x] = b;
    ws_sync(A, ctl);
    for (int t = threadIdx.x; t < 2 * G; t += blockDim.x) gvi[t] = pv[t];
    __syncthreads();
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (w < 2) {
      VI x{-1.f, 0x7fffffff};
      for (int k = l; k < G; k += 32) x = vi_max(x, gvi[w * G + k]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        VI y;
        y.v = __shfl_xor_sync(0xffffffffu, x.v, o);
        y.i = __shfl_xor_sync(0xffffffffu, x.i, o);
        x = vi_max(x, y);
      }
      if (l == 0) resv[w] = x;
    }
    __syncthreads();
    a = resv[0], b = resv[1];
  }
  __device__ void max2(float& a, float& b) {
    a = block_max(a, shf);
    b = block_max(b, shf);
    put(6, a), put(7, b);
    ws_sync(A, ctl);
    gather(6, 2);
    combine(2, false);
    a = res[0], b = res[1];
  }
  __device__ void done() {}
};

__device__ __forceinline__ int ws_split(int n, int c, int G) { return int((long long)n * c / G); }

// A block's float64 sum: warps by xor shuffles, then the first warp over the
// warps' sums (the float64 order does not reach the float32 results of the
// LayerNorm but in a last-ulp tie, as for k_wln).
__device__ __forceinline__ double ws_sum_d(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    double r = threadIdx.x < nw ? sh[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (threadIdx.x == 0) sh[32] = r;
  }
  __syncthreads();
  const double r = sh[32];
  __syncthreads();  // sh is reused by the next sum
  return r;
}

// whisper/mathx.go:55-75 over a row in shared memory (as k_wln).
__device__ __noinline__ void ws_ln(const float* x, float* y, const float* w, const float* b, int n, double* shd) {
  double s = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += double(x[i]);
  s = ws_sum_d(s, shd);
  const float mean = float(s / double(n));
  double vs = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double d = double(__fsub_rn(x[i], mean));
    vs += d * d;
  }
  vs = ws_sum_d(vs, shd);
  const float inv = float(1.0 / sqrt(vs / double(n) + 1e-5));
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    y[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x[i], mean), inv), w[i]), b[i]);
  __syncthreads();
}

// ---- async copies into shared memory (cp.async, for the strided V columns
// of self-attention; completion per thread, then a CTA barrier before other
// threads read)
__device__ __forceinline__ void cpa8(void* s, const void* g) {
  const unsigned sa = unsigned(__cvta_generic_to_shared(s));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(sa), "l"(g) : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

enum { WS_STORE = 0, WS_RESID = 1, WS_GELU = 2 };

// One product's rows for ws_rows: the rows [r0, r0 + R) of a float16
// matrix staged at s (rows of 2K + 16 bytes), their outputs y[r0 + r] (bias
// optional; RESID adds res[r0 + r]).
struct WsOut {
  const unsigned char* s;
  int r0, R;
  const float* bias;
  float* y;
  const float* res;
};

// Up to three products with the same K and input row, and their epilogue.
struct WsProd {
  WsOut o[3];
  int np, epi;
};

// The rows of the products in P (y = W·x (+ bias), x a row of K values in
// shared memory) in k_flin's order (dot4f16avx): eight lanes l each with two
// chains, elements 16c + l and 16c + 8 + l over c in order, the two added,
// then the HSUM ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7)). When the rows fit the
// block at 16 threads a row each thread runs one chain (thread l + 8 the
// second chain of l); otherwise 4 threads a row run four chains each (thread
// t the elements 4t..4t+3 of every 16, read as vectors; threads 2 and 3 the
// second chains of 0 and 1). A call of its own: its loops are scheduled
// apart from the persistent kernel's other state (inlined they lost 3-4x).
// The matrices are float16 (Q8_0 ones widened beforehand as f16(q·d), the
// values whisper/model.go:486-490 gives every product). RESID stores
// res + (dot + bias), GELU geluAVX(dot + bias).
__device__ __noinline__ void ws_product(const WsProd& P, const float* x, int K) {
  const int np = P.np, epi = P.epi, nc = K / 16;
  int tot = 0;
  for (int m = 0; m < np; m++) tot += P.o[m].R;
  const int tpr = tot * 16 <= int(blockDim.x) ? 16 : 4;
  const int g = threadIdx.x / tpr, t = threadIdx.x % tpr, ng = blockDim.x / tpr;
  for (int rb = 0; rb < tot; rb += ng) {  // whole warps through every round
    int r = min(rb + g, tot - 1), m = 0;
    while (m + 1 < np && r >= P.o[m].R) r -= P.o[m].R, m++;
    const WsOut& O = P.o[m];
    const unsigned char* wrow = O.s + r * (2 * K + 16);
    const int n = O.r0 + r;
    const float bv = O.bias && t == 0 ? __ldg(O.bias + n) : 0.f;  // in flight during the chains
    float v;
    if (tpr == 16) {
      const float* xr = x + t;
      const uint16_t* wr = reinterpret_cast<const uint16_t*>(wrow) + t;
      float a = 0.f;
#pragma unroll 8
      for (int c = 0; c < nc; c++) a = __fmaf_rn(xr[16 * c], h2f(wr[16 * c]), a);
      v = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 8));  // threads l < 8: a_l + a1_l
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
    } else {
      const float4* x4 = reinterpret_cast<const float4*>(x) + t;
      const uint2* w2 = reinterpret_cast<const uint2*>(wrow) + t;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
      for (int c = 0; c < nc; c++) {
        const float4 xv = x4[4 * c];
        const uint2 wv = w2[4 * c];
        a0 = __fmaf_rn(xv.x, h2f(uint16_t(wv.x)), a0);
        a1 = __fmaf_rn(xv.y, h2f(uint16_t(wv.x >> 16)), a1);
        a2 = __fmaf_rn(xv.z, h2f(uint16_t(wv.y)), a2);
        a3 = __fmaf_rn(xv.w, h2f(uint16_t(wv.y >> 16)), a3);
      }
      // v_l = a_l + a1_l (threads 0 and 1 take the second chains from 2 and 3)
      a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 2));
      a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 2));
      a2 = __fadd_rn(a2, __shfl_down_sync(0xffffffffu, a2, 2));
      a3 = __fadd_rn(a3, __shfl_down_sync(0xffffffffu, a3, 2));
      // thread 0: v_j + v_(j+4), then the pairs
      a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 1));
      a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 1));
      a2 = __fadd_rn(a2, __shfl_down_sync(0xffffffffu, a2, 1));
      a3 = __fadd_rn(a3, __shfl_down_sync(0xffffffffu, a3, 1));
      v = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    }
    if (t == 0 && rb + g < tot) {
      const float ov = O.bias ? __fadd_rn(v, bv) : v;
      if (epi == WS_RESID)
        O.y[n] = __fadd_rn(O.res[n], ov);
      else if (epi == WS_GELU)
        O.y[n] = gelu_avx(ov);
      else
        O.y[n] = ov;
    }
  }
}

__device__ __forceinline__ void ws_rows(int epi, const WsOut& a, const float* x, int K) {
  WsProd P;
  P.o[0] = a, P.np = 1, P.epi = epi;
  ws_product(P, x, K);
}

// n floats from global memory (16-byte aligned, n a multiple of 4) into
// shared memory, up to four vectors a thread in flight before their stores;
// read through L2 (data other CTAs wrote before the last grid barrier).
__device__ __forceinline__ void ws_load(float* dst, const float* src, int n) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  const int n4 = n >> 2, bd = blockDim.x;
  for (int i0 = 0; i0 < n4; i0 += 4 * bd) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int i = i0 + u * bd + int(threadIdx.x);
      if (i < n4) v[u] = __ldcg(s4 + i);
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int i = i0 + u * bd + int(threadIdx.x);
      if (i < n4) d4[i] = v[u];
    }
  }
  __syncthreads();
}

// This CTA's rows of a layer's eight matrices in the order q, k, v, o, xq,
// xo, fc1, fc2: their offsets in a weight buffer.
struct WsPlan {
  int off[9];
};

__device__ WsPlan ws_plan(const WS1Layer& Y, int st, int ff, int R, int Rf) {
  WsPlan p;
  p.off[0] = 0;
  for (int i = 0; i < 8; i++)
    p.off[i + 1] = p.off[i] + ws_slice_bytes(true, i == 6 ? Rf : R, i == 7 ? ff : st);
  return p;
}

// Self-attention of head h over keys 0..n-1 (decoder.go:70-87, as k_wself),
// outputs d0..d0+nd-1 of the head: every CTA of the head takes the scores
// and softmax, its nd columns of V staged by async copies meanwhile.
__device__ __noinline__ void ws_self(const float* q, const float* sk, const float* sv, int st, int n, int h, int d0, int nd,
                        float* sc, float* qh, float* vs, float* sh, float* att) {
  for (int t = threadIdx.x; t < n * (nd / 2); t += blockDim.x) {
    const int j = t / (nd / 2), c = t - j * (nd / 2);
    cpa8(vs + j * nd + 2 * c, sv + (size_t)j * st + h * 64 + d0 + 2 * c);
  }
  cpa_commit();
  if (threadIdx.x < 64) qh[threadIdx.x] = q[h * 64 + threadIdx.x];
  __syncthreads();
  const float scale = float(1.0 / sqrt(double(64)));
  const float* kb = sk + h * 64;
  float mx = NINF;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float* kj = kb + (size_t)j * st;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int i = 0; i < 64; i += 4) {
      const float4 k4 = *reinterpret_cast<const float4*>(kj + i);
      s0 = __fadd_rn(s0, __fmul_rn(qh[i], k4.x));
      s1 = __fadd_rn(s1, __fmul_rn(qh[i + 1], k4.y));
      s2 = __fadd_rn(s2, __fmul_rn(qh[i + 2], k4.z));
      s3 = __fadd_rn(s3, __fmul_rn(qh[i + 3], k4.w));
    }
    const float v = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3), scale);
    sc[j] = v;
    mx = fmaxf(mx, v);
  }
  mx = block_max(mx, sh);
  const float sum = exp_sub(sc, n, mx, sh);
  const float inv = __fdiv_rn(1.f, sum);
  for (int j = threadIdx.x; j < n; j += blockDim.x) sc[j] = __fmul_rn(sc[j], inv);
  cpa_wait<0>();
  __syncthreads();
  if (threadIdx.x < nd) {
    float o = 0.f;
#pragma unroll 8
    for (int j = 0; j < n; j++) o = __fadd_rn(o, __fmul_rn(sc[j], vs[j * nd + threadIdx.x]));
    att[h * 64 + d0 + threadIdx.x] = o;
  }
  __syncthreads();
}

// ---- bulk copies into this CTA's own shared memory, completing on an
// mbarrier (no cluster-wide forms); thread 0 waits, bounded like the grid
// barrier, and a wait that runs out sets the error word.
__device__ __forceinline__ bool ws_bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void ws_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
// One contiguous copy (16-byte aligned ends, a multiple of 16 bytes). The
// proxy fence orders the CTA's earlier reads of the destination (behind a
// CTA barrier) before the copy's writes.
__device__ __forceinline__ void ws_bulk(void* dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   unsigned(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ bool ws_bar_wait(const WStep1Args& A, WsCtl& ctl, uint32_t bar, uint32_t parity) {
  if (threadIdx.x == 0 && !ctl.fail) {
    const unsigned long long t0 = wtime();
    bool got = ws_bar_try(bar, parity);
    while (!got && wtime() - t0 < kWsWaitNs) got = ws_bar_try(bar, parity);
    if (!got) {
      atomicCAS(A.err, 0, 1);
      ctl.fail = 1;
    }
  }
  __syncthreads();
  if (ctl.fail) return false;
  ws_bar_try(bar, parity);  // every thread observes the completed phase itself
  return true;
}
// Before leaving: the last fill of a barrier landed (bounded), so no copy
// is in flight into shared memory the CTA releases.
__device__ void ws_bar_drain(uint32_t bar, unsigned fills) {
  if (threadIdx.x == 0 && fills > 0) {
    const unsigned long long t0 = wtime();
    while (!ws_bar_try(bar, (fills - 1) & 1) && wtime() - t0 < kWsWaitNs) {
    }
  }
}

// h[i] = f16(q[i]·d[i/32]): the float16 value every Whisper product widens
// a Q8_0 value to (whisper/model.go:486-490).
__global__ void k_wwiden(const int8_t* q, const uint16_t* d, uint16_t* h, size_t n) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) h[i] = __half_as_ushort(__float2half_rn(__fmul_rn(float(q[i]), h2f(d[i / QK]))));
}

// The cross scores of keys [j0, j1) from staged rows and the values of
// outputs d0..d0+nd-1 from staged Vᵀ rows, as calls of their own (their
// loops scheduled apart from the persistent kernel's other state).
__device__ __noinline__ float ws_xscores(const float* qh, const float* kb, int j0, int j1, bool tail, int ctx, float* sc,
                                         const float* ks) {
  return wcross_scores(qh, kb, j0, j1, tail, ctx, sc, ks);
}

__device__ __noinline__ void ws_xout(const float* p, const float* vs, int ctx, int d0, int nd, float* att) {
  wcross_out<1>(p, vs, ctx, d0, att, d0, nd);
}

// process + sample of step i: the rules and maxima first unless the
// previous step's logits phase took them (`prepped`: their partials in the
// reduction slots 0-2).
__device__ __noinline__ void ws_proc(GridRed& red, const WStep1Args& A, int i, int v0, int v1, bool writer,
                                     bool prepped, int* amb) {
  const WSample q = *A.state;
  float mx, mts, mtx;
  if (prepped) {
    red.maxima(mx, mts, mtx);
  } else {
    proc_prep(A.logits, A.voc, q, v0, v1, amb, mx, mts, mtx);
    red.max3(mx, mts, mtx);
  }
  proc_finish(red, A.logits, A.scratch, A.voc, A.state, q, A.out + 4 * i, A.row_tok, v0, v1, writer, amb, mx, mts,
              mtx);
}

// The rules and this CTA's maxima of the logits just made, for the next
// step's process (its state is the one the current step's sample left).
__device__ __noinline__ void ws_prep(GridRed& red, const WStep1Args& A, int v0, int v1, int* amb) {
  const WSample q = *A.state;
  float mx, mts, mtx;
  proc_prep(A.logits, A.voc, q, v0, v1, amb, mx, mts, mtx);
  mx = block_max(mx, red.shf);
  mts = block_max(mts, red.shf);
  mtx = block_max(mtx, red.shf);
  red.put(0, mx), red.put(1, mts), red.put(2, mtx);
}

__global__ void __launch_bounds__(WS_NT, 1) k_wstep1(const WStep1Args* __restrict__ Ap, int pos0, int steps) {
  const WStep1Args& A = *Ap;
  extern __shared__ __align__(128) float ws1m[];
  const int st = A.st, ff = A.ff, ctx = A.ctx, nh = A.nh, G = gridDim.x, cta = blockIdx.x, L = A.L;
  float* xs = ws1m;                       // [st] the residual row
  float* cur = xs + st;                   // [max(st, ff)] a product's input
  float* sc = cur + max(st, ff);          // [max(ctx, text_ctx)] scores
  float* qh = sc + max(ctx, A.text_ctx);  // [64]
  float* xv = qh + 64;                    // [xv_floats] staged V columns
  float* xk = xv + A.xv_floats;           // [xk_floats] staged cross K rows
  unsigned char* wbuf = reinterpret_cast<unsigned char*>(xk + A.xk_floats);  // [2][wb] weight rows
  __shared__ float shf[40];
  __shared__ VI shv[32];
  __shared__ double shd[32];
  __shared__ float gcol[3 * WS1_MAX_GRID];
  __shared__ VI gvi[2 * WS1_MAX_GRID];
  __shared__ float gres[3];
  __shared__ VI gresv[2];
  __shared__ WsCtl ctl;
  __shared__ int amb;  // process/sample's "recompute in order" flag
  __shared__ __align__(8) uint64_t mbar[4];  // weight buffers 0 and 1, cross K rows, cross V rows
  if (threadIdx.x == 0) {
    ctl.bar_k = 0, ctl.fail = 0;
    for (int b = 0; b < 4; b++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_addr(&mbar[b])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  unsigned fills[4] = {0, 0, 0, 0};
  GridRed red{A, ctl, shf, shv, gcol, gvi, gres, gresv};
  // this CTA's rows: [r0, r1) of the state-sized products, [f0, f1) of fc1,
  // [v0, v1) of the logits in chunks of A.lrows
  const int r0 = ws_split(st, cta, G), r1 = ws_split(st, cta + 1, G);
  const int f0 = ws_split(ff, cta, G), f1 = ws_split(ff, cta + 1, G);
  const int v0 = ws_split(A.vocab, cta, G), v1 = ws_split(A.vocab, cta + 1, G);
  const int nchunk = max(1, (v1 - v0 + A.lrows - 1) / A.lrows);
  const int items = L + nchunk;  // staged items a step: the layers, then the logits chunks
  // item t of a step into weight buffer b: a bulk copy a row (thread c the
  // c-th row of the layer's eight slices, or of the logits chunk)
  auto stage = [&](int t, int b) {
    unsigned char* buf = wbuf + size_t(b) * A.wb;
    const uint32_t bar = smem_addr(&mbar[b]);
    fills[b]++;
    if (t < L) {
      const WS1Layer& Y = A.layers[t];
      const WsPlan p = ws_plan(Y, st, ff, r1 - r0, f1 - f0);
      const int R = r1 - r0, Rf = f1 - f0;
      if (threadIdx.x == 0) ws_expect(bar, uint32_t(2 * (6 * R * st + Rf * st + R * ff)));
      const WMat* m[8] = {&Y.q, &Y.k, &Y.v, &Y.o, &Y.xq, &Y.xo, &Y.fc1, &Y.fc2};
      for (int c = threadIdx.x; c < 7 * R + Rf; c += blockDim.x) {
        int k = c, i = 0;
        while (k >= (i == 6 ? Rf : R)) k -= (i == 6 ? Rf : R), i++;
        const int K = i == 7 ? ff : st, row = (i == 6 ? f0 : r0) + k;
        ws_bulk(buf + p.off[i] + k * (2 * K + 16), m[i]->h + (size_t)row * K, uint32_t(2 * K), bar);
      }
    } else {
      const int a = min(v1, v0 + (t - L) * A.lrows), e = min(v1, a + A.lrows);
      if (threadIdx.x == 0) ws_expect(bar, uint32_t(2 * (e - a) * st));
      for (int c = threadIdx.x; c < e - a; c += blockDim.x)
        ws_bulk(buf + c * (2 * st + 16), A.emb.h + (size_t)(a + c) * st, uint32_t(2 * st), bar);
    }
  };
  // item t of the step is consumed from buffer qi & 1 (that buffer's fill
  // qi / 2); on entry the next item goes to the other buffer (whose last
  // reader finished behind a CTA barrier), then this one's copies are waited
  // for. nullptr when the wait ran out.
  int qi = 0;
  auto consume = [&](int t) -> const unsigned char* {
    stage((t + 1) % items, (qi + 1) & 1);
    const int b = qi & 1;
    if (!ws_bar_wait(A, ctl, smem_addr(&mbar[b]), (qi >> 1) & 1)) return nullptr;
    qi++;
    return wbuf + size_t(b) * A.wb;
  };
  stage(0, 0);
  // the cross scores' key chunks: about G / nh per head, whole groups of 16
  const int ctx4 = ctx & ~3;
  int ks = max(1, G / nh);
  const int ch = ((ctx4 + ks - 1) / ks + 15) / 16 * 16;
  ks = (ctx4 + ch - 1) / ch;
  const int so_s = 64 / A.so_nd, xo_s = 64 / A.xo_nd;  // CTAs a head for self-attention and the values
  int i = 0;
  for (; i < steps; i++) {
    // ---- process + sample of the last logits (transcribe.go:370-494)
    ws_proc(red, A, i, v0, v1, cta == 0, i > 0, &amb);
    if (!ws_sync(A, ctl)) break;
    const int pos = pos0 + i, tok = A.row_tok[0];
    // ---- decode of the token at pos (decoder.go:33-140): the embedding
    for (int j = threadIdx.x; j < st; j += blockDim.x)
      xs[j] = __fadd_rn(wmat_at(A.emb, tok, j), A.dec_pos[(size_t)pos * st + j]);
    __syncthreads();
    for (int l = 0; l < L; l++) {
      const WS1Layer& Y = A.layers[l];
      const unsigned char* wl = consume(l);
      if (!wl) break;
      const WsPlan p = ws_plan(Y, st, ff, r1 - r0, f1 - f0);
      if (cta < nh * ks && threadIdx.x == 0) {  // this CTA's cross K rows, for the scores four phases on
        const int h = cta / ks, j0 = (cta % ks) * ch, j1 = min(ctx4, j0 + ch);
        ws_expect(smem_addr(&mbar[2]), uint32_t((j1 - j0) * 256));
        ws_bulk(xk, Y.ck + ((size_t)h * ctx + j0) * 64, uint32_t((j1 - j0) * 256), smem_addr(&mbar[2]));
      }
      if (cta < nh * ks) fills[2]++;
      ws_ln(xs, cur, Y.ln1w, Y.ln1b, st, shd);
      {
        const WsProd P = {{{wl + p.off[0], r0, r1 - r0, Y.qb, A.q, nullptr},
                           {wl + p.off[1], r0, r1 - r0, nullptr, Y.sk + (size_t)pos * st, nullptr},
                           {wl + p.off[2], r0, r1 - r0, Y.vb, Y.sv + (size_t)pos * st, nullptr}},
                          3,
                          WS_STORE};
        ws_product(P, cur, st);
      }
      if (!ws_sync(A, ctl)) break;
      if (cta < nh * so_s)
        ws_self(A.q, Y.sk, Y.sv, st, pos + 1, cta / so_s, (cta % so_s) * A.so_nd, A.so_nd, sc, qh, xv, shf, A.att);
      if (!ws_sync(A, ctl)) break;
      if (cta < nh * xo_s) {  // the Vᵀ rows of this CTA's cross outputs, for three phases on
        const int h = cta / xo_s, d0 = (cta % xo_s) * A.xo_nd;
        if (threadIdx.x == 0) {
          ws_expect(smem_addr(&mbar[3]), uint32_t(A.xo_nd * ctx * 4));
          ws_bulk(xv, Y.cvt + ((size_t)h * 64 + d0) * ctx, uint32_t(A.xo_nd * ctx * 4), smem_addr(&mbar[3]));
        }
        fills[3]++;
      }
      ws_load(cur, A.att, st);
      ws_rows(WS_RESID, WsOut{wl + p.off[3], r0, r1 - r0, Y.ob, A.x, xs}, cur, st);
      if (!ws_sync(A, ctl)) break;
      ws_load(xs, A.x, st);
      ws_ln(xs, cur, Y.ln2w, Y.ln2b, st, shd);
      ws_rows(WS_STORE, WsOut{wl + p.off[4], r0, r1 - r0, Y.xqb, A.q, nullptr}, cur, st);
      if (!ws_sync(A, ctl)) break;
      if (cta < nh * ks) {  // cross scores of key chunk cta % ks of head cta / ks
        const int h = cta / ks, kc = cta % ks, j0 = kc * ch, j1 = min(ctx4, j0 + ch);
        if (threadIdx.x < 64) qh[threadIdx.x] = A.q[h * 64 + threadIdx.x];
        if (!ws_bar_wait(A, ctl, smem_addr(&mbar[2]), (fills[2] - 1) & 1)) break;
        float mx = ws_xscores(qh, Y.ck + (size_t)h * ctx * 64, j0, j1, kc == ks - 1, ctx, A.sg + (size_t)h * ctx, xk);
        mx = block_max(mx, shf);
        if (threadIdx.x == 0) A.mg[h * ks + kc] = mx;
      }
      if (!ws_sync(A, ctl)) break;
      if (cta < nh * xo_s) {  // softmax and outputs d0..d0+xo_nd-1 of head h
        const int h = cta / xo_s, d0 = (cta % xo_s) * A.xo_nd;
        float mx = threadIdx.x < ks ? A.mg[h * ks + threadIdx.x] : NINF;
        mx = block_max(mx, shf);
        ws_load(sc, A.sg + (size_t)h * ctx, ctx);
        wcross_softmax(sc, ctx, mx, shf);
        if (!ws_bar_wait(A, ctl, smem_addr(&mbar[3]), (fills[3] - 1) & 1)) break;
        ws_xout(sc, xv, ctx, d0, A.xo_nd, A.att + h * 64);
      }
      if (!ws_sync(A, ctl)) break;
      ws_load(cur, A.att, st);
      ws_rows(WS_RESID, WsOut{wl + p.off[5], r0, r1 - r0, Y.xob, A.x, xs}, cur, st);
      if (!ws_sync(A, ctl)) break;
      ws_load(xs, A.x, st);
      ws_ln(xs, cur, Y.ln3w, Y.ln3b, st, shd);
      ws_rows(WS_GELU, WsOut{wl + p.off[6], f0, f1 - f0, Y.fc1b, A.ffb, nullptr}, cur, st);
      if (!ws_sync(A, ctl)) break;
      ws_load(cur, A.ffb, ff);
      ws_rows(WS_RESID, WsOut{wl + p.off[7], r0, r1 - r0, Y.fc2b, A.x, xs}, cur, ff);
      if (!ws_sync(A, ctl)) break;
      ws_load(xs, A.x, st);
    }
    if (ctl.fail) break;
    // ---- the final LayerNorm and the logits (no bias), chunk by chunk
    ws_ln(xs, cur, A.lnw, A.lnb, st, shd);
    for (int c = 0; c < nchunk; c++) {
      const unsigned char* wl = consume(L + c);
      if (!wl) break;
      const int a = min(v1, v0 + c * A.lrows), b = min(v1, a + A.lrows);
      ws_rows(WS_STORE, WsOut{wl, a, b - a, nullptr, A.logits, nullptr}, cur, st);
      __syncthreads();
    }
    if (ctl.fail) break;
    if (i + 1 < steps) ws_prep(red, A, v0, v1, &amb);  // the last step's logits stay as made
    if (!ws_sync(A, ctl)) break;
  }
  // no copy in flight into the shared memory the CTA releases: the prefetch
  // for a next step, and any a failed wait left
  for (int b = 0; b < 4; b++) ws_bar_drain(smem_addr(&mbar[b]), fills[b]);
  cpa_wait<0>();
  // the positions and the run's step counter, as the per-kernel path leaves them
  if (cta == 0 && threadIdx.x == 0 && !ctl.fail) {
    A.row_pos[0] = pos0 + steps;
    A.dst_row[0] = pos0 + steps;
    *A.step = steps;
  }
}

}  // namespace

void launch_wembed(const WRows& r, const WMat& emb, const float* pos, float* x, cudaStream_t st) {
  k_wembed<<<r.rows, 128, 0, st>>>(r, emb, pos, x);
}

void launch_wln(const float* x, float* y, const float* w, const float* b, int rows, int n, cudaStream_t st) {
  k_wln<<<rows, 128, 0, st>>>(x, y, w, b, n);
}

void launch_wself(const WRows& r, const float* q, const float* sk, const float* sv, float* att, cudaStream_t st) {
  k_wself<<<dim3(r.rows, r.nh), 128, (r.text_ctx + 64) * 4, st>>>(r, q, sk, sv, att);
}

void launch_wcross(const WRows& r, const float* q, const float* ck, const float* cvt, float* att, float* scratch,
                   size_t scratch_floats, cudaStream_t st) {
  // One CTA per (row, head) when those fill the GPU; otherwise a head's keys
  // (chunks of at most 256) and its outputs are spread over more CTAs, their
  // rows staged by bulk copies (same bits either way).
  const int heads = r.rows * r.nh, ctx = r.audio_ctx, ctx4 = ctx & ~3;
  const int target = 4 * 148;
  int ks = std::min((target + heads - 1) / heads, std::max(1, ctx4 / 64));
  const int ch = std::min(256, ((ctx4 + ks - 1) / ks + 15) / 16 * 16);
  ks = std::max(1, (ctx4 + ch - 1) / ch);
  const size_t need = size_t(heads) * ctx + size_t(heads) * ks;
  if (heads >= 2 * 148 || r.nh * 64 != r.st || !scratch || need > scratch_floats || ctx4 == 0 || ctx % 4 ||
      ctx > 1500) {
    k_wcross<<<dim3(r.rows, r.nh), 256, (ctx + 64) * 4, st>>>(r, q, ck, cvt, att);
    return;
  }
  float* sg = scratch;
  float* mg = scratch + size_t(heads) * ctx;
  k_wcross_sc<<<dim3(r.rows, r.nh, ks), 128, size_t(ch) * 64 * 4, st>>>(r, q, ck, ch, sg, mg);
  if (heads * 16 <= target)
    k_wcross_o<4, true><<<dim3(r.rows, r.nh, 16), 64, size_t(ctx) * 4 * 5, st>>>(r, cvt, ks, sg, mg, att);
  else if (heads * 8 <= target)
    k_wcross_o<8, true><<<dim3(r.rows, r.nh, 8), 128, size_t(ctx) * 4 * 9, st>>>(r, cvt, ks, sg, mg, att);
  else  // 16 outputs a CTA: staging them would leave two CTAs an SM
    k_wcross_o<16, false><<<dim3(r.rows, r.nh, 4), 256, size_t(ctx) * 4, st>>>(r, cvt, ks, sg, mg, att);
}

void launch_wmm(const WmmArgs& a, int groups, cudaStream_t st) {
  // the 128-wide kernel when the product fills its tiles, is at least one
  // 256-deep pass deep and its rows are float4-aligned; the 64-wide one
  // otherwise (both give the same bits)
  const int K = a.w.cols;
  const bool aligned = K % 4 == 0 && a.lda % 4 == 0 && a.a_zs % 4 == 0 && (reinterpret_cast<uintptr_t>(a.a) & 15) == 0 &&
                       (a.w.f ? (reinterpret_cast<uintptr_t>(a.w.f) & 15) == 0 && a.w_zs % 4 == 0
                              : a.w.h ? (reinterpret_cast<uintptr_t>(a.w.h) & 7) == 0 : K % QK == 0);
  if (aligned && a.m >= 96 && a.w.rows >= 96 && K >= 256) {
    dim3 grid((a.w.rows + G_BM - 1) / G_BM, (a.m + G_BM - 1) / G_BM, groups);
    if (a.w.f)
      k_wmm2<0><<<grid, 256, 0, st>>>(a);
    else if (a.w.h)
      k_wmm2<1><<<grid, 256, 0, st>>>(a);
    else
      k_wmm2<2><<<grid, 256, 0, st>>>(a);
    return;
  }
  dim3 grid((a.w.rows + MM_T - 1) / MM_T, (a.m + MM_T - 1) / MM_T, groups);
  k_wmm<<<grid, 256, 0, st>>>(a);
}

// Whether a cluster of `cl` 1024-thread CTAs of k_wproc can be resident
// (asked once per size and device).
bool wproc_cluster_fits(int cl) {
  static int known[64][4] = {};  // 0 unknown, 1 fits, 2 does not
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = cl == 8 ? 0 : cl == 4 ? 1 : 2;
  if (dev < 0 || dev >= 64) return false;
  if (known[dev][slot] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl);
    cfg.blockDim = dim3(1024);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cl;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    const cudaError_t e = cl == 8   ? cudaOccupancyMaxActiveClusters(&n, k_wproc<8>, &cfg)
                          : cl == 4 ? cudaOccupancyMaxActiveClusters(&n, k_wproc<4>, &cfg)
                                    : cudaOccupancyMaxActiveClusters(&n, k_wproc<2>, &cfg);
    if (e != cudaSuccess) cudaGetLastError();
    known[dev][slot] = e == cudaSuccess && n > 0 ? 1 : 2;
  }
  return known[dev][slot] == 1;
}

void wdecode_init() {
  for (int cl : {8, 4, 2}) wproc_cluster_fits(cl);
  cudaFuncSetAttribute(k_wcross_sc, cudaFuncAttributeMaxDynamicSharedMemorySize, 256 * 64 * 4);
  cudaFuncSetAttribute(k_wcross_o<8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 9 * 1500 * 4);
}

void launch_wproc(const WRows& r, float* logits, float* scratch, const WVocabDev& v, WSample* state, int* out,
                  const int* step, int* next_tok, cudaStream_t st) {
  // Each row on a cluster of 8, 4 or 2 CTAs (one CTA an SM) while the rows
  // leave SMs idle, else one CTA per row.
  int cl = r.rows * 8 <= 148 ? 8 : r.rows * 4 <= 148 ? 4 : r.rows * 2 <= 148 ? 2 : 1;
  while (cl > 1 && !wproc_cluster_fits(cl)) cl /= 2;
  if (cl == 1) {
    k_wproc<1><<<r.rows, 1024, 0, st>>>(r, logits, scratch, v, state, out, step, next_tok);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(r.rows * cl);
  cfg.blockDim = dim3(1024);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cl;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cl == 8)
    cudaLaunchKernelEx(&cfg, k_wproc<8>, r, logits, scratch, v, state, out, step, next_tok);
  else if (cl == 4)
    cudaLaunchKernelEx(&cfg, k_wproc<4>, r, logits, scratch, v, state, out, step, next_tok);
  else
    cudaLaunchKernelEx(&cfg, k_wproc<2>, r, logits, scratch, v, state, out, step, next_tok);
}

void launch_wtick(int rows, int* row_pos, int* dst_row, int text_ctx, int advance, int* step, cudaStream_t st) {
  k_wtick<<<(rows + 127) / 128, 128, 0, st>>>(rows, row_pos, dst_row, text_ctx, advance, step);
}

void launch_wnospeech(const float* logits, int vocab, int nosp, float* scratch, float* out, int rows, cudaStream_t st) {
  k_wnospeech<<<rows, 1024, 0, st>>>(logits, vocab, nosp, scratch, out);
}

void launch_wenc_conv1(const float* mel, float* x1, int nmel, int n, cudaStream_t st) {
  k_wenc_conv1<<<dim3((3000 * nmel * 3 + 255) / 256, n), 256, 0, st>>>(mel, x1, nmel);
}

void launch_wenc_conv2(const float* h1, float* x2, int state, int ctx, int n, cudaStream_t st) {
  k_wenc_conv2<<<dim3((ctx * state * 3 + 255) / 256, n), 256, 0, st>>>(h1, x2, state, ctx);
}

void launch_wenc_heads(const float* q, const float* k, const float* v, float* qh, float* kh, float* vt, int ctx,
                       int state, int nh, float sc, int n, cudaStream_t st) {
  k_wenc_heads<<<dim3((ctx * state + 255) / 256, n), 256, 0, st>>>(q, k, v, qh, kh, vt, ctx, state, nh, sc);
}

void launch_wenc_softmax(float* x, int len, long rows, cudaStream_t st) {
  if (len <= kSmRow)
    k_wenc_softmax_reg<<<unsigned((rows + 7) / 8), 256, 0, st>>>(x, len, rows);
  else
    k_wenc_softmax<<<unsigned((rows + 7) / 8), 256, 0, st>>>(x, len, rows);
}

void whisper_kernels_init() {}

void launch_wwiden(const WMat& w, uint16_t* h, cudaStream_t st) {
  const size_t n = size_t(w.rows) * w.cols;
  k_wwiden<<<unsigned((n + 255) / 256), 256, 0, st>>>(w.q, w.d, h, n);
}

size_t wstep1_smem(const WStep1Args& a) {
  const size_t floats = size_t(a.st) + size_t(std::max(a.st, a.ff)) + size_t(std::max(a.ctx, a.text_ctx)) + 64 +
                        size_t(a.xv_floats) + size_t(a.xk_floats);
  return sizeof(float) * floats + 2 * size_t(a.wb);
}

int wstep1_max_active(size_t smem) {
  int n = 0;
  if (cudaFuncSetAttribute(k_wstep1, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_wstep1, WS_NT, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

cudaError_t launch_wstep1(const WStep1Args* d_args, int grid, size_t smem, int pos0, int steps, cudaStream_t st) {
  void* args[] = {(void*)&d_args, (void*)&pos0, (void*)&steps};
  return cudaLaunchCooperativeKernel((const void*)k_wstep1, dim3(grid), dim3(WS_NT), args, smem, st);
}

}  // namespace grx
