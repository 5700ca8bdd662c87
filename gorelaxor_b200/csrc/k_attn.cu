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

#include <algorithm>

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

// dotF32Go (gemm.go:294-308) of n values: four strided unfused sums.
template <class X, class Y>
__device__ __forceinline__ float dot_go(X x, Y y, int n) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int i = 0;
  for (; i + 4 <= n; i += 4) {
    s0 = __fadd_rn(s0, __fmul_rn(x(i), y(i)));
    s1 = __fadd_rn(s1, __fmul_rn(x(i + 1), y(i + 1)));
    s2 = __fadd_rn(s2, __fmul_rn(x(i + 2), y(i + 2)));
    s3 = __fadd_rn(s3, __fmul_rn(x(i + 3), y(i + 3)));
  }
  for (; i < n; i++) s0 = __fadd_rn(s0, __fmul_rn(x(i), y(i)));
  return __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(uint32_t(__cvta_generic_to_shared(dst))),
               "l"(src));
}

// transformer.attend for T queries of one stream (nn.go:200-243, T > 1),
// one block per (head, stream, query t). The reference makes each head's
// T × nk scores one kern.MatMulF32 (nk = pos0 + T, the call's keys) and, for
// T ≥ 4, the values another (kern.go:205 → gemm.go:116-185), and those
// choose the arithmetic: up to 16 rows of A, gemvRows (dot4f32avx per group
// of four B rows of the product, dotF32Go past the last group, and a
// dotF32Go of any K tail added); with more, the packed kernel for rows below
// T/6·6 (each output starts at 0 and adds the fused chain of every 256-deep
// pass). Here one thread computes one output in that order. Scores past the
// query's own position are cleared by the reference before the values;
// they are never computed here and enter the value products as zeros. For
// T < 4 the values are added key by key (AddScaled), skipping zero weights.
__global__ void __launch_bounds__(128) k_attn_rows(AttnRowsArgs a) {
  extern __shared__ __align__(16) float rsc[];  // [nk] scores, then weights; then (vstage) V rows
  __shared__ float qh[HD];
  __shared__ float red[8];
  const int h = blockIdx.x, si = blockIdx.y, t = blockIdx.z;
  const int T = a.T[si];
  if (t >= T) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s = a.slot[si], pos0 = a.pos0[si], row = a.row0[si] + t;
  // keys lo0 .. pos0 + T − 1 are the call's (indices j below are relative
  // to lo0); this query sees lo .. p
  const int p = pos0 + t, lo0 = a.context > 0 ? max(0, pos0 - a.context + 1) : 0;
  const int lo = a.context > 0 ? max(lo0, p - a.context + 1) : lo0;
  const int nk = pos0 + T - lo0, v0 = lo - lo0, nvis = p + 1 - lo0;  // visible: v0 .. nvis − 1
  auto krow = [&](int j) {  // cache row of relative key j
    const int ab = lo0 + j;
    return a.ring ? ab % a.ring : ab;
  };
  const size_t kbase = ((((size_t)s * a.layers + a.layer) * 2 + 0) * a.heads + h) * (size_t)a.cap * HD;
  const size_t vbase = ((((size_t)s * a.layers + a.layer) * 2 + 1) * a.heads + h) * (size_t)a.cap * HD;
  const float* K = a.kv + kbase;
  const float* V = a.kv + vbase;
  if (tid < HD) qh[tid] = a.q[(size_t)row * a.d + h * HD + tid];
  // With vstage, the call's value rows come into shared memory while the
  // scores are computed (rows [nk][64] after vstage score slots).
  float* vsm = rsc + a.vstage;
  if (a.vstage) {
    for (int i = tid; i < nk * (HD / 4); i += 128) {
      const int j = i / (HD / 4), c = (i % (HD / 4)) * 4;
      cp_async16(vsm + j * HD + c, V + (size_t)krow(j) * HD + c);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }
  __syncthreads();
  const bool packed = T > 16 && t < T / 6 * 6;  // this query row goes through the packed kernel
  const int nk4 = nk & ~3;

  // --- scores of the visible keys, ·1/√64 ---
  float mx = -__int_as_float(0x7f800000);
  if (packed) {
    for (int j = v0 + tid; j < nvis; j += 128) {
      const float* kj = K + (size_t)krow(j) * HD;
      float acc = 0.f;
      for (int k = 0; k < HD; k++) acc = __fmaf_rn(qh[k], kj[k], acc);
      const float sj = __fmul_rn(__fadd_rn(0.f, acc), 0.125f);
      rsc[j] = sj;
      mx = fmaxf(mx, sj);
    }
  } else {
    // dot4f32avx for keys below nk&~3: 16 lanes per key, lane l the AVX
    // accumulator of elements 16c + l (lanes 8-15 the second register),
    // two keys per warp pass and U pairs in flight
    const int half = lane >> 4, l = lane & 15, jend = min(nvis, nk4);
    const float q0 = qh[l], q1 = qh[16 + l], q2 = qh[32 + l], q3 = qh[48 + l];
    constexpr int U = 4;
    for (int j0 = v0 + warp * 2 * U; j0 < jend; j0 += 4 * 2 * U) {
      float k[U][4];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int j = j0 + 2 * u + half;
        if (j < jend) {
          const float* kr = K + (size_t)krow(j) * HD + l;
          k[u][0] = kr[0];
          k[u][1] = kr[16];
          k[u][2] = kr[32];
          k[u][3] = kr[48];
        } else {
          k[u][0] = k[u][1] = k[u][2] = k[u][3] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int j = j0 + 2 * u + half;
        float acc = __fmaf_rn(q0, k[u][0], 0.f);
        acc = __fmaf_rn(q1, k[u][1], acc);
        acc = __fmaf_rn(q2, k[u][2], acc);
        acc = __fmaf_rn(q3, k[u][3], acc);
        const float sum = hsum8_lanes(__fadd_rn(acc, __shfl_down_sync(FULL, acc, 8)));
        if (l == 0 && j < jend) {
          const float sj = __fmul_rn(sum, 0.125f);
          rsc[j] = sj;
          mx = fmaxf(mx, sj);
        }
      }
    }
    // keys from nk&~3 on: dotF32Go
    for (int j = max(v0, nk4) + tid; j < nvis; j += 128) {
      const float* kj = K + (size_t)krow(j) * HD;
      const float sj = __fmul_rn(dot_go([&](int i) { return qh[i]; }, [&](int i) { return kj[i]; }, HD), 0.125f);
      rsc[j] = sj;
      mx = fmaxf(mx, sj);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  // --- softmax over the visible keys (expSub over the slice v0 .. nvis − 1:
  // EXP8 lanes for its first count&~7, HSUM, Go tail) ---
  const int cnt = nvis - v0, n8 = v0 + (cnt & ~7);
  for (int j = v0 + tid; j < nvis; j += 128) {
    const float x = __fsub_rn(rsc[j], mx);
    rsc[j] = j < n8 ? exp_avx(x) : expf_go(x);
  }
  __syncthreads();
  if (warp == 0) {
    float part = 0.f;
    if (lane < 8)
      for (int c = v0 + lane; c < n8; c += 8) part = __fadd_rn(part, rsc[c]);
    const float savx = hsum8_lanes(part);
    if (lane == 0) {
      float tail = 0.f;
      for (int j = n8; j < nvis; j++) tail = __fadd_rn(tail, rsc[j]);
      red[4] = __fdiv_rn(1.f, __fadd_rn(savx, tail));
    }
  }
  __syncthreads();
  const float inv = red[4];
  for (int j = tid; j < nk; j += 128) rsc[j] = j >= v0 && j < nvis ? __fmul_rn(rsc[j], inv) : 0.f;
  __syncthreads();

  // --- values: thread d owns output d ---
  if (a.vstage) {
    asm volatile("cp.async.wait_all;\n" ::);
    __syncthreads();
  }
  if (tid < HD) {
    const int d = tid;
    const float* vd = V + d;  // element j of the transposed row d is vd[krow(j)·64]
    const float* vsd = vsm + d;
    auto vat = [&](int j) { return a.vstage ? vsd[j * HD] : vd[(size_t)krow(j) * HD]; };
    float o;
    if (T < 4) {
      // AddScaled skips zero weights, and every key outside v0 .. nvis − 1
      // has one; the values come eight at a time ahead of their products
      o = 0.f;
      for (int j0 = v0; j0 < nvis; j0 += 8) {
        float vv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) vv[u] = j0 + u < nvis ? vat(j0 + u) : 0.f;
#pragma unroll
        for (int u = 0; u < 8; u++) {
          const float w = j0 + u < nvis ? rsc[j0 + u] : 0.f;
          if (w != 0.f) o = __fmaf_rn(w, vv[u], o);
        }
      }
    } else if (packed) {
      o = 0.f;
      for (int k0 = 0; k0 < nk; k0 += 256) {
        const int k1 = min(nk, k0 + 256);
        float acc = 0.f;
        for (int j0 = k0; j0 < k1; j0 += 8) {
          float vv[8];
#pragma unroll
          for (int u = 0; u < 8; u++) vv[u] = j0 + u < k1 ? vat(j0 + u) : 0.f;
#pragma unroll
          for (int u = 0; u < 8; u++)
            if (j0 + u < k1) acc = __fmaf_rn(rsc[j0 + u], vv[u], acc);
        }
        o = __fadd_rn(o, acc);
      }
    } else {
      const int kk = nk & ~15;
      float av[8], bv[8];
#pragma unroll
      for (int l = 0; l < 8; l++) av[l] = bv[l] = 0.f;
      for (int c = 0; c < kk; c += 16)
#pragma unroll
        for (int l = 0; l < 8; l++) {
          av[l] = __fmaf_rn(rsc[c + l], vat(c + l), av[l]);
          bv[l] = __fmaf_rn(rsc[c + 8 + l], vat(c + 8 + l), bv[l]);
        }
      if (kk > 0) {
#pragma unroll
        for (int l = 0; l < 8; l++) av[l] = __fadd_rn(av[l], bv[l]);
        o = __fadd_rn(__fadd_rn(__fadd_rn(av[0], av[4]), __fadd_rn(av[1], av[5])),
                      __fadd_rn(__fadd_rn(av[2], av[6]), __fadd_rn(av[3], av[7])));
      } else {
        o = 0.f;
      }
      if (kk < nk)
        o = __fadd_rn(o, dot_go([&](int i) { return rsc[kk + i]; }, [&](int i) { return vat(kk + i); }, nk - kk));
    }
    if (a.out) a.out[(size_t)row * a.d + h * HD + d] = o;
    float sc;
    const int8_t qv = quant_lane(o, &sc);
    a.q8[(size_t)row * a.d + h * HD + d] = qv;
    if (lane == 0) a.q8s[(size_t)row * (a.d / QK) + h * 2 + warp] = make_float2(sc, sc);
  }
}

__global__ void k_embed_rows(float* x, const float* embed, const int* ids, int rows, int d) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* src = embed + (size_t)ids[r] * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) x[(size_t)r * d + i] = src[i];
}

// The most keys whose value rows k_attn_rows stages in shared memory.
constexpr int kVStageRows = 384;

}  // namespace

void launch_attn_rows(const AttnRowsArgs& a0, int nstreams, int tmax, cudaStream_t st) {
  if (nstreams < 1 || tmax < 1) return;
  // the scores of one query: at most the call's keys; up to kVStageRows of
  // them, the value rows too
  AttnRowsArgs a = a0;
  const int nk = a.context > 0 ? std::min(a.cap, a.context - 1 + tmax) : a.cap;
  a.vstage = nk <= kVStageRows ? (nk + 3) & ~3 : 0;
  const size_t sm = (a.vstage ? size_t(a.vstage) * (1 + HD) : size_t(nk)) * sizeof(float);
  k_attn_rows<<<dim3(a.heads, nstreams, tmax), 128, sm, st>>>(a);
}

// Dynamic shared memory up to 200 KB (the per-block limit less the kernels'
// static arrays, with room to spare).
void attn_kernels_init() {
  cudaFuncSetAttribute(k_attn_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaFuncSetAttribute(k_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

void launch_embed_rows(float* x, const float* embed, const int* ids, int rows, int d, cudaStream_t st) {
  if (rows > 0) k_embed_rows<<<rows, 256, 0, st>>>(x, embed, ids, rows, d);
}

void launch_attn(const AttnArgs& a, int M, cudaStream_t st) {
  dim3 grid(a.heads, M);
  k_attn<<<grid, 64, size_t(a.cap) * sizeof(float), st>>>(a);
}

}  // namespace grx
