// The FastConformer encoder (conformer/encoder.go:41-480) on the device, for
// one utterance per call, rows [time][channels]: the subsampling's
// convolutions, the elementwise steps between the int8 products, and the
// relative-position attention. Every kernel keeps the reference's float32
// operations element by element; the products are the int8 path of k_q8.cu
// (the loader packs the encoder's matrices and drops their rows).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

constexpr uint32_t FULL = 0xffffffffu;

unsigned nblk(long n) { return unsigned((n + 255) / 256); }

// subsample's input (encoder.go:125-131): in[t][f] = mel[f][t] for t < valid.
__global__ void k_fc_mel_in(const float* mel, float* in, int frames, int nm, int valid) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= long(frames) * nm) return;
  const int t = int(i / nm), f = int(i % nm);
  in[i] = t < valid ? mel[long(f) * frames + t] : 0.f;
}

// conv0 (encoder.go:41-75), then maskRows and relu: output (t, f, ch) starts
// at the bias; each nonzero tap v adds v·w through AddScaled (fused for the
// channels below c&~7, Go's unfused step beyond).
__global__ void k_fc_conv0(const float* in, int T, int F, const float* w, const float* b, int c, float* out, int T1,
                           int F1, int L) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= long(T1) * F1 * c) return;
  const int ch = int(i % c), f = int((i / c) % F1), t = int(i / (long(c) * F1));
  float o = b[ch];
  const bool fused = ch < (c & ~7);
  for (int kt = 0; kt < 3; kt++)
    for (int kf = 0; kf < 3; kf++) {
      const int ti = 2 * t + kt - 1, fi = 2 * f + kf - 1;
      const float v = ti >= 0 && ti < T && fi >= 0 && fi < F ? in[long(ti) * F + fi] : 0.f;
      if (v != 0.f) {
        const float wv = w[(kt * 3 + kf) * c + ch];
        o = fused ? __fmaf_rn(wv, v, o) : __fadd_rn(o, __fmul_rn(v, wv));
      }
    }
  out[i] = t >= L ? 0.f : (o < 0.f ? 0.f : o);
}

// dwConv2 (encoder.go:77-111) then maskRows: o = b + Σ w·x, unfused, taps in
// order.
__global__ void k_fc_dwconv2(const float* in, int T, int F, int c, const float* w, const float* b, float* out, int T1,
                             int F1, int L) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= long(T1) * F1 * c) return;
  const int ch = int(i % c), f = int((i / c) % F1), t = int(i / (long(c) * F1));
  float o = b[ch];
  for (int kt = 0; kt < 3; kt++) {
    const int ti = 2 * t + kt - 1;
    if (ti < 0 || ti >= T) continue;
    for (int kf = 0; kf < 3; kf++) {
      const int fi = 2 * f + kf - 1;
      if (fi < 0 || fi >= F) continue;
      o = __fadd_rn(o, __fmul_rn(w[(kt * 3 + kf) * c + ch], in[(long(ti) * F + fi) * c + ch]));
    }
  }
  out[i] = t >= L ? 0.f : o;
}

// maskRows then relu over rows of `width` values.
__global__ void k_fc_mask_relu(float* x, long n, long width, int L) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  x[i] = i / width >= L ? 0.f : (v < 0.f ? 0.f : v);
}

// [t][f][c] → [t][c·F + f] (encoder.go:155-165).
__global__ void k_fc_flatten(const float* y, float* flat, int T, int F, int c) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= long(T) * F * c) return;
  const int f = int(i % F), ch = int((i / F) % c), t = int(i / (long(F) * c));
  flat[i] = y[(long(t) * F + f) * c + ch];
}

__global__ void k_fc_scale(float* x, long n, float s) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fmul_rn(x[i], s);
}

// siluVec over an array of n values (kernels_amd64.go:241-250): siluAVX for
// the first n&~7, siluGo for the rest.
__global__ void k_fc_silu(float* x, long n) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  x[i] = i < (n & ~7L) ? silu_avx(x[i]) : silu_go(x[i]);
}

// AddScaled(x, y, 0.5) over n values (axpy): fused below n&~7.
__global__ void k_fc_axpy_half(float* x, const float* y, long n) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  x[i] = i < (n & ~7L) ? __fmaf_rn(y[i], 0.5f, x[i]) : __fadd_rn(x[i], __fmul_rn(0.5f, y[i]));
}

// qu = q + pos_bias_u, qv = q + pos_bias_v (encoder.go:269-278).
__global__ void k_fc_qpos(const float* q, const float* pu, const float* pv, float* qu, float* qv, long n, int D) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int c = int(i % D);
  qu[i] = __fadd_rn(q[i], pu[c]);
  qv[i] = __fadd_rn(q[i], pv[c]);
}

// The conv module's gate (encoder.go:347-357): g = a·sigmoid(b), Go's expf,
// rows from L on zero.
__global__ void k_fc_glu(const float* a, float* g, int T, int D, int L) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= long(T) * D) return;
  const int t = int(i / D), c = int(i % D);
  const float* r = a + long(t) * 2 * D;
  g[i] = t >= L ? 0.f : __fmul_rn(r[c], sigmoid_go(r[D + c]));
}

// The depthwise convolution over time (encoder.go:359-381, offline: zero
// padding), o = bias (or 0) + Σ w·g unfused, taps in order; then, unless
// the module normalizes with layer norm, the folded batch norm o·s + b and
// siluVec over the T·D array.
__global__ void k_fc_dwconv(const float* g, const float* w, const float* dwb, const float* cnw, const float* cnb,
                            float* out, int T, int D, int K, int padL, int bn_silu) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  const long n = long(T) * D;
  if (i >= n) return;
  const int t = int(i / D), c = int(i % D);
  float o = dwb ? dwb[c] : 0.f;
  for (int j = 0; j < K; j++) {
    const int ti = t + j - padL;
    if (ti < 0 || ti >= T) continue;
    o = __fadd_rn(o, __fmul_rn(w[long(j) * D + c], g[long(ti) * D + c]));
  }
  if (bn_silu) {
    o = __fadd_rn(__fmul_rn(o, cnw[c]), cnb[c]);
    o = i < (n & ~7L) ? silu_avx(o) : silu_go(o);
  }
  out[i] = o;
}

// --- attention ---

// dot4f32avx of n values (n % 16 == 0): two 8-lane fused chains, added, HSUM.
__device__ __forceinline__ float dot4_avx(const float* x, const float* y, int n) {
  float a[8], b[8];
#pragma unroll
  for (int l = 0; l < 8; l++) a[l] = b[l] = 0.f;
  for (int c = 0; c < n; c += 16)
#pragma unroll
    for (int l = 0; l < 8; l++) {
      a[l] = __fmaf_rn(x[c + l], y[c + l], a[l]);
      b[l] = __fmaf_rn(x[c + 8 + l], y[c + 8 + l], b[l]);
    }
#pragma unroll
  for (int l = 0; l < 8; l++) a[l] = __fadd_rn(a[l], b[l]);
  return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[1], a[5])),
                   __fadd_rn(__fadd_rn(a[2], a[6]), __fadd_rn(a[3], a[7])));
}

// dotF32Go: four strided unfused sums.
__device__ __forceinline__ float dot_go(const float* x, const float* y, int n) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int i = 0;
  for (; i + 4 <= n; i += 4) {
    s0 = __fadd_rn(s0, __fmul_rn(x[i], y[i]));
    s1 = __fadd_rn(s1, __fmul_rn(x[i + 1], y[i + 1]));
    s2 = __fadd_rn(s2, __fmul_rn(x[i + 2], y[i + 2]));
    s3 = __fadd_rn(s3, __fmul_rn(x[i + 3], y[i + 3]));
  }
  for (; i < n; i++) s0 = __fadd_rn(s0, __fmul_rn(x[i], y[i]));
  return __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
}

// One output of a MatMulF32 (gemm.go:116-185) row against B row j of an
// n-row B, K = k: the packed kernel's order (0 + the fused chain of each
// 256-deep pass) or gemvRows' (dotF32x4 for j below n&~3 — dot4f32avx of
// k&~15, plus dotF32Go of the rest — else dotF32Go).
__device__ __forceinline__ float mm_dot(const float* x, const float* y, int k, bool packed, int j, int n) {
  if (packed) {
    float c = 0.f;
    for (int k0 = 0; k0 < k; k0 += 256) {
      const int k1 = min(k, k0 + 256);
      float acc = 0.f;
      for (int kb = k0; kb < k1; kb += 16) {  // sixteen loads ahead of the chain
        float yv[16];
#pragma unroll
        for (int u = 0; u < 16; u++) yv[u] = kb + u < k1 ? y[kb + u] : 0.f;
#pragma unroll
        for (int u = 0; u < 16; u++)
          if (kb + u < k1) acc = __fmaf_rn(x[kb + u], yv[u], acc);
      }
      c = __fadd_rn(c, acc);
    }
    return c;
  }
  if (j < (n & ~3)) {
    const int kv = k & ~15;
    float s = kv > 0 ? dot4_avx(x, y, kv) : 0.f;
    if (kv < k) s = __fadd_rn(s, dot_go(x + kv, y + kv, k - kv));
    return s;
  }
  return dot_go(x, y, k);
}

// attention (encoder.go:259-331), offline: a block per (head, query q).
// Queries go in blocks of 32; q's block [q0, q1) makes its MatMulF32 calls
// with nq = q1 − q0 rows, so row i = q − q0 takes the packed order when
// nq > 16 and i < nq/6·6, gemvRows otherwise. Keys [0, L) for q < L
// (nk = L for a block with a valid query, else the rows are zero); scores
// (qu·k + qv·pp[jlo + nq − 1 − i + kk])·scale, masked keys −inf, expSub over
// the row, × 1/Σ; then the values, MatMulF32 of the weights against the
// head's value columns (K = nk). smem: qu, qv [hd], the row [nk], a key
// tile and a position tile [kTile][hd + 1].
constexpr int kTile = 64;  // keys per staged tile of k_fc_attn

__global__ void __launch_bounds__(128) k_fc_attn(const float* qu, const float* qv, const float* k, const float* v,
                                                 const float* pp, float* out, int T, int D, int H, int L, float scale,
                                                 int gemv_only) {
  extern __shared__ float fsm[];
  const int h = blockIdx.x, q = blockIdx.y, tid = threadIdx.x;
  const int hd = D / H, bl = 32;
  const int q0 = q / bl * bl, q1 = min(T, q0 + bl), nq = q1 - q0, i = q - q0;
  if (gemv_only && nq > 16 && i < nq / 6 * 6) return;  // k_fc_attn_blk's row
  const int k0 = 0, nk = q0 < L ? L : 0;
  float* o = out + long(q) * D + h * hd;
  if (nk <= 0) {
    for (int d = tid; d < hd; d += blockDim.x) o[d] = 0.f;
    return;
  }
  float* xu = fsm;
  float* xv = fsm + hd;
  float* row = fsm + 2 * hd;
  __shared__ float red[8];
  for (int d = tid; d < hd; d += blockDim.x) {
    xu[d] = qu[long(q) * D + h * hd + d];
    xv[d] = qv[long(q) * D + h * hd + d];
  }
  __syncthreads();
  const int np = nq + nk - 1, jlo = T - 1 - (q1 - 1) + k0;
  const int lo = 0, hi = q < L ? L : 0;
  const bool packed = nq > 16 && i < nq / 6 * 6;
  // keys in tiles of kTile: their key rows and position rows come into
  // shared memory with coalesced loads (rows padded to an odd stride so that
  // a warp's threads, one row each, read different banks), then thread j
  // computes key t0 + j's two dots from there
  float* kt = row + nk;
  float* pt = kt + kTile * (hd + 1);
  const int hs = hd + 1, h4 = hd >> 2;
  float mx = -__int_as_float(0x7f800000);
  for (int t0 = 0; t0 < nk; t0 += kTile) {
    const int nt = min(kTile, nk - t0);
    __syncthreads();  // the last tile's readers are done
    for (int e = tid; e < nt * h4; e += blockDim.x) {
      const int r = e / h4, c = (e - r * h4) * 4;
      const float4 a = *reinterpret_cast<const float4*>(k + long(k0 + t0 + r) * D + h * hd + c);
      const float4 b = *reinterpret_cast<const float4*>(pp + long(jlo + nq - 1 - i + t0 + r) * D + h * hd + c);
      float* kr = kt + r * hs + c;
      float* pr = pt + r * hs + c;
      kr[0] = a.x, kr[1] = a.y, kr[2] = a.z, kr[3] = a.w;
      pr[0] = b.x, pr[1] = b.y, pr[2] = b.z, pr[3] = b.w;
    }
    __syncthreads();
    if (tid < nt) {
      const int kk = t0 + tid, kq = k0 + kk;
      if (kq < lo || kq >= hi) {
        row[kk] = -__int_as_float(0x7f800000);
      } else {
        const float sc = mm_dot(xu, kt + tid * hs, hd, packed, kk, nk);
        const int jj = nq - 1 - i + kk;
        const float bd = mm_dot(xv, pt + tid * hs, hd, packed, jj, np);
        const float val = __fmul_rn(__fadd_rn(sc, bd), scale);
        row[kk] = val;
        mx = fmaxf(mx, val);
      }
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, s));
  const int warp = tid >> 5, lane = tid & 31;
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const bool empty = mx == -__int_as_float(0x7f800000);
  __syncthreads();
  if (empty) {
    for (int kk = tid; kk < nk; kk += blockDim.x) row[kk] = 0.f;
  } else {
    // expSub: EXP8 for the first nk&~7 with eight lane sums and HSUM, Go's
    // expf for the rest summed in order; then × 1/Σ
    const int n8 = nk & ~7;
    for (int kk = tid; kk < nk; kk += blockDim.x) {
      const float e = __fsub_rn(row[kk], mx);
      row[kk] = kk < n8 ? exp_avx(e) : expf_go(e);
    }
    __syncthreads();
    if (warp == 0) {
      float part = 0.f;
      if (lane < 8)
        for (int c = lane; c < n8; c += 8) part = __fadd_rn(part, row[c]);
      const float savx = hsum8_lanes(part);
      if (lane == 0) {
        float tail = 0.f;
        for (int j = n8; j < nk; j++) tail = __fadd_rn(tail, row[j]);
        red[4] = __fdiv_rn(1.f, __fadd_rn(savx, tail));
      }
    }
    __syncthreads();
    const float inv = red[4];
    for (int kk = tid; kk < nk; kk += blockDim.x) row[kk] = __fmul_rn(row[kk], inv);
  }
  __syncthreads();
  // values: output d is MatMulF32 row i against B row d (value column d of
  // the head, K = nk)
  for (int d = tid; d < hd; d += blockDim.x) {
    const float* vd = v + long(k0) * D + h * hd + d;  // element kk at vd[kk·D]
    float r;
    if (packed) {
      r = 0.f;
      for (int c0 = 0; c0 < nk; c0 += 256) {
        const int c1 = min(nk, c0 + 256);
        float acc = 0.f;
        for (int kb = c0; kb < c1; kb += 16) {  // sixteen loads ahead of the chain
          float vv[16];
#pragma unroll
          for (int u = 0; u < 16; u++) vv[u] = kb + u < c1 ? vd[long(kb + u) * D] : 0.f;
#pragma unroll
          for (int u = 0; u < 16; u++)
            if (kb + u < c1) acc = __fmaf_rn(row[kb + u], vv[u], acc);
        }
        r = __fadd_rn(r, acc);
      }
    } else if (d < (hd & ~3)) {
      const int kv = nk & ~15;
      float a[8], b[8];
#pragma unroll
      for (int l = 0; l < 8; l++) a[l] = b[l] = 0.f;
      for (int c = 0; c < kv; c += 16)
#pragma unroll
        for (int l = 0; l < 8; l++) {
          a[l] = __fmaf_rn(row[c + l], vd[long(c + l) * D], a[l]);
          b[l] = __fmaf_rn(row[c + 8 + l], vd[long(c + 8 + l) * D], b[l]);
        }
      if (kv > 0) {
#pragma unroll
        for (int l = 0; l < 8; l++) a[l] = __fadd_rn(a[l], b[l]);
        r = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[1], a[5])),
                      __fadd_rn(__fadd_rn(a[2], a[6]), __fadd_rn(a[3], a[7])));
      } else {
        r = 0.f;
      }
      if (kv < nk) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        int kk = kv;
        for (; kk + 4 <= nk; kk += 4) {
          s0 = __fadd_rn(s0, __fmul_rn(row[kk], vd[long(kk) * D]));
          s1 = __fadd_rn(s1, __fmul_rn(row[kk + 1], vd[long(kk + 1) * D]));
          s2 = __fadd_rn(s2, __fmul_rn(row[kk + 2], vd[long(kk + 2) * D]));
          s3 = __fadd_rn(s3, __fmul_rn(row[kk + 3], vd[long(kk + 3) * D]));
        }
        for (; kk < nk; kk++) s0 = __fadd_rn(s0, __fmul_rn(row[kk], vd[long(kk) * D]));
        r = __fadd_rn(r, __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3));
      }
    } else {
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
      int kk = 0;
      for (; kk + 4 <= nk; kk += 4) {
        s0 = __fadd_rn(s0, __fmul_rn(row[kk], vd[long(kk) * D]));
        s1 = __fadd_rn(s1, __fmul_rn(row[kk + 1], vd[long(kk + 1) * D]));
        s2 = __fadd_rn(s2, __fmul_rn(row[kk + 2], vd[long(kk + 2) * D]));
        s3 = __fadd_rn(s3, __fmul_rn(row[kk + 3], vd[long(kk + 3) * D]));
      }
      for (; kk < nk; kk++) s0 = __fadd_rn(s0, __fmul_rn(row[kk], vd[long(kk) * D]));
      r = __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
    }
    o[d] = r;
  }
}

// The packed-order rows of attention (those k_fc_attn returns on with
// gemv_only), a block per (head, query block of 32): rows i < nq/6·6 of a
// block with nq > 16. All its rows' scores against every key are computed
// from shared-memory tiles of 32 key rows and of the position rows they
// need (each score two fused chains over hd, 0 + the chain, as the packed
// kernel does for K ≤ 256), kept in shared memory for the softmax (a warp
// per row: EXP8 lanes, eight running sums, HSUM, Go's expf for the tail,
// × 1/Σ), then each output runs the packed order over the keys (the chain
// folded into C at every 256-deep boundary) from shared tiles of value rows.
// Padded queries (q ≥ L) get zero rows, as the reference clears them.
constexpr int kBQ = 32, kKT = 32, kBlkRows = 16;  // queries per block, keys per tile, rows per thread (values)

size_t fc_blk_smem(int hd, int nk) {
  const int hs = hd + 1;
  return (size_t(2) * kBQ * hs + size_t(kKT) * hs + size_t(kKT + kBQ - 1) * hs + size_t(kBQ) * nk) * sizeof(float);
}

__global__ void __launch_bounds__(256) k_fc_attn_blk(const float* qu, const float* qv, const float* k, const float* v,
                                                     const float* pp, float* out, int T, int D, int H, int L,
                                                     float scale) {
  extern __shared__ float bsm[];
  const int h = blockIdx.x, blk = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd = D / H, hs = hd + 1;
  const int q0 = blk * kBQ, q1 = min(T, q0 + kBQ), nq = q1 - q0;
  if (nq <= 16) return;  // gemvRows throughout: k_fc_attn's
  const int nr = nq / 6 * 6;  // the packed rows of this block
  const int nk = q0 < L ? L : 0;
  if (nk <= 0) {
    for (int e = tid; e < nr * hd; e += blockDim.x) out[long(q0 + e / hd) * D + h * hd + e % hd] = 0.f;
    return;
  }
  const int jlo = T - q1;  // T − 1 − (q1 − 1) + k0, k0 = 0
  float* xu = bsm;
  float* xv = xu + kBQ * hs;
  float* kt = xv + kBQ * hs;           // key rows, later value rows [kKT][hs]
  float* pt = kt + kKT * hs;           // position rows [kKT + kBQ − 1][hs]
  float* S = pt + (kKT + kBQ - 1) * hs;  // [nr][nk]
  const float NEG = -__int_as_float(0x7f800000);
  for (int e = tid; e < nr * hd; e += blockDim.x) {
    const int i = e / hd, d = e - i * hd;
    xu[i * hs + d] = qu[long(q0 + i) * D + h * hd + d];
    xv[i * hs + d] = qv[long(q0 + i) * D + h * hd + d];
  }
  // scores: warp w has rows w, w + 8, w + 16, w + 24; lane the tile's key
  for (int t0 = 0; t0 < nk; t0 += kKT) {
    const int nt = min(kKT, nk - t0);
    // the tile's position rows: pair (i, t0 + j) reads row jlo + nq − 1 − i + t0 + j,
    // i.e. staged row (nr − 1 − i) + j from pbase
    const int pbase = jlo + nq - nr + t0, np_t = nr - 1 + nt;
    __syncthreads();
    for (int e = tid; e < nt * hd; e += blockDim.x) {
      const int r = e / hd, d = e - r * hd;
      kt[r * hs + d] = k[long(t0 + r) * D + h * hd + d];
    }
    for (int e = tid; e < np_t * hd; e += blockDim.x) {
      const int r = e / hd, d = e - r * hd;
      pt[r * hs + d] = pp[long(pbase + r) * D + h * hd + d];
    }
    __syncthreads();
    if (lane < nt) {
      float as[4], ab[4];
      bool live[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        as[u] = ab[u] = 0.f;
        const int i = warp + 8 * u;
        live[u] = i < nr && q0 + i < L;
      }
      const float* kr = kt + lane * hs;
      for (int d = 0; d < hd; d++) {
        const float kv = kr[d];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int i = warp + 8 * u;
          if (live[u]) {
            as[u] = __fmaf_rn(xu[i * hs + d], kv, as[u]);
            ab[u] = __fmaf_rn(xv[i * hs + d], pt[(nr - 1 - i + lane) * hs + d], ab[u]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int i = warp + 8 * u;
        if (i >= nr) continue;
        S[i * nk + t0 + lane] =
            live[u] ? __fmul_rn(__fadd_rn(__fadd_rn(0.f, as[u]), __fadd_rn(0.f, ab[u])), scale) : NEG;
      }
    }
  }
  __syncthreads();
  // softmax of each row, a warp per row
  for (int i = warp; i < nr; i += 8) {
    float* r = S + i * nk;
    float mx = NEG;
    for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, r[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    if (mx == NEG) {
      for (int j = lane; j < nk; j += 32) r[j] = 0.f;
      continue;
    }
    const int n8 = nk & ~7;
    for (int j = lane; j < nk; j += 32) {
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
      for (int j = n8; j < nk; j++) tail = __fadd_rn(tail, r[j]);
      sum = __fdiv_rn(1.f, __fadd_rn(sum, tail));
    }
    const float inv = __shfl_sync(FULL, sum, 0);
    __syncwarp();
    for (int j = lane; j < nk; j += 32) r[j] = __fmul_rn(r[j], inv);
  }
  // values: thread (g, d) has output column d of rows g, g + G, ... (G = 256 / hd)
  const int G = blockDim.x / hd, g = tid / hd, d = tid - g * hd;
  float acc[kBlkRows], c[kBlkRows];
#pragma unroll
  for (int j = 0; j < kBlkRows; j++) acc[j] = c[j] = 0.f;
  for (int t0 = 0; t0 < nk; t0 += kKT) {
    const int nt = min(kKT, nk - t0);
    __syncthreads();  // score/softmax readers or the last value tile's are done
    for (int e = tid; e < nt * hd; e += blockDim.x) {
      const int r = e / hd, dd = e - r * hd;
      kt[r * hs + dd] = v[long(t0 + r) * D + h * hd + dd];
    }
    __syncthreads();
    if (g < G) {
      if ((t0 & 255) == 0) {
#pragma unroll
        for (int j = 0; j < kBlkRows; j++) acc[j] = 0.f;
      }
      for (int kk = 0; kk < nt; kk++) {
        const float vv = kt[kk * hs + d];
#pragma unroll
        for (int j = 0; j < kBlkRows; j++) {
          const int i = g + j * G;
          if (i < nr) acc[j] = __fmaf_rn(S[i * nk + t0 + kk], vv, acc[j]);
        }
      }
      if (((t0 + kKT) & 255) == 0 || t0 + nt == nk) {
#pragma unroll
        for (int j = 0; j < kBlkRows; j++) c[j] = __fadd_rn(c[j], acc[j]);
      }
    }
  }
  if (g < G)
#pragma unroll
    for (int j = 0; j < kBlkRows; j++) {
      const int i = g + j * G;
      if (i < nr) out[long(q0 + i) * D + h * hd + d] = c[j];
    }
}

}  // namespace

void launch_fc_mel_in(const float* mel, float* in, int frames, int nm, int valid, cudaStream_t st) {
  k_fc_mel_in<<<nblk(long(frames) * nm), 256, 0, st>>>(mel, in, frames, nm, valid);
}
void launch_fc_conv0(const float* in, int T, int F, const float* w, const float* b, int c, float* out, int T1, int F1,
                     int L, cudaStream_t st) {
  k_fc_conv0<<<nblk(long(T1) * F1 * c), 256, 0, st>>>(in, T, F, w, b, c, out, T1, F1, L);
}
void launch_fc_dwconv2(const float* in, int T, int F, int c, const float* w, const float* b, float* out, int T1, int F1,
                       int L, cudaStream_t st) {
  k_fc_dwconv2<<<nblk(long(T1) * F1 * c), 256, 0, st>>>(in, T, F, c, w, b, out, T1, F1, L);
}
void launch_fc_mask_relu(float* x, long n, long width, int L, cudaStream_t st) {
  k_fc_mask_relu<<<nblk(n), 256, 0, st>>>(x, n, width, L);
}
void launch_fc_flatten(const float* y, float* flat, int T, int F, int c, cudaStream_t st) {
  k_fc_flatten<<<nblk(long(T) * F * c), 256, 0, st>>>(y, flat, T, F, c);
}
void launch_fc_scale(float* x, long n, float s, cudaStream_t st) { k_fc_scale<<<nblk(n), 256, 0, st>>>(x, n, s); }
void launch_fc_silu(float* x, long n, cudaStream_t st) { k_fc_silu<<<nblk(n), 256, 0, st>>>(x, n); }
void launch_fc_axpy_half(float* x, const float* y, long n, cudaStream_t st) {
  k_fc_axpy_half<<<nblk(n), 256, 0, st>>>(x, y, n);
}
void launch_fc_qpos(const float* q, const float* pu, const float* pv, float* qu, float* qv, long n, int D,
                    cudaStream_t st) {
  k_fc_qpos<<<nblk(n), 256, 0, st>>>(q, pu, pv, qu, qv, n, D);
}
void launch_fc_glu(const float* a, float* g, int T, int D, int L, cudaStream_t st) {
  k_fc_glu<<<nblk(long(T) * D), 256, 0, st>>>(a, g, T, D, L);
}
void launch_fc_dwconv(const float* g, const float* w, const float* dwb, const float* cnw, const float* cnb, float* out,
                      int T, int D, int K, int padL, bool bn_silu, cudaStream_t st) {
  k_fc_dwconv<<<nblk(long(T) * D), 256, 0, st>>>(g, w, dwb, cnw, cnb, out, T, D, K, padL, bn_silu ? 1 : 0);
}
void launch_fc_attn(const float* qu, const float* qv, const float* k, const float* v, const float* pp, float* out,
                    int T, int D, int H, int L, float scale, cudaStream_t st) {
  const int hd = D / H, nk = L;
  // the block kernel takes the packed rows when their scores fit in shared
  // memory (and a thread's rows in registers); the per-query kernel the rest
  const size_t bsm = fc_blk_smem(hd, nk);
  const bool blk = nk > 0 && bsm <= size_t(200) * 1024 && hd <= 256 && (kBQ + 256 / hd - 1) / (256 / hd) <= kBlkRows;
  if (blk) k_fc_attn_blk<<<dim3(H, (T + kBQ - 1) / kBQ), 256, bsm, st>>>(qu, qv, k, v, pp, out, T, D, H, L, scale);
  const size_t sm = (size_t(2) * hd + size_t(T) + size_t(2) * kTile * (hd + 1)) * sizeof(float);
  k_fc_attn<<<dim3(H, T), 128, sm, st>>>(qu, qv, k, v, pp, out, T, D, H, L, scale, blk ? 1 : 0);
}
void fconf_kernels_init() {
  cudaFuncSetAttribute(k_fc_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaFuncSetAttribute(k_fc_attn_blk, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

}  // namespace grx
