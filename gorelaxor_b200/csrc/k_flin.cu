// The float path of products with one row of activations per stream
// (internal/kern/gemm.go:195-259, kern.go:189 false branch; whisper/gemm.go:
// 212-256): the flow head, the TDT encoder projection of a single frame,
// the Whisper decoder's products and the generic grx_linear float path.
//
// Eight lanes compute one output exactly as one AVX row accumulator does:
//  * Q8_0 weight with rows kept (dot4q8avx, kernels_amd64.s:343-399): per
//    block, lane l forms q[l]·x[l] and three fused steps over q[8+l],
//    q[16+l], q[24+l], then fuses that into its accumulator by the block's
//    f16 scale; HSUM at the end;
//  * F32 or F16 weight (dot4f32avx / dot4f16avx, kernels_amd64.s:99-204;
//    whisper/kernels_amd64.s:88-190): lane l keeps two accumulators for
//    elements 16c+l and 16c+8+l, adds them, HSUM. F16 values widen exactly;
//    a Q8_0 weight read the Whisper way widens through f16(q·d) first.
// Rows past the last group of four take the scalar Go dots (gemm.go:239-
// 249, whisper/gemm.go:240-247), and for F32/F16 a K that is not a
// multiple of 16 adds dotF32Go/dotF16Go of its tail. The bias is added after
// the dot, then the epilogue the caller asked for (FEpi).
//
// Tiling: a CTA holds TS streams' activations and TN weight rows of a K chunk
// in shared memory; each group of 8 lanes (one AVX register) keeps R rows ×
// M streams of accumulators in registers, so every activation loaded from
// shared memory feeds R rows and every weight value M streams. Activations
// are stream-minor, XS = TS + 4 (or + 8) floats per k: the 8 lanes of a group
// (k = … + l) then read 8 disjoint bank quads. Q8_0 blocks are re-laid at
// staging so lane l's four bytes (q[l], q[8+l], q[16+l], q[24+l]) are one
// 32-bit word. The lanes' accumulation runs over k in order, so chunking K
// does not change a result.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

enum WMode { W_F32 = 0, W_Q8 = 1, W_H16 = 2, W_Q8H = 3 };

// Row stride (bytes) ≡ 32 mod 128: the four groups of a warp, on four
// consecutive rows, read four different 8-bank sets.
__host__ __device__ constexpr int fl_wstride(int bytes) { return bytes + ((160 - bytes % 128) % 128); }

constexpr int KC = 256;  // K per shared-memory chunk (small enough for several CTAs per SM)

template <int WM, int R, int M, int GR, int NTH>
struct FlinTile {
  static constexpr int GM = NTH / 8 / GR;  // stream groups
  static_assert(GM * GR * 8 == NTH, "groups of 8 lanes tile the block");
  static constexpr int TN = GR * R;   // weight rows per CTA
  static constexpr int TS = GM * M;   // streams per CTA
  static constexpr int XS = TS + (TS % 8 == 0 ? 4 : 8);
  static_assert(M % 4 == 0 && R * M >= 8, "streams in fours; at least one output per lane after the HSUM");
  static constexpr int wbytes = fl_wstride(WM == W_Q8 ? KC : WM == W_F32 ? 4 * KC : 2 * KC);
  static constexpr int dstride = (KC / QK) | 1;
  static constexpr int wbufs = (WM == W_F32 || WM == W_H16) ? 2 : 1;  // async-copied weights double-buffer
  static constexpr size_t smem =
      size_t(KC) * XS * 4 + size_t(TN) * wbytes * wbufs + (WM == W_Q8 ? size_t(TN) * dstride * 4 : 0);
};

__device__ __forceinline__ float q8h(int8_t q, float d) { return __half2float(__float2half_rn(__fmul_rn(float(q), d))); }

// The weight value (row n, column k) the product multiplies by, from global
// memory (the scalar tails).
__device__ __forceinline__ float w_at(const FArgs& a, int n, int k) {
  if (a.wf) return a.wf[(size_t)n * a.K + k];
  if (a.wh) return __half2float(__ushort_as_half(a.wh[(size_t)n * a.K + k]));
  return q8h(a.wq[(size_t)n * a.K + k], h2f(a.wd[(size_t)n * (a.K / QK) + k / QK]));
}

// dotF32Go / dotF16Go (gemm.go:294-325) of x[k0, k1) against row n: four
// strided unfused sums. x(k) reads the staged activation.
template <class X>
__device__ float go_dot(const FArgs& a, int n, int k0, int k1, X x) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int i = k0;
  for (; i + 4 <= k1; i += 4) {
    s0 = __fadd_rn(s0, __fmul_rn(x(i), w_at(a, n, i)));
    s1 = __fadd_rn(s1, __fmul_rn(x(i + 1), w_at(a, n, i + 1)));
    s2 = __fadd_rn(s2, __fmul_rn(x(i + 2), w_at(a, n, i + 2)));
    s3 = __fadd_rn(s3, __fmul_rn(x(i + 3), w_at(a, n, i + 3)));
  }
  for (; i < k1; i++) s0 = __fadd_rn(s0, __fmul_rn(x(i), w_at(a, n, i)));
  return __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
}

// dotQ8Go (kern.go:249-266): per block four strided unfused sums, scaled.
template <class X>
__device__ float q8_go(const FArgs& a, int n, X x) {
  const int nb = a.K / QK;
  const int8_t* q = a.wq + (size_t)n * a.K;
  float s = 0.f;
  for (int b = 0; b < nb; b++) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int i = 0; i < QK; i += 4) {
      const int k = b * QK + i;
      a0 = __fadd_rn(a0, __fmul_rn(x(k), float(q[k])));
      a1 = __fadd_rn(a1, __fmul_rn(x(k + 1), float(q[k + 1])));
      a2 = __fadd_rn(a2, __fmul_rn(x(k + 2), float(q[k + 2])));
      a3 = __fadd_rn(a3, __fmul_rn(x(k + 3), float(q[k + 3])));
    }
    s = __fadd_rn(s, __fmul_rn(h2f(a.wd[(size_t)n * nb + b]), __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3)));
  }
  return s;
}

// The physical rows of logical row m in x and y (FArgs row groups).
__device__ __forceinline__ int fl_row(const FArgs& a, int m) {
  return a.rg_len ? (m / a.rg_len) * a.rg_stride + a.rg_off + m % a.rg_len : m;
}
__device__ __forceinline__ int fl_yrow(const FArgs& a, int m) {
  return a.rg_len ? (m / a.rg_len) * a.ry_stride + a.ry_off + m % a.rg_len : m;
}

// Output (m, n) of the dot r: bias, then the epilogue.
__device__ __forceinline__ void fl_out(const FArgs& a, int m, int n, float r) {
  const float v = a.bias ? __fadd_rn(r, a.bias[n]) : r;
  float* yp = a.y + (size_t)fl_yrow(a, m) * a.ldy + n;
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
      const float* aux =
          a.aux_noise ? a.io->noise + ((size_t)a.io->frame * a.io->rows + a.io->row0) * a.ldaux : a.aux;
      const float cur = __fadd_rn(aux[(size_t)m * a.ldaux + n], __fdiv_rn(v, a.steps));
      *yp = cur;
      const float sc = __fadd_rn(__fmul_rn(cur, a.stdv[n]), a.mean[n]);
      if (a.out2) a.out2[(size_t)m * a.ldy + n] = cur;
      if (a.out3) a.out3[(size_t)m * a.ldy + n] = sc;
      if (a.io_out) {
        const size_t o = ((size_t)a.io->frame * a.io->rows + a.io->row0 + m) * a.ldy + n;
        if (a.io->latent) a.io->latent[o] = cur;
        if (a.io->scaled) a.io->scaled[o] = sc;
      }
      break;
    }
    case FE_RESID:
      *yp = __fadd_rn(*yp, v);
      break;
    case FE_GELU:
      *yp = gelu_avx(v);
      break;
    case FE_ROWPOS:
      a.y[(size_t)a.dst_row[m] * a.ldy + n] = v;
      break;
    case FE_QKV: {
      const int sg = n / a.seg, c = n - sg * a.seg;
      const float* b = a.qkv_bias[sg];
      const float w = b ? __fadd_rn(r, b[c]) : r;
      if (sg == 0)
        a.y[(size_t)m * a.ldy + c] = w;
      else
        a.qkv_y[sg - 1][(size_t)a.dst_row[m] * a.ldy + c] = w;
      break;
    }
    default:
      *yp = v;
  }
}

__device__ __forceinline__ void cp16f(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(uint32_t(__cvta_generic_to_shared(dst))), "l"(src));
}

// Lane word l of a 32-byte Q8_0 block (w[j] = bytes 4j..4j+3): bytes l,
// 8+l, 16+l, 24+l.
__device__ __forceinline__ uint32_t lane_word(const uint32_t (&w)[8], int l) {
  const int h = l >> 2, p = l & 3;
  const uint32_t sel = uint32_t(p | ((4 + p) << 4));
  const uint32_t lo = __byte_perm(w[h], w[2 + h], sel), hi = __byte_perm(w[4 + h], w[6 + h], sel);
  return __byte_perm(lo, hi, 0x5410);
}

template <int WM, int R, int M, int GR, int NTH>
__global__ void __launch_bounds__(NTH) k_flin(FArgs a) {
  using T = FlinTile<WM, R, M, GR, NTH>;
  constexpr int TS = T::TS, TN = T::TN, XS = T::XS, NC = M / 4, RM = R * M;
  extern __shared__ __align__(16) uint8_t fsm[];
  const int K = a.K;
  const int tid = threadIdx.x, g = tid >> 3, l = tid & 7, rg = g % GR, sg = g / GR;
  const int n0 = blockIdx.x * TN, m0 = blockIdx.y * TS;
  const int mt = min(TS, a.M - m0), nrows = min(TN, a.N - n0);
  float* xs = reinterpret_cast<float*>(fsm);
  uint8_t* ws = fsm + size_t(KC) * XS * 4;
  constexpr int wst = T::wbytes, dst = T::dstride;
  float* ds = reinterpret_cast<float*>(ws + size_t(TN) * wst);
  const float* xsrc = a.x_noise ? a.io->noise + ((size_t)a.io->frame * a.io->rows + a.io->row0) * a.ldx : a.x;
  const int kfull = WM == W_Q8 ? K : (K & ~15);  // the vector part of the dot

  f2 acc[R][M / 2], acc1[R][M / 2];
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int p = 0; p < M / 2; p++) acc[r][p] = acc1[r][p] = 0;

  // Chunk c+1's operands come from global memory into registers (the F32 and
  // F16 weights by async copy into the other of two buffers) while chunk c is
  // multiplied, so a product waits on memory once rather than once per chunk
  // and per load.
  constexpr bool WASYNC = WM == W_F32 || WM == W_H16;
  constexpr int XI = (TS * (KC / 8) + NTH - 1) / NTH;   // activation items: (stream, 8 values)
  constexpr int WQI = (TN * (KC / QK) + NTH - 1) / NTH;  // Q8_0 items: (row, block)
  constexpr int WHI = (TN * (KC / 8) + NTH - 1) / NTH;   // widened Q8_0 items: (row, 8 values)
  constexpr int WDI = WQI > WHI ? WQI : WHI;
  float4 xr0[XI], xr1[XI];
  uint4 qr0[WQI], qr1[WQI];
  uint2 hr[WHI];
  uint16_t qd[WDI];
  const size_t wrow_bytes = WM == W_F32 ? 4 : 2;
  auto fetch = [&](int kc0) {
    const int kn = min(KC, kfull - kc0);
#pragma unroll
    for (int u = 0; u < XI; u++) {
      const int i = tid + u * NTH, m = i % TS, k8 = i / TS;
      if (k8 < kn / 8 && m < mt) {
        const float4* p = reinterpret_cast<const float4*>(xsrc + (size_t)fl_row(a, m0 + m) * a.ldx + kc0 + k8 * 8);
        xr0[u] = p[0];
        xr1[u] = p[1];
      }
    }
    if (WM == W_Q8) {
#pragma unroll
      for (int u = 0; u < WQI; u++) {
        const int i = tid + u * NTH, r = i / (KC / QK), b = i % (KC / QK);
        if (r < nrows && b < kn / QK) {
          const uint4* src = reinterpret_cast<const uint4*>(a.wq + (size_t)(n0 + r) * K + kc0 + b * QK);
          qr0[u] = __ldg(src);
          qr1[u] = __ldg(src + 1);
          qd[u] = a.wd[(size_t)(n0 + r) * (K / QK) + kc0 / QK + b];
        }
      }
    } else if (WM == W_Q8H) {
#pragma unroll
      for (int u = 0; u < WHI; u++) {
        const int i = tid + u * NTH, r = i / (KC / 8), c8 = i % (KC / 8);
        if (r < nrows && c8 < kn / 8) {
          const int k = kc0 + c8 * 8;
          hr[u] = __ldg(reinterpret_cast<const uint2*>(a.wq + (size_t)(n0 + r) * K + k));
          qd[u] = a.wd[(size_t)(n0 + r) * (K / QK) + k / QK];
        }
      }
    }
  };
  auto fetch_async = [&](int kc0, int buf) {
    const int kn = min(KC, kfull - kc0), cpr = kn * int(wrow_bytes) / 16;
    const uint8_t* wsrc = WM == W_F32 ? reinterpret_cast<const uint8_t*>(a.wf) : reinterpret_cast<const uint8_t*>(a.wh);
    uint8_t* wb = ws + size_t(buf) * TN * wst;
    for (int i = tid; i < nrows * cpr; i += NTH) {
      const int r = i / cpr, c = i - r * cpr;
      cp16f(wb + size_t(r) * wst + c * 16, wsrc + ((size_t)(n0 + r) * K + kc0) * wrow_bytes + c * 16);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
  // The fetched registers to shared memory: activations stream-minor, Q8_0
  // blocks re-laid into lane words, widened values as halves.
  auto stage = [&](int kc0) {
    const int kn = min(KC, kfull - kc0);
#pragma unroll
    for (int u = 0; u < XI; u++) {
      const int i = tid + u * NTH, m = i % TS, k8 = i / TS;
      if (k8 < kn / 8) {
        const bool ok = m < mt;
        const float v[8] = {ok ? xr0[u].x : 0.f, ok ? xr0[u].y : 0.f, ok ? xr0[u].z : 0.f, ok ? xr0[u].w : 0.f,
                            ok ? xr1[u].x : 0.f, ok ? xr1[u].y : 0.f, ok ? xr1[u].z : 0.f, ok ? xr1[u].w : 0.f};
#pragma unroll
        for (int j = 0; j < 8; j++) xs[(k8 * 8 + j) * XS + m] = v[j];
      }
    }
    if (WM == W_Q8) {
#pragma unroll
      for (int u = 0; u < WQI; u++) {
        const int i = tid + u * NTH, r = i / (KC / QK), b = i % (KC / QK);
        if (r < nrows && b < kn / QK) {
          const uint32_t w[8] = {qr0[u].x, qr0[u].y, qr0[u].z, qr0[u].w, qr1[u].x, qr1[u].y, qr1[u].z, qr1[u].w};
          uint4* dstp = reinterpret_cast<uint4*>(ws + size_t(r) * wst + b * 32);
          dstp[0] = make_uint4(lane_word(w, 0), lane_word(w, 1), lane_word(w, 2), lane_word(w, 3));
          dstp[1] = make_uint4(lane_word(w, 4), lane_word(w, 5), lane_word(w, 6), lane_word(w, 7));
          ds[r * dst + b] = h2f(qd[u]);
        }
      }
    } else if (WM == W_Q8H) {
#pragma unroll
      for (int u = 0; u < WHI; u++) {
        const int i = tid + u * NTH, r = i / (KC / 8), c8 = i % (KC / 8);
        if (r < nrows && c8 < kn / 8) {
          const float d = h2f(qd[u]);
          const int8_t* qb = reinterpret_cast<const int8_t*>(&hr[u]);
          __half h[8];
#pragma unroll
          for (int j = 0; j < 8; j++) h[j] = __float2half_rn(__fmul_rn(float(qb[j]), d));
          *reinterpret_cast<uint4*>(ws + size_t(r) * wst + c8 * 16) = *reinterpret_cast<const uint4*>(h);
        }
      }
    }
  };

  const int nch = (kfull + KC - 1) / KC;
  if (nch > 0) {
    fetch(0);
    if (WASYNC) fetch_async(0, 0);
  }
  for (int ch = 0; ch < nch; ch++) {
    const int kc0 = ch * KC, kn = min(KC, kfull - kc0), nb = kn / QK;
    if (ch > 0) __syncthreads();  // the previous chunk's readers are done
    stage(kc0);
    if (ch + 1 < nch) {
      fetch(kc0 + KC);
      if (WASYNC) fetch_async(kc0 + KC, (ch + 1) & 1);
    }
    if (WASYNC) {
      if (ch + 1 < nch)
        asm volatile("cp.async.wait_group 1;\n" ::);
      else
        asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    const uint8_t* wsb = ws + (WASYNC ? size_t(ch & 1) * TN * wst : 0);

    // ---- the dots over this chunk: rows rg·R + r, streams sg·M + 4c + e
    const float* xg = xs + sg * M;
    if (WM == W_Q8) {
      const uint8_t* wr = wsb + size_t(rg * R) * wst + 4 * l;
      const float* dr = ds + rg * R * dst;
      for (int b = 0; b < nb; b++) {
        uint32_t qw[R];
        float dv[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
          qw[r] = *reinterpret_cast<const uint32_t*>(wr + size_t(r) * wst + b * 32);
          dv[r] = dr[r * dst + b];
        }
        f2 y[R][M / 2];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float* xk = xg + (b * QK + l + 8 * i) * XS;
          ulonglong2 X[NC];
#pragma unroll
          for (int c = 0; c < NC; c++) X[c] = *reinterpret_cast<const ulonglong2*>(xk + 4 * c);
#pragma unroll
          for (int r = 0; r < R; r++) {
            const f2 q = f2dup(float(int8_t(qw[r] >> (8 * i))));
#pragma unroll
            for (int c = 0; c < NC; c++) {
              if (i == 0) {
                y[r][2 * c] = f2mul(q, X[c].x);
                y[r][2 * c + 1] = f2mul(q, X[c].y);
              } else {
                y[r][2 * c] = f2fma(q, X[c].x, y[r][2 * c]);
                y[r][2 * c + 1] = f2fma(q, X[c].y, y[r][2 * c + 1]);
              }
            }
          }
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
          const f2 D = f2dup(dv[r]);
#pragma unroll
          for (int p = 0; p < M / 2; p++) acc[r][p] = f2fma(y[r][p], D, acc[r][p]);
        }
      }
    } else {
      for (int c16 = 0; c16 < kn; c16 += 16) {
        const float* x0 = xg + (c16 + l) * XS;
        const float* x1 = x0 + 8 * XS;
        ulonglong2 X0[NC], X1[NC];
#pragma unroll
        for (int c = 0; c < NC; c++) {
          X0[c] = *reinterpret_cast<const ulonglong2*>(x0 + 4 * c);
          X1[c] = *reinterpret_cast<const ulonglong2*>(x1 + 4 * c);
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
          const uint8_t* wrow = wsb + size_t(rg * R + r) * wst;
          float w0, w1;
          if (WM == W_F32) {
            w0 = reinterpret_cast<const float*>(wrow)[c16 + l];
            w1 = reinterpret_cast<const float*>(wrow)[c16 + 8 + l];
          } else {
            w0 = __half2float(reinterpret_cast<const __half*>(wrow)[c16 + l]);
            w1 = __half2float(reinterpret_cast<const __half*>(wrow)[c16 + 8 + l]);
          }
          const f2 W0 = f2dup(w0), W1 = f2dup(w1);
#pragma unroll
          for (int c = 0; c < NC; c++) {
            acc[r][2 * c] = f2fma(X0[c].x, W0, acc[r][2 * c]);
            acc[r][2 * c + 1] = f2fma(X0[c].y, W0, acc[r][2 * c + 1]);
            acc1[r][2 * c] = f2fma(X1[c].x, W1, acc1[r][2 * c]);
            acc1[r][2 * c + 1] = f2fma(X1[c].y, W1, acc1[r][2 * c + 1]);
          }
        }
      }
    }
  }
  if (WM != W_Q8)
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int p = 0; p < M / 2; p++) acc[r][p] = f2add(acc[r][p], acc1[r][p]);

  // ---- HSUM ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7)) of every output, spread:
  // after the exchanges over lane bits 2, 0 and 1 each lane of the group
  // holds RM/8 finished outputs.
  float v[RM];
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int p = 0; p < M / 2; p++) {
      v[r * M + 2 * p] = f2lo(acc[r][p]);
      v[r * M + 2 * p + 1] = f2hi(acc[r][p]);
    }
  const bool hA = l & 4, hB = l & 1, hC = l & 2;
#pragma unroll
  for (int j = 0; j < RM / 2; j++) {
    const float keep = hA ? v[RM / 2 + j] : v[j], send = hA ? v[j] : v[RM / 2 + j];
    v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
#pragma unroll
  for (int j = 0; j < RM / 4; j++) {
    const float keep = hB ? v[RM / 4 + j] : v[j], send = hB ? v[j] : v[RM / 4 + j];
    v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 1));
  }
#pragma unroll
  for (int j = 0; j < RM / 8; j++) {
    const float keep = hC ? v[RM / 8 + j] : v[j], send = hC ? v[j] : v[RM / 8 + j];
    v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 2));
  }
  const int obase = (hA ? RM / 2 : 0) + (hB ? RM / 4 : 0) + (hC ? RM / 8 : 0);
  const int ntail = a.N & ~3;
#pragma unroll
  for (int j = 0; j < RM / 8; j++) {
    const int o = obase + j, r = o / M, mm = o % M;
    const int nl = rg * R + r, ml = sg * M + mm;
    if (nl >= nrows || ml >= mt) continue;
    const int n = n0 + nl, m = m0 + ml;
    const float* xrow = xsrc + (size_t)fl_row(a, m) * a.ldx;
    auto xg = [&](int k) { return xrow[k]; };
    float r_;
    if (n >= ntail)  // a row past the last group of four: the scalar Go dot
      r_ = WM == W_Q8 ? q8_go(a, n, xg) : go_dot(a, n, 0, K, xg);
    else if (WM != W_Q8 && kfull < K)  // dotF32x4/dotF16x4: + the Go dot of the tail
      r_ = __fadd_rn(v[j], go_dot(a, n, kfull, K, xg));
    else
      r_ = v[j];
    fl_out(a, m, n, r_);
  }
}

template <int WM, int R, int M, int GR, int NTH>
void fl_init() {
  cudaFuncSetAttribute(k_flin<WM, R, M, GR, NTH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       int(FlinTile<WM, R, M, GR, NTH>::smem));
}

template <int WM, int R, int M, int GR, int NTH>
void fl_launch(const FArgs& a, cudaStream_t st) {
  using T = FlinTile<WM, R, M, GR, NTH>;
  dim3 grid((a.N + T::TN - 1) / T::TN, (a.M + T::TS - 1) / T::TS);
  k_flin<WM, R, M, GR, NTH><<<grid, NTH, T::smem, st>>>(a);
}

template <int WM, int R, int M, int GR, int NTH>
int fl_ctas(const FArgs& a) {
  using T = FlinTile<WM, R, M, GR, NTH>;
  return ((a.N + T::TN - 1) / T::TN) * ((a.M + T::TS - 1) / T::TS);
}

// Per weight kind and shape. Every configuration gives the same bits (the
// lanes' order over k is fixed), so the choice is by speed, from timings of
// the path's product shapes on B200: a product too small to fill the GPU is
// bound by one block's latency through K, so the tile shrinks until the
// blocks cover the SMs; K of one chunk or less wants square tiles (a tall
// weight tile is re-read once per stream tile).
constexpr int kFillCtas = 148;
template <int WM>
void fl_dispatch(const FArgs& a, cudaStream_t st) {
  if (a.M <= 8) {
    // 64 rows × 4 streams for wide products (the Whisper logits: 24.7 µs
    // against 50.6 at one stream), else 8 rows × 8 streams
    if (fl_ctas<WM, 2, 4, 32, 256>(a) >= 2 * kFillCtas)
      fl_launch<WM, 2, 4, 32, 256>(a, st);
    else
      fl_launch<WM, 1, 8, 8, 64>(a, st);
  } else if (fl_ctas<WM, 4, 16, 16, 256>(a) >= 2 * kFillCtas) {
    // 64 rows × 32 streams: each staged activation tile serves twice the
    // rows (the Whisper logits at 32 streams: 30.7 k tokens/s against 30.0 k)
    fl_launch<WM, 4, 16, 16, 256>(a, st);
  } else if (fl_ctas<WM, 2, 16, 16, 256>(a) >= 2 * kFillCtas) {
    fl_launch<WM, 2, 16, 16, 256>(a, st);  // 32 rows × 32 streams
  } else if (a.K <= 64 || (a.M <= 32 && fl_ctas<WM, 2, 8, 8, 128>(a) >= kFillCtas)) {
    // 16 rows × 16 streams; at up to 32 streams also for deep products that
    // still fill the SMs (Whisper's stacked q/k/v and fc1 at 32 streams:
    // 30.1 k tokens/s against 29.3 k), which at 128 streams (the FlowLM flow
    // head) measured slower than 64 × 4
    fl_launch<WM, 2, 8, 8, 128>(a, st);
  } else if (fl_ctas<WM, 2, 4, 32, 256>(a) >= kFillCtas) {
    fl_launch<WM, 2, 4, 32, 256>(a, st);  // 64 rows × 4 streams
  } else {
    fl_launch<WM, 1, 8, 8, 64>(a, st);  // 8 rows × 8 streams
  }
}

template <int WM>
void fl_init_all() {
  fl_init<WM, 2, 4, 32, 256>();
  fl_init<WM, 4, 16, 16, 256>();
  fl_init<WM, 2, 16, 16, 256>();
  fl_init<WM, 2, 8, 8, 128>();
  fl_init<WM, 1, 8, 8, 64>();
}

}  // namespace

void launch_flin(const FArgs& a0, int M, cudaStream_t st) {
  FArgs a = a0;
  a.M = M;
  if (a.wq && a.q8_as_f16)
    fl_dispatch<W_Q8H>(a, st);
  else if (a.wq)
    fl_dispatch<W_Q8>(a, st);
  else if (a.wh)
    fl_dispatch<W_H16>(a, st);
  else
    fl_dispatch<W_F32>(a, st);
}

void flin_kernels_init() {
  fl_init_all<W_F32>();
  fl_init_all<W_Q8>();
  fl_init_all<W_H16>();
  fl_init_all<W_Q8H>();
}

// K is chunked, so any K that the weight format allows is taken.
int flin_max_k_q8() { return 1 << 16; }

int flin_max_k() { return 1 << 16; }

}  // namespace grx
