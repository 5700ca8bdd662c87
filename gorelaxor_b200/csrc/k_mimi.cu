// Mimi's decoder (pockettts/mimi.go:24-150, nn.go:52-64 and 258-327) on
// the device: the steps between and inside its products, for n streams
// decoding one latent each per call, rows laid out [stream][time][channel].
// Each keeps the reference's float32 operations element by element.
//
// Grids are (per-stream work, stream), so index arithmetic stays in 32 bits;
// rows move as float4 (every channel count here is a multiple of 4).
//
// A causal convolution of stride 1 and dilation 1 never materialises its
// im2col matrix: k_mimi_stage writes [carried rows; ELU(x)] contiguously per
// stream, and output row t's window is then the k·cin values from staged
// row t on — a row of stride cin that the products read in place.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// elu (nn.go:52-64) of the value at index e of its stream's len-value
// array: per 512-value chunk t = min(v, 0) through ExpSub(t, 0) — EXP8 for
// the chunk's first len&~7 values, Go's expf for the rest — then
// max(v, 0) + (t − 1).
__device__ __forceinline__ float elu_at(float v, int e, int len) {
  const int c0 = e & ~511, clen = min(512, len - c0);
  const float t = __fsub_rn(v < 0.f ? v : 0.f, 0.f);
  const float ex = e - c0 < (clen & ~7) ? exp_avx(t) : expf_go(t);
  return __fadd_rn(v > 0.f ? v : 0.f, __fsub_rn(ex, 1.f));
}

__device__ __forceinline__ float4 elu4(float4 v, int e, int len) {
  return make_float4(elu_at(v.x, e, len), elu_at(v.y, e + 1, len), elu_at(v.z, e + 2, len), elu_at(v.w, e + 3, len));
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// decode's depthwise ConvTranspose1d for one latent (mimi.go:130-145): with
// z the projected latent, row j < 2S of the full output is 0 + z[c]·up[c][j]
// (cleared, then +=); rows j < S get the partial carried from the last call
// added and are the transformer's input, rows S.. are the next partial.
__global__ void k_mimi_up(const float* z, const float* up, const float* part_in, float* x, float* part_out, int S,
                          int C) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * S * C) return;
  const int j = i / C, c = i - j * C;
  const float v = __fadd_rn(0.f, __fmul_rn(z[size_t(s) * C + c], up[size_t(c) * 2 * S + j]));
  const size_t o = size_t(s) * S * C;
  if (j < S)
    x[o + i] = __fadd_rn(v, part_in[o + i]);
  else
    part_out[o + i - S * C] = v;
}

// The ELU of every stream's len values (len % 4 == 0).
__global__ void k_mimi_elu(const float* in, float* out, int len) {
  const int s = blockIdx.y, i = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= len) return;
  const size_t o = size_t(s) * len + i;
  st4(out + o, elu4(ld4(in + o), i, len));
}

// Rows [carry (P); x (T), through the ELU when elu] of C values into
// stage [P + T]; carry_out gets the last P of those rows (the next call's).
__global__ void k_mimi_stage(const float* x, const float* carry_in, float* carry_out, float* stage, int T, int C,
                             int P, int elu) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  const int C4 = C >> 2, nst = (P + T) * C4;
  if (i >= nst + P * C4) return;
  const int q = i < nst ? i : i - nst;
  const int rq = q / C4, c = (q - rq * C4) * 4, r = rq + (i < nst ? 0 : T);
  float4 v;
  if (r < P) {
    v = ld4(carry_in + (size_t(s) * P + r) * C + c);
  } else {
    v = ld4(x + (size_t(s) * T + r - P) * C + c);
    if (elu) v = elu4(v, (r - P) * C + c, T * C);
  }
  if (i < nst)
    st4(stage + (size_t(s) * (P + T) + r) * C + c, v);
  else
    st4(carry_out + (size_t(s) * P + r - T) * C + c, v);
}

// k_mimi_stage for a channel count that is not a multiple of four (the
// encoder's first convolution reads one channel): one value per thread.
__global__ void k_mimi_stage_s(const float* x, const float* carry_in, float* carry_out, float* stage, int T, int C,
                               int P, int elu) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  const int nst = (P + T) * C;
  if (i >= nst + P * C) return;
  const int q = i < nst ? i : i - nst;
  const int rq = q / C, c = q - rq * C, r = rq + (i < nst ? 0 : T);
  float v;
  if (r < P) {
    v = carry_in[(size_t(s) * P + r) * C + c];
  } else {
    v = x[(size_t(s) * T + r - P) * C + c];
    if (elu) v = elu_at(v, (r - P) * C + c, T * C);
  }
  if (i < nst)
    stage[(size_t(s) * (P + T) + r) * C + c] = v;
  else
    carry_out[(size_t(s) * P + r - T) * C + c] = v;
}

// gemvRows (gemm.go:195-259) of a float32 weight with K < 16 columns for
// rows [off, T) of every stream: every dot is dotF32Go (four strided
// unfused sums, gemm.go:294-308); an output in a group of four is
// 0 + dot (dotF32x4's zeroed start, kernels_amd64.go:75-95), the last n % 4
// the dot itself; then + bias, stored or (resid) added to y.
__global__ void k_mimi_gemv_small(const float* x, int ldx, int sstride, int T, int off, const float* w, int N, int K,
                                  const float* bias, float* y, int resid) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x, rows = T - off;
  if (i >= rows * N) return;
  const int t = off + i / N, j = i - (i / N) * N;
  const float* xr = x + (size_t(s) * sstride + t) * ldx;
  const float* wr = w + size_t(j) * K;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int k = 0;
  for (; k + 4 <= K; k += 4) {
    s0 = __fadd_rn(s0, __fmul_rn(xr[k], wr[k]));
    s1 = __fadd_rn(s1, __fmul_rn(xr[k + 1], wr[k + 1]));
    s2 = __fadd_rn(s2, __fmul_rn(xr[k + 2], wr[k + 2]));
    s3 = __fadd_rn(s3, __fmul_rn(xr[k + 3], wr[k + 3]));
  }
  for (; k < K; k++) s0 = __fadd_rn(s0, __fmul_rn(xr[k], wr[k]));
  float v = __fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3);
  if (j < (N & ~3)) v = __fadd_rn(0.f, v);
  if (bias) v = __fadd_rn(v, bias[j]);
  float* yp = y + (size_t(s) * T + t) * N + j;
  *yp = resid ? __fadd_rn(*yp, v) : v;
}

// The row tables of a call of T rows per stream (the encoder's last piece
// can be shorter than the others): row r belongs to stream slot r / T,
// call-stream i starts at row i·T, runs T rows and uses slot i.
__global__ void k_mimi_rowtab(int T, int n, int* rowslot, int* crow0, int* cT, int* cslot) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n * T) rowslot[i] = i / T;
  if (i < n) {
    crow0[i] = i * T;
    cT[i] = T;
    cslot[i] = i;
  }
}

// The encoder's downsampling convolution pads its first call with copies of
// the first row ("replicate", model.go:308-313): carry[s][p] = x[s][0] for
// p < P.
__global__ void k_mimi_replicate(const float* x, int T, int C, float* carry, int P) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P * C) return;
  carry[size_t(s) * P * C + i] = x[size_t(s) * T * C + i % C];
}

// conv.run's window (nn.go:275-300) for any stride and dilation: rows
// [prev (P); x (T)] of cin values; output row t takes rows t·stride + j·dil
// for j < k. The last P rows become the next call's prev.
__global__ void k_mimi_im2col(const float* x, const float* prev_in, float* prev_out, float* col, int T, int cin,
                              int k, int stride, int dil, int P) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  const int C4 = cin >> 2, To = T / stride, ncol = To * k * C4;
  if (i >= ncol + P * C4) return;
  auto row = [&](int r, int c) {
    return r < P ? ld4(prev_in + (size_t(s) * P + r) * cin + c) : ld4(x + (size_t(s) * T + r - P) * cin + c);
  };
  if (i < ncol) {
    const int c4 = i % C4, tj = i / C4, j = tj % k, t = tj / k;
    st4(col + size_t(s) * To * k * cin + size_t(i) * 4, row(t * stride + j * dil, c4 * 4));
  } else {
    const int q = i - ncol, r = q / C4, c = (q % C4) * 4;
    st4(prev_out + (size_t(s) * P + r) * cin + c, row(T + r, c));
  }
}

// The int8 path's activation rounding (quantU8, q8int.go:88-105) of rows of
// K values: row t of stream s at x + (s·sstride + t)·ldx (rows may overlap:
// a staged convolution window), through the ELU first when elu_len (x then
// dense, the element's index in its stream's array is t·K + k). Eight values
// per thread, a 32-value block over four lanes; outputs dense [n·T][K].
__global__ void k_mimi_quant(const float* x, int ldx, int sstride, int T, int K, int elu_len, int8_t* q, float2* qs) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  const int K8 = K >> 3;
  const bool live = i < T * K8;
  const int t = live ? i / K8 : 0, k = live ? (i - t * K8) * 8 : 0;
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (live) {
    const float* src = x + (size_t(s) * sstride + t) * ldx + k;
    float4 a = ld4(src), b = ld4(src + 4);
    if (elu_len) {
      a = elu4(a, t * K + k, elu_len);
      b = elu4(b, t * K + k + 4, elu_len);
    }
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
  float amax = 0.f;
#pragma unroll
  for (int u = 0; u < 8; u++) amax = fmaxf(amax, fabsf(v[u]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  if (!live) return;
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int u = 0; u < 4; u++) {
    w0 |= uint32_t(uint8_t(quant_val(v[u], amax))) << (8 * u);
    w1 |= uint32_t(uint8_t(quant_val(v[4 + u], amax))) << (8 * u);
  }
  const size_t row = size_t(s) * T + t;
  *reinterpret_cast<uint2*>(q + row * K + k) = make_uint2(w0, w1);
  if ((k & 31) == 0) {
    const float sc = quant_scale(amax);
    qs[row * (K >> 5) + (k >> 5)] = make_float2(sc, sc);
  }
}

// MatMul's packed kernel for a float32 weight (gemm.go k6x16, the rows
// below m/6·6 of a call): every output starts at its bias (or 0) and gets
// += the fused chain of each 256-deep pass. Here for a convolution over
// staged rows: output row t of stream s reads the K = k·cin values from
// x + (s·sstride + t)·cin on. Rows t < mf; y dense [n·T][N], stored or added
// to (resid: y = y + c, the residual block's x + o).
//
// A CTA holds TM output rows of one stream and all N ≤ 64 columns: the
// TM + k − 1 input rows (padded by 4 floats) and the weight (as float4s
// [k/4][4][column group]) sit in shared memory. Thread (cg, rg) — column
// group fastest, so a warp's lanes span consecutive columns — keeps RM rows
// rg + i·TMG × the four columns 4cg.. in registers and walks k in order,
// four values per step: weight reads are consecutive float4s, row reads
// broadcasts or rows apart, and the outputs leave as whole float4 rows.
//
// Fused (a.virt): the rows are not staged beforehand; x is dense [n][T][cin]
// and row r of the window is carry row r (r < P) or ELU?(x row r − P), as
// k_mimi_stage would write them; the stream's first CTA writes the next
// call's carried rows.
template <int RM>
__global__ void __launch_bounds__(256) k_mimi_fconv(FconvArgs a) {
  extern __shared__ __align__(16) float fsm[];
  const int cin = a.cin, K = a.K, T = a.T, N = a.N, ngp = a.ngp, P = a.P;
  const int tmg = 256 / ngp, TM = tmg * RM, k = K / cin;
  const int s = blockIdx.y, t0 = blockIdx.x * TM;
  const int rows = TM + k - 1, cinp = cin + 4, C4 = cin >> 2, K4 = K >> 2;
  float* xs = fsm;
  float4* ws = reinterpret_cast<float4*>(fsm + rows * cinp);
  const int tid = threadIdx.x;
  const int total = a.virt ? P + T : a.sstride;  // window rows of the stream
  auto window_row = [&](int vr, int c) {
    if (!a.virt) return ld4(a.x + (size_t(s) * a.sstride + vr) * cin + c);
    if (vr < P) return ld4(a.carry_in + (size_t(s) * P + vr) * cin + c);
    const float4 v = ld4(a.x + (size_t(s) * T + vr - P) * cin + c);
    return a.elu ? elu4(v, (vr - P) * cin + c, T * cin) : v;
  };
  for (int i = tid; i < rows * C4; i += 256) {
    const int r = i / C4, c = (i - r * C4) * 4;
    st4(xs + r * cinp + c, t0 + r < total ? window_row(t0 + r, c) : make_float4(0, 0, 0, 0));
  }
  if (a.virt && P > 0 && blockIdx.x == 0)
    for (int i = tid; i < P * C4; i += 256) {
      const int r = i / C4, c = (i - r * C4) * 4;
      st4(a.carry_out + (size_t(s) * P + r) * cin + c, window_row(T + r, c));
    }
  const float* w = a.w;
  const float* bias = a.bias;
  for (int i = tid; i < K4 * 4 * ngp; i += 256) {
    const int kq = i / (4 * ngp), rem = i - kq * 4 * ngp, u = rem / ngp, g = rem - u * ngp, n = g * 4 + u;
    ws[i] = n < N ? ld4(w + size_t(n) * K + kq * 4) : make_float4(0, 0, 0, 0);
  }
  __syncthreads();
  const int cg = tid % ngp, rg = tid / ngp;
  if (cg * 4 >= N) return;
  float cv[RM][4];
#pragma unroll
  for (int u = 0; u < 4; u++) {
    const int n = cg * 4 + u;
    const float b = bias && n < N ? bias[n] : 0.f;
#pragma unroll
    for (int i = 0; i < RM; i++) cv[i][u] = b;
  }
  for (int k0 = 0; k0 < K; k0 += 256) {
    const int k1 = min(K, k0 + 256);
    float acc[RM][4];
#pragma unroll
    for (int i = 0; i < RM; i++)
#pragma unroll
      for (int u = 0; u < 4; u++) acc[i][u] = 0.f;
    int j = k0 / cin, c = k0 - j * cin;
    for (int kk = k0; kk < k1; kk += 4) {
      float4 wv[4];
#pragma unroll
      for (int u = 0; u < 4; u++) wv[u] = ws[((kk >> 2) * 4 + u) * ngp + cg];
#pragma unroll
      for (int i = 0; i < RM; i++) {
        const float4 a = ld4(xs + (rg + i * tmg + j) * cinp + c);
#pragma unroll
        for (int u = 0; u < 4; u++) {
          float r = acc[i][u];
          r = __fmaf_rn(a.x, wv[u].x, r);
          r = __fmaf_rn(a.y, wv[u].y, r);
          r = __fmaf_rn(a.z, wv[u].z, r);
          r = __fmaf_rn(a.w, wv[u].w, r);
          acc[i][u] = r;
        }
      }
      c += 4;
      if (c == cin) c = 0, j++;
    }
#pragma unroll
    for (int i = 0; i < RM; i++)
#pragma unroll
      for (int u = 0; u < 4; u++) cv[i][u] = __fadd_rn(cv[i][u], acc[i][u]);
  }
  const bool vec = (N & 3) == 0;
#pragma unroll
  for (int i = 0; i < RM; i++) {
    const int t = t0 + rg + i * tmg;
    if (t >= a.mf) continue;
    float* yp = a.y + (size_t(s) * T + t) * N + cg * 4;
    if (vec) {
      float4 v = make_float4(cv[i][0], cv[i][1], cv[i][2], cv[i][3]);
      if (a.resid) v = add4(ld4(yp), v);
      st4(yp, v);
    } else {
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (cg * 4 + u < N) yp[u] = a.resid ? __fadd_rn(yp[u], cv[i][u]) : cv[i][u];
    }
  }
}

// convtr.run (nn.go:305-327): output row q of cout values starts at the bias
// and adds tap q − t·S of every input row t in order; rows below k − S then
// add the carried partial. Rows below T·S are the output, the rest (less the
// bias) the next partial. Four channels per thread.
__global__ void k_mimi_convtr(const float* z, const float* bias, const float* part_in, float* y, float* part_out,
                              int T, int co, int k, int S) {
  const int s = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
  const int L = (T - 1) * S + k, PT = k - S, C4 = co >> 2;
  if (i >= L * C4) return;
  const int q = i / C4, c = (i - q * C4) * 4;
  const float4 b = ld4(bias + c);
  float4 v = b;
  const int t0 = q >= k ? (q - k) / S + 1 : 0, t1 = min(T - 1, q / S);
  const float* zs = z + size_t(s) * T * k * co;
  for (int t = t0; t <= t1; t++) v = add4(v, ld4(zs + (size_t(t) * k + (q - t * S)) * co + c));
  if (q < PT) v = add4(v, ld4(part_in + (size_t(s) * PT + q) * co + c));
  if (q < T * S)
    st4(y + (size_t(s) * T * S + q) * co + c, v);
  else
    st4(part_out + (size_t(s) * PT + q - T * S) * co + c,
        make_float4(__fsub_rn(v.x, b.x), __fsub_rn(v.y, b.y), __fsub_rn(v.z, b.z), __fsub_rn(v.w, b.w)));
}

// Row r of a call is stream r / S at position pos[r / S] + r % S.
__global__ void k_mimi_rows(const int* pos, int S, int R, int* rowpos) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < R) rowpos[r] = pos[r / S] + r % S;
}

__global__ void k_mimi_advance(int* pos, int S, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) pos[i] += S;
}

// speakChunk's fade-in (speak.go:185-190) on a stream's first frame:
// sample i < fade is multiplied by float32(i)/float32(fade − 1). One block
// per stream; the stream is started afterwards.
__global__ void k_mimi_fade(float* pcm, int* started, int frame, int fade) {
  const int s = blockIdx.x;
  if (started[s]) return;
  const int nf = min(fade, frame);
  for (int i = threadIdx.x; i < nf; i += blockDim.x) {
    float* p = pcm + size_t(s) * frame + i;
    *p = __fmul_rn(*p, __fdiv_rn(float(i), float(fade - 1)));
  }
  __syncthreads();
  if (threadIdx.x == 0) started[s] = 1;
}

dim3 grid2(int per_stream, int n) { return dim3(unsigned((per_stream + 255) / 256), unsigned(n)); }

// k_mimi_fconv's tiling: column groups of four, rounded up to a power of two
// (ngp lanes per row), and rows per thread: a CTA holds 256 output rows for
// N ≤ 8, 128 for N ≤ 32 and 64 beyond.
int fconv_ngp(int N) {
  const int ncg = (N + 3) / 4;
  int p = 1;
  while (p < ncg) p *= 2;
  return p;
}

int fconv_rm(int ngp) { return ngp <= 2 ? ngp : ngp <= 8 ? 128 * ngp / 256 : 4; }

size_t fconv_smem(int cin, int K, int N) {
  const int ngp = fconv_ngp(N), TM = 256 / ngp * fconv_rm(ngp);
  return (size_t(TM + K / cin - 1) * (cin + 4) + size_t(K) * 4 * ngp) * sizeof(float);
}

constexpr size_t kFconvSmemMax = 200 * 1024;

}  // namespace

void launch_mimi_up(const float* z, const float* up, const float* part_in, float* x, float* part_out, int n, int S,
                    int C, cudaStream_t st) {
  k_mimi_up<<<grid2(2 * S * C, n), 256, 0, st>>>(z, up, part_in, x, part_out, S, C);
}

void launch_mimi_elu(const float* in, float* out, int n, int len, cudaStream_t st) {
  k_mimi_elu<<<grid2(len / 4, n), 256, 0, st>>>(in, out, len);
}

void launch_mimi_stage(const float* x, const float* carry_in, float* carry_out, float* stage, int n, int T, int C,
                       int P, bool elu, cudaStream_t st) {
  if (C % 4)
    k_mimi_stage_s<<<grid2((2 * P + T) * C, n), 256, 0, st>>>(x, carry_in, carry_out, stage, T, C, P, elu ? 1 : 0);
  else
    k_mimi_stage<<<grid2((2 * P + T) * (C / 4), n), 256, 0, st>>>(x, carry_in, carry_out, stage, T, C, P, elu ? 1 : 0);
}

void launch_mimi_gemv_small(const float* x, int ldx, int sstride, int T, int off, const float* w, int N, int K,
                            const float* bias, float* y, bool resid, int n, cudaStream_t st) {
  k_mimi_gemv_small<<<grid2((T - off) * N, n), 256, 0, st>>>(x, ldx, sstride, T, off, w, N, K, bias, y, resid ? 1 : 0);
}

void launch_mimi_rowtab(int T, int n, int* rowslot, int* crow0, int* cT, int* cslot, cudaStream_t st) {
  k_mimi_rowtab<<<(n * T + 255) / 256, 256, 0, st>>>(T, n, rowslot, crow0, cT, cslot);
}

void launch_mimi_replicate(const float* x, int T, int C, float* carry, int P, int n, cudaStream_t st) {
  k_mimi_replicate<<<grid2(P * C, n), 256, 0, st>>>(x, T, C, carry, P);
}

void launch_mimi_im2col(const float* x, const float* prev_in, float* prev_out, float* col, int n, int T, int cin, int k,
                        int stride, int dil, int P, cudaStream_t st) {
  k_mimi_im2col<<<grid2((T / stride * k + P) * (cin / 4), n), 256, 0, st>>>(x, prev_in, prev_out, col, T, cin, k,
                                                                              stride, dil, P);
}

void launch_mimi_quant(const float* x, int ldx, int sstride, int n, int T, int K, int elu_len, int8_t* q, float2* qs,
                       cudaStream_t st) {
  k_mimi_quant<<<grid2(T * (K / 8), n), 256, 0, st>>>(x, ldx, sstride, T, K, elu_len, q, qs);
}

bool mimi_fconv_fits(int cin, int K, int N) {
  return N >= 1 && N <= 64 && cin % 4 == 0 && K % cin == 0 && fconv_smem(cin, K, N) <= kFconvSmemMax;
}

void launch_mimi_fconv(const FconvArgs& a0, int n, cudaStream_t st) {
  FconvArgs a = a0;
  a.ngp = fconv_ngp(a.N);
  const int rm = fconv_rm(a.ngp), TM = 256 / a.ngp * rm;
  const size_t sm = fconv_smem(a.cin, a.K, a.N);
  const dim3 grid(unsigned((a.mf + TM - 1) / TM), unsigned(n));
  switch (rm) {
    case 1:
      k_mimi_fconv<1><<<grid, 256, sm, st>>>(a);
      break;
    case 2:
      k_mimi_fconv<2><<<grid, 256, sm, st>>>(a);
      break;
    default:
      k_mimi_fconv<4><<<grid, 256, sm, st>>>(a);
  }
}

void launch_mimi_convtr(const float* z, const float* bias, const float* part_in, float* y, float* part_out, int n, int T,
                        int co, int k, int S, cudaStream_t st) {
  k_mimi_convtr<<<grid2(((T - 1) * S + k) * (co / 4), n), 256, 0, st>>>(z, bias, part_in, y, part_out, T, co, k, S);
}

void launch_mimi_rows(const int* pos, int S, int R, int* rowpos, cudaStream_t st) {
  k_mimi_rows<<<(R + 255) / 256, 256, 0, st>>>(pos, S, R, rowpos);
}

void launch_mimi_advance(int* pos, int S, int n, cudaStream_t st) {
  k_mimi_advance<<<(n + 255) / 256, 256, 0, st>>>(pos, S, n);
}

void launch_mimi_fade(float* pcm, int* started, int n, int frame, int fade, cudaStream_t st) {
  k_mimi_fade<<<n, 128, 0, st>>>(pcm, started, frame, fade);
}

void mimi_kernels_init() {
  const int sm = int(kFconvSmemMax);
  cudaFuncSetAttribute(k_mimi_fconv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  cudaFuncSetAttribute(k_mimi_fconv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  cudaFuncSetAttribute(k_mimi_fconv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
}

}  // namespace grx
