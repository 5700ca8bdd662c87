// Mimi's decoder (pockettts/mimi.go:24-150, nn.go:52-64 and 258-327) on
// the device: the elementwise steps between its products, for n streams
// decoding one latent each per call, rows laid out [stream][time][channel].
// Each keeps the reference's float32 operations element by element; the
// products themselves are the int8 path (Q8_0 weights) and the float path
// (float32 weights) of k_q8.cu, k_flin.cu and k_whisper.cu's packed-order
// kernel.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

// decode's depthwise ConvTranspose1d for one latent (mimi.go:130-145): with
// z the projected latent, row j < 2S of the full output is 0 + z[c]·up[c][j]
// (cleared, then +=), rows j < S get the partial carried from the last call
// added and are the transformer's input, rows S.. are the next partial.
__global__ void k_mimi_up(const float* z, const float* up, const float* part_in, float* x, float* part_out, int n,
                          int S, int C) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t total = size_t(n) * 2 * S * C;
  if (i >= total) return;
  const int c = int(i % C), j = int((i / C) % (2 * S)), s = int(i / (size_t(C) * 2 * S));
  const float v = __fadd_rn(0.f, __fmul_rn(z[size_t(s) * C + c], up[size_t(c) * 2 * S + j]));
  if (j < S)
    x[(size_t(s) * S + j) * C + c] = __fadd_rn(v, part_in[(size_t(s) * S + j) * C + c]);
  else
    part_out[(size_t(s) * S + j - S) * C + c] = v;
}

// elu (nn.go:52-64) of every stream's len values: per 512-value chunk of
// the stream's array, t = min(v, 0) through ExpSub(t, 0) — EXP8 for the
// chunk's first len&~7 values, Go's expf for the rest — then
// max(v, 0) + (t − 1).
__global__ void k_mimi_elu(const float* in, float* out, int n, int len) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= size_t(n) * len) return;
  const int e = int(i % len), c0 = e / 512 * 512, clen = min(512, len - c0);
  const float v = in[i];
  const float t = v < 0.f ? v : 0.f;
  const float x = __fsub_rn(t, 0.f);
  const float ex = e - c0 < (clen & ~7) ? exp_avx(x) : expf_go(x);
  out[i] = __fadd_rn(v > 0.f ? v : 0.f, __fsub_rn(ex, 1.f));
}

// conv.run's window (nn.go:275-300): rows [prev (P); x (T)] of cin values;
// output row t takes rows t·stride + j·dil for j < k. The last P rows
// become the next call's prev (a separate buffer: the old one is read here).
__global__ void k_mimi_im2col(const float* x, const float* prev_in, float* prev_out, float* col, int n, int T, int cin,
                              int k, int stride, int dil, int P) {
  const int To = T / stride;
  const size_t cols = size_t(k) * cin;
  const size_t ncol = size_t(n) * To * cols, nprev = size_t(n) * P * cin;
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  auto row = [&](int s, int r, int c) {
    return r < P ? prev_in[(size_t(s) * P + r) * cin + c] : x[(size_t(s) * T + r - P) * cin + c];
  };
  if (i < ncol) {
    const int c = int(i % cin), j = int((i / cin) % k), t = int((i / cols) % To), s = int(i / (cols * To));
    col[i] = row(s, t * stride + j * dil, c);
  } else if (i < ncol + nprev) {
    const size_t q = i - ncol;
    const int c = int(q % cin), r = int((q / cin) % P), s = int(q / (size_t(P) * cin));
    prev_out[q] = row(s, T + r, c);
  }
}

// convtr.run (nn.go:305-327): output row q of cout values starts at the bias
// and adds tap q − t·S of every input row t in order; rows below k − S then
// add the carried partial. Rows below T·S are the output, the rest (less the
// bias) the next partial.
__global__ void k_mimi_convtr(const float* z, const float* bias, const float* part_in, float* y, float* part_out, int n,
                              int T, int co, int k, int S) {
  const int L = (T - 1) * S + k, PT = k - S;
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= size_t(n) * L * co) return;
  const int c = int(i % co), q = int((i / co) % L), s = int(i / (size_t(co) * L));
  float v = bias[c];
  const int t0 = q >= k ? (q - k) / S + 1 : 0, t1 = min(T - 1, q / S);
  for (int t = t0; t <= t1; t++) v = __fadd_rn(v, z[((size_t(s) * T + t) * k + (q - t * S)) * co + c]);
  if (q < PT) v = __fadd_rn(v, part_in[(size_t(s) * PT + q) * co + c]);
  if (q < T * S)
    y[(size_t(s) * T * S + q) * co + c] = v;
  else
    part_out[(size_t(s) * PT + q - T * S) * co + c] = __fsub_rn(v, bias[c]);
}

__global__ void k_mimi_add(const float* a, const float* b, float* y, size_t n) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fadd_rn(a[i], b[i]);
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

unsigned blocks_for(size_t n) { return unsigned((n + 255) / 256); }

}  // namespace

void launch_mimi_up(const float* z, const float* up, const float* part_in, float* x, float* part_out, int n, int S,
                    int C, cudaStream_t st) {
  k_mimi_up<<<blocks_for(size_t(n) * 2 * S * C), 256, 0, st>>>(z, up, part_in, x, part_out, n, S, C);
}

void launch_mimi_elu(const float* in, float* out, int n, int len, cudaStream_t st) {
  k_mimi_elu<<<blocks_for(size_t(n) * len), 256, 0, st>>>(in, out, n, len);
}

void launch_mimi_im2col(const float* x, const float* prev_in, float* prev_out, float* col, int n, int T, int cin, int k,
                        int stride, int dil, int P, cudaStream_t st) {
  const size_t total = size_t(n) * (T / stride) * k * cin + size_t(n) * P * cin;
  k_mimi_im2col<<<blocks_for(total), 256, 0, st>>>(x, prev_in, prev_out, col, n, T, cin, k, stride, dil, P);
}

void launch_mimi_convtr(const float* z, const float* bias, const float* part_in, float* y, float* part_out, int n, int T,
                        int co, int k, int S, cudaStream_t st) {
  k_mimi_convtr<<<blocks_for(size_t(n) * ((T - 1) * S + k) * co), 256, 0, st>>>(z, bias, part_in, y, part_out, n, T,
                                                                                 co, k, S);
}

void launch_mimi_rows(const int* pos, int S, int R, int* rowpos, cudaStream_t st) {
  k_mimi_rows<<<blocks_for(size_t(R)), 256, 0, st>>>(pos, S, R, rowpos);
}

void launch_mimi_advance(int* pos, int S, int n, cudaStream_t st) {
  k_mimi_advance<<<blocks_for(size_t(n)), 256, 0, st>>>(pos, S, n);
}

void launch_mimi_fade(float* pcm, int* started, int n, int frame, int fade, cudaStream_t st) {
  k_mimi_fade<<<n, 128, 0, st>>>(pcm, started, frame, fade);
}

void launch_mimi_add(const float* a, const float* b, float* y, size_t n, cudaStream_t st) {
  k_mimi_add<<<blocks_for(n), 256, 0, st>>>(a, b, y, n);
}

}  // namespace grx
