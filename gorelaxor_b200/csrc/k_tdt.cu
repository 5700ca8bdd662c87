// The greedy TDT / RNN-T decode loop (conformer/rnnt.go:111-173) for a batch
// of independent streams, one loop iteration per round of four kernels:
//
//   k_tdt_lin<LSTM> ×layers  predict (rnnt.go:46-68) for the streams whose
//                            last iteration emitted (the "dirty" list):
//                            gates = (Wx·x + b) + Wh·h, then the LSTM cell
//   k_tdt_lin<PROJ>          predProj = jPred·pred + b for the same streams
//                            (the reference recomputes it every iteration
//                            from an unchanged pred; caching it is exact)
//   k_tdt_lin<JOINT>         logits = jOut·act(encProj[step] + predProj) + b
//                            for every stream still decoding
//   k_tdt_decide             argmaxes, softmaxAt, the token, frame skipping
//                            and max_symbols, the state swap; builds the
//                            next iteration's stream lists
//
// All products are the reference's m = 1 float path on Q8_0 weights with
// rows kept (dot4q8avx lanes, kernels_amd64.s:343-399; dotQ8Go for rows
// past the last group of four, kern.go:249-266), as in k_flow.cu: 8 lanes
// per output, 16 streams per CTA sharing each staged weight row.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

constexpr int TM = 16;       // streams per CTA
constexpr int TROWS = 32;    // weight rows per CTA (8 warps × 4 groups of 8 lanes)

// x[m][k] at k·TM + 4·((m/4) ^ ((k/2) mod 4)) + m mod 4: the 16-byte group of
// streams 4g..4g+3 at the 8 consecutive k of a lane group falls on 8
// different bank quads, so a group's 16-byte loads are conflict-free.
__device__ __forceinline__ int tx_at(int k, int m) { return k * TM + 4 * ((m >> 2) ^ ((k >> 1) & 3)) + (m & 3); }

__host__ __device__ constexpr int t_wstride(int K) { return K + 16; }

// Shared memory: one input [K][TM] floats, 32 weight rows, their f16 block
// scales, and a [32][TM] tile for the epilogue.
__host__ __device__ constexpr size_t tdt_smem(int K) {
  return size_t(TM) * K * 4 + size_t(TROWS) * t_wstride(K) + size_t(TROWS) * (K / QK) * 2 + size_t(TROWS) * TM * 4;
}

// dot4q8avx's lanes for one weight row against TM staged streams: lane l of
// the 8-lane group accumulates block by block (q[l]x[l], three fused steps
// over q[8+l], q[16+l], q[24+l], then one fused step by the block scale).
__device__ __forceinline__ void row_lanes(const int8_t* wr, const uint16_t* sd, const float* sx, int nb, int l,
                                          f2 (&acc)[TM / 2]) {
  for (int b = 0; b < nb; b++) {
    const int k = b * QK + l;
    f2 Q[4];
#pragma unroll
    for (int i = 0; i < 4; i++) Q[i] = f2dup(float(wr[k + 8 * i]));
    const f2 D = f2dup(h2f(sd[b]));
#pragma unroll
    for (int g4 = 0; g4 < TM / 4; g4++) {
      f2 X[4][2];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(&sx[tx_at(k + 8 * i, 4 * g4)]);
        X[i][0] = v.x;
        X[i][1] = v.y;
      }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        f2 y = f2mul(Q[0], X[0][h]);
        y = f2fma(Q[1], X[1][h], y);
        y = f2fma(Q[2], X[2][h], y);
        y = f2fma(Q[3], X[3][h], y);
        acc[2 * g4 + h] = f2fma(y, D, acc[2 * g4 + h]);
      }
    }
  }
}

// dotQ8Go (kern.go:249-266) of one row against staged stream m: four
// strided unfused sums per block, scaled by the block's f16 value.
__device__ float row_go(const int8_t* wr, const uint16_t* sd, const float* sx, int nb, int m) {
  float s = 0.f;
  for (int b = 0; b < nb; b++) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int i = 0; i < QK; i += 4) {
      const int k = b * QK + i;
      a0 = __fadd_rn(a0, __fmul_rn(sx[tx_at(k, m)], float(wr[k])));
      a1 = __fadd_rn(a1, __fmul_rn(sx[tx_at(k + 1, m)], float(wr[k + 1])));
      a2 = __fadd_rn(a2, __fmul_rn(sx[tx_at(k + 2, m)], float(wr[k + 2])));
      a3 = __fadd_rn(a3, __fmul_rn(sx[tx_at(k + 3, m)], float(wr[k + 3])));
    }
    s = __fadd_rn(s, __fmul_rn(h2f(sd[b]), __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3)));
  }
  return s;
}

__device__ __forceinline__ void cp16t(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(uint32_t(__cvta_generic_to_shared(dst))), "l"(src));
}

// tanh32, rnnt.go:42: float64 tanh of the widened value.
__device__ __forceinline__ float tanh32(float x) { return float(tanh(double(x))); }

// Go's builtin max(v, 0) on float32: NaN stays NaN, -0 gives +0.
__device__ __forceinline__ float relu_go(float v) { return v != v ? v : (v > 0.f ? v : 0.f); }

enum TMode { T_LSTM = 0, T_PROJ = 1, T_JOINT = 2 };

// One product round. Grid: (row tiles, stream groups of TM); the streams
// are list[0 .. *count) of the parity's list.
//  LSTM  (layer l): rows = the 4 gates × 8 units of unit group blockIdx.x;
//                   inputs x (embedding row, zeros, or layer l-1's new h)
//                   and h (layer l's current h); writes the new h, c.
//  PROJ:            rows of jPred on the top layer's new h; writes predProj.
//  JOINT:           rows of jOut on act(encProj[step] + predProj); writes
//                   logits.
// The round's weights, chosen on the host (no run-time index into the
// parameter block).
struct TLin {
  DQ8 w0, w1;  // LSTM: Wx, Wh of the layer; PROJ: jPred; JOINT: jOut
  const float* bias = nullptr;
  int layer = 0;
};

template <int MODE>
__global__ void __launch_bounds__(256, MODE == T_JOINT ? 2 : 3) k_tdt_lin(TdtArgs a, TLin t, int parity) {
  const int layer = t.layer;
  extern __shared__ __align__(16) uint8_t tsm[];
  // The LSTM's two products (Wx·x, Wh·h) pass through the same tiles one
  // after the other, which keeps the shared memory of a CTA to one input.
  constexpr int NPASS = MODE == T_LSTM ? 2 : 1;
  if (MODE == T_LSTM && layer == 0 && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
    // the next iteration's lists start empty (k_tdt_decide fills them)
    a.counts[2 * (parity ^ 1)] = 0;
    a.counts[2 * (parity ^ 1) + 1] = 0;
  }
  const bool dirty_list = MODE != T_JOINT;
  const int count = a.counts[2 * parity + (dirty_list ? 1 : 0)];
  const int* list = (dirty_list ? a.dirty : a.active) + size_t(parity) * a.n;
  const int g0 = blockIdx.y * TM;
  if (g0 >= count) return;
  const int mt = min(TM, count - g0);
  const int K = MODE == T_JOINT ? a.J : a.H;
  const int nb = K / QK, ws = t_wstride(K);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = lane >> 3, l = lane & 7;
  const int r = warp * 4 + grp;  // this group's row within the tile
  float* sx = reinterpret_cast<float*>(tsm);
  int8_t* sw = reinterpret_cast<int8_t*>(tsm + size_t(TM) * K * 4);
  uint16_t* sd = reinterpret_cast<uint16_t*>(tsm + size_t(TM) * K * 4 + size_t(TROWS) * ws);
  float* tile = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sd) + size_t(TROWS) * nb * 2);
  __shared__ int s_stream[TM];
  if (threadIdx.x < TM) s_stream[threadIdx.x] = threadIdx.x < mt ? list[g0 + threadIdx.x] : -1;
  const int nrows = MODE == T_LSTM ? TROWS : min(TROWS, t.w0.rows - int(blockIdx.x) * TROWS);
  float out[TM];

  for (int in = 0; in < NPASS; in++) {
    if (in > 0) __syncthreads();  // every group is done with the previous pass's tiles
    // ---- the tile's weight rows and scales, by async copies
    {
      // tile row tr holds global row (LSTM) gate tr/8, unit 8·blockIdx.x + tr%8,
      // or (PROJ, JOINT) row 32·blockIdx.x + tr
      auto grow = [&](int tr) {
        return MODE == T_LSTM ? (tr >> 3) * a.H + int(blockIdx.x) * 8 + (tr & 7) : int(blockIdx.x) * TROWS + tr;
      };
      const int cpr = K / 16;
      const DQ8& W = in == 0 ? t.w0 : t.w1;
      for (int i = threadIdx.x; i < nrows * cpr; i += blockDim.x) {
        const int tr = i / cpr, c = i - tr * cpr;
        cp16t(sw + size_t(tr) * ws + c * 16, W.q + size_t(grow(tr)) * K + c * 16);
      }
      // scales: every load of the tile issued before the first store
      constexpr int SI = (TROWS * (1024 / QK) + 255) / 256;
      uint16_t dv[SI];
#pragma unroll
      for (int u = 0; u < SI; u++) {
        const int i = threadIdx.x + u * 256, tr = i / nb, b = i - tr * nb;
        if (i < nrows * nb) dv[u] = W.d[size_t(grow(tr)) * nb + b];
      }
#pragma unroll
      for (int u = 0; u < SI; u++) {
        const int i = threadIdx.x + u * 256, tr = i / nb, b = i - tr * nb;
        if (i < nrows * nb) sd[size_t(tr) * nb + b] = dv[u];
      }
      asm volatile("cp.async.commit_group;\n" ::);
    }
    if (in == 0) __syncthreads();  // s_stream

    // ---- the streams' inputs, stream-minor: an item is four consecutive k
    // of one stream (16-byte loads along the stream's row); BATCH items'
    // loads are in flight before the first is stored.
    constexpr int BATCH = 8;
    const int k4n = K / 4, items = TM * k4n;
    for (int i0 = 0; i0 < items; i0 += BATCH * 256) {
      float4 v[BATCH], e[BATCH];
#pragma unroll
      for (int u = 0; u < BATCH; u++) {
        const int i = i0 + threadIdx.x + u * 256;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        e[u] = v[u];
        if (i >= items) continue;
        const int m = i / k4n, k = 4 * (i - m * k4n), s = s_stream[m];
        if (s < 0) continue;
        const int cur = a.cur[s];
        const float* src = nullptr;
        if (MODE == T_LSTM) {
          if (in == 0) {
            if (layer == 0) {
              const int last = a.last[s];
              if (last >= 0 && last != a.blank) src = a.embed + size_t(last) * a.H;
            } else {
              src = a.h + ((size_t(cur ^ 1) * a.layers + layer - 1) * a.n + s) * a.H;
            }
          } else {
            src = a.h + ((size_t(cur) * a.layers + layer) * a.n + s) * a.H;
          }
        } else if (MODE == T_PROJ) {
          src = a.h + ((size_t(cur ^ 1) * a.layers + a.layers - 1) * a.n + s) * a.H;
        } else {
          src = a.enc_proj + (size_t(s) * a.max_t + a.step[s]) * a.J;
          e[u] = *reinterpret_cast<const float4*>(a.pred_proj + size_t(s) * a.J + k);
        }
        if (src) v[u] = *reinterpret_cast<const float4*>(src + k);
      }
#pragma unroll
      for (int u = 0; u < BATCH; u++) {
        const int i = i0 + threadIdx.x + u * 256;
        if (i >= items) continue;
        const int m = i / k4n, k = 4 * (i - m * k4n);
        float x[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        if (MODE == T_JOINT) {
          const float p[4] = {e[u].x, e[u].y, e[u].z, e[u].w};
#pragma unroll
          for (int j = 0; j < 4; j++) {
            float w = __fadd_rn(x[j], p[j]);
            if (a.act == 1) w = sigmoid_go(w);
            else if (a.act == 2) w = tanh32(w);
            else w = relu_go(w);
            x[j] = s_stream[m] >= 0 ? w : 0.f;
          }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) sx[tx_at(k + j, m)] = x[j];
      }
    }
    asm volatile("cp.async.wait_all;\n" ::);
    __syncthreads();

    // ---- the product: row r of the tile for all TM streams
    f2 acc[TM / 2];
#pragma unroll
    for (int p = 0; p < TM / 2; p++) acc[p] = 0;
    if (r < nrows) row_lanes(sw + size_t(r) * ws, sd + size_t(r) * nb, sx, nb, l, acc);
    if (in == 0) {
#pragma unroll
      for (int p = 0; p < TM / 2; p++) {
        out[2 * p] = hsum8_lanes(f2lo(acc[p]));
        out[2 * p + 1] = hsum8_lanes(f2hi(acc[p]));
      }
    } else {
      // gates[j] = (Wx·x + b)[j], then kern.Add of Wh·h (rnnt.go:57-59)
      const int gr = (r >> 3) * a.H + blockIdx.x * 8 + (r & 7);
      const float b = t.bias[gr];
#pragma unroll
      for (int p = 0; p < TM / 2; p++) {
        const float h0 = hsum8_lanes(f2lo(acc[p])), h1 = hsum8_lanes(f2hi(acc[p]));
        out[2 * p] = __fadd_rn(__fadd_rn(out[2 * p], b), h0);
        out[2 * p + 1] = __fadd_rn(__fadd_rn(out[2 * p + 1], b), h1);
      }
    }
  }
  if (MODE == T_LSTM) {
    if (l == 0)
#pragma unroll
      for (int m = 0; m < TM; m++) tile[r * TM + m] = out[m];
    __syncthreads();
    // the cell for 8 units × TM streams (rnnt.go:60-66), unfused
    if (threadIdx.x < 8 * TM) {
      const int u = threadIdx.x / TM, m = threadIdx.x % TM, s = s_stream[m];
      if (s >= 0) {
        const int cur = a.cur[s], j = blockIdx.x * 8 + u;
        const float i = sigmoid_go(tile[u * TM + m]);
        const float f = sigmoid_go(tile[(8 + u) * TM + m]);
        const float g = tanh32(tile[(16 + u) * TM + m]);
        const float o = sigmoid_go(tile[(24 + u) * TM + m]);
        const size_t cs = ((size_t(cur) * a.layers + layer) * a.n + s) * a.H + j;
        const size_t ns = ((size_t(cur ^ 1) * a.layers + layer) * a.n + s) * a.H + j;
        const float c = __fadd_rn(__fmul_rn(f, a.c[cs]), __fmul_rn(i, g));
        a.c[ns] = c;
        a.h[ns] = __fmul_rn(o, tanh32(c));
      }
    }
    return;
  }
  // PROJ / JOINT: + bias (gemm.go:251-255); rows past the last group of
  // four take dotQ8Go (gemm.go:239-249), serially by the group's lane 0.
  if (l != 0 || r >= nrows) return;
  const float* bias = t.bias;
  const int n = blockIdx.x * TROWS + r;
  const bool tail = n >= (t.w0.rows & ~3);
#pragma unroll
  for (int m = 0; m < TM; m++) {
    if (m >= mt) break;
    const int s = s_stream[m];
    float v = tail ? row_go(sw + size_t(r) * ws, sd + size_t(r) * nb, sx, nb, m) : out[m];
    v = __fadd_rn(v, bias[n]);
    if (MODE == T_PROJ) a.pred_proj[size_t(s) * a.J + n] = v;
    else a.logits[size_t(s) * a.nout + n] = v;
  }
}

// One warp per stream of the active list: the rest of the loop body
// (rnnt.go:139-171).
__global__ void __launch_bounds__(128) k_tdt_decide(TdtArgs a, int parity) {
  const int w = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int count = a.counts[2 * parity];
  if (w >= count) return;
  const int s = a.active[size_t(parity) * a.n + w];
  const float* lg = a.logits + size_t(s) * a.nout;
  // argmax over the tokens, strict '>' from index 0: the first of equal
  // maxima wins (rnnt.go:70-78)
  float bv = lg[lane < a.V ? lane : 0];
  int bi = lane < a.V ? lane : 0;
  for (int i = lane + 32; i < a.V; i += 32)
    if (lg[i] > bv) bv = lg[i], bi = i;
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
  }
  const int tok = bi;
  const bool blank = tok == a.blank;
  // softmaxAt (rnnt.go:80-89): float32 differences, float64 exp and sum
  float p = 0.f;
  if (!blank) {
    double sum = 0;
    for (int i = lane; i < a.V; i += 32) sum += exp(double(__fsub_rn(lg[i], bv)));
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    p = float(exp(double(__fsub_rn(lg[tok], bv))) / sum);
  }
  if (lane != 0) return;
  int duration = 1;
  if (a.tdt) {
    int di = 0;
    for (int i = 1; i < a.ndur; i++)
      if (lg[a.V + i] > lg[a.V + di]) di = i;
    duration = a.durations[di];
  }
  int step = a.step[s], nsym = a.nsym[s];
  bool dirty = false;
  if (!blank) {
    const int k = a.ntok[s];
    if (k < a.cap) {
      int4* t = reinterpret_cast<int4*>(a.tokens) + size_t(s) * a.cap + k;
      *t = make_int4(tok, a.frame_offset[s] + step, duration, __float_as_int(p));
    }
    a.ntok[s] = k + 1;
    a.last[s] = tok;
    a.cur[s] ^= 1;
    dirty = true;
  }
  if (!a.tdt) {
    if (blank) {
      step++;
      nsym = 0;
    } else if (++nsym, a.max_symbols > 0 && nsym >= a.max_symbols) {
      step++;
      nsym = 0;
    }
  } else {
    step += duration;
    nsym++;
    if (duration != 0) {
      nsym = 0;
    } else if (a.max_symbols > 0 && nsym >= a.max_symbols) {
      step++;
      nsym = 0;
    }
  }
  a.step[s] = step;
  a.nsym[s] = nsym;
  const int iter = a.iter[s] + 1;
  a.iter[s] = iter;
  if (step < a.T[s] && iter < 16 * a.T[s] + 1024) {
    const int q = parity ^ 1;
    a.active[size_t(q) * a.n + atomicAdd(&a.counts[2 * q], 1)] = s;
    if (dirty) a.dirty[size_t(q) * a.n + atomicAdd(&a.counts[2 * q + 1], 1)] = s;
  }
}

// The first iteration's lists: every stream with frames left is active and
// dirty (Decode starts with a prediction from the state, rnnt.go:130-141).
__global__ void k_tdt_begin(TdtArgs a) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s == 0) a.counts[0] = a.counts[1] = a.counts[2] = a.counts[3] = 0;
  if (s >= a.n) return;
  a.step[s] = 0;
  a.nsym[s] = 0;
  a.iter[s] = 0;
  a.ntok[s] = 0;
}

__global__ void k_tdt_begin_lists(TdtArgs a) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= a.n || a.T[s] <= 0) return;
  a.active[atomicAdd(&a.counts[0], 1)] = s;
  a.dirty[atomicAdd(&a.counts[1], 1)] = s;
}

}  // namespace

size_t tdt_lin_smem(int K, bool lstm) { return (void)lstm, tdt_smem(K); }

void tdt_kernels_init() {
  const size_t a = tdt_smem(1024);
  cudaFuncSetAttribute(k_tdt_lin<T_LSTM>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(a));
  cudaFuncSetAttribute(k_tdt_lin<T_PROJ>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(tdt_smem(1024)));
  cudaFuncSetAttribute(k_tdt_lin<T_JOINT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(tdt_smem(1024)));
}

void launch_tdt_begin(const TdtArgs& a, cudaStream_t st) {
  k_tdt_begin<<<(a.n + 255) / 256, 256, 0, st>>>(a);
  k_tdt_begin_lists<<<(a.n + 255) / 256, 256, 0, st>>>(a);
}

void launch_tdt_iteration(const TdtArgs& a, int parity, cudaStream_t st) {
  const int sg = (a.n + TM - 1) / TM;
  for (int l = 0; l < a.layers; l++) {
    TLin t;
    t.w0 = a.lstm_wx[l];
    t.w1 = a.lstm_wh[l];
    t.bias = a.lstm_b[l];
    t.layer = l;
    k_tdt_lin<T_LSTM><<<dim3(a.H / 8, sg), 256, tdt_smem(a.H), st>>>(a, t, parity);
  }
  TLin p;
  p.w0 = p.w1 = a.jpred;
  p.bias = a.jpred_b;
  k_tdt_lin<T_PROJ><<<dim3((a.J + TROWS - 1) / TROWS, sg), 256, tdt_smem(a.H), st>>>(a, p, parity);
  TLin j;
  j.w0 = j.w1 = a.jout;
  j.bias = a.jout_b;
  k_tdt_lin<T_JOINT><<<dim3((a.nout + TROWS - 1) / TROWS, sg), 256, tdt_smem(a.J), st>>>(a, j, parity);
  k_tdt_decide<<<(a.n + 3) / 4, 128, 0, st>>>(a, parity);
}

}  // namespace grx
