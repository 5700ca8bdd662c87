// One stream's FlowLM frames in one persistent kernel: flowLM.step
// (pockettts/lm.go:185-195 → transformer.forward, nn.go:142-182) and
// flowHead.sample (lm.go:108-160) with speakChunk's feedback of the latent
// (speak.go:146-175), for every frame of a run, with the reference's
// arithmetic kept value for value (the same orders as the per-kernel path:
// k_q8.cu's int8 chain, k_flin.cu's dot4q8avx / dot4f32avx lanes, k_attn.cu's
// scores, EXP8 sums and value chains, k_ln.cu's float64 LayerNorm).
//
// Why one kernel: at one stream a frame is ~35 dependent steps over 83 MB of
// weights; as separate launches each step pays a launch and a ramp, so the
// frame is bound by launch latency far from the HBM roofline. Here one CTA
// per SM (cooperative launch, so all are resident) runs every step, and the
// steps are separated by a grid barrier instead of a kernel boundary.
//
// Weights stream independently of the barriers: each CTA's slice of every
// product (its contiguous rows, int8 values and f16 scales, or float32 rows)
// is a "task", and the CTA keeps F1_SLOTS tasks in flight with bulk async
// copies (cp.async.bulk, no multicast) into a ring of shared-memory slots,
// issued as soon as a slot frees up — several steps ahead of the barrier
// chain. Everything a step needs beyond its own rows (LayerNorm of the
// residual, the rounding of the attention output) is computed by every CTA
// from the 4 KB vector in L2, which costs less than another barrier.
//
// Every wait is bounded (about a second of %globaltimer): a barrier or a
// copy that does not arrive sets the run's error word, every CTA leaves, and
// the host reports GRX_ETIMEDOUT; in-flight copies are drained before a CTA
// exits.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

// Phase marks for timing studies: a build may define F1_MARK(kind) to record
// them (kind: 1 barrier passed, 2 prologue done, 3 weights ready, 4 phase
// done, 6 barrier reached); the library defines it empty.
#ifndef F1_MARK
#define F1_MARK(kind)
#endif

namespace grx {

namespace {

constexpr int NT = F1_THREADS, NW = NT / 32;
constexpr uint32_t FULL = 0xffffffffu;
constexpr unsigned long long kWaitNs = 1000000000ull;  // one second per wait

// ------------------------------------------------------------ the tasks --

struct Region {
  const void* src;
  uint32_t bytes, off;
};
constexpr int kMaxRegions = 2 * (F1_MAX_DEPTH + 1) + 2;

__host__ __device__ inline int split(int n, int c, int G) { return int((long long)n * c / G); }
__host__ __device__ inline uint32_t up128(uint32_t v) { return (v + 127u) & ~127u; }

// Rows [r0, r1) of a Q8_0 matrix: the int8 values then the f16 scales.
__host__ __device__ inline void q8_slice(const DQ8& w, int r0, int r1, Region* r, int& n, uint32_t& off) {
  if (r1 <= r0) return;
  const uint32_t qb = uint32_t(r1 - r0) * uint32_t(w.cols), db = uint32_t(r1 - r0) * uint32_t(w.cols / QK) * 2u;
  r[n++] = {w.q + (size_t)r0 * w.cols, qb, off};
  off = up128(off + qb);
  r[n++] = {w.d + (size_t)r0 * (w.cols / QK), db, off};
  off = up128(off + db);
}
__host__ __device__ inline void f32_slice(const float* w, int cols, int r0, int r1, Region* r, int& n, uint32_t& off) {
  if (r1 <= r0) return;
  const uint32_t b = uint32_t(r1 - r0) * uint32_t(cols) * 4u;
  r[n++] = {w + (size_t)r0 * cols, b, off};
  off = up128(off + b);
}

// Tasks within a frame: per layer qkv, out, ff1, ff2; then cond (with the
// flow input rows), every adaLN projection, per residual block fc1 and fc2,
// and lm.input (the next frame's input projection). -1 is lm.input alone.
__host__ __device__ inline int frame_tasks(const Frame1Args& A) { return 4 * A.L + 3 + 2 * A.depth; }

__host__ __device__ inline int task_regions(const Frame1Args& A, int i, int c, int G, Region* r) {
  int n = 0;
  uint32_t off = 0;
  const int d = A.d, fd = A.fd;
  if (i < 0 || i == frame_tasks(A) - 1) {
    f32_slice(A.win, A.ldim, split(d, c, G), split(d, c + 1, G), r, n, off);
    return n;
  }
  if (i < 4 * A.L) {
    const F1Layer& ly = A.layers[i / 4];
    switch (i % 4) {
      case 0: {
        const int P = 3 * d / 2;
        q8_slice(ly.qkv, 2 * split(P, c, G), 2 * split(P, c + 1, G), r, n, off);
        break;
      }
      case 1:
        q8_slice(ly.out, split(d, c, G), split(d, c + 1, G), r, n, off);
        break;
      case 2: {
        const int NB = A.ff / QK;
        q8_slice(ly.ff1, QK * split(NB, c, G), QK * split(NB, c + 1, G), r, n, off);
        break;
      }
      default:
        q8_slice(ly.ff2, split(d, c, G), split(d, c + 1, G), r, n, off);
    }
    return n;
  }
  const int j = i - 4 * A.L;
  if (j == 0) {
    q8_slice(A.cond, split(fd, c, G), split(fd, c + 1, G), r, n, off);
    f32_slice(A.fin, A.ldim, split(fd, c, G), split(fd, c + 1, G), r, n, off);
  } else if (j == 1) {
    for (int k = 0; k < A.depth; k++) q8_slice(A.res[k].ada, split(3 * fd, c, G), split(3 * fd, c + 1, G), r, n, off);
    q8_slice(A.fada, split(2 * fd, c, G), split(2 * fd, c + 1, G), r, n, off);
  } else {
    const F1Res& rb = A.res[(j - 2) / 2];
    q8_slice((j - 2) % 2 == 0 ? rb.fc1 : rb.fc2, split(fd, c, G), split(fd, c + 1, G), r, n, off);
  }
  return n;
}

// ------------------------------------------------------- synchronisation --

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// The run's shared state in shared memory.
struct Ctl {
  int fail;           // this CTA gives up
  unsigned bar_k;     // grid barriers passed
  int issued;         // tasks issued (their copies started)
  int stall;          // the watchdog check: no barrier completes
};

// Grid barrier: a monotonically increasing arrival counter (zeroed before
// the launch); the k-th barrier waits for k·G arrivals. Bounded.
__device__ bool grid_sync(const Frame1Args& A, Ctl& ctl) {
  __syncthreads();
  F1_MARK(6);
  if (threadIdx.x == 0) {
    ctl.bar_k += 1;
    const unsigned target = ctl.stall ? 0xffffffffu : ctl.bar_k * gridDim.x;
    asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;\n" ::"l"(A.bar) : "memory");
    const unsigned long long t0 = gtime();
    for (int it = 0;; it++) {
      unsigned v;
      asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(A.bar) : "memory");
      if (v >= target) break;
      if ((it & 63) == 63) {
        if (*(volatile int*)A.err) {
          ctl.fail = 1;
          break;
        }
        if (gtime() - t0 > kWaitNs) {
          atomicCAS(A.err, 0, 1);
          ctl.fail = 1;
          break;
        }
      }
    }
    asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
  }
  __syncthreads();
  F1_MARK(1);
  return !ctl.fail;
}

// --------------------------------------------------------- shared memory --

struct Smem {
  uint8_t* slot[F1_SLOTS];
  uint64_t* mbar;    // [F1_SLOTS]
  int8_t* xq;        // [max(d, ff)] activations rounded to Q8_0
  float* xs;         // [max(d, ff)/32] their scales
  float* vf;         // [max(d, 2fd)] a float vector (LayerNorm output, flow-head input)
  float* vf2;        // [max(d, fd)]
  float* sc;         // [cap] attention scores
  float* vst;        // [cap][8] a CTA's value columns
  float* red;        // [64] reduction scratch (as doubles: 32)
  float* lat;        // [ldim] the latent
  Ctl* ctl;
};

__host__ __device__ inline size_t smem_layout(const Frame1Args& A, uint32_t slot_bytes, size_t* off) {
  const int vmax = A.d > A.ff ? A.d : A.ff;
  const int fmax = A.d > 2 * A.fd ? A.d : 2 * A.fd;
  size_t o = 0;
  for (int s = 0; s < F1_SLOTS; s++) {
    off[s] = o;
    o += slot_bytes;
  }
  off[F1_SLOTS + 0] = o;  // mbarriers
  o += 8 * F1_SLOTS;
  o = (o + 127) & ~size_t(127);
  off[F1_SLOTS + 1] = o;  // xq
  o += size_t(vmax);
  o = (o + 127) & ~size_t(127);
  off[F1_SLOTS + 2] = o;  // xs
  o += size_t(vmax / QK) * 4;
  o = (o + 127) & ~size_t(127);
  off[F1_SLOTS + 3] = o;  // vf
  o += size_t(fmax) * 4;
  off[F1_SLOTS + 4] = o;  // vf2
  o += size_t(fmax) * 4;
  off[F1_SLOTS + 5] = o;  // sc
  o += size_t(A.cap + 8) * 4;
  o = (o + 127) & ~size_t(127);
  off[F1_SLOTS + 9] = o;  // vst
  o += size_t(A.cap) * 32;
  off[F1_SLOTS + 6] = o;  // red (doubles)
  o += 64 * 4;
  off[F1_SLOTS + 7] = o;  // lat
  o += size_t(A.ldim) * 4;
  o = (o + 15) & ~size_t(15);
  off[F1_SLOTS + 8] = o;  // ctl
  o += sizeof(Ctl);
  return (o + 127) & ~size_t(127);
}

// ------------------------------------------------------------ the copies --

// Issues task g (sequence number in the run: 0 is lm.input for the first
// frame, then frame f's task i is 1 + f·W + i) into its slot.
__device__ void issue_task(const Frame1Args& A, const Smem& S, int g) {
  const int W = frame_tasks(A);
  const int i = g == 0 ? -1 : (g - 1) % W;
  Region r[kMaxRegions];
  const int n = task_regions(A, i, blockIdx.x, gridDim.x, r);
  uint32_t total = 0;
  for (int k = 0; k < n; k++) total += r[k].bytes;
  const int s = g % F1_SLOTS;
  const uint32_t bar = smem_addr(S.mbar + s), base = smem_addr(S.slot[s]);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(total) : "memory");
  for (int k = 0; k < n; k++)
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            base + r[k].off),
        "l"(r[k].src), "r"(r[k].bytes), "r"(bar)
        : "memory");
}

// Waits (thread 0, bounded) for task g's copies; false if they did not come.
__device__ bool wait_task(const Frame1Args& A, const Smem& S, int g) {
  if (threadIdx.x == 0) {
    const int s = g % F1_SLOTS;
    const uint32_t bar = smem_addr(S.mbar + s), parity = uint32_t(g / F1_SLOTS) & 1u;
    if (!mbar_try(bar, parity)) {
      const unsigned long long t0 = gtime();
      while (!mbar_try(bar, parity))
        if (gtime() - t0 > kWaitNs) {
          atomicCAS(A.err, 0, 2);
          S.ctl->fail = 1;
          break;
        }
    }
  }
  __syncthreads();
  if (S.ctl->fail) return false;
  // every thread observes the completed phase itself (acquiring the copies)
  mbar_try(smem_addr(S.mbar + g % F1_SLOTS), uint32_t(g / F1_SLOTS) & 1u);
  F1_MARK(3);
  return true;
}

// Frees task g's slot and starts the copies of task g + F1_SLOTS into it.
__device__ void release_task(const Frame1Args& A, const Smem& S, int g, int ntasks) {
  __syncthreads();  // every thread is done reading the slot
  F1_MARK(4);
  if (threadIdx.x == 0 && g + F1_SLOTS < ntasks) {
    issue_task(A, S, g + F1_SLOTS);
    S.ctl->issued = g + F1_SLOTS + 1;
  }
}

// Before leaving: every copy issued into this CTA's shared memory has landed
// (bounded; a copy still in flight after that is abandoned with the error set).
__device__ void drain(const Frame1Args& A, const Smem& S, int consumed) {
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int g = consumed; g < S.ctl->issued; g++) {
      const int s = g % F1_SLOTS;
      const uint32_t bar = smem_addr(S.mbar + s), parity = uint32_t(g / F1_SLOTS) & 1u;
      const unsigned long long t0 = gtime();
      while (!mbar_try(bar, parity) && gtime() - t0 < kWaitNs) {
      }
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------ block math --

__device__ __forceinline__ double block_sum_d(double v, float* red_) {
  double* red = reinterpret_cast<double*>(red_);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double t = 0;
  for (int i = 0; i < NW; i++) t += red[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = red[0];
  for (int i = 1; i < NW; i++) t = fmaxf(t, red[i]);
  return t;
}

// LayerNorm of D values from x (global) into out (shared), pockettts/nn.go:
// 27-49: float64 mean and biased variance, o = float((x − mean)·inv), then
// o·w + b in float32 when w, then (mod) o·(1 + scale) + shift.
__device__ void layer_norm(const float* x, int D, const float* w, const float* b, double eps, const float* shift,
                           const float* scale, float* out, float* red) {
  double s = 0;
  for (int i = threadIdx.x; i < D; i += NT) {
    const float v = __ldcg(x + i);
    out[i] = v;
    s += double(v);
  }
  const double mean = block_sum_d(s, red) / double(D);
  double q = 0;
  for (int i = threadIdx.x; i < D; i += NT) {
    const double dd = double(out[i]) - mean;
    q += dd * dd;
  }
  const double inv = 1.0 / sqrt(block_sum_d(q, red) / double(D) + eps);
  for (int i = threadIdx.x; i < D; i += NT) {
    float o = float((double(out[i]) - mean) * inv);
    if (w) o = __fadd_rn(__fmul_rn(o, w[i]), b[i]);
    if (shift) o = __fadd_rn(__fmul_rn(o, __fadd_rn(1.f, __ldcg(scale + i))), __ldcg(shift + i));
    out[i] = o;
  }
  __syncthreads();
}

// Q8_0 rounding of D shared values (quantU8, q8int.go:88-105), a warp per block.
__device__ void quant_smem(const float* v, int D, int8_t* q, float* s) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int b = w; b < D / QK; b += NW) {
    float sc;
    q[b * QK + l] = quant_lane(v[b * QK + l], &sc);
    if (l == 0) s[b] = sc;
  }
  __syncthreads();
}

// ---------------------------------------------------------- the products --

// R rows of the int8 path (q8int.go:148-223) by one warp: row r's values at
// wq + r·K (shared), scales wd + r·nb; lanes split the blocks, each block's
// exact int32 dot becomes t = float(s)·dw, and the chain c = fma(t, da, c)
// runs in block order (every lane holds the result).
template <int R>
__device__ __forceinline__ void q8_rows(const int8_t* wq, const uint16_t* wd, int K, const int8_t* xq, const float* xs,
                                        float (&c)[R]) {
  const int lane = threadIdx.x & 31, nb = K / QK;
#pragma unroll
  for (int r = 0; r < R; r++) c[r] = 0.f;
  for (int it = 0; it * 32 < nb; it++) {
    const int b = it * 32 + lane;
    float t[R];
    if (b < nb) {
      const int4 a0 = *reinterpret_cast<const int4*>(xq + b * QK), a1 = *reinterpret_cast<const int4*>(xq + b * QK + 16);
#pragma unroll
      for (int r = 0; r < R; r++) {
        const int4 w0 = *reinterpret_cast<const int4*>(wq + (size_t)r * K + b * QK);
        const int4 w1 = *reinterpret_cast<const int4*>(wq + (size_t)r * K + b * QK + 16);
        int s = __dp4a(w0.x, a0.x, 0);
        s = __dp4a(w0.y, a0.y, s);
        s = __dp4a(w0.z, a0.z, s);
        s = __dp4a(w0.w, a0.w, s);
        s = __dp4a(w1.x, a1.x, s);
        s = __dp4a(w1.y, a1.y, s);
        s = __dp4a(w1.z, a1.z, s);
        s = __dp4a(w1.w, a1.w, s);
        t[r] = __fmul_rn(i2f_small(s), h2f(wd[(size_t)r * nb + b]));
      }
    } else {
#pragma unroll
      for (int r = 0; r < R; r++) t[r] = 0.f;
    }
    const int lim = min(32, nb - it * 32);
    for (int l = 0; l < lim; l++) {
      const float da = xs[it * 32 + l];
#pragma unroll
      for (int r = 0; r < R; r++) c[r] = __fmaf_rn(__shfl_sync(FULL, t[r], l), da, c[r]);
    }
  }
}

// One row of the float path with a Q8_0 weight (dot4q8avx,
// kernels_amd64.s:343-399) by an 8-lane group: lane l of the group; the
// result lands in lane 0 of the group. x is shared.
__device__ __forceinline__ float q8f_row(const int8_t* wq, const uint16_t* wd, int K, const float* x) {
  const int l = threadIdx.x & 7;
  float acc = 0.f;
  for (int b = 0; b < K / QK; b++) {
    const int8_t* q = wq + b * QK;
    const float* xs = x + b * QK;
    float y = __fmul_rn(float(q[l]), xs[l]);
    y = __fmaf_rn(float(q[8 + l]), xs[8 + l], y);
    y = __fmaf_rn(float(q[16 + l]), xs[16 + l], y);
    y = __fmaf_rn(float(q[24 + l]), xs[24 + l], y);
    acc = __fmaf_rn(y, h2f(wd[b]), acc);
  }
  return hsum8_lanes(acc);
}

// One row of the float path with a float32 weight (dot4f32avx,
// kernels_amd64.s:157-204), K a multiple of 16, by an 8-lane group.
__device__ __forceinline__ float f32_row(const float* w, int K, const float* x) {
  const int l = threadIdx.x & 7;
  float a = 0.f, b = 0.f;
  for (int c = 0; c < K; c += 16) {
    a = __fmaf_rn(x[c + l], w[c + l], a);
    b = __fmaf_rn(x[c + 8 + l], w[c + 8 + l], b);
  }
  return hsum8_lanes(__fadd_rn(a, b));
}

// RoPE pair rotation (nn.go:80-93), unfused, as k_q8.cu.
__device__ __forceinline__ void rope(float& x0, float& x1, float2 cs) {
  const float r = x0, im = x1;
  x0 = __fsub_rn(__fmul_rn(r, cs.x), __fmul_rn(im, cs.y));
  x1 = __fadd_rn(__fmul_rn(r, cs.y), __fmul_rn(im, cs.x));
}

// ------------------------------------------------------------ the phases --

// x rows of this CTA = lm.input · latent (the frame's input projection).
__device__ void phase_input(const Frame1Args& A, const Smem& S, const uint8_t* slot) {
  const int c = blockIdx.x, G = gridDim.x, r0 = split(A.d, c, G), r1 = split(A.d, c + 1, G);
  const float* w = reinterpret_cast<const float*>(slot);
  const int g = threadIdx.x >> 3;  // 8-lane groups
  for (int rr = 0; rr * (NT / 8) < r1 - r0; rr++) {
    const int row = rr * (NT / 8) + g;  // whole warps iterate together
    const bool ok = row < r1 - r0;
    const float v = f32_row(w + (size_t)(ok ? row : 0) * A.ldim, A.ldim, S.lat);
    if (ok && (threadIdx.x & 7) == 0) A.x[r0 + row] = v;
  }
}

__device__ void phase_qkv(const Frame1Args& A, const Smem& S, const uint8_t* slot, int l, int pos) {
  const int c = blockIdx.x, G = gridDim.x, P = 3 * A.d / 2;
  const int p0 = split(P, c, G), p1 = split(P, c + 1, G), nrow = 2 * (p1 - p0), K = A.d;
  const int8_t* wq = reinterpret_cast<const int8_t*>(slot);
  const uint16_t* wd = reinterpret_cast<const uint16_t*>(slot + up128(uint32_t(nrow) * K));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, hd = 64, H = A.heads;
  for (int pr = warp; pr < p1 - p0; pr += NW) {
    float cc[2];
    q8_rows<2>(wq + (size_t)2 * pr * K, wd + (size_t)2 * pr * (K / QK), K, S.xq, S.xs, cc);
    if (lane == 0) {
      const int n = 2 * (p0 + pr), region = n / A.d, w = n - region * A.d, h = w / hd, i = w - h * hd;
      if (region < 2) rope(cc[0], cc[1], reinterpret_cast<const float2*>(A.rope)[(size_t)pos * (hd / 2) + i / 2]);
      if (region == 0) {
        *reinterpret_cast<float2*>(A.q + w) = make_float2(cc[0], cc[1]);
      } else {
        const size_t base = (((size_t)l * 2 + (region - 1)) * H + h) * (size_t)A.cap;
        *reinterpret_cast<float2*>(A.kv + (base + pos) * hd + i) = make_float2(cc[0], cc[1]);
      }
    }
  }
}

// transformer.attend for one query (nn.go:200-243): CTA c < 8·H takes head
// c/8 and value columns 8·(c%8) .. +7; every CTA of a head computes all its
// scores and the softmax (the same values), then its columns' chains.
__device__ void phase_attn(const Frame1Args& A, const Smem& S, int l, int pos) {
  const int c = blockIdx.x, H = A.heads;
  if (c >= 8 * H) return;
  const int h = c >> 3, cg = c & 7, nk = pos + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* K = A.kv + (((size_t)l * 2 + 0) * H + h) * (size_t)A.cap * 64;
  const float* V = A.kv + (((size_t)l * 2 + 1) * H + h) * (size_t)A.cap * 64;
  const float* q = A.q + h * 64;
  float* sc = S.sc;
  // scores, keys in groups of four (dot4f32avx), two keys per warp pass
  const int half = lane >> 4, li = lane & 15;
  const float q0 = __ldcg(q + li), q1 = __ldcg(q + 16 + li), q2 = __ldcg(q + 32 + li), q3 = __ldcg(q + 48 + li);
  const int nk4 = nk & ~3;
  constexpr int U = 8;
  for (int p0 = warp * U; 2 * p0 < nk4; p0 += NW * U) {
    float k[U][4];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = 2 * (p0 + u) + half;
      if (j < nk4) {
        const float* kr = K + (size_t)j * 64 + li;
        k[u][0] = __ldcg(kr);
        k[u][1] = __ldcg(kr + 16);
        k[u][2] = __ldcg(kr + 32);
        k[u][3] = __ldcg(kr + 48);
      } else {
        k[u][0] = k[u][1] = k[u][2] = k[u][3] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = 2 * (p0 + u) + half;
      float acc = __fmaf_rn(q0, k[u][0], 0.f);
      acc = __fmaf_rn(q1, k[u][1], acc);
      acc = __fmaf_rn(q2, k[u][2], acc);
      acc = __fmaf_rn(q3, k[u][3], acc);
      const float p = __fadd_rn(acc, __shfl_down_sync(FULL, acc, 8));
      const float s = hsum8_lanes(p);
      if (li == 0 && j < nk4) sc[j] = __fmul_rn(s, 0.125f);
    }
  }
  if (warp == NW - 1) {  // the last nk%4 keys: dotF32Go
    for (int j = nk4; j < nk; j++) {
      float s = 0.f;
      if (lane < 4)
        for (int i = lane; i < 64; i += 4) s = __fadd_rn(s, __fmul_rn(__ldcg(q + i), __ldcg(K + (size_t)j * 64 + i)));
      const float s1 = __shfl_sync(FULL, s, 1), s2 = __shfl_sync(FULL, s, 2), s3 = __shfl_sync(FULL, s, 3);
      if (lane == 0) sc[j] = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3), 0.125f);
    }
  }
  // this CTA's value columns, staged while the scores finish
  float* vs = S.vst;  // [nk][8]
  for (int t = tid; t < 2 * nk; t += NT) {
    const int j = t >> 1, hf = t & 1;
    reinterpret_cast<float4*>(vs)[t] = __ldcg(reinterpret_cast<const float4*>(V + (size_t)j * 64 + cg * 8 + hf * 4));
  }
  __syncthreads();
  float mx = -__int_as_float(0x7f800000);
  for (int j = tid; j < nk; j += NT) mx = fmaxf(mx, sc[j]);
  mx = block_max(mx, S.red + 32);
  const int n8 = nk & ~7;
  for (int j = tid; j < nk; j += NT) {
    const float x = __fsub_rn(sc[j], mx);
    sc[j] = j < n8 ? exp_avx(x) : expf_go(x);
  }
  __syncthreads();
  if (warp == 0) {
    float part = 0.f;
    if (lane < 8)
      for (int j = lane; j < n8; j += 8) part = __fadd_rn(part, sc[j]);
    const float savx = hsum8_lanes(part);
    if (lane == 0) {
      float tail = 0.f;
      for (int j = n8; j < nk; j++) tail = __fadd_rn(tail, sc[j]);
      S.red[0] = __fdiv_rn(1.f, __fadd_rn(savx, tail));
    }
  }
  __syncthreads();
  const float inv = S.red[0];
  for (int j = tid; j < nk; j += NT) sc[j] = __fmul_rn(sc[j], inv);
  __syncthreads();
  if (tid < 8) {
    float o = 0.f;
    int j = 0;
    for (; j + 8 <= nk; j += 8) {
      float w[8], v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        w[u] = sc[j + u];
        v[u] = vs[(j + u) * 8 + tid];
      }
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (w[u] != 0.f) o = __fmaf_rn(w[u], v[u], o);
    }
    for (; j < nk; j++) {
      const float w = sc[j];
      if (w != 0.f) o = __fmaf_rn(w, vs[j * 8 + tid], o);
    }
    A.att[h * 64 + cg * 8 + tid] = o;
  }
}

// Rows [r0, r1) of an int8-path product, K deep, R rows per warp at a time;
// out(n, c) receives each result (lane 0 of the warp).
template <class Out>
__device__ void q8_slice_rows(const uint8_t* slot, int nrow, int K, const Smem& S, Out out) {
  const int8_t* wq = reinterpret_cast<const int8_t*>(slot);
  const uint16_t* wd = reinterpret_cast<const uint16_t*>(slot + up128(uint32_t(nrow) * K));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int r = warp * 2;
  for (; r + 1 < nrow; r += 2 * NW) {
    float cc[2];
    q8_rows<2>(wq + (size_t)r * K, wd + (size_t)r * (K / QK), K, S.xq, S.xs, cc);
    if (lane == 0) {
      out(r, cc[0]);
      out(r + 1, cc[1]);
    }
  }
  if (r < nrow) {
    float cc[1];
    q8_rows<1>(wq + (size_t)r * K, wd + (size_t)r * (K / QK), K, S.xq, S.xs, cc);
    if (lane == 0) out(r, cc[0]);
  }
}

// Rows of a float-path product (Q8_0 rows kept) by 8-lane groups: out(row,
// v) in lane 0 of each group.
template <class Out>
__device__ void q8f_slice_rows(const uint8_t* slot, uint32_t off, int nrow, int K, const float* x, Out out) {
  const int8_t* wq = reinterpret_cast<const int8_t*>(slot + off);
  const uint16_t* wd = reinterpret_cast<const uint16_t*>(slot + off + up128(uint32_t(nrow) * K));
  const int g = threadIdx.x >> 3;
  for (int r0 = 0; r0 < nrow; r0 += NT / 8) {
    const int r = r0 + g;
    const bool ok = r < nrow;
    const int rr = ok ? r : 0;
    const float v = q8f_row(wq + (size_t)rr * K, wd + (size_t)rr * (K / QK), K, x);
    if (ok && (threadIdx.x & 7) == 0) out(r, v);
  }
}

// The size of a Q8_0 slice of nrow rows in a slot.
__device__ __forceinline__ uint32_t q8_bytes(int nrow, int K) {
  return up128(uint32_t(nrow) * K) + up128(uint32_t(nrow) * (K / QK) * 2u);
}

// ------------------------------------------------------------ the kernel --

__global__ void __launch_bounds__(NT, 1) k_frame1(const Frame1Args* __restrict__ Ap, uint32_t slot_bytes, int frames,
                                                  int stall) {
  extern __shared__ __align__(128) uint8_t f1_smem[];
  const Frame1Args& A = *Ap;
  Smem S;
  {
    size_t off[F1_SLOTS + 10];
    smem_layout(A, slot_bytes, off);
    for (int s = 0; s < F1_SLOTS; s++) S.slot[s] = f1_smem + off[s];
    S.mbar = reinterpret_cast<uint64_t*>(f1_smem + off[F1_SLOTS]);
    S.xq = reinterpret_cast<int8_t*>(f1_smem + off[F1_SLOTS + 1]);
    S.xs = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 2]);
    S.vf = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 3]);
    S.vf2 = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 4]);
    S.sc = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 5]);
    S.vst = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 9]);
    S.red = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 6]);
    S.lat = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 7]);
    S.ctl = reinterpret_cast<Ctl*>(f1_smem + off[F1_SLOTS + 8]);
  }
  const int tid = threadIdx.x, c = blockIdx.x, G = gridDim.x;
  const int W = frame_tasks(A), ntasks = 1 + frames * W;
  const int frame0 = A.io->frame, pos0 = A.pos[0];
  FrameIO io = *A.io;
  if (tid == 0) {
    S.ctl->fail = 0;
    S.ctl->bar_k = 0;
    S.ctl->issued = 0;
    S.ctl->stall = stall;
    for (int s = 0; s < F1_SLOTS; s++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_addr(S.mbar + s)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    const int first = ntasks < F1_SLOTS ? ntasks : F1_SLOTS;
    for (int g = 0; g < first; g++) issue_task(A, S, g);
    S.ctl->issued = first;
  }
  for (int i = tid; i < A.ldim; i += NT) S.lat[i] = A.lat[i];
  __syncthreads();
  int g = 0;  // the next task to consume

  // the first frame's input projection from the latent the set holds
  if (!wait_task(A, S, g)) goto out;
  phase_input(A, S, S.slot[g % F1_SLOTS]);
  release_task(A, S, g, ntasks);
  g++;

  for (int f = 0; f < frames; f++) {
    const int pos = pos0 + f, frame = frame0 + f;
    const float* noise = io.noise + ((size_t)frame * io.rows + io.row0) * A.ldim;
    for (int l = 0; l < A.L; l++) {
      const F1Layer& ly = A.layers[l];
      // ---- qkv (LayerNorm 1 → Q8_0 in every CTA) ----
      if (!grid_sync(A, *S.ctl)) goto out;
      layer_norm(A.x, A.d, ly.n1w, ly.n1b, 1e-5, nullptr, nullptr, S.vf, S.red);
      quant_smem(S.vf, A.d, S.xq, S.xs);
      F1_MARK(2);
      if (!wait_task(A, S, g)) goto out;
      phase_qkv(A, S, S.slot[g % F1_SLOTS], l, pos);
      release_task(A, S, g, ntasks);
      g++;
      // ---- attention ----
      if (!grid_sync(A, *S.ctl)) goto out;
      phase_attn(A, S, l, pos);
      __syncthreads();
      F1_MARK(4);
      // ---- out (+ residual) ----
      if (!grid_sync(A, *S.ctl)) goto out;
      for (int i = tid; i < A.d; i += NT) S.vf[i] = __ldcg(A.att + i);
      __syncthreads();
      quant_smem(S.vf, A.d, S.xq, S.xs);
      if (!wait_task(A, S, g)) goto out;
      {
        const int r0 = split(A.d, c, G), nrow = split(A.d, c + 1, G) - r0;
        float* x = A.x + r0;
        q8_slice_rows(S.slot[g % F1_SLOTS], nrow, A.d, S, [&](int r, float v) { x[r] = __fadd_rn(__ldcg(x + r), v); });
      }
      release_task(A, S, g, ntasks);
      g++;
      // ---- ff1 (LayerNorm 2 → Q8_0; GELU and the rounding of whole blocks here) ----
      if (!grid_sync(A, *S.ctl)) goto out;
      layer_norm(A.x, A.d, ly.n2w, ly.n2b, 1e-5, nullptr, nullptr, S.vf, S.red);
      quant_smem(S.vf, A.d, S.xq, S.xs);
      if (!wait_task(A, S, g)) goto out;
      {
        const int NB = A.ff / QK, b0 = split(NB, c, G), nrow = QK * (split(NB, c + 1, G) - b0);
        float* gv = S.vf2;
        q8_slice_rows(S.slot[g % F1_SLOTS], nrow, A.d, S, [&](int r, float v) { gv[r] = gelu_avx(v); });
        __syncthreads();
        const int warp = tid >> 5, lane = tid & 31;
        for (int b = warp; b < nrow / QK; b += NW) {
          float s;
          const int8_t qv = quant_lane(gv[b * QK + lane], &s);
          A.ffq[(b0 + b) * QK + lane] = qv;
          if (lane == 0) A.ffs[b0 + b] = s;
        }
      }
      release_task(A, S, g, ntasks);
      g++;
      // ---- ff2 (+ residual) ----
      if (!grid_sync(A, *S.ctl)) goto out;
      for (int i = tid; i < A.ff / 16; i += NT)
        reinterpret_cast<int4*>(S.xq)[i] = __ldcg(reinterpret_cast<const int4*>(A.ffq) + i);
      for (int i = tid; i < A.ff / QK; i += NT) S.xs[i] = __ldcg(A.ffs + i);
      __syncthreads();
      if (!wait_task(A, S, g)) goto out;
      {
        const int r0 = split(A.d, c, G), nrow = split(A.d, c + 1, G) - r0;
        float* x = A.x + r0;
        q8_slice_rows(S.slot[g % F1_SLOTS], nrow, A.ff, S, [&](int r, float v) { x[r] = __fadd_rn(__ldcg(x + r), v); });
      }
      release_task(A, S, g, ntasks);
      g++;
    }
    // ---- out_norm → lm_out, EOS; cond (→ SiLU) and the flow input h ----
    if (!grid_sync(A, *S.ctl)) goto out;
    layer_norm(A.x, A.d, A.outw, A.outb, 1e-5, nullptr, nullptr, S.vf, S.red);
    if (c == 0) {
      for (int i = tid; i < A.d; i += NT) A.lm_out[i] = S.vf[i];
      if (tid < 32) {  // eos = dotF32Go(lm_out, eosw) + b (gemm.go:294-308, lm.go:193-194)
        const int D4 = A.d & ~3;
        float s = 0.f;
        if (tid < 4)
          for (int i = tid; i < D4; i += 4) s = __fadd_rn(s, __fmul_rn(S.vf[i], A.eosw[i]));
        const float s1 = __shfl_sync(FULL, s, 1), s2 = __shfl_sync(FULL, s, 2), s3 = __shfl_sync(FULL, s, 3);
        if (tid == 0) {
          for (int i = D4; i < A.d; i++) s = __fadd_rn(s, __fmul_rn(S.vf[i], A.eosw[i]));
          const float e = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3), A.eosb);
          A.eos[0] = e;
          if (io.eos) io.eos[(size_t)frame * io.rows + io.row0] = e;
        }
      }
    }
    for (int i = tid; i < A.ldim; i += NT) S.vf2[i] = __ldcg(noise + i);
    __syncthreads();
    if (!wait_task(A, S, g)) goto out;
    {
      const int r0 = split(A.fd, c, G), nrow = split(A.fd, c + 1, G) - r0;
      const uint8_t* slot = S.slot[g % F1_SLOTS];
      q8f_slice_rows(slot, 0, nrow, A.d, S.vf, [&](int r, float v) {
        A.sy[r0 + r] = silu_avx(__fadd_rn(__fadd_rn(v, A.condb[r0 + r]), A.tc[r0 + r]));
      });
      const float* fw = reinterpret_cast<const float*>(slot + (nrow > 0 ? q8_bytes(nrow, A.d) : 0));
      const int gi = tid >> 3;
      for (int rr = 0; rr < nrow; rr += NT / 8) {
        const int r = rr + gi;
        const bool ok = r < nrow;
        const float v = f32_row(fw + (size_t)(ok ? r : 0) * A.ldim, A.ldim, S.vf2);
        if (ok && (tid & 7) == 0) A.h[r0 + r] = __fadd_rn(v, A.finb[r0 + r]);
      }
    }
    release_task(A, S, g, ntasks);
    g++;
    // ---- the adaLN projections of SiLU(y) ----
    if (!grid_sync(A, *S.ctl)) goto out;
    for (int i = tid; i < A.fd; i += NT) S.vf[i] = __ldcg(A.sy + i);
    __syncthreads();
    if (!wait_task(A, S, g)) goto out;
    {
      const uint8_t* slot = S.slot[g % F1_SLOTS];
      uint32_t off = 0;
      for (int k = 0; k <= A.depth; k++) {
        const bool fin = k == A.depth;
        const int N = fin ? 2 * A.fd : 3 * A.fd, r0 = split(N, c, G), nrow = split(N, c + 1, G) - r0;
        const float* bias = fin ? A.fadab : A.res[k].adab;
        float* y = fin ? A.mod2 : A.mod + (size_t)k * 3 * A.fd;
        q8f_slice_rows(slot, off, nrow, A.fd, S.vf, [&](int r, float v) { y[r0 + r] = __fadd_rn(v, bias[r0 + r]); });
        if (nrow > 0) off += q8_bytes(nrow, A.fd);
      }
    }
    release_task(A, S, g, ntasks);
    g++;
    // ---- the residual blocks ----
    for (int k = 0; k < A.depth; k++) {
      const F1Res& rb = A.res[k];
      const float* mod = A.mod + (size_t)k * 3 * A.fd;
      if (!grid_sync(A, *S.ctl)) goto out;
      layer_norm(A.h, A.fd, rb.nw, rb.nb, 1e-6, mod, mod + A.fd, S.vf, S.red);
      if (!wait_task(A, S, g)) goto out;
      {
        const int r0 = split(A.fd, c, G), nrow = split(A.fd, c + 1, G) - r0;
        q8f_slice_rows(S.slot[g % F1_SLOTS], 0, nrow, A.fd, S.vf,
                       [&](int r, float v) { A.mm[r0 + r] = silu_avx(__fadd_rn(v, rb.b1[r0 + r])); });
      }
      release_task(A, S, g, ntasks);
      g++;
      if (!grid_sync(A, *S.ctl)) goto out;
      for (int i = tid; i < A.fd; i += NT) S.vf[i] = __ldcg(A.mm + i);
      __syncthreads();
      if (!wait_task(A, S, g)) goto out;
      {
        const int r0 = split(A.fd, c, G), nrow = split(A.fd, c + 1, G) - r0;
        q8f_slice_rows(S.slot[g % F1_SLOTS], 0, nrow, A.fd, S.vf, [&](int r, float v) {
          const int n = r0 + r;
          A.h[n] = __fadd_rn(__ldcg(A.h + n), __fmul_rn(__ldcg(mod + 2 * A.fd + n), __fadd_rn(v, rb.b2[n])));
        });
      }
      release_task(A, S, g, ntasks);
      g++;
    }
    // ---- the final adaLN, the latent (every CTA), the next input rows ----
    if (!grid_sync(A, *S.ctl)) goto out;
    layer_norm(A.h, A.fd, nullptr, nullptr, 1e-6, A.mod2, A.mod2 + A.fd, S.vf, S.red);
    {
      const int gi = tid >> 3;
      for (int rr = 0; rr < A.ldim; rr += NT / 8) {
        const int r = rr + gi;
        const bool ok = r < A.ldim;
        const float v = f32_row(A.fout + (size_t)(ok ? r : 0) * A.fd, A.fd, S.vf);
        if (ok && (tid & 7) == 0) {
          const float cur = __fadd_rn(__ldcg(noise + r), __fdiv_rn(__fadd_rn(v, A.foutb[r]), 1.f));
          S.lat[r] = cur;
          if (c == 0) {
            const float scv = __fadd_rn(__fmul_rn(cur, A.stdv[r]), A.mean[r]);
            A.lat[r] = cur;
            const size_t o = ((size_t)frame * io.rows + io.row0) * A.ldim + r;
            if (io.latent) io.latent[o] = cur;
            if (io.scaled) io.scaled[o] = scv;
          }
        }
      }
    }
    __syncthreads();
    if (!wait_task(A, S, g)) goto out;
    phase_input(A, S, S.slot[g % F1_SLOTS]);
    release_task(A, S, g, ntasks);
    g++;
  }
  if (c == 0 && tid == 0) {
    A.pos[0] = pos0 + frames;
    A.io->frame = frame0 + frames;
  }
out:
  drain(A, S, g);
}

}  // namespace

bool frame1_suits(const Frame1Args& A, size_t* smem, uint32_t* slot_bytes, int G) {
  // (scales slices start on 16-byte boundaries: K % 256 == 0)
  if (A.d % 256 || A.heads * 64 != A.d || A.ff % 256 || A.fd % 256 || A.ldim % 16 || A.ldim > 64 || A.L < 1 ||
      A.L > F1_MAX_LAYERS || A.depth < 1 || A.depth > F1_MAX_DEPTH || A.d > 4096 || A.ff > 8192 || A.fd > 2048 ||
      A.cap < 1 || 8 * A.heads > G)
    return false;
  // a CTA's ff1 rows (whole Q8_0 blocks) fit the GELU buffer vf2
  const int fmax = A.d > 2 * A.fd ? A.d : 2 * A.fd, nbk = A.ff / QK;
  if (QK * ((nbk + G - 1) / G) > fmax) return false;
  uint32_t sb = 0;
  Region r[kMaxRegions];
  for (int i = -1; i < frame_tasks(A); i++)
    for (int c = 0; c < G; c++) {
      const int n = task_regions(A, i, c, G, r);
      if (n > kMaxRegions) return false;
      for (int k = 0; k < n; k++) sb = sb > r[k].off + r[k].bytes ? sb : up128(r[k].off + r[k].bytes);
    }
  size_t off[F1_SLOTS + 10];
  const size_t need = smem_layout(A, sb, off);
  *smem = need;
  *slot_bytes = sb;
  return need <= 227 * 1024;
}

cudaError_t launch_frame1(const Frame1Args* d_args, size_t smem, uint32_t slot_bytes, int G, int frames, int stall,
                          cudaStream_t st) {
  static thread_local int last_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != last_dev) {
    cudaError_t e = cudaFuncSetAttribute(k_frame1, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    last_dev = dev;
  }
  void* args[] = {(void*)&d_args, (void*)&slot_bytes, (void*)&frames, (void*)&stall};
  return cudaLaunchCooperativeKernel((const void*)k_frame1, dim3(G), dim3(NT), args, smem, st);
}

int frame1_max_active(size_t smem) {
  int n = 0;
  cudaFuncSetAttribute(k_frame1, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_frame1, NT, smem) != cudaSuccess) return 0;
  return n;
}

}  // namespace grx
