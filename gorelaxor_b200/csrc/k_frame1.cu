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
// copies (plain cp.async.bulk, this CTA only) into a ring of shared-memory slots,
// issued as soon as a slot frees up — several steps ahead of the barrier
// chain. What a step needs beyond its own rows (the LayerNorm of the
// residual, the rounding of the attention output) every CTA computes from
// the 4 KB vector in L2, each warp reducing it on its own so that no
// block-wide reduction stands in the way. The residual rows a CTA owns stay
// in its shared memory (every product that updates them uses the same row
// split), so updating them reads nothing back from L2.
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
constexpr int kOwnMax = 64;                            // rows of x or h one CTA may own

// ------------------------------------------------------------ the tasks --

struct Region {
  const void* src;
  uint32_t bytes, off;
};
constexpr int kMaxRegions = 2 * (F1_MAX_DEPTH + 1) + 2;
// Regions of every task of a frame plus lm.input alone: per layer at most 2
// per product, cond 3, the adaLN projections 2·(depth + 1), fc1 / fc2 2 each.
constexpr int kTableRegions = 8 * F1_MAX_LAYERS + 3 + 2 * (F1_MAX_DEPTH + 1) + 4 * F1_MAX_DEPTH + 2;
constexpr int kMaxTasks = 4 * F1_MAX_LAYERS + 3 + 2 * F1_MAX_DEPTH + 1;

// CTA c's share of n items over G CTAs starts here (n·c < 2^31 for every
// shape the kernel takes).
__host__ __device__ inline int split(int n, int c, int G) { return (n * c) / G; }
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
  int fail;        // this CTA gives up
  unsigned bar_k;  // grid barriers passed
  int issued;      // tasks issued (their copies started)
  int stall;       // the watchdog check: no barrier completes
  int pending;     // a task to issue once this CTA has arrived at the next barrier (−1: none)
  int ntab;        // regions in the task table
  uint16_t tstart[kMaxTasks + 1], tcount[kMaxTasks + 1];  // per task (index i + 1)
};

// Grid barrier: a monotonically increasing arrival counter (zeroed before
// the launch); the k-th barrier waits for k·G arrivals. The arrival is a
// release (the CTA's writes, ordered before it by the block barrier, become
// visible with it) and the polling load an acquire. Bounded.
template <class Arrived>
__device__ bool grid_sync(const Frame1Args& A, Ctl& ctl, Arrived arrived) {
  __syncthreads();
  F1_MARK(6);
  if (threadIdx.x == 0) {
    ctl.bar_k += 1;
    const unsigned target = ctl.stall ? 0xffffffffu : ctl.bar_k * gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(A.bar) : "memory");
    arrived();  // work that overlaps the wait
    const unsigned long long t0 = gtime();
    for (int it = 0;; it++) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(A.bar) : "memory");
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
  }
  __syncthreads();
  F1_MARK(1);
  return !ctl.fail;
}

// --------------------------------------------------------- shared memory --

struct Smem {
  uint8_t* slot[F1_SLOTS];
  uint64_t* mbar;    // [F1_SLOTS]
  Region* tab;       // [kTableRegions] every task's copies, this CTA
  int8_t* xq;        // [max(d, ff)] activations rounded to Q8_0
  float* xs;         // [max(d, ff)/32] their scales
  float* vf;         // [max(d, 2fd)] a float vector (LayerNorm output, flow-head input)
  float* vf2;        // [max(d, 2fd)]
  float* sc;         // [cap] attention scores
  float* vst;        // [max(cap·8, NW·2·128)] value columns, or the warps' chain scratch
  float* red;        // [128] reduction scratch: 2·NW doubles, then floats from 64
  float* lat;        // [ldim] the latent
  float* xo;         // [kOwnMax] the rows of x this CTA owns
  float* ho;         // [kOwnMax] the rows of h this CTA owns
  Ctl* ctl;
};

constexpr int kChainPerWarp = 2 * 128;  // two rows of up to 128 blocks

__host__ __device__ inline size_t smem_layout(const Frame1Args& A, uint32_t slot_bytes, size_t* off) {
  const int vmax = A.d > A.ff ? A.d : A.ff;
  const int fmax = A.d > 2 * A.fd ? A.d : 2 * A.fd;
  const size_t vst = size_t(A.cap) * 8 > size_t(NW) * kChainPerWarp ? size_t(A.cap) * 8 : size_t(NW) * kChainPerWarp;
  size_t o = 0;
  auto take = [&](int k, size_t bytes) {
    off[k] = o;
    o = (o + bytes + 127) & ~size_t(127);
  };
  for (int s = 0; s < F1_SLOTS; s++) take(s, slot_bytes);
  take(F1_SLOTS + 0, 8 * F1_SLOTS);                    // mbarriers
  take(F1_SLOTS + 1, sizeof(Region) * kTableRegions);  // task table
  take(F1_SLOTS + 2, size_t(vmax));                    // xq
  take(F1_SLOTS + 3, size_t(vmax / QK) * 4);           // xs
  take(F1_SLOTS + 4, size_t(fmax) * 4);                // vf
  take(F1_SLOTS + 5, size_t(fmax) * 4);                // vf2
  take(F1_SLOTS + 6, size_t(A.cap + 8) * 4);           // sc
  take(F1_SLOTS + 7, vst * 4);                         // vst
  take(F1_SLOTS + 8, 128 * 4);                         // red: 2·NW doubles, then NW floats
  take(F1_SLOTS + 9, size_t(A.ldim) * 4);              // lat
  take(F1_SLOTS + 10, kOwnMax * 4);                    // xo
  take(F1_SLOTS + 11, kOwnMax * 4);                    // ho
  take(F1_SLOTS + 12, sizeof(Ctl));                    // ctl
  return o;
}
constexpr int kSmemParts = F1_SLOTS + 13;

// ------------------------------------------------------------ the copies --

// Issues task g (sequence number in the run: 0 is lm.input for the first
// frame, then frame f's task i is 1 + f·W + i) into its slot, from the table.
__device__ void issue_task(const Smem& S, int W, int g) {
  const int i = g == 0 ? -1 : (g - 1) % W;
  const Ctl& ctl = *S.ctl;
  const int t0 = ctl.tstart[i + 1], n = ctl.tcount[i + 1];
  uint32_t total = 0;
  for (int k = 0; k < n; k++) total += S.tab[t0 + k].bytes;
  const int s = g % F1_SLOTS;
  const uint32_t bar = smem_addr(S.mbar + s), base = smem_addr(S.slot[s]);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(total) : "memory");
  for (int k = 0; k < n; k++) {
    const Region& r = S.tab[t0 + k];
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            base + r.off),
        "l"(r.src), "r"(r.bytes), "r"(bar)
        : "memory");
  }
}

// Waits (thread 0, bounded) for task g's copies; false if they did not come.
__device__ bool wait_task(const Frame1Args& A, const Smem& S, int g) {
  const int s = g % F1_SLOTS;
  const uint32_t bar = smem_addr(S.mbar + s), parity = uint32_t(g / F1_SLOTS) & 1u;
  if (threadIdx.x == 0 && !mbar_try(bar, parity)) {
    const unsigned long long t0 = gtime();
    while (!mbar_try(bar, parity))
      if (gtime() - t0 > kWaitNs) {
        atomicCAS(A.err, 0, 2);
        S.ctl->fail = 1;
        break;
      }
  }
  __syncthreads();
  if (S.ctl->fail) return false;
  // every thread observes the completed phase itself (acquiring the copies)
  mbar_try(bar, parity);
  F1_MARK(3);
  return true;
}

// Frees task g's slot; the copies of task g + F1_SLOTS into it start once
// this CTA has arrived at the next grid barrier (sync below), so that they
// overlap the wait instead of delaying the arrival.
__device__ void release_task(const Smem& S, int W, int g, int ntasks) {
  __syncthreads();  // every thread is done reading the slot
  F1_MARK(4);
  if (threadIdx.x == 0 && g + F1_SLOTS < ntasks) S.ctl->pending = g + F1_SLOTS;
}

__device__ void issue_pending(const Smem& S, int W) {
  Ctl& ctl = *S.ctl;
  if (ctl.pending >= 0) {
    issue_task(S, W, ctl.pending);
    ctl.issued = ctl.pending + 1;
    ctl.pending = -1;
  }
}

// The grid barrier with the pending copies issued after this CTA's arrival.
__device__ __forceinline__ bool sync(const Frame1Args& A, const Smem& S, int W) {
  return grid_sync(A, *S.ctl, [&] { issue_pending(S, W); });
}

// Before leaving: every copy issued into this CTA's shared memory has landed
// (bounded; a copy still in flight after that is abandoned with the error set).
__device__ void drain(const Smem& S, int consumed) {
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

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}

// A double summed over the block: lanes, then the warps' partials, in the
// same tree order in every warp, so every thread returns the same value.
__device__ __forceinline__ double block_sum_d(double v, double* red) {
  v = warp_sum_d(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  // every lane sums all 32 (lanes past NW hold 0): each butterfly step adds
  // the same two values in both lanes of a pair, so all lanes end equal
  return warp_sum_d(l < NW ? red[l] : 0.0);
}

// LayerNorm of D values (D ≤ 2·NT, a multiple of 32) from x (global) into out
// (shared), pockettts/nn.go:27-49: float64 mean and biased variance,
// o = float((x − mean)·inv), then o·w + b in float32 when w, then (shift)
// o·(1 + scale) + shift. Each thread keeps its values in registers; thread
// t holds elements t and t + NT, so every warp holds whole 32-value blocks.
// With q, each warp rounds its blocks to Q8_0 (quantU8, q8int.go:88-105)
// into q / qs instead of writing out.
__device__ void layer_norm(const float* x, int D, const float* w, const float* b, double eps, const float* shift,
                           const float* scale, float* out, int8_t* q, float* qs, float* red_) {
  double* red = reinterpret_cast<double*>(red_);
  const int t = threadIdx.x, lane = t & 31;
  const bool h0 = t < D, h1 = t + NT < D;
  const float v0 = h0 ? __ldcg(x + t) : 0.f, v1 = h1 ? __ldcg(x + t + NT) : 0.f;
  const double mean = block_sum_d((h0 ? double(v0) : 0.0) + (h1 ? double(v1) : 0.0), red) / double(D);
  const double d0 = h0 ? double(v0) - mean : 0.0, d1 = h1 ? double(v1) - mean : 0.0;
  const double inv = 1.0 / sqrt(block_sum_d(d0 * d0 + d1 * d1, red + NW) / double(D) + eps);
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int i = t + k * NT;
    if (i >= D) break;  // (warp-uniform: D is a multiple of 32)
    float o = float(((k ? double(v1) : double(v0)) - mean) * inv);
    if (w) o = __fadd_rn(__fmul_rn(o, w[i]), b[i]);
    if (shift) o = __fadd_rn(__fmul_rn(o, __fadd_rn(1.f, __ldcg(scale + i))), __ldcg(shift + i));
    if (q) {
      float sc;
      q[i] = quant_lane(o, &sc);
      if (lane == 0) qs[i / QK] = sc;
    } else {
      out[i] = o;
    }
  }
  __syncthreads();
}

// Q8_0 rounding of D values from global memory into q / qs, a warp per block.
__device__ void quant_global(const float* v, int D, int8_t* q, float* s) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int b = w; b < D / QK; b += NW) {
    float sc;
    q[b * QK + l] = quant_lane(__ldcg(v + b * QK + l), &sc);
    if (l == 0) s[b] = sc;
  }
  __syncthreads();
}

// ---------------------------------------------------------- the products --

// R rows of the int8 path (q8int.go:148-223) by one warp: row r's values at
// wq + r·K (shared), scales wd + r·nb. Lanes split the blocks; each block's
// exact int32 dot becomes t = float(s)·dw in the warp's scratch tb, then the
// chain c = fma(t, da, c) runs in block order in every lane from there.
template <int R>
__device__ __forceinline__ void q8_rows(const int8_t* wq, const uint16_t* wd, int K, const int8_t* xq, const float* xs,
                                        float* tb, float (&c)[R]) {
  const int lane = threadIdx.x & 31, nb = K / QK;
  for (int b = lane; b < nb; b += 32) {
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
      tb[r * nb + b] = __fmul_rn(i2f_small(s), h2f(wd[(size_t)r * nb + b]));
    }
  }
  __syncwarp();
#pragma unroll
  for (int r = 0; r < R; r++) c[r] = 0.f;
#pragma unroll 16
  for (int b = 0; b < nb; b++) {
    const float da = xs[b];
#pragma unroll
    for (int r = 0; r < R; r++) c[r] = __fmaf_rn(tb[r * nb + b], da, c[r]);
  }
  __syncwarp();  // the scratch is free again
}

// One row of the float path with a Q8_0 weight (dot4q8avx,
// kernels_amd64.s:343-399) by an 8-lane group: lane l of the group; the
// result lands in lane 0 of the group. x is shared.
__device__ __forceinline__ float q8f_row(const int8_t* wq, const uint16_t* wd, int K, const float* x) {
  const int l = threadIdx.x & 7;
  float acc = 0.f;
#pragma unroll 4
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
#pragma unroll 4
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

// Rows [0, nrow) of an int8-path product K deep from a slot, two rows per
// warp at a time; out(r, c) receives each result in lane 0.
template <class Out>
__device__ void q8_slice_rows(const uint8_t* slot, int nrow, int K, const Smem& S, Out out) {
  const int8_t* wq = reinterpret_cast<const int8_t*>(slot);
  const uint16_t* wd = reinterpret_cast<const uint16_t*>(slot + up128(uint32_t(nrow) * K));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* tb = S.vst + warp * kChainPerWarp;
  int r = warp * 2;
  for (; r + 1 < nrow; r += 2 * NW) {
    float cc[2];
    q8_rows<2>(wq + (size_t)r * K, wd + (size_t)r * (K / QK), K, S.xq, S.xs, tb, cc);
    if (lane == 0) {
      out(r, cc[0]);
      out(r + 1, cc[1]);
    }
  }
  if (r < nrow) {
    float cc[1];
    q8_rows<1>(wq + (size_t)r * K, wd + (size_t)r * (K / QK), K, S.xq, S.xs, tb, cc);
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

// ------------------------------------------------------------ the phases --

// The x rows this CTA owns = lm.input · latent (the frame's input
// projection), kept in xo and written through to x.
__device__ void phase_input(const Frame1Args& A, const Smem& S, const uint8_t* slot) {
  const int c = blockIdx.x, G = gridDim.x, r0 = split(A.d, c, G), nrow = split(A.d, c + 1, G) - r0;
  const float* w = reinterpret_cast<const float*>(slot);
  const int g = threadIdx.x >> 3;
  for (int rr = 0; rr < nrow; rr += NT / 8) {
    const int row = rr + g;
    const bool ok = row < nrow;
    const float v = f32_row(w + (size_t)(ok ? row : 0) * A.ldim, A.ldim, S.lat);
    if (ok && (threadIdx.x & 7) == 0) {
      S.xo[row] = v;
      A.x[r0 + row] = v;
    }
  }
}

__device__ void phase_qkv(const Frame1Args& A, const Smem& S, const uint8_t* slot, int l, int pos) {
  const int c = blockIdx.x, G = gridDim.x, P = 3 * A.d / 2;
  const int p0 = split(P, c, G), p1 = split(P, c + 1, G), nrow = 2 * (p1 - p0), K = A.d;
  const int8_t* wq = reinterpret_cast<const int8_t*>(slot);
  const uint16_t* wd = reinterpret_cast<const uint16_t*>(slot + up128(uint32_t(nrow) * K));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, hd = 64, H = A.heads;
  float* tb = S.vst + warp * kChainPerWarp;
  for (int pr = warp; pr < p1 - p0; pr += NW) {
    float cc[2];
    q8_rows<2>(wq + (size_t)2 * pr * K, wd + (size_t)2 * pr * (K / QK), K, S.xq, S.xs, tb, cc);
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
  float* vs = S.vst;  // [nk][8]
  // this CTA's value columns: loads issued first, stored once the scores are done
  constexpr int VP = 2;
  float4 vreg[VP];
#pragma unroll
  for (int u = 0; u < VP; u++) {
    const int t = tid + u * NT;
    if (t < 2 * nk) vreg[u] = __ldcg(reinterpret_cast<const float4*>(V + (size_t)(t >> 1) * 64 + cg * 8 + (t & 1) * 4));
  }
  // scores, keys in groups of four (dot4f32avx), two keys per warp pass;
  // each warp keeps the largest score it wrote
  const int half = lane >> 4, li = lane & 15;
  const float q0 = __ldcg(q + li), q1 = __ldcg(q + 16 + li), q2 = __ldcg(q + 32 + li), q3 = __ldcg(q + 48 + li);
  const int nk4 = nk & ~3;
  float wmax = -__int_as_float(0x7f800000);
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
      const float s = __fmul_rn(hsum8_lanes(p), 0.125f);
      if (li == 0 && j < nk4) {
        sc[j] = s;
        wmax = fmaxf(wmax, s);
      }
    }
  }
  if (warp == NW - 1) {  // the last nk%4 keys: dotF32Go
    for (int j = nk4; j < nk; j++) {
      float s = 0.f;
      if (lane < 4)
        for (int i = lane; i < 64; i += 4) s = __fadd_rn(s, __fmul_rn(__ldcg(q + i), __ldcg(K + (size_t)j * 64 + i)));
      const float s1 = __shfl_sync(FULL, s, 1), s2 = __shfl_sync(FULL, s, 2), s3 = __shfl_sync(FULL, s, 3);
      if (lane == 0) {
        const float v = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3), 0.125f);
        sc[j] = v;
        wmax = fmaxf(wmax, v);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wmax = fmaxf(wmax, __shfl_xor_sync(FULL, wmax, o));
  float* fred = S.red + 64;
  if (lane == 0) fred[warp] = wmax;
#pragma unroll
  for (int u = 0; u < VP; u++) {
    const int t = tid + u * NT;
    if (t < 2 * nk) reinterpret_cast<float4*>(vs)[t] = vreg[u];
  }
  for (int t = tid + VP * NT; t < 2 * nk; t += NT)
    reinterpret_cast<float4*>(vs)[t] = __ldcg(reinterpret_cast<const float4*>(V + (size_t)(t >> 1) * 64 + cg * 8 + (t & 1) * 4));
  __syncthreads();
  float mx = fred[0];
  for (int i = 1; i < NW; i++) mx = fmaxf(mx, fred[i]);
  // expSub: EXP8 over the first nk&~7 scores, Go's expf for the rest
  const int n8 = nk & ~7;
  for (int j = tid; j < nk; j += NT) {
    const float x = __fsub_rn(sc[j], mx);
    sc[j] = j < n8 ? exp_avx(x) : expf_go(x);
  }
  __syncthreads();
  if (warp != 0) return;
  // warp 0: the 8 lane sums in key order, HSUM, the scalar tail, 1/Σ; then
  // lanes 0-7 run the value chains with w_j = e_j·(1/Σ) (kern.Scale then
  // AddScaled, nn.go:228-236), skipping w_j == 0
  float part = 0.f;
  if (lane < 8)
    for (int j = lane; j < n8; j += 8) part = __fadd_rn(part, sc[j]);
  const float savx = hsum8_lanes(part);
  float inv = 0.f;
  if (lane == 0) {
    float tail = 0.f;
    for (int j = n8; j < nk; j++) tail = __fadd_rn(tail, sc[j]);
    inv = __fdiv_rn(1.f, __fadd_rn(savx, tail));
  }
  inv = __shfl_sync(FULL, inv, 0);
  if (lane < 8) {
    float o = 0.f;
    int j = 0;
    for (; j + 8 <= nk; j += 8) {
      float w[8], v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        w[u] = __fmul_rn(sc[j + u], inv);
        v[u] = vs[(j + u) * 8 + lane];
      }
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (w[u] != 0.f) o = __fmaf_rn(w[u], v[u], o);
    }
    for (; j < nk; j++) {
      const float w = __fmul_rn(sc[j], inv);
      if (w != 0.f) o = __fmaf_rn(w, vs[j * 8 + lane], o);
    }
    A.att[h * 64 + cg * 8 + lane] = o;
  }
}

// ------------------------------------------------------------ the kernel --

__global__ void __launch_bounds__(NT, 1) k_frame1(const Frame1Args* __restrict__ Ap, uint32_t slot_bytes, int frames,
                                                  int stall) {
  extern __shared__ __align__(128) uint8_t f1_smem[];
  const Frame1Args& A = *Ap;
  Smem S;
  {
    size_t off[kSmemParts];
    smem_layout(A, slot_bytes, off);
    for (int s = 0; s < F1_SLOTS; s++) S.slot[s] = f1_smem + off[s];
    S.mbar = reinterpret_cast<uint64_t*>(f1_smem + off[F1_SLOTS]);
    S.tab = reinterpret_cast<Region*>(f1_smem + off[F1_SLOTS + 1]);
    S.xq = reinterpret_cast<int8_t*>(f1_smem + off[F1_SLOTS + 2]);
    S.xs = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 3]);
    S.vf = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 4]);
    S.vf2 = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 5]);
    S.sc = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 6]);
    S.vst = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 7]);
    S.red = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 8]);
    S.lat = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 9]);
    S.xo = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 10]);
    S.ho = reinterpret_cast<float*>(f1_smem + off[F1_SLOTS + 11]);
    S.ctl = reinterpret_cast<Ctl*>(f1_smem + off[F1_SLOTS + 12]);
  }
  const int tid = threadIdx.x, c = blockIdx.x, G = gridDim.x;
  const int W = frame_tasks(A), ntasks = 1 + frames * W;
  const int frame0 = A.io->frame, pos0 = A.pos[0];
  const FrameIO io = *A.io;
  const int last = G - 1;  // the CTA that writes the frame's outputs (it has no attention work)
  if (tid == 0) {
    Ctl& ctl = *S.ctl;
    ctl.fail = 0;
    ctl.bar_k = 0;
    ctl.stall = stall;
    ctl.pending = -1;
    int n = 0;
    for (int i = -1; i < W; i++) {  // this CTA's copies of every task, once per launch
      ctl.tstart[i + 1] = uint16_t(n);
      ctl.tcount[i + 1] = uint16_t(task_regions(A, i, c, G, S.tab + n));
      n += ctl.tcount[i + 1];
    }
    ctl.ntab = n;
    for (int s = 0; s < F1_SLOTS; s++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_addr(S.mbar + s)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    const int first = ntasks < F1_SLOTS ? ntasks : F1_SLOTS;
    for (int g = 0; g < first; g++) issue_task(S, W, g);
    ctl.issued = first;
  }
  for (int i = tid; i < A.ldim; i += NT) S.lat[i] = A.lat[i];
  __syncthreads();
  int g = 0;  // the next task to consume

  // the first frame's input projection from the latent the set holds
  if (!wait_task(A, S, g)) goto out;
  phase_input(A, S, S.slot[g % F1_SLOTS]);
  release_task(S, W, g, ntasks);
  g++;

  for (int f = 0; f < frames; f++) {
    const int pos = pos0 + f, frame = frame0 + f;
    const float* noise = io.noise + ((size_t)frame * io.rows + io.row0) * A.ldim;
    for (int l = 0; l < A.L; l++) {
      const F1Layer& ly = A.layers[l];
      // ---- qkv (LayerNorm 1 → Q8_0 in every CTA) ----
      if (!sync(A, S, W)) goto out;
      layer_norm(A.x, A.d, ly.n1w, ly.n1b, 1e-5, nullptr, nullptr, S.vf, S.xq, S.xs, S.red);
      F1_MARK(2);
      if (!wait_task(A, S, g)) goto out;
      phase_qkv(A, S, S.slot[g % F1_SLOTS], l, pos);
      release_task(S, W, g, ntasks);
      g++;
      // ---- attention ----
      if (!sync(A, S, W)) goto out;
      phase_attn(A, S, l, pos);
      __syncthreads();
      F1_MARK(4);
      // ---- out (+ residual) ----
      if (!sync(A, S, W)) goto out;
      quant_global(A.att, A.d, S.xq, S.xs);
      if (!wait_task(A, S, g)) goto out;
      {
        const int r0 = split(A.d, c, G), nrow = split(A.d, c + 1, G) - r0;
        q8_slice_rows(S.slot[g % F1_SLOTS], nrow, A.d, S, [&](int r, float v) {
          const float nx = __fadd_rn(S.xo[r], v);
          S.xo[r] = nx;
          A.x[r0 + r] = nx;
        });
      }
      release_task(S, W, g, ntasks);
      g++;
      // ---- ff1 (LayerNorm 2 → Q8_0; GELU and the rounding of whole blocks here) ----
      if (!sync(A, S, W)) goto out;
      layer_norm(A.x, A.d, ly.n2w, ly.n2b, 1e-5, nullptr, nullptr, S.vf, S.xq, S.xs, S.red);
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
      release_task(S, W, g, ntasks);
      g++;
      // ---- ff2 (+ residual) ----
      if (!sync(A, S, W)) goto out;
      for (int i = tid; i < A.ff / 16; i += NT)
        reinterpret_cast<int4*>(S.xq)[i] = __ldcg(reinterpret_cast<const int4*>(A.ffq) + i);
      for (int i = tid; i < A.ff / QK; i += NT) S.xs[i] = __ldcg(A.ffs + i);
      __syncthreads();
      if (!wait_task(A, S, g)) goto out;
      {
        const int r0 = split(A.d, c, G), nrow = split(A.d, c + 1, G) - r0;
        q8_slice_rows(S.slot[g % F1_SLOTS], nrow, A.ff, S, [&](int r, float v) {
          const float nx = __fadd_rn(S.xo[r], v);
          S.xo[r] = nx;
          A.x[r0 + r] = nx;
        });
      }
      release_task(S, W, g, ntasks);
      g++;
    }
    // ---- out_norm → lm_out, EOS; cond (→ SiLU) and the flow input h ----
    if (!sync(A, S, W)) goto out;
    layer_norm(A.x, A.d, A.outw, A.outb, 1e-5, nullptr, nullptr, S.vf, nullptr, nullptr, S.red);
    if (c == last) {
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
        if (ok && (tid & 7) == 0) {
          const float hv = __fadd_rn(v, A.finb[r0 + r]);
          S.ho[r] = hv;
          A.h[r0 + r] = hv;
        }
      }
    }
    release_task(S, W, g, ntasks);
    g++;
    // ---- the adaLN projections of SiLU(y) ----
    if (!sync(A, S, W)) goto out;
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
    release_task(S, W, g, ntasks);
    g++;
    // ---- the residual blocks ----
    for (int k = 0; k < A.depth; k++) {
      const F1Res& rb = A.res[k];
      const float* mod = A.mod + (size_t)k * 3 * A.fd;
      if (!sync(A, S, W)) goto out;
      layer_norm(A.h, A.fd, rb.nw, rb.nb, 1e-6, mod, mod + A.fd, S.vf, nullptr, nullptr, S.red);
      if (!wait_task(A, S, g)) goto out;
      {
        const int r0 = split(A.fd, c, G), nrow = split(A.fd, c + 1, G) - r0;
        q8f_slice_rows(S.slot[g % F1_SLOTS], 0, nrow, A.fd, S.vf,
                       [&](int r, float v) { A.mm[r0 + r] = silu_avx(__fadd_rn(v, rb.b1[r0 + r])); });
      }
      release_task(S, W, g, ntasks);
      g++;
      if (!sync(A, S, W)) goto out;
      for (int i = tid; i < A.fd; i += NT) S.vf[i] = __ldcg(A.mm + i);
      __syncthreads();
      if (!wait_task(A, S, g)) goto out;
      {
        const int r0 = split(A.fd, c, G), nrow = split(A.fd, c + 1, G) - r0;
        q8f_slice_rows(S.slot[g % F1_SLOTS], 0, nrow, A.fd, S.vf, [&](int r, float v) {
          const int n = r0 + r;
          const float hv = __fadd_rn(S.ho[r], __fmul_rn(__ldcg(mod + 2 * A.fd + n), __fadd_rn(v, rb.b2[n])));
          S.ho[r] = hv;
          A.h[n] = hv;
        });
      }
      release_task(S, W, g, ntasks);
      g++;
    }
    // ---- the final adaLN, the latent (every CTA), the next input rows ----
    if (!sync(A, S, W)) goto out;
    layer_norm(A.h, A.fd, nullptr, nullptr, 1e-6, A.mod2, A.mod2 + A.fd, S.vf, nullptr, nullptr, S.red);
    {
      const int gi = tid >> 3;
      for (int rr = 0; rr < A.ldim; rr += NT / 8) {
        const int r = rr + gi;
        const bool ok = r < A.ldim;
        const float v = f32_row(A.fout + (size_t)(ok ? r : 0) * A.fd, A.fd, S.vf);
        if (ok && (tid & 7) == 0) {
          const float cur = __fadd_rn(__ldcg(noise + r), __fdiv_rn(__fadd_rn(v, A.foutb[r]), 1.f));
          S.lat[r] = cur;
          if (c == last) {
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
    release_task(S, W, g, ntasks);
    g++;
  }
  if (c == last && tid == 0) {
    A.pos[0] = pos0 + frames;
    A.io->frame = frame0 + frames;
  }
out:
  drain(S, g);
}

}  // namespace

bool frame1_suits(const Frame1Args& A, size_t* smem, uint32_t* slot_bytes, int G) {
  // (scales slices start on 16-byte boundaries: K % 256 == 0)
  if (A.d % 256 || A.heads * 64 != A.d || A.ff % 256 || A.fd % 256 || A.ldim % 16 || A.ldim > 64 || A.L < 1 ||
      A.L > F1_MAX_LAYERS || A.depth < 1 || A.depth > F1_MAX_DEPTH || A.d > 2 * NT || A.ff > 4096 || A.fd > 2 * NT ||
      A.cap < 1 || 8 * A.heads > G)
    return false;
  // a CTA's rows of x and h fit xo / ho, its ff1 rows (whole Q8_0 blocks) the GELU buffer vf2
  const int fmax = A.d > 2 * A.fd ? A.d : 2 * A.fd, nbk = A.ff / QK;
  if (QK * ((nbk + G - 1) / G) > fmax || (A.d + G - 1) / G > kOwnMax || (A.fd + G - 1) / G > kOwnMax) return false;
  uint32_t sb = 0;
  Region r[kMaxRegions];
  for (int c = 0; c < G; c++) {
    int total = 0;
    for (int i = -1; i < frame_tasks(A); i++) {
      const int n = task_regions(A, i, c, G, r);
      total += n;
      for (int k = 0; k < n; k++) sb = sb > r[k].off + r[k].bytes ? sb : up128(r[k].off + r[k].bytes);
    }
    if (total > kTableRegions) return false;
  }
  size_t off[kSmemParts];
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
