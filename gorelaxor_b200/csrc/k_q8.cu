// The int8 path of Q8_0 products (internal/kern/q8int.go:148-223) on the
// GPU: C[m][n] = Σ_b fma(float(s_b)·dw[n][b], da[m][b], ·), blocks b in
// order 0..nb-1, where s_b is the exact int32 dot of block b's 32 int8
// activations and 32 int8 weights. Keeping that order per output makes the
// float32 results identical to the reference's VNNI tile (FIN,
// vnni_amd64.s:58-69), not just close.
//
// Two kernels share the arithmetic:
//  * k_q8_gemv for M ≤ 8 (one stream, or a few): HBM-bound, one warp per
//    weight row, lanes split K into blocks, dp4a block dots, then the
//    block chain in order through warp shuffles.
//  * k_q8_gemm for more rows (batched streams): mma.sync m16n8k32 s8 — one
//    MMA k-step is exactly one Q8_0 block, so each block's int32 tile comes
//    out of the tensor core whole and is folded into float32 accumulators
//    with the per-block scales before the next block.
// Both fuse what follows the product in the transformer (see Epi).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace grx {

namespace {

constexpr uint32_t FULL = 0xffffffffu;

// ------------------------------------------------------------ epilogues --

// RoPE pair rotation, pockettts/nn.go:80-93 (x0 = r·c − i·s, x1 = r·s + i·c,
// unfused), cos/sin from the host table made with the reference's float64
// trigonometry.
__device__ __forceinline__ void rope_pair(float& x0, float& x1, float2 cs) {
  float r = x0, im = x1;
  x0 = __fsub_rn(__fmul_rn(r, cs.x), __fmul_rn(im, cs.y));
  x1 = __fadd_rn(__fmul_rn(r, cs.y), __fmul_rn(im, cs.x));
}

// Stores the qkv product's pair (n, n+1) of row m: q rotated to the query
// buffer, k rotated and v as they are to the cache row at pos[m].
__device__ __forceinline__ void store_qkv_pair(const KVArgs& kv, int m, int n, float c0, float c1) {
  int d = kv.d, hd = d / kv.heads;
  int region = n / d, w = n - region * d, h = w / hd, i = w - h * hd;
  int p = kv.pos[m];
  if (region < 2) {
    float2 cs = reinterpret_cast<const float2*>(kv.rope)[(size_t)p * (hd / 2) + i / 2];
    rope_pair(c0, c1, cs);
  }
  if (region == 0) {
    *reinterpret_cast<float2*>(kv.q + (size_t)m * d + w) = make_float2(c0, c1);
    return;
  }
  size_t base = ((((size_t)m * kv.layers + kv.layer) * 2 + (region - 1)) * kv.heads + h) * (size_t)kv.cap;
  *reinterpret_cast<float2*>(kv.kv + (base + p) * hd + i) = make_float2(c0, c1);
}

// ------------------------------------------------------------- GEMV ------

template <int MAXM>
__global__ void __launch_bounds__(256) k_q8_gemv(const int8_t* __restrict__ a, const float* __restrict__ as, int M,
                                                 const int8_t* __restrict__ wq, const uint16_t* __restrict__ wd,
                                                 int N, int K, EpiArgs e) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = K / QK;
  int8_t* sa = reinterpret_cast<int8_t*>(smem);
  float* ss = reinterpret_cast<float*>(smem + MAXM * K);
  float* sg = ss + MAXM * nb;  // GELU outputs [MAXM][32]
  for (int i = threadIdx.x; i < M * K / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(sa)[i] = reinterpret_cast<const uint4*>(a)[i];
  for (int i = threadIdx.x; i < M * nb; i += blockDim.x) ss[i] = as[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nrow0 = blockIdx.x * 32 + warp * 4;
  float c[4][MAXM];
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int n = nrow0 + r;
    const int8_t* wr = wq + (size_t)n * K;
    const uint16_t* dr = wd + (size_t)n * nb;
    // c starts at the bias, or 0 (q8int.go:175-182).
    const float c0 = e.bias ? e.bias[n] : 0.f;
    float cm[MAXM];
#pragma unroll
    for (int m = 0; m < MAXM; m++) cm[m] = c0;
    for (int it = 0; it * 32 < nb; it++) {
      const int b = it * 32 + lane;
      float t[MAXM];
#pragma unroll
      for (int m = 0; m < MAXM; m++) t[m] = 0.f;
      if (b < nb) {
        const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(wr + b * QK));
        const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(wr + b * QK + 16));
        const float dw = h2f(__ldg(dr + b));
#pragma unroll
        for (int m = 0; m < MAXM; m++) {
          if (m < M) {
            const uint4* ap = reinterpret_cast<const uint4*>(sa + m * K + b * QK);
            const uint4 a0 = ap[0], a1 = ap[1];
            int s = __dp4a(int(w0.x), int(a0.x), 0);
            s = __dp4a(int(w0.y), int(a0.y), s);
            s = __dp4a(int(w0.z), int(a0.z), s);
            s = __dp4a(int(w0.w), int(a0.w), s);
            s = __dp4a(int(w1.x), int(a1.x), s);
            s = __dp4a(int(w1.y), int(a1.y), s);
            s = __dp4a(int(w1.z), int(a1.z), s);
            s = __dp4a(int(w1.w), int(a1.w), s);
            t[m] = __fmul_rn(i2f_small(s), dw);
          }
        }
      }
      const int lim = min(32, nb - it * 32);
      for (int l = 0; l < lim; l++) {
#pragma unroll
        for (int m = 0; m < MAXM; m++) {
          const float tv = __shfl_sync(FULL, t[m], l);
          if (m < M) cm[m] = __fmaf_rn(tv, ss[m * nb + it * 32 + l], cm[m]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MAXM; m++) c[r][m] = cm[m];
  }
  // Every lane holds every result; lane m writes row m.
  if (e.epi == EPI_ROPE_KV) {
#pragma unroll
    for (int m = 0; m < MAXM; m++)
      if (m < M && lane == m) {
        store_qkv_pair(e.kv, m, nrow0, c[0][m], c[1][m]);
        store_qkv_pair(e.kv, m, nrow0 + 2, c[2][m], c[3][m]);
      }
    return;
  }
  if (e.epi == EPI_GELU_Q8) {
#pragma unroll
    for (int m = 0; m < MAXM; m++)
      if (m < M && lane == m)
#pragma unroll
        for (int r = 0; r < 4; r++) sg[m * 32 + warp * 4 + r] = gelu_avx(c[r][m]);
    __syncthreads();
    if (warp < M) {
      float sc;
      const int8_t q = quant_lane(sg[warp * 32 + lane], &sc);
      e.q8[(size_t)warp * N + blockIdx.x * 32 + lane] = q;
      if (lane == 0) e.q8s[(size_t)warp * (N / QK) + blockIdx.x] = sc;
    }
    return;
  }
#pragma unroll
  for (int m = 0; m < MAXM; m++)
    if (m < M && lane == m)
#pragma unroll
      for (int r = 0; r < 4; r++) {
        float* yp = e.y + (size_t)m * e.ldy + nrow0 + r;
        const float v = c[r][m];
        if (e.epi == EPI_RESID)
          *yp = __fadd_rn(*yp, v);
        else
          *yp = v;
      }
}

// ------------------------------------------------------------- GEMM ------

constexpr int BM = 64, BN = 64, BKB = 128, STAGES = 4;  // BKB: bytes of K per stage = 4 blocks

struct __align__(16) Stage {
  int8_t A[BM * BKB];
  int8_t W[BN * BKB];
  float sa[BM * 4];
  uint16_t sw[BN * 4];
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 8 : 0));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void load_stage(Stage& st, int kt, const int8_t* a, const float* as, int M,
                                           const int8_t* wq, const uint16_t* wd, int N, int K, int m0, int n0) {
  const int tid = threadIdx.x, nb = K / QK, kb0 = kt * 4;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int idx = tid + i * 128, r = idx >> 3, c = idx & 7;
    const int gk = kb0 * QK + c * 16;
    const int swz = ((c ^ (r & 7)) << 4);
    const int gm = m0 + r, gn = n0 + r;
    const bool va = gm < M && gk < K, vw = gn < N && gk < K;
    cp_async16(&st.A[r * BKB + swz], va ? a + (size_t)gm * K + gk : a, va);
    cp_async16(&st.W[r * BKB + swz], vw ? wq + (size_t)gn * K + gk : wq, vw);
  }
  if (tid < 64) {
    const int gm = m0 + tid;
    const bool v = gm < M;
    cp_async16(&st.sa[tid * 4], v ? as + (size_t)gm * nb + kb0 : as, v);
  } else {
    const int r = tid - 64, gn = n0 + r;
    const bool v = gn < N;
    cp_async8(&st.sw[r * 4], v ? wd + (size_t)gn * nb + kb0 : wd, v);
  }
}

__global__ void __launch_bounds__(128) k_q8_gemm(const int8_t* __restrict__ a, const float* __restrict__ as, int M,
                                                 const int8_t* __restrict__ wq, const uint16_t* __restrict__ wd,
                                                 int N, int K, EpiArgs e) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Stage* st = reinterpret_cast<Stage*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int wm = warp >> 1, wn = warp & 1;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nb = K / QK, nkt = (nb + 3) / 4;

  // Each output's chain starts at its bias, or 0 (q8int.go:175-182).
  float acc[2][4][4];
#pragma unroll
  for (int j = 0; j < 4; j++)
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int col = n0 + wn * 32 + j * 8 + 2 * t4 + (q & 1);
      const float b0 = (e.bias && col < N) ? e.bias[col] : 0.f;
#pragma unroll
      for (int i = 0; i < 2; i++) acc[i][j][q] = b0;
    }

#pragma unroll
  for (int s = 0; s < STAGES - 1; s++) {
    if (s < nkt) load_stage(st[s], s, a, as, M, wq, wd, N, K, m0, n0);
    cp_commit();
  }
  for (int kt = 0; kt < nkt; kt++) {
    cp_wait<STAGES - 2>();
    __syncthreads();
    {
      const int nk = kt + STAGES - 1;
      if (nk < nkt) load_stage(st[nk % STAGES], nk, a, as, M, wq, wd, N, K, m0, n0);
      cp_commit();
    }
    const Stage& S = st[kt % STAGES];
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      if (kt * 4 + kk >= nb) break;
      uint32_t af[2][4], bf[4][2];
#pragma unroll
      for (int i = 0; i < 2; i++) {
        const int mat = lane >> 3, row = wm * 32 + i * 16 + (lane & 7) + (mat & 1) * 8;
        const int chunk = 2 * kk + (mat >> 1);
        ldsm_x4(af[i][0], af[i][1], af[i][2], af[i][3], &S.A[row * BKB + ((chunk ^ (row & 7)) << 4)]);
      }
#pragma unroll
      for (int p = 0; p < 2; p++) {
        const int mat = lane >> 3, row = wn * 32 + p * 16 + (lane & 7) + (mat >> 1) * 8;
        const int chunk = 2 * kk + (mat & 1);
        ldsm_x4(bf[2 * p][0], bf[2 * p][1], bf[2 * p + 1][0], bf[2 * p + 1][1],
                &S.W[row * BKB + ((chunk ^ (row & 7)) << 4)]);
      }
      float da[2][2], dw[4][2];
#pragma unroll
      for (int i = 0; i < 2; i++)
#pragma unroll
        for (int h = 0; h < 2; h++) da[i][h] = S.sa[(wm * 32 + i * 16 + g + h * 8) * 4 + kk];
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int h = 0; h < 2; h++) dw[j][h] = h2f(S.sw[(wn * 32 + j * 8 + 2 * t4 + h) * 4 + kk]);
#pragma unroll
      for (int i = 0; i < 2; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
          int c[4];
          mma_s8(c, af[i], bf[j][0], bf[j][1]);
#pragma unroll
          for (int q = 0; q < 4; q++)
            acc[i][j][q] = __fmaf_rn(__fmul_rn(i2f_small(c[q]), dw[j][q & 1]), da[i][q >> 1], acc[i][j][q]);
        }
    }
  }
  cp_wait<0>();

  // Epilogue: thread holds rows (g, g+8) of each m16 tile, column pairs.
#pragma unroll
  for (int i = 0; i < 2; i++)
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int row = m0 + wm * 32 + i * 16 + g + h * 8;
      const bool rv = row < M;
      if (e.epi == EPI_GELU_Q8) {
        float v[8], amax = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
          for (int q = 0; q < 2; q++) {
            v[j * 2 + q] = gelu_avx(acc[i][j][h * 2 + q]);
            amax = fmaxf(amax, fabsf(v[j * 2 + q]));
          }
        amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, 2));
        if (rv) {
          const int colb = n0 + wn * 32;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const uint16_t pk = uint16_t(uint8_t(quant_val(v[j * 2], amax))) |
                                uint16_t(uint16_t(uint8_t(quant_val(v[j * 2 + 1], amax))) << 8);
            *reinterpret_cast<uint16_t*>(e.q8 + (size_t)row * N + colb + j * 8 + 2 * t4) = pk;
          }
          if (t4 == 0) e.q8s[(size_t)row * (N / QK) + colb / QK] = quant_scale(amax);
        }
        continue;
      }
      if (!rv) continue;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int col = n0 + wn * 32 + j * 8 + 2 * t4;
        if (col >= N) continue;
        const float c0 = acc[i][j][h * 2], c1 = acc[i][j][h * 2 + 1];
        if (e.epi == EPI_ROPE_KV) {
          store_qkv_pair(e.kv, row, col, c0, c1);
          continue;
        }
        float2* yp = reinterpret_cast<float2*>(e.y + (size_t)row * e.ldy + col);
        if (e.epi == EPI_RESID) {
          float2 o = *yp;
          *yp = make_float2(__fadd_rn(o.x, c0), __fadd_rn(o.y, c1));
        } else {
          *yp = make_float2(c0, c1);
        }
      }
    }
}

}  // namespace

void launch_q8_product(const int8_t* a, const float* as, int M, const DQ8& w, const EpiArgs& e, cudaStream_t st) {
  const int N = w.rows, K = w.cols;
  if (M <= 8) {
    const int nb = K / QK;
    const size_t sm = size_t(8) * K + size_t(8) * nb * 4 + 8 * 32 * 4;
    dim3 grid(N / 32);
    if (M == 1)
      k_q8_gemv<1><<<grid, 256, sm, st>>>(a, as, M, w.q, w.d, N, K, e);
    else if (M == 2)
      k_q8_gemv<2><<<grid, 256, sm, st>>>(a, as, M, w.q, w.d, N, K, e);
    else if (M <= 4)
      k_q8_gemv<4><<<grid, 256, sm, st>>>(a, as, M, w.q, w.d, N, K, e);
    else
      k_q8_gemv<8><<<grid, 256, sm, st>>>(a, as, M, w.q, w.d, N, K, e);
    return;
  }
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  k_q8_gemm<<<grid, 128, sizeof(Stage) * STAGES, st>>>(a, as, M, w.q, w.d, N, K, e);
}

// Raises the kernels' dynamic shared memory limits once per device.
void q8_kernels_init() {
  cudaFuncSetAttribute(k_q8_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(Stage) * STAGES));
  const int gv = 8 * 4096 + 8 * 128 * 4 + 8 * 32 * 4;
  cudaFuncSetAttribute(k_q8_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
}

}  // namespace grx
