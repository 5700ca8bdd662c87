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
//  * k_q8_gemm2 for more rows (batched streams): mma.sync m16n8k32 s8 — one
//    MMA k-step is exactly one Q8_0 block, so each block's int32 tile comes
//    out of the tensor core whole and is folded into float32 accumulators
//    with the per-block scales before the next block.
// Both fuse what follows the product in the transformer (see Epi).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <type_traits>
#include <unordered_map>

#include <cstddef>
#include <cstdlib>
#include <cstdint>

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
// buffer, k rotated and v as they are to the cache row at pos[m] of the
// row's stream.
__device__ __forceinline__ void store_qkv_pair(const KVArgs& kv, int m, int n, float c0, float c1) {
  int d = kv.d, hd = d / kv.heads;
  int region = n / d, w = n - region * d, h = w / hd, i = w - h * hd;
  int p = kv.pos[m];
  const int slot = kv.row_stream ? kv.row_stream[m] : m;
  const int pc = kv.ring ? p % kv.ring : p;  // the cache row
  if (region < 2) {
    float2 cs = reinterpret_cast<const float2*>(kv.rope)[(size_t)p * (hd / 2) + i / 2];
    rope_pair(c0, c1, cs);
  }
  if (region == 0) {
    *reinterpret_cast<float2*>(kv.q + (size_t)m * d + w) = make_float2(c0, c1);
    return;
  }
  size_t base = ((((size_t)slot * kv.layers + kv.layer) * 2 + (region - 1)) * kv.heads + h) * (size_t)kv.cap;
  *reinterpret_cast<float2*>(kv.kv + (base + pc) * hd + i) = make_float2(c0, c1);
}

// ------------------------------------------------------------- GEMV ------

template <int MAXM>
__global__ void __launch_bounds__(256) k_q8_gemv(const int8_t* __restrict__ a, const float2* __restrict__ as, int M,
                                                 const int8_t* __restrict__ wq, const uint16_t* __restrict__ wd,
                                                 int N, int K, EpiArgs e) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = K / QK;
  int8_t* sa = reinterpret_cast<int8_t*>(smem);
  float* ss = reinterpret_cast<float*>(smem + MAXM * K);
  float* sg = ss + MAXM * nb;  // GELU outputs [MAXM][32]
  for (int i = threadIdx.x; i < M * K / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(sa)[i] = reinterpret_cast<const uint4*>(a)[i];
  for (int i = threadIdx.x; i < M * nb; i += blockDim.x) ss[i] = as[i].x;
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
      if (lane == 0) e.q8s[(size_t)warp * (N / QK) + blockIdx.x] = make_float2(sc, sc);
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
          *yp = __fadd_rn(*yp, e.ls ? __fmul_rn(e.ls[nrow0 + r], v) : v);
        else
          *yp = v;
      }
}

// ------------------------------------------------------------- GEMM ------
//
// The chain over K blocks cannot be split, so the parallelism of a product
// is its M×N outputs (at M = 256 streams and N = 1024 only 256K). A warp
// owns TM×TN m16n8 tiles (TM·TN MMAs per block, the A fragment shared by the
// TN column tiles), WGM×WGN warps a CTA tile. The tile shape is chosen per
// product shape (launch_q8_product).

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_n(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(bytes));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t a) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ f2 lds64(uint32_t a) {
  f2 v;
  asm volatile("ld.shared.b64 %0, [%1];\n" : "=l"(v) : "r"(a));
  return v;
}

// The same block split in two, so the MMAs of a whole stage can be issued
// before the first of their results is folded into the chains: the MMA
// (into the magic-initialized pairs) ...
__device__ __forceinline__ void q8_mma(f2& p01, f2& p23, const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("{\n"
      " .reg .b32 d0, d1, d2, d3;\n"
      " mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {d0,d1,d2,d3}, {%2,%3,%4,%5}, {%6,%7}, {%8,%8,%8,%8};\n"
      " mov.b64 %0, {d0, d1};\n"
      " mov.b64 %1, {d2, d3};\n"
      "}\n"
      : "=l"(p01), "=l"(p23)
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(MAGIC_BITS));
}
// ... and the two roundings of the reference's FIN (see q8_block).
__device__ __forceinline__ void q8_fold(f2& acc01, f2& acc23, f2 p01, f2 p23, f2 dw, f2 nm, f2 da0, f2 da1) {
  acc01 = f2fma(f2fma(p01, dw, nm), da0, acc01);
  acc23 = f2fma(f2fma(p23, dw, nm), da1, acc23);
}

// One finished output pair (row, col..col+1), every epilogue but the Q8_0
// rounding: the RoPE'd K/V append, the residual add (with the layer scale),
// or a plain store.
__device__ __forceinline__ void epi_pair(const EpiArgs& e, int row, int col, float c0v, float c1v) {
  if (e.epi == EPI_ROPE_KV) {
    store_qkv_pair(e.kv, row, col, c0v, c1v);
    return;
  }
  float2* yp = reinterpret_cast<float2*>(e.y + (size_t)row * e.ldy + col);
  if (e.epi == EPI_RESID) {
    const float2 o = *yp;
    const float a0 = e.ls ? __fmul_rn(e.ls[col], c0v) : c0v, a1 = e.ls ? __fmul_rn(e.ls[col + 1], c1v) : c1v;
    *yp = make_float2(__fadd_rn(o.x, a0), __fadd_rn(o.y, a1));
  } else {
    *yp = make_float2(c0v, c1v);
  }
}

// The epilogue of both GEMM kernels: each thread's accumulators (rows g and
// g+8 of its m-tiles, column pairs of its n-tiles) go where e says.
template <int TM, int TN, int NWARPS>
__device__ __forceinline__ void gemm_epilogue(f2 (&acc)[TM][TN][2], const EpiArgs& e, uint8_t* smem_raw, int m0,
                                              int n0, int arow, int brow, int g, int t4, int warp, int lane, int M,
                                              int N, int BM, int BN) {
  if (e.epi == EPI_GELU_Q8) {
    // A row's 32-column blocks span several warps: gather the tile in shared
    // memory, then one warp per (row, block) rounds its block to Q8_0.
    __syncthreads();
    float* tile = reinterpret_cast<float*>(smem_raw);  // [BM][BN + 1]
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
      for (int j = 0; j < TN; j++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int r = arow + i * 16 + g + h * 8, c = brow + j * 8 + 2 * t4;
          tile[r * (BN + 1) + c] = gelu_avx(f2lo(acc[i][j][h]));
          tile[r * (BN + 1) + c + 1] = gelu_avx(f2hi(acc[i][j][h]));
        }
    __syncthreads();
    for (int rb = warp; rb < BM * (BN / 32); rb += NWARPS) {
      const int r = rb / (BN / 32), cb = rb % (BN / 32), row = m0 + r;
      float sc;
      const int8_t qv = quant_lane(tile[r * (BN + 1) + cb * 32 + lane], &sc);
      if (row < M) {
        e.q8[(size_t)row * N + n0 + cb * 32 + lane] = qv;
        if (lane == 0) e.q8s[(size_t)row * (N / QK) + (n0 + cb * 32) / QK] = make_float2(sc, sc);
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++)
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int row = m0 + arow + i * 16 + g + h * 8, col = n0 + brow + j * 8 + 2 * t4;
        if (row < M && col < N) epi_pair(e, row, col, f2lo(acc[i][j][h]), f2hi(acc[i][j][h]));
      }
}

// ------------------------------------------------ GEMM, lean inner loop --
//
// k_q8_gemm2: a stage is four Q8_0 blocks (128 bytes of K). Every thread's async-copy
// sources and destinations are computed once and only advance per stage;
// the weight scales come as {dw[n], dw[n+1], nm[n], nm[n+1]} quads (one
// 16-byte read per column pair, DQ8::dwnm); B fragments come two column
// tiles per ldmatrix.x4. Per block a warp issues its TM·TN MMAs, then folds
// them (four packed FMAs each).
template <int TM, int TN, int WGM, int WGN>
struct Cfg2 {
  static constexpr int BM = 16 * TM * WGM, BN = 8 * TN * WGN, NT = 32 * WGM * WGN, KB = 4;
  static constexpr int OFF_A = 0, OFF_W = BM * 128, OFF_SA = OFF_W + BN * 128, OFF_DN = OFF_SA + BM * KB * 8,
                       SST = (OFF_DN + KB * BN * 8 + 1023) / 1024 * 1024;
  static constexpr int CA = BM * 8, CW = BN * 8, CS = BM * 2, CD = KB * BN / 2;  // 16-byte chunks per stage
  static constexpr int PA = (CA + NT - 1) / NT, PW = (CW + NT - 1) / NT, PS = (CS + NT - 1) / NT,
                       PD = (CD + NT - 1) / NT;
};

template <int TM, int TN, int WGM, int WGN, int STAGES, int PB = 1>
__global__ void __launch_bounds__(32 * WGM * WGN) k_q8_gemm2(const int8_t* __restrict__ a,
                                                            const float2* __restrict__ as, int M,
                                                            const int8_t* __restrict__ wq,
                                                            const float4* __restrict__ dwnm, int N, int K, EpiArgs e) {
  using C = Cfg2<TM, TN, WGM, WGN>;
  constexpr int BM = C::BM, BN = C::BN, NT = C::NT;
  static_assert(TN % 2 == 0, "B fragments two column tiles at a time");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int wm = warp / WGN, wn = warp % WGN;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nb = K / QK, nkt = (nb + 3) / 4, np2 = (N + 1) / 2;  // a last stage may hold fewer blocks
  const int arow = wm * 16 * TM, brow = wn * 8 * TN;
  const uint32_t sbase = smem_u32(smem_raw);

  // ---- this thread's copies of a stage: sources (advance per stage) and
  // destinations within a stage
  const int8_t* srcA[C::PA];
  uint32_t dstA[C::PA];
  bool okA[C::PA];
  int blA[C::PA], blW[C::PW], blS[C::PS], blD[C::PD];  // the first block of the chunk within a stage
#pragma unroll
  for (int u = 0; u < C::PA; u++) {
    const int i = tid + u * NT, r = i >> 3, c = i & 7;
    blA[u] = c >> 1;
    okA[u] = i < C::CA && m0 + r < M;
    srcA[u] = a + (size_t)(okA[u] ? m0 + r : 0) * K + c * 16;
    dstA[u] = C::OFF_A + r * 128 + ((c ^ (r & 7)) << 4);
  }
  const int8_t* srcW[C::PW];
  uint32_t dstW[C::PW];
  bool okW[C::PW];
#pragma unroll
  for (int u = 0; u < C::PW; u++) {
    const int i = tid + u * NT, r = i >> 3, c = i & 7;
    blW[u] = c >> 1;
    okW[u] = i < C::CW && n0 + r < N;
    srcW[u] = wq + (size_t)(okW[u] ? n0 + r : 0) * K + c * 16;
    dstW[u] = C::OFF_W + r * 128 + ((c ^ (r & 7)) << 4);
  }
  const float2* srcS[C::PS];
  uint32_t dstS[C::PS];
  bool okS[C::PS];
#pragma unroll
  for (int u = 0; u < C::PS; u++) {
    const int i = tid + u * NT, r = i >> 1, h = i & 1;
    blS[u] = 2 * h;
    okS[u] = i < C::CS && m0 + r < M;
    srcS[u] = as + (size_t)(okS[u] ? m0 + r : 0) * nb + 2 * h;
    dstS[u] = C::OFF_SA + r * 32 + h * 16;
  }
  const float4* srcD[C::PD];
  uint32_t dstD[C::PD];
  bool okD[C::PD];
#pragma unroll
  for (int u = 0; u < C::PD; u++) {
    const int i = tid + u * NT, kb = i / (BN / 2), p = i % (BN / 2);
    blD[u] = kb;
    okD[u] = i < C::CD && n0 + 2 * p < N;
    srcD[u] = dwnm + (size_t)kb * np2 + (okD[u] ? n0 / 2 + p : 0);
    dstD[u] = C::OFF_DN + (kb * (BN / 2) + p) * 16;
  }
  // Chunks past the last block are zero-filled without a read (an odd
  // block count ends with a half scale chunk).
  auto load = [&](int kt, uint32_t st) {
    const int left = nb - kt * 4;
#pragma unroll
    for (int u = 0; u < C::PA; u++)
      if (tid + u * NT < C::CA) cp_async16(st + dstA[u], srcA[u] + kt * 128, okA[u] && blA[u] < left);
#pragma unroll
    for (int u = 0; u < C::PW; u++)
      if (tid + u * NT < C::CW) cp_async16(st + dstW[u], srcW[u] + kt * 128, okW[u] && blW[u] < left);
#pragma unroll
    for (int u = 0; u < C::PS; u++)
      if (tid + u * NT < C::CS)
        cp_async_n(st + dstS[u], srcS[u] + kt * 4, okS[u] ? (blS[u] + 1 < left ? 16 : blS[u] < left ? 8 : 0) : 0);
#pragma unroll
    for (int u = 0; u < C::PD; u++)
      if (tid + u * NT < C::CD) cp_async16(st + dstD[u], srcD[u] + (size_t)kt * 4 * np2, okD[u] && blD[u] < left);
  };

  // ---- fragment offsets within a stage
  const int mat = lane >> 3;
  uint32_t aoff[TM], boff[TN / 2];
#pragma unroll
  for (int i = 0; i < TM; i++) {
    const int ra = arow + i * 16 + (lane & 7) + (mat & 1) * 8;
    aoff[i] = C::OFF_A + ra * 128 + (((mat >> 1) ^ (ra & 7)) << 4);
  }
#pragma unroll
  for (int j = 0; j < TN / 2; j++) {
    const int rb = brow + j * 16 + (lane & 7) + (mat >> 1) * 8;
    boff[j] = C::OFF_W + rb * 128 + (((mat & 1) ^ (rb & 7)) << 4);
  }
  uint32_t soff[TM], doff[TN];
#pragma unroll
  for (int i = 0; i < TM; i++) soff[i] = C::OFF_SA + (arow + i * 16 + g) * 32;
#pragma unroll
  for (int j = 0; j < TN; j++) doff[j] = C::OFF_DN + ((brow + j * 8) / 2 + t4) * 16;

  // Each output's chain starts at its bias, or 0 (q8int.go:175-182).
  f2 acc[TM][TN][2];
#pragma unroll
  for (int j = 0; j < TN; j++) {
    const int c0 = n0 + brow + j * 8 + 2 * t4;
    const f2 b = f2make(e.bias && c0 < N ? e.bias[c0] : 0.f, e.bias && c0 + 1 < N ? e.bias[c0 + 1] : 0.f);
#pragma unroll
    for (int i = 0; i < TM; i++) acc[i][j][0] = acc[i][j][1] = b;
  }

#pragma unroll
  for (int s = 0; s < STAGES - 1; s++) {
    if (s < nkt) load(s, sbase + s * C::SST);
    cp_commit();
  }
  int rs = 0, ws = STAGES - 1;
  for (int kt = 0; kt < nkt; kt++) {
    cp_wait<STAGES - 2>();
    __syncthreads();
    if (kt + STAGES - 1 < nkt) load(kt + STAGES - 1, sbase + ws * C::SST);
    cp_commit();
    ws = ws + 1 == STAGES ? 0 : ws + 1;
    const uint32_t cur = sbase + rs * C::SST;
    rs = rs + 1 == STAGES ? 0 : rs + 1;
    // PB blocks at a time: their MMAs are all issued before the first of
    // their results is folded, so the MMA latencies overlap; the folds then
    // run in block order, which is all the chain needs.
#pragma unroll
    for (int k0 = 0; k0 < 4; k0 += PB) {
      if (kt * 4 + k0 >= nb) break;
      f2 p[PB][TM][TN][2];
#pragma unroll
      for (int kb = 0; kb < PB; kb++) {
        const int kk = k0 + kb;
        if (kt * 4 + kk >= nb) break;
        const uint32_t kl = uint32_t(2 * kk) << 4;  // the block's first chunk (the swizzle keeps bit 0)
        uint32_t af[TM][4], bf[TN][2];
#pragma unroll
        for (int i = 0; i < TM; i++) ldsm_x4(af[i][0], af[i][1], af[i][2], af[i][3], (cur + aoff[i]) ^ kl);
#pragma unroll
        for (int j = 0; j < TN / 2; j++)
          ldsm_x4(bf[2 * j][0], bf[2 * j][1], bf[2 * j + 1][0], bf[2 * j + 1][1], (cur + boff[j]) ^ kl);
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
          for (int j = 0; j < TN; j++) q8_mma(p[kb][i][j][0], p[kb][i][j][1], af[i], bf[j][0], bf[j][1]);
      }
#pragma unroll
      for (int kb = 0; kb < PB; kb++) {
        const int kk = k0 + kb;
        if (kt * 4 + kk >= nb) break;
#pragma unroll
        for (int j = 0; j < TN; j++) {
          f2 dw, nm;
          asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];\n" : "=l"(dw), "=l"(nm) : "r"(cur + doff[j] + kk * (BN / 2) * 16));
#pragma unroll
          for (int i = 0; i < TM; i++) {
            const uint32_t sa = cur + soff[i] + kk * 8;
            q8_fold(acc[i][j][0], acc[i][j][1], p[kb][i][j][0], p[kb][i][j][1], dw, nm, lds64(sa), lds64(sa + 8 * 32));
          }
        }
      }
    }
  }
  cp_wait<0>();
  gemm_epilogue<TM, TN, WGM * WGN>(acc, e, smem_raw, m0, n0, arow, brow, g, t4, warp, lane, M, N, BM, BN);
}

template <int TM, int TN, int WGM, int WGN, int STAGES, int PB = 1>
struct Gemm2 {
  using C = Cfg2<TM, TN, WGM, WGN>;
  static constexpr size_t smem() {
    const size_t s = size_t(C::SST) * STAGES, t = size_t(C::BM) * (C::BN + 1) * 4;
    return s > t ? s : t;
  }
  static void init() {
    cudaFuncSetAttribute(k_q8_gemm2<TM, TN, WGM, WGN, STAGES, PB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(smem()));
  }
  static void launch(const int8_t* a, const float2* as, int M, const DQ8& w, const EpiArgs& e, cudaStream_t st) {
    dim3 grid((w.rows + C::BN - 1) / C::BN, (M + C::BM - 1) / C::BM);
    k_q8_gemm2<TM, TN, WGM, WGN, STAGES, PB><<<grid, C::NT, smem(), st>>>(a, as, M, w.q, w.dwnm, w.rows, w.cols, e);
  }
};

// ------------------------------------------ GEMM on the 5th-gen tensor core --
//
// k_q8_tc: the same per-block chain with the int8 block products from
// tcgen05.mma (kind::i8, M = 128 activation rows, N = BN weight rows, K = 32 =
// one Q8_0 block per instruction) into Tensor Memory. A stage is four blocks
// of K (one 128-byte swizzle row of both operands). Warp roles:
//  * warp 0, one thread: the TMA loads of a stage (activation and weight
//    tiles in the 128-byte swizzled K-major layout the MMA reads, the
//    activation scales and the {dw, dw', nm, nm'} quads);
//  * warp 1: allocates TMEM; one thread issues a stage's four MMAs into one
//    of two groups of four int32 tiles and commits the group once;
//  * the epilogue warps: thread r of lane quarter q owns activation row
//    32q + r and a slice of CW columns. Per block it loads its row of the
//    int32 tile (tcgen05.ld), adds the magic bits (1.5·2^23 + s as float, as
//    the mma.sync path gets from its accumulator initialisation) and folds
//    it into the chain with two packed FMAs per column pair; per stage it
//    frees the group and the stage's shared memory.
// Synchronisation is per stage, not per block: the barrier operations of the
// single issuing thread cost more than an MMA. Every wait is bounded (about a
// second of clocks); one that runs out sets the kernel's fault word, every
// role then leaves its loop, and the block still reaches the TMEM release.
constexpr int TC_BM = 128, TC_KB = 4, TC_STAGES = 4, TC_GROUPS = 2;

template <int BN, int EPW>
struct TcCfg {
  static constexpr int NT = 64 + 32 * EPW;  // producer warp, MMA warp, epilogue warps
  static constexpr int CW = BN / (EPW / 4);  // columns per epilogue thread
  static_assert(EPW % 4 == 0 && CW % 16 == 0, "epilogue warps cover the lane quarters evenly");
  static constexpr int TMEM_COLS = TC_GROUPS * TC_KB * BN;  // power of two for BN = 16, 32, 64
  static constexpr int A_BYTES = TC_BM * 128, B_BYTES = BN * 128, S_BYTES = TC_BM * TC_KB * 8,
                       D_BYTES = TC_KB * BN * 8;
  static constexpr int OFF_B = A_BYTES, OFF_S = OFF_B + B_BYTES, OFF_D = OFF_S + S_BYTES;
  static constexpr int STAGE = (OFF_D + D_BYTES + 1023) / 1024 * 1024;
  static constexpr int TX = A_BYTES + B_BYTES + S_BYTES + D_BYTES;
  static constexpr int OFF_BAR = STAGE * TC_STAGES;
  static constexpr int NBAR = 2 * TC_STAGES + 2 * TC_GROUPS + 1;
  static constexpr int SMEM = 1024 + OFF_BAR + NBAR * 8 + 16;  // + alignment slack
  // Shared memory bounds how many blocks share an SM (228 KB), so their TMEM
  // allocations together never exceed the 512 columns and never wait.
  static_assert((228 * 1024 / SMEM) * TMEM_COLS <= 512, "co-resident blocks must fit in TMEM");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "allocation size");
};

__device__ int g_q8_tc_fault = 0;

__device__ __forceinline__ bool mb_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false once about 2^31 clocks passed or another role gave up.
__device__ __forceinline__ bool mb_wait(uint32_t bar, uint32_t parity, volatile int* dead) {
  if (mb_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mb_try(bar, parity)) {
    if (*dead || clock64() - t0 > (1LL << 31)) {
      if (!*dead) {
        *dead = 1;
        atomicExch(&g_q8_tc_fault, 1);
      }
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void mb_init(uint32_t bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
// The single-thread instructions below are executed by a whole warp in
// step and issued by the one lane elect.sync picks, so the warp's control
// flow and operands stay uniform.
__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n"
      "@p cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n}\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mb_expect_one(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n@p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n}\n" ::"r"(bar),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n"
      "@p tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(bar)
      : "memory");
}
// K-major operand in the 128-byte swizzle: rows of 128 bytes, groups of 8
// rows 1024 bytes apart; the start moves 32 bytes per block within a row.
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}
// D += A·Bᵀ (the tile holds the magic bits, so D ends as 1.5·2^23 + s).
__device__ __forceinline__ void tc_mma_i8(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, 1, 0;\n elect.sync _|e, 0xffffffff;\n"
      "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(ad), "l"(bd), "r"(idesc)
      : "memory");
}
// 16 consecutive int32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t* d) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]), "=r"(d[8]),
        "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
      : "r"(taddr)
      : "memory");
}
// 16 consecutive columns of this thread's TMEM lane set to v.
__device__ __forceinline__ void tc_st16(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};\n" ::"r"(taddr),
      "r"(v)
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

template <int BN, int EPW>
__global__ void __launch_bounds__(TcCfg<BN, EPW>::NT, 1)
    k_q8_tc(const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mw,
            const __grid_constant__ CUtensorMap ms, const __grid_constant__ CUtensorMap md, int M, int N, int nb,
            EpiArgs e) {
  using C = TcCfg<BN, EPW>;
  constexpr int S = TC_STAGES, G = TC_GROUPS, CW = C::CW;
  extern __shared__ uint8_t tc_raw[];
  const uint32_t raw = smem_u32(tc_raw), base = (raw + 1023) & ~1023u;
  uint8_t* gbase = tc_raw + (base - raw);
  const uint32_t bars = base + C::OFF_BAR;
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (S + s); };
  auto tfull = [&](int g) { return bars + 8 * (2 * S + g); };
  auto tempty = [&](int g) { return bars + 8 * (2 * S + G + g); };
  const uint32_t done = bars + 8 * (2 * S + 2 * G);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + C::OFF_BAR + C::NBAR * 8);
  __shared__ int dead_s;
  volatile int* dead = &dead_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * TC_BM;
  if (threadIdx.x == 0) {
    dead_s = 0;
    for (int s = 0; s < S; s++) {
      mb_init(full(s), 1);
      mb_init(empty(s), EPW);
    }
    for (int g = 0; g < G; g++) {
      mb_init(tfull(g), 1);
      mb_init(tempty(g), EPW);
    }
    mb_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile(
        "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
        "tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::"r"(smem_u32(tmem_slot)),
        "r"(C::TMEM_COLS)
        : "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nst = (nb + TC_KB - 1) / TC_KB;
  if (warp >= 2) {  // every tile starts as the magic bits; the epilogue restores them after each read
    const uint32_t t0 = tmem + (uint32_t((warp & 3) * 32) << 16) + uint32_t(((warp - 2) >> 2) * CW);
    for (int b = 0; b < TC_GROUPS * TC_KB; b++)
#pragma unroll
      for (int c = 0; c < CW / 16; c++) tc_st16(t0 + uint32_t(b * BN + 16 * c), uint32_t(MAGIC_BITS));
    tc_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    {
      int issued = 0;
      for (int st = 0; st < nst; st++) {
        const int s = st % S;
        if (!__all_sync(FULL, mb_wait(empty(s), ((st / S) & 1) ^ 1, dead))) break;
        const uint32_t sb = base + s * C::STAGE;
        mb_expect_one(full(s), C::TX);
        tma2d(sb, &ma, st * 128, m0, full(s));
        tma2d(sb + C::OFF_B, &mw, st * 128, n0, full(s));
        tma2d(sb + C::OFF_S, &ms, st * 8, m0, full(s));
        tma2d(sb + C::OFF_D, &md, n0 * 2, st * TC_KB, full(s));
        issued = st + 1;
      }
      // After a failure, let this block's copies land before it exits.
      if (*dead)
        for (int st = issued > S ? issued - S : 0; st < issued; st++) {
          const long long t0 = clock64();
          while (!mb_try(full(st % S), (st / S) & 1) && clock64() - t0 < (1LL << 30)) {
          }
        }
    }
  } else if (warp == 1) {
    {
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(TC_BM >> 4) << 24);
      for (int st = 0; st < nst; st++) {
        const int s = st % S, g = st % G, nbl = min(TC_KB, nb - st * TC_KB);
        if (!__all_sync(FULL, mb_wait(full(s), (st / S) & 1, dead))) break;
        if (!__all_sync(FULL, mb_wait(tempty(g), ((st / G) & 1) ^ 1, dead))) break;
        tc_fence_after();
        const uint32_t sb = base + s * C::STAGE;
        for (int kk = 0; kk < nbl; kk++)
          tc_mma_i8(tmem + uint32_t((g * TC_KB + kk) * BN), tc_desc(sb + kk * 32), tc_desc(sb + C::OFF_B + kk * 32),
                    idesc);
        tc_commit(tfull(g));
      }
      // Every MMA issued has completed before the TMEM is released.
      tc_commit(done);
      const long long t0 = clock64();
      while (!mb_try(done, 0) && clock64() - t0 < (1LL << 31)) {
      }
    }
  } else {
    // lane quarter q (TMEM lanes 32q..32q+31 are this warp's), column slice h
    const int q = warp & 3, h = (warp - 2) >> 2, r = q * 32 + lane, m = m0 + r, c0 = h * CW;
    const uint32_t trow = tmem + (uint32_t(q * 32) << 16) + uint32_t(c0);
    f2 acc[CW / 2];
#pragma unroll
    for (int j = 0; j < CW / 2; j++) {
      const int c = n0 + c0 + 2 * j;
      acc[j] = f2make(e.bias && c < N ? e.bias[c] : 0.f, e.bias && c + 1 < N ? e.bias[c + 1] : 0.f);
    }
    for (int st = 0; st < nst; st++) {
      const int s = st % S, g = st % G, nbl = min(TC_KB, nb - st * TC_KB);
      // (warp-uniform outcomes: the TMEM loads below are warp-collective)
      if (!__all_sync(FULL, mb_wait(full(s), (st / S) & 1, dead))) break;
      if (!__all_sync(FULL, mb_wait(tfull(g), (st / G) & 1, dead))) break;
      tc_fence_after();
      const uint32_t sb = base + s * C::STAGE;
      const uint8_t* sg = gbase + (sb - base);
      const float4 da4 = *reinterpret_cast<const float4*>(sg + C::OFF_S + r * 32);
      const float4 da4b = *reinterpret_cast<const float4*>(sg + C::OFF_S + r * 32 + 16);
#pragma unroll
      for (int kk = 0; kk < TC_KB; kk++) {
        if (kk >= nbl) break;
        const uint32_t tb = trow + uint32_t((g * TC_KB + kk) * BN);
        uint32_t d[CW];
#pragma unroll
        for (int c = 0; c < CW / 16; c++) tc_ld16(tb + 16 * c, d + 16 * c);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < CW / 16; c++) tc_st16(tb + 16 * c, uint32_t(MAGIC_BITS));
        const float dsc = kk == 0 ? da4.x : kk == 1 ? da4.z : kk == 2 ? da4b.x : da4b.z;
        const f2 da = f2dup(dsc);
        const float4* dq = reinterpret_cast<const float4*>(sg + C::OFF_D) + kk * (BN / 2) + c0 / 2;
        // in three independent passes, so the packed FMAs issue back to back
        float4 qd[CW / 2];  // {dw[n], dw[n+1], nm[n], nm[n+1]}
#pragma unroll
        for (int j = 0; j < CW / 2; j++) qd[j] = dq[j];
        f2 t[CW / 2];
#pragma unroll
        for (int j = 0; j < CW / 2; j++)
          t[j] = f2fma(f2make(__uint_as_float(d[2 * j]), __uint_as_float(d[2 * j + 1])), f2make(qd[j].x, qd[j].y),
                       f2make(qd[j].z, qd[j].w));
#pragma unroll
        for (int j = 0; j < CW / 2; j++) acc[j] = f2fma(t[j], da, acc[j]);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mb_arrive(tempty(g));
        mb_arrive(empty(s));
      }
    }
    if (!*dead && m < M) {
      if (e.epi == EPI_GELU_Q8) {
#pragma unroll
        for (int cb = 0; cb < CW / 32; cb++) {
          float g[32], amax = 0.f;
#pragma unroll
          for (int j = 0; j < 16; j++) {
            g[2 * j] = gelu_avx(f2lo(acc[cb * 16 + j]));
            g[2 * j + 1] = gelu_avx(f2hi(acc[cb * 16 + j]));
          }
#pragma unroll
          for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(g[j]));
          const int col = n0 + c0 + cb * 32;
          if (col < N) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
              uint32_t v = 0;
#pragma unroll
              for (int b = 0; b < 4; b++) v |= uint32_t(uint8_t(quant_val(g[4 * j + b], amax))) << (8 * b);
              w[j] = v;
            }
            uint4* dst = reinterpret_cast<uint4*>(e.q8 + (size_t)m * N + col);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            const float sc = quant_scale(amax);
            e.q8s[(size_t)m * (N / QK) + col / QK] = make_float2(sc, sc);
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < CW / 2; j++) {
          const int col = n0 + c0 + 2 * j;
          if (col >= N) continue;
          const float c0v = f2lo(acc[j]), c1v = f2hi(acc[j]);
          if (e.epi == EPI_ROPE_KV) {
            store_qkv_pair(e.kv, m, col, c0v, c1v);
            continue;
          }
          float2* yp = reinterpret_cast<float2*>(e.y + (size_t)m * e.ldy + col);
          if (e.epi == EPI_RESID) {
            const float2 o = *yp;
            const float a0 = e.ls ? __fmul_rn(e.ls[col], c0v) : c0v, a1 = e.ls ? __fmul_rn(e.ls[col + 1], c1v) : c1v;
            *yp = make_float2(__fadd_rn(o.x, a0), __fadd_rn(o.y, a1));
          } else {
            *yp = make_float2(c0v, c1v);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
  }
}


// ------------------------------------- GEMM, mma.sync fed by TMA --
//
// k_q8_gemm4: k_q8_gemm2's tiles, fold order and epilogues, with the loads
// taken off the computing warps. One producer warp issues each stage's four
// TMA copies (activation and weight tiles in the 128-byte swizzle — the
// XOR layout k_q8_gemm2's ldmatrix addressing already reads — the
// activation scales and the {dw, dw', nm, nm'} quads) on a full barrier;
// the consumer warps wait on it, run the stage's four blocks (their MMAs
// issued before the first fold) and arrive on the stage's empty barrier.
// A full stage runs without block-count checks; the activation scales of a
// stage are read once. Waits are bounded as in k_q8_tc (its fault word).
template <int TM, int TN, int WGM, int WGN, int STAGES>
struct Cfg4 {
  using B = Cfg2<TM, TN, WGM, WGN>;
  static constexpr int NWC = WGM * WGN, NT = 32 * (NWC + 1);
  static constexpr int TX = B::BM * 128 + B::BN * 128 + B::BM * B::KB * 8 + B::KB * B::BN * 8;
  static constexpr int OFF_BAR = STAGES * B::SST;
  static constexpr int SMEM = 1024 + OFF_BAR + 2 * STAGES * 8;  // + alignment slack
  static_assert(B::BM % 8 == 0 && B::SST % 1024 == 0, "swizzled tiles start on 1024-byte boundaries");
};

template <int TM, int TN, int WGM, int WGN, int STAGES>
__global__ void __launch_bounds__(Cfg4<TM, TN, WGM, WGN, STAGES>::NT)
    k_q8_gemm4(const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mw,
               const __grid_constant__ CUtensorMap ms, const __grid_constant__ CUtensorMap md, int M, int N, int nb,
               EpiArgs e) {
  using C4 = Cfg4<TM, TN, WGM, WGN, STAGES>;
  using C = typename C4::B;
  constexpr int BM = C::BM, BN = C::BN, NWC = C4::NWC, KB = C::KB;
  static_assert(TN % 2 == 0, "B fragments two column tiles at a time");
  extern __shared__ uint8_t g4_raw[];
  const uint32_t raw = smem_u32(g4_raw), sbase = (raw + 1023) & ~1023u;
  uint8_t* gbase = g4_raw + (sbase - raw);
  const uint32_t bars = sbase + C4::OFF_BAR;
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (STAGES + s); };
  __shared__ int dead_s;
  volatile int* dead = &dead_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nkt = (nb + KB - 1) / KB;
  if (tid == 0) {
    dead_s = 0;
    for (int s = 0; s < STAGES; s++) {
      mb_init(full(s), 1);
      mb_init(empty(s), NWC);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  f2 acc[TM][TN][2];
  const int wm = warp / WGN, wn = warp % WGN, arow = wm * 16 * TM, brow = wn * 8 * TN;
  if (warp == NWC) {
    // ---- the producer warp
    int issued = 0;
    for (int kt = 0; kt < nkt; kt++) {
      const int s = kt % STAGES;
      if (!__all_sync(FULL, mb_wait(empty(s), ((kt / STAGES) & 1) ^ 1, dead))) break;
      const uint32_t sb = sbase + s * C::SST;
      mb_expect_one(full(s), C4::TX);
      tma2d(sb + C::OFF_A, &ma, kt * 128, m0, full(s));
      tma2d(sb + C::OFF_W, &mw, kt * 128, n0, full(s));
      tma2d(sb + C::OFF_SA, &ms, kt * 8, m0, full(s));
      tma2d(sb + C::OFF_DN, &md, n0 * 2, kt * KB, full(s));
      issued = kt + 1;
    }
    // After a failure, let this block's copies land before it goes on.
    if (*dead)
      for (int kt = issued > STAGES ? issued - STAGES : 0; kt < issued; kt++) {
        const long long t0 = clock64();
        while (!mb_try(full(kt % STAGES), (kt / STAGES) & 1) && clock64() - t0 < (1LL << 30)) {
        }
      }
  } else {
    // ---- the consumer warps: fragment offsets within a stage
    const int mat = lane >> 3;
    uint32_t aoff[TM], boff[TN / 2];
#pragma unroll
    for (int i = 0; i < TM; i++) {
      const int ra = arow + i * 16 + (lane & 7) + (mat & 1) * 8;
      aoff[i] = C::OFF_A + ra * 128 + (((mat >> 1) ^ (ra & 7)) << 4);
    }
#pragma unroll
    for (int j = 0; j < TN / 2; j++) {
      const int rb = brow + j * 16 + (lane & 7) + (mat >> 1) * 8;
      boff[j] = C::OFF_W + rb * 128 + (((mat & 1) ^ (rb & 7)) << 4);
    }
    uint32_t soff[TM], doff[TN];
#pragma unroll
    for (int i = 0; i < TM; i++) soff[i] = C::OFF_SA + (arow + i * 16 + g) * 32;
#pragma unroll
    for (int j = 0; j < TN; j++) doff[j] = C::OFF_DN + ((brow + j * 8) / 2 + t4) * 16;
    // Each output's chain starts at its bias, or 0 (q8int.go:175-182).
#pragma unroll
    for (int j = 0; j < TN; j++) {
      const int c0 = n0 + brow + j * 8 + 2 * t4;
      const f2 b = f2make(e.bias && c0 < N ? e.bias[c0] : 0.f, e.bias && c0 + 1 < N ? e.bias[c0 + 1] : 0.f);
#pragma unroll
      for (int i = 0; i < TM; i++) acc[i][j][0] = acc[i][j][1] = b;
    }
    // The MMAs of a stage's first nbl blocks, then their folds in block order.
    auto stage = [&](uint32_t cur, int nbl, auto whole_c) {
      constexpr bool whole = decltype(whole_c)::value;
      f2 da[TM][2][KB];
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
          for (int kk = 0; kk < KB; kk += 2)
            asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];\n"
                         : "=l"(da[i][h][kk]), "=l"(da[i][h][kk + 1])
                         : "r"(cur + soff[i] + h * 8 * 32 + kk * 8));
      f2 p[KB][TM][TN][2];
#pragma unroll
      for (int kk = 0; kk < KB; kk++) {
        if (!whole && kk >= nbl) break;
        const uint32_t kl = uint32_t(2 * kk) << 4;  // the block's first chunk (the swizzle keeps bit 0)
        uint32_t af[TM][4], bf[TN][2];
#pragma unroll
        for (int i = 0; i < TM; i++) ldsm_x4(af[i][0], af[i][1], af[i][2], af[i][3], (cur + aoff[i]) ^ kl);
#pragma unroll
        for (int j = 0; j < TN / 2; j++)
          ldsm_x4(bf[2 * j][0], bf[2 * j][1], bf[2 * j + 1][0], bf[2 * j + 1][1], (cur + boff[j]) ^ kl);
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
          for (int j = 0; j < TN; j++) q8_mma(p[kk][i][j][0], p[kk][i][j][1], af[i], bf[j][0], bf[j][1]);
      }
#pragma unroll
      for (int kk = 0; kk < KB; kk++) {
        if (!whole && kk >= nbl) break;
#pragma unroll
        for (int j = 0; j < TN; j++) {
          f2 dw, nm;
          asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];\n" : "=l"(dw), "=l"(nm) : "r"(cur + doff[j] + kk * (BN / 2) * 16));
#pragma unroll
          for (int i = 0; i < TM; i++)
            q8_fold(acc[i][j][0], acc[i][j][1], p[kk][i][j][0], p[kk][i][j][1], dw, nm, da[i][0][kk], da[i][1][kk]);
        }
      }
    };
    for (int kt = 0; kt < nkt; kt++) {
      const int s = kt % STAGES;
      if (!__all_sync(FULL, mb_wait(full(s), (kt / STAGES) & 1, dead))) break;
      const uint32_t cur = sbase + s * C::SST;
      const int nbl = nb - kt * KB;
      if (nbl >= KB)
        stage(cur, KB, std::true_type{});
      else
        stage(cur, nbl, std::false_type{});
      __syncwarp();
      if (lane == 0) mb_arrive(empty(s));
    }
  }
  __syncthreads();  // every stage consumed (or abandoned), every copy landed
  if (e.epi == EPI_GELU_Q8) {
    // A row's 32-column blocks span several warps: gather the tile in shared
    // memory, then one warp per (row, block) rounds its block to Q8_0.
    float* tile = reinterpret_cast<float*>(gbase);  // [BM][BN + 1]
    if (warp < NWC)
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++)
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int r = arow + i * 16 + g + h * 8, c = brow + j * 8 + 2 * t4;
            tile[r * (BN + 1) + c] = gelu_avx(f2lo(acc[i][j][h]));
            tile[r * (BN + 1) + c + 1] = gelu_avx(f2hi(acc[i][j][h]));
          }
    __syncthreads();
    for (int rb = warp; rb < BM * (BN / 32); rb += NWC + 1) {
      const int r = rb / (BN / 32), cb = rb % (BN / 32), row = m0 + r;
      float sc;
      const int8_t qv = quant_lane(tile[r * (BN + 1) + cb * 32 + lane], &sc);
      if (row < M) {
        e.q8[(size_t)row * N + n0 + cb * 32 + lane] = qv;
        if (lane == 0) e.q8s[(size_t)row * (N / QK) + (n0 + cb * 32) / QK] = make_float2(sc, sc);
      }
    }
    return;
  }
  if (warp == NWC) return;
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++)
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int row = m0 + arow + i * 16 + g + h * 8, col = n0 + brow + j * 8 + 2 * t4;
        if (row < M && col < N) epi_pair(e, row, col, f2lo(acc[i][j][h]), f2hi(acc[i][j][h]));
      }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool tmap2d(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t outer,
            uint64_t stride_bytes, uint32_t box_in, uint32_t box_out, CUtensorMapSwizzle sw) {
  const cuuint64_t dims[2] = {inner, outer}, strides[1] = {stride_bytes};
  const cuuint32_t box[2] = {box_in, box_out}, es[2] = {1, 1};
  return g_encode(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A product's four tensor maps and launch shape, encoded once (a captured
// graph replays the launch with them).
struct TcLaunch {
  CUtensorMap ma, mw, ms, md;
  int M = 0, N = 0, nb = 0;
};

bool tc_prepare(TcLaunch& L, const int8_t* a, const float2* as, int M, const DQ8& w, int bn) {
  const int N = w.rows, K = w.cols, nb = K / QK, np2 = (N + 1) / 2;
  if (!g_encode || nb % 2 || ((uintptr_t(a) | uintptr_t(as) | uintptr_t(w.q) | uintptr_t(w.dwnm)) & 15)) return false;
  L.M = M, L.N = N, L.nb = nb;
  return tmap2d(&L.ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, K, M, K, 128, TC_BM, CU_TENSOR_MAP_SWIZZLE_128B) &&
         tmap2d(&L.mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q, K, N, K, 128, bn, CU_TENSOR_MAP_SWIZZLE_128B) &&
         tmap2d(&L.ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, as, 2 * nb, M, 8 * nb, 2 * TC_KB, TC_BM,
                CU_TENSOR_MAP_SWIZZLE_NONE) &&
         tmap2d(&L.md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.dwnm, 4 * np2, nb, 16 * np2, 2 * bn, TC_KB,
                CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int BN, int EPW>
struct GemmTc {
  using C = TcCfg<BN, EPW>;
  static void init() {
    cudaFuncSetAttribute(k_q8_tc<BN, EPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  }
  static bool suits(const DQ8& w, const EpiArgs& e) { return !(e.epi == EPI_GELU_Q8 && (w.rows % 32 || C::CW % 32)); }
  static void run(const TcLaunch& L, const EpiArgs& e, cudaStream_t st) {
    dim3 grid((L.N + BN - 1) / BN, (L.M + TC_BM - 1) / TC_BM);
    k_q8_tc<BN, EPW><<<grid, C::NT, C::SMEM, st>>>(L.ma, L.mw, L.ms, L.md, L.M, L.N, L.nb, e);
  }
  // False when the shape or the buffers do not suit the tensor maps (the
  // caller then takes the mma.sync kernel, which gives identical results).
  static bool launch(const int8_t* a, const float2* as, int M, const DQ8& w, const EpiArgs& e, cudaStream_t st) {
    TcLaunch L;
    if (!suits(w, e) || !tc_prepare(L, a, as, M, w, BN)) return false;
    run(L, e, st);
    return true;
  }
};

// A product's four tensor maps, kept per host thread and keyed by the
// buffers and the tile, so a product launched again with the same operands
// (a decode loop's layers, call after call) is not re-encoded.
struct G4Key {
  const void *a, *as, *wq, *dwnm;
  int M, N, K, bm, bn;
  bool operator==(const G4Key& o) const {
    return a == o.a && as == o.as && wq == o.wq && dwnm == o.dwnm && M == o.M && N == o.N && K == o.K &&
           bm == o.bm && bn == o.bn;
  }
};
struct G4KeyHash {
  size_t operator()(const G4Key& k) const {
    size_t h = std::hash<const void*>()(k.a) ^ (std::hash<const void*>()(k.wq) * 31u);
    return h ^ (size_t(k.M) * 1000003u) ^ (size_t(k.bm * 131 + k.bn) << 20);
  }
};
struct G4Maps {
  CUtensorMap ma, mw, ms, md;
};

const G4Maps* g4_maps(const int8_t* a, const float2* as, int M, const DQ8& w, int bm, int bn) {
  thread_local std::unordered_map<G4Key, G4Maps, G4KeyHash> cache;
  const int N = w.rows, K = w.cols, nb = K / QK, np2 = (N + 1) / 2;
  const G4Key key{a, as, w.q, w.dwnm, M, N, K, bm, bn};
  auto it = cache.find(key);
  if (it != cache.end()) return &it->second;
  G4Maps m;
  if (!tmap2d(&m.ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, K, M, K, 128, bm, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tmap2d(&m.mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q, K, N, K, 128, bn, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tmap2d(&m.ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, as, 2 * nb, M, 8 * nb, 8, bm, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !tmap2d(&m.md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.dwnm, 4 * np2, nb, 16 * np2, 2 * bn, 4,
              CU_TENSOR_MAP_SWIZZLE_NONE))
    return nullptr;
  if (cache.size() >= 4096) cache.clear();
  return &cache.emplace(key, m).first->second;
}

template <int TM, int TN, int WGM, int WGN, int STAGES>
struct Gemm4 {
  using C4 = Cfg4<TM, TN, WGM, WGN, STAGES>;
  using C = typename C4::B;
  static constexpr int kTile = C::BM * (C::BN + 1) * 4 + 1024;  // the GELU epilogue's tile
  static constexpr int kSmem = C4::SMEM > kTile ? C4::SMEM : kTile;
  static void init() {
    cudaFuncSetAttribute(k_q8_gemm4<TM, TN, WGM, WGN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  }
  // False when the shape or the buffers do not suit the tensor maps; the
  // caller then takes k_q8_gemm2 (identical results).
  static bool launch(const int8_t* a, const float2* as, int M, const DQ8& w, const EpiArgs& e, cudaStream_t st) {
    const int N = w.rows, nb = w.cols / QK;
    if (!g_encode || nb % 2 || ((uintptr_t(a) | uintptr_t(as) | uintptr_t(w.q) | uintptr_t(w.dwnm)) & 15)) return false;
    const G4Maps* m = g4_maps(a, as, M, w, C::BM, C::BN);
    if (!m) return false;
    dim3 grid((N + C::BN - 1) / C::BN, (M + C::BM - 1) / C::BM);
    k_q8_gemm4<TM, TN, WGM, WGN, STAGES><<<grid, C4::NT, kSmem, st>>>(m->ma, m->mw, m->ms, m->md, M, N, nb, e);
    return true;
  }
};

void tc_init_encode() {
  if (g_encode) return;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

// The tensor-core kernel gives the same bits as the mma.sync one but was
// slower at every product shape timed on B200 (one tcgen05.mma per 32-deep
// Q8_0 block costs about 100 clocks to issue, and the exact per-block chain
// rules out split-K), so it runs only when GRX_Q8_TC=1 is set at
// initialisation.
bool g_q8_tc = false;

// The TMA-fed kernel's shapes (bit-identical to the others; graph-timed on
// B200 at M = 128): 16×32 tiles of two 16×16 warps, six stages, for the
// narrow products (attn_out 4.80 µs against 5.73, ff2 13.1 against 16.8);
// 32×32 for qkv (7.07 against 7.56); 64×32 for ff1 (7.22 against 8.21) and,
// at 129–256 rows, for the narrow ones (attn_out 5.82 against 6.49, ff2 15.4
// against 19.4). Above 256 rows k_q8_gemm2 stays: Mimi's decoder at 512
// rows per product ran 8 % slower on this kernel.
bool g_q8_g4 = true;  // GRX_Q8_G4=0 at initialisation keeps every product on k_q8_gemm2
using G4Narrow = Gemm4<1, 2, 1, 2, 6>;
using G4Mid = Gemm4<1, 2, 2, 2, 4>;
using G4Wide = Gemm4<2, 2, 2, 2, 4>;

// Tile shapes per product shape, the fastest of those timed on B200, every
// one bit-identical to the others. PB = 4: each warp issues the MMAs of four
// Q8_0 blocks before folding them into its chains in block order, so the
// tensor-pipe latency of one block overlaps the issue of the next three.
// At M ≤ 128 (one part of a FlowLM set): 32×32 CTA tiles of four 16×16
// warps (qkv 7.78 µs, attn_out 5.56, ff2 16.8 per product), and 64×64 tiles
// of eight 32×16 warps for the widest (ff1 8.2).
using GemmSmall = Gemm2<1, 2, 2, 2, 4, 4>;
using GemmSmallWide = Gemm2<2, 2, 2, 4, 4>;  // N > 3072
// At M > 128: 64×32 tiles of four 32×16 warps for qkv-wide products (qkv
// 10.6 at M = 256), the 32×32 tiles above where N ≤ 2048 (attn_out 6.5,
// ff2 19.5: twice the CTAs), 64×64 of four 32×32 warps for the widest
// (ff1 11.7).
using GemmMid = Gemm2<2, 2, 2, 2, 4, 4>;
using GemmWide = Gemm2<2, 4, 2, 2, 4>;  // N > 3072

}  // namespace

int q8_tc_fault() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_q8_tc_fault, sizeof v);
  return v;
}

void launch_q8_product(const int8_t* a, const float2* as, int M, const DQ8& w, const EpiArgs& e, cudaStream_t st) {
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
  if (g_q8_tc && GemmTc<32, 4>::launch(a, as, M, w, e, st)) return;
  if (!g_q8_g4 || M > 256) {
    // the larger products (Mimi's, the TDT encoder projection, prefills)
    // measured as fast or faster on k_q8_gemm2
  } else if (M <= 128) {
    if (N <= 2048 ? G4Narrow::launch(a, as, M, w, e, st)
                  : N <= 3072 ? G4Mid::launch(a, as, M, w, e, st) : G4Wide::launch(a, as, M, w, e, st))
      return;
  } else if (N <= 2048 && G4Wide::launch(a, as, M, w, e, st)) {
    return;
  }
  if (M <= 128) {
    if (N > 3072)
      GemmSmallWide::launch(a, as, M, w, e, st);
    else
      GemmSmall::launch(a, as, M, w, e, st);
  } else if (N > 3072) {
    GemmWide::launch(a, as, M, w, e, st);
  } else if (N > 2048) {
    GemmMid::launch(a, as, M, w, e, st);
  } else {
    GemmSmall::launch(a, as, M, w, e, st);
  }
}

// Raises the kernels' dynamic shared memory limits once per device.
void q8_kernels_init() {
  tc_init_encode();
  const char* tc = getenv("GRX_Q8_TC");
  g_q8_tc = tc && tc[0] == '1';
  const char* g4 = getenv("GRX_Q8_G4");
  g_q8_g4 = !(g4 && g4[0] == '0');
  GemmTc<32, 4>::init();
  G4Narrow::init();
  G4Mid::init();
  G4Wide::init();
  GemmMid::init();
  GemmWide::init();
  GemmSmall::init();
  GemmSmallWide::init();
  const int gv = 8 * kQ8GemvMaxK + 8 * (kQ8GemvMaxK / QK) * 4 + 8 * 32 * 4;
  cudaFuncSetAttribute(k_q8_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
}

}  // namespace grx
