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
#include <cuda_runtime.h>

#include <cstddef>

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
          *yp = __fadd_rn(*yp, v);
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
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, uint32_t a) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(a));
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
        if (row >= M || col >= N) continue;
        const float c0v = f2lo(acc[i][j][h]), c1v = f2hi(acc[i][j][h]);
        if (e.epi == EPI_ROPE_KV) {
          store_qkv_pair(e.kv, row, col, c0v, c1v);
          continue;
        }
        float2* yp = reinterpret_cast<float2*>(e.y + (size_t)row * e.ldy + col);
        if (e.epi == EPI_RESID) {
          const float2 o = *yp;
          *yp = make_float2(__fadd_rn(o.x, c0v), __fadd_rn(o.y, c1v));
        } else {
          *yp = make_float2(c0v, c1v);
        }
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

template <int TM, int TN, int WGM, int WGN, int STAGES>
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
  const int nb = K / QK, nkt = nb / 4, np2 = (N + 1) / 2;
  const int arow = wm * 16 * TM, brow = wn * 8 * TN;
  const uint32_t sbase = smem_u32(smem_raw);

  // ---- this thread's copies of a stage: sources (advance per stage) and
  // destinations within a stage
  const int8_t* srcA[C::PA];
  uint32_t dstA[C::PA];
  bool okA[C::PA];
#pragma unroll
  for (int u = 0; u < C::PA; u++) {
    const int i = tid + u * NT, r = i >> 3, c = i & 7;
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
    okD[u] = i < C::CD && n0 + 2 * p < N;
    srcD[u] = dwnm + (size_t)kb * np2 + (okD[u] ? n0 / 2 + p : 0);
    dstD[u] = C::OFF_DN + (kb * (BN / 2) + p) * 16;
  }
  auto load = [&](int kt, uint32_t st) {
#pragma unroll
    for (int u = 0; u < C::PA; u++)
      if (tid + u * NT < C::CA) cp_async16(st + dstA[u], srcA[u] + kt * 128, okA[u]);
#pragma unroll
    for (int u = 0; u < C::PW; u++)
      if (tid + u * NT < C::CW) cp_async16(st + dstW[u], srcW[u] + kt * 128, okW[u]);
#pragma unroll
    for (int u = 0; u < C::PS; u++)
      if (tid + u * NT < C::CS) cp_async16(st + dstS[u], srcS[u] + kt * 4, okS[u]);
#pragma unroll
    for (int u = 0; u < C::PD; u++)
      if (tid + u * NT < C::CD) cp_async16(st + dstD[u], srcD[u] + (size_t)kt * 4 * np2, okD[u]);
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
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const uint32_t kl = uint32_t(2 * kk) << 4;  // the block's first chunk (the swizzle keeps bit 0)
      uint32_t af[TM][4], bf[TN][2];
#pragma unroll
      for (int i = 0; i < TM; i++) ldsm_x4(af[i][0], af[i][1], af[i][2], af[i][3], (cur + aoff[i]) ^ kl);
#pragma unroll
      for (int j = 0; j < TN / 2; j++)
        ldsm_x4(bf[2 * j][0], bf[2 * j][1], bf[2 * j + 1][0], bf[2 * j + 1][1], (cur + boff[j]) ^ kl);
      f2 p[TM][TN][2];
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) q8_mma(p[i][j][0], p[i][j][1], af[i], bf[j][0], bf[j][1]);
#pragma unroll
      for (int j = 0; j < TN; j++) {
        f2 dw, nm;
        asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];\n" : "=l"(dw), "=l"(nm) : "r"(cur + doff[j] + kk * (BN / 2) * 16));
#pragma unroll
        for (int i = 0; i < TM; i++) {
          const uint32_t sa = cur + soff[i] + kk * 8;
          q8_fold(acc[i][j][0], acc[i][j][1], p[i][j][0], p[i][j][1], dw, nm, lds64(sa), lds64(sa + 8 * 32));
        }
      }
    }
  }
  cp_wait<0>();
  gemm_epilogue<TM, TN, WGM * WGN>(acc, e, smem_raw, m0, n0, arow, brow, g, t4, warp, lane, M, N, BM, BN);
}

template <int TM, int TN, int WGM, int WGN, int STAGES>
struct Gemm2 {
  using C = Cfg2<TM, TN, WGM, WGN>;
  static constexpr size_t smem() {
    const size_t s = size_t(C::SST) * STAGES, t = size_t(C::BM) * (C::BN + 1) * 4;
    return s > t ? s : t;
  }
  static void init() {
    cudaFuncSetAttribute(k_q8_gemm2<TM, TN, WGM, WGN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(smem()));
  }
  static void launch(const int8_t* a, const float2* as, int M, const DQ8& w, const EpiArgs& e, cudaStream_t st) {
    dim3 grid((w.rows + C::BN - 1) / C::BN, (M + C::BM - 1) / C::BM);
    k_q8_gemm2<TM, TN, WGM, WGN, STAGES><<<grid, C::NT, smem(), st>>>(a, as, M, w.q, w.dwnm, w.rows, w.cols, e);
  }
};

// Tile shapes per product shape, the fastest of those timed at M = 256 on
// B200, every one bit-identical to the others: 64×32 CTA tiles of four 32×16
// warps for most (qkv 11.3 µs, attn_out 7.6, ff2 18.5 per product), 64×64
// of four 32×32 warps for the widest (ff1 12.4).
using GemmMid = Gemm2<2, 2, 2, 2, 4>;
using GemmWide = Gemm2<2, 4, 2, 2, 4>;  // N > 3072

}  // namespace

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
  if (N > 3072)
    GemmWide::launch(a, as, M, w, e, st);
  else
    GemmMid::launch(a, as, M, w, e, st);
}

// Raises the kernels' dynamic shared memory limits once per device.
void q8_kernels_init() {
  GemmMid::init();
  GemmWide::init();
  const int gv = 8 * 4096 + 8 * 128 * 4 + 8 * 32 * 4;
  cudaFuncSetAttribute(k_q8_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
}

}  // namespace grx
