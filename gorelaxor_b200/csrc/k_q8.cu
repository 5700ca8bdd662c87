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
// TN column tiles), eight warps a CTA tile; a stage carries KB blocks of K.
// Every shared-memory address is a 32-bit offset computed once, and the
// scale operands are read as ready-made pairs. The tile shape is chosen per
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

// One Q8_0 block of a 16×8 tile, in one piece of PTX so every value stays
// in its register pair: D = A·B + MAGIC_BITS (the tensor core's int32 sum
// lands on the bits of the float 1.5·2^23 + s, |s| ≤ 32·128·128 = 2^19), then
// t = fma(1.5·2^23 + s, dw, −1.5·2^23·dw) = fl(float(s)·dw) — one rounding
// of the exact product, as the reference's VMULPS (vnni_amd64.s:63-64) —
// and acc = fma(t, da, acc) (its VFMADD213PS, :66-67), both as f32x2 pairs.
__device__ __forceinline__ void q8_block(f2& acc01, f2& acc23, const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                         f2 dw, f2 nm, f2 da0, f2 da1) {
  asm("{\n"
      " .reg .b32 d0, d1, d2, d3;\n"
      " .reg .b64 p01, p23;\n"
      " mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {d0,d1,d2,d3}, {%2,%3,%4,%5}, {%6,%7}, {%12,%12,%12,%12};\n"
      " mov.b64 p01, {d0, d1};\n"
      " mov.b64 p23, {d2, d3};\n"
      " fma.rn.f32x2 p01, p01, %8, %9;\n"
      " fma.rn.f32x2 p23, p23, %8, %9;\n"
      " fma.rn.f32x2 %0, p01, %10, %0;\n"
      " fma.rn.f32x2 %1, p23, %11, %1;\n"
      "}\n"
      : "+l"(acc01), "+l"(acc23)
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "l"(dw), "l"(nm), "l"(da0), "l"(da1),
        "r"(MAGIC_BITS));
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

template <int TM, int TN, int WGM, int WGN, int KB>
struct GemmCfg {
  static constexpr int BM = 16 * TM * WGM, BN = 8 * TN * WGN, BKB = KB * QK;
  static constexpr int OFF_A = 0, OFF_W = OFF_A + BM * BKB, OFF_SA = OFF_W + BN * BKB,
                       OFF_DW = OFF_SA + BM * KB * 8, OFF_NM = OFF_DW + KB * BN * 4,
                       SST = (OFF_NM + KB * BN * 4 + 1023) / 1024 * 1024;  // stages 1 KB aligned: the swizzle
                                                                          // XORs address bits 4-6
  static constexpr int CPR = BKB / 16;  // 16-byte chunks per tile row
};

template <int TM, int TN, int WGM, int WGN, int KB, int STAGES, bool PIPE>
__global__ void __launch_bounds__(256) k_q8_gemm(const int8_t* __restrict__ a, const float2* __restrict__ as, int M,
                                                 const int8_t* __restrict__ wq, const float* __restrict__ dwT,
                                                 const float* __restrict__ nmT, int N, int K, EpiArgs e) {
  using C = GemmCfg<TM, TN, WGM, WGN, KB>;
  constexpr int BM = C::BM, BN = C::BN, BKB = C::BKB, CPR = C::CPR;
  static_assert(WGM * WGN == 8, "eight warps");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const int wm = warp / WGN, wn = warp % WGN;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nb = K / QK, nkt = (nb + KB - 1) / KB;
  const int arow = wm * 16 * TM, brow = wn * 8 * TN;
  const uint32_t sbase = smem_u32(smem_raw);

  // ---- the copies of one stage: A and W tiles (rows × CPR chunks), the
  // (da, da) pairs (BM rows × KB/2 chunks) and dw, nm (KB × BN/4 chunks each).
  constexpr int NA = BM * CPR, NW = BN * CPR, NS = BM * KB / 2, ND = KB * BN / 4;
  auto load = [&](int kt, uint32_t st) {
    const int kb0 = kt * KB;
    for (int i = tid; i < NA + NW; i += 256) {
      const bool isw = i >= NA;
      const int j = isw ? i - NA : i, r = j / CPR, c = j % CPR;
      const int swz = ((c & ~7) | ((c & 7) ^ (r & 7))) << 4;
      const int gr = (isw ? n0 : m0) + r, kc = kb0 * QK + c * 16;
      const bool v = gr < (isw ? N : M) && kc < K;
      const int8_t* src = (isw ? wq : a) + (size_t)(v ? gr : 0) * K + (v ? kc : 0);
      cp_async16(st + (isw ? C::OFF_W : C::OFF_A) + r * BKB + swz, src, v);
    }
    for (int i = tid; i < NS + 2 * ND; i += 256) {
      if (i < NS) {
        const int r = i / (KB / 2), q = i % (KB / 2), gr = m0 + r;
        const bool v = gr < M && kb0 + 2 * q < nb;
        cp_async16(st + C::OFF_SA + (r * KB + 2 * q) * 8, as + (size_t)(v ? gr : 0) * nb + (v ? kb0 + 2 * q : 0), v);
      } else {
        const int j = i - NS, which = j / ND, jj = j % ND, kb = jj / (BN / 4), c4 = (jj % (BN / 4)) * 4;
        const bool v = kb0 + kb < nb && n0 + c4 < N;
        const float* src = (which ? nmT : dwT) + (v ? (size_t)(kb0 + kb) * N + n0 + c4 : 0);
        cp_async16(st + (which ? C::OFF_NM : C::OFF_DW) + (kb * BN + c4) * 4, src, v);
      }
    }
  };

  // ---- the warp's fragment and operand offsets within a stage.
  const int mat = lane >> 3;
  uint32_t aoff[TM], boff[TN];
#pragma unroll
  for (int i = 0; i < TM; i++) {
    const int ra = arow + i * 16 + (lane & 7) + (mat & 1) * 8;
    aoff[i] = C::OFF_A + ra * BKB + (((mat >> 1) ^ (ra & 7)) << 4);
  }
#pragma unroll
  for (int j = 0; j < TN; j++) {
    const int rb = brow + j * 8 + (lane & 7);
    boff[j] = C::OFF_W + rb * BKB + ((((lane >> 3) & 1) ^ (rb & 7)) << 4);
  }

  // Each output's chain starts at its bias, or 0 (q8int.go:175-182).
  // acc[i][j][0]: rows g of m-tile i, columns (c, c+1) of n-tile j; [1]: row g+8.
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
  int rs = 0, ws = STAGES - 1;  // read and write stage
  for (int kt = 0; kt < nkt; kt++) {
    cp_wait<STAGES - 2>();
    __syncthreads();
    if (kt + STAGES - 1 < nkt) load(kt + STAGES - 1, sbase + ws * C::SST);
    cp_commit();
    ws = ws + 1 == STAGES ? 0 : ws + 1;
    const uint32_t cur = sbase + rs * C::SST;
    rs = rs + 1 == STAGES ? 0 : rs + 1;
    const int nblk = min(KB, nb - kt * KB);
    if (PIPE && nblk == KB) {
      // all MMAs of the stage first, then the chains: the tensor-core latency
      // is paid once per stage, not once per block.
      f2 p[KB][TM][TN][2];
#pragma unroll
      for (int kk = 0; kk < KB; kk++) {
        const uint32_t kx = (uint32_t)((2 * kk) & ~7) << 4, kl = (uint32_t)((2 * kk) & 7) << 4;
        uint32_t af[TM][4];
#pragma unroll
        for (int i = 0; i < TM; i++) ldsm_x4(af[i][0], af[i][1], af[i][2], af[i][3], (cur + aoff[i] + kx) ^ kl);
#pragma unroll
        for (int j = 0; j < TN; j++) {
          uint32_t b0, b1;
          ldsm_x2(b0, b1, (cur + boff[j] + kx) ^ kl);
#pragma unroll
          for (int i = 0; i < TM; i++) q8_mma(p[kk][i][j][0], p[kk][i][j][1], af[i], b0, b1);
        }
      }
#pragma unroll
      for (int kk = 0; kk < KB; kk++)
#pragma unroll
        for (int j = 0; j < TN; j++) {
          const uint32_t so = cur + kk * BN * 4 + (brow + j * 8 + 2 * t4) * 4;
          const f2 dw = lds64(so + C::OFF_DW), nm = lds64(so + C::OFF_NM);
#pragma unroll
          for (int i = 0; i < TM; i++) {
            const uint32_t sa = cur + C::OFF_SA + ((arow + i * 16 + g) * KB + kk) * 8;
            q8_fold(acc[i][j][0], acc[i][j][1], p[kk][i][j][0], p[kk][i][j][1], dw, nm, lds64(sa),
                    lds64(sa + 8 * KB * 8));
          }
        }
      continue;
    }
#pragma unroll
    for (int kk = 0; kk < KB; kk++) {
      if (kk < nblk) {
        // chunk 2kk (k 0..15 of the block) and 2kk+1: the swizzle keeps the
        // chunk's high bits, so the block's offset is added before it.
        const uint32_t kx = (uint32_t)((2 * kk) & ~7) << 4;
        const uint32_t kl = (uint32_t)((2 * kk) & 7) << 4;
        uint32_t af[TM][4];
#pragma unroll
        for (int i = 0; i < TM; i++) ldsm_x4(af[i][0], af[i][1], af[i][2], af[i][3], (cur + aoff[i] + kx) ^ kl);
#pragma unroll
        for (int j = 0; j < TN; j++) {
          uint32_t b0, b1;
          ldsm_x2(b0, b1, (cur + boff[j] + kx) ^ kl);
          const uint32_t so = cur + kk * BN * 4 + (brow + j * 8 + 2 * t4) * 4;
          const f2 dw = lds64(so + C::OFF_DW), nm = lds64(so + C::OFF_NM);
#pragma unroll
          for (int i = 0; i < TM; i++) {
            const uint32_t sa = cur + C::OFF_SA + ((arow + i * 16 + g) * KB + kk) * 8;
            const f2 da0 = lds64(sa), da1 = lds64(sa + 8 * KB * 8);
            q8_block(acc[i][j][0], acc[i][j][1], af[i], b0, b1, dw, nm, da0, da1);
          }
        }
      }
    }
  }
  cp_wait<0>();

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
    for (int rb = warp; rb < BM * (BN / 32); rb += 8) {
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

template <int TM, int TN, int WGM, int WGN, int KB, int STAGES, bool PIPE = true>
struct Gemm {
  using C = GemmCfg<TM, TN, WGM, WGN, KB>;
  static constexpr size_t smem() {
    const size_t s = size_t(C::SST) * STAGES, t = size_t(C::BM) * (C::BN + 1) * 4;
    return s > t ? s : t;
  }
  static void init() {
    cudaFuncSetAttribute(k_q8_gemm<TM, TN, WGM, WGN, KB, STAGES, PIPE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(smem()));
  }
  static void launch(const int8_t* a, const float2* as, int M, const DQ8& w, const EpiArgs& e, cudaStream_t st) {
    dim3 grid((w.rows + C::BN - 1) / C::BN, (M + C::BM - 1) / C::BM);
    k_q8_gemm<TM, TN, WGM, WGN, KB, STAGES, PIPE><<<grid, 256, smem(), st>>>(a, as, M, w.q, w.dwT, w.nmT, w.rows,
                                                                             w.cols, e);
  }
};

// Tile shapes per product shape, the fastest of those timed at M = 256 on
// B200 (qkv 16.6 µs, attn_out 10.4, ff1 21.4, ff2 26.8 per product).
using GemmNarrow = Gemm<1, 1, 2, 4, 4, 4>;  // N ≤ 2048, K ≤ 2048
using GemmWide = Gemm<2, 2, 2, 4, 4, 4>;    // N > 2048
using GemmDeep = Gemm<1, 2, 2, 4, 8, 4>;    // K > 2048

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
  if (K > 2048)
    GemmDeep::launch(a, as, M, w, e, st);
  else if (N > 2048)
    GemmWide::launch(a, as, M, w, e, st);
  else
    GemmNarrow::launch(a, as, M, w, e, st);
}

// Raises the kernels' dynamic shared memory limits once per device.
void q8_kernels_init() {
  GemmNarrow::init();
  GemmWide::init();
  GemmDeep::init();
  const int gv = 8 * 4096 + 8 * 128 * 4 + 8 * 32 * 4;
  cudaFuncSetAttribute(k_q8_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
  cudaFuncSetAttribute(k_q8_gemv<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, gv);
}

}  // namespace grx
