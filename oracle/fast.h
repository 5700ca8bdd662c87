// TEST INFRASTRUCTURE ONLY: the oracle's fast mode, the timed CPU baseline.
// Nothing in the product links, loads or calls this code.
//
// The same arithmetic as the exact mode (kern.h, flowlm.h), written with the
// SIMD instructions the reference's amd64 assembly uses and in its lane
// order, so every result is bit-identical to the exact mode (tests check it):
//  * int8 products (matmulQ8Int, internal/kern/q8int.go:148-223, with the
//    tile of vnni_amd64.s:58-138): weight panels of 16 rows laid out for
//    vpdpbusd ([8 groups][16 rows][4 bytes] per block, then the rows' scales
//    and their 128·Σw), unsigned activations q+128, per block the exact
//    int32 sums, then FIN: cvt(s − 128·Σw)·dw and one fused ·da + c;
//  * the float path's dot4q8avx / dot4f32avx / dot4f16avx
//    (kernels_amd64.s:99-204,343-399): 8 lanes per row, HSUM at the end;
//  * one-query attention (pockettts/nn.go:200-243): dot4f32avx scores,
//    EXP8 lane sums (kernels_amd64.s:238-283), axpy values;
//  * GELU / SiLU over 8 lanes (kernels_amd64.s:301-339,441-459).
// The kernels are chosen at run time: AVX-512 VNNI (as the reference's
// q8tileEVEX) where the processor has it, else a 256-bit form whose int32
// block sums are the same exact integers. Products of one row split their
// weight panels (or row groups) over a pool of threads, as the reference
// splits a product's columns over goroutines (gemm.go:327-351).
#pragma once
#include <immintrin.h>

#include <atomic>
#include <condition_variable>
#include <cstdlib>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "kern.h"

namespace orc {

// ------------------------------------------------------------ the mode ---

inline std::atomic<int>& fast_flag() {
  static std::atomic<int> f{0};
  return f;
}
inline bool fast_on() { return fast_flag().load(std::memory_order_relaxed) != 0; }

inline bool cpu_avx2() {
  static const bool ok = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") &&
                         __builtin_cpu_supports("f16c");
  return ok;
}
// ORC_FAST_AVX2=1 takes the 256-bit kernels even where AVX-512 VNNI exists
// (tests check that both give the exact mode's values).
inline bool cpu_vnni512() {
  static const bool ok = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
                         __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("avx512vnni") &&
                         !(getenv("ORC_FAST_AVX2") && getenv("ORC_FAST_AVX2")[0] == '1');
  return ok;
}

// ------------------------------------------------------------ the pool ---
//
// Fork-join over `items` work items; workers spin briefly between jobs (a
// frame makes dozens of short parallel calls) and then sleep.
class Pool {
 public:
  explicit Pool(int threads) : n_(std::max(1, threads)) {
    for (int t = 1; t < n_; t++) ts_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    stop_.store(true);
    {
      std::lock_guard<std::mutex> lk(mu_);
      cv_.notify_all();
    }
    for (auto& t : ts_) t.join();
  }
  int size() const { return n_; }
  void run(int items, const std::function<void(int)>& fn) {
    if (items <= 0) return;
    if (n_ == 1 || items == 1) {
      for (int i = 0; i < items; i++) fn(i);
      return;
    }
    fn_ = &fn;
    items_ = items;
    next_.store(0);
    done_.store(0);
    {
      std::lock_guard<std::mutex> lk(mu_);
      gen_.fetch_add(1, std::memory_order_release);
      cv_.notify_all();
    }
    grab();
    while (done_.load(std::memory_order_acquire) < n_ - 1) _mm_pause();
    fn_ = nullptr;
  }

 private:
  void grab() {
    for (;;) {
      const int i = next_.fetch_add(1);
      if (i >= items_) return;
      (*fn_)(i);
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      int spins = 0;
      while (gen_.load(std::memory_order_acquire) == seen) {
        if (stop_.load()) return;
        if (++spins < 200000) {
          _mm_pause();
        } else {
          std::unique_lock<std::mutex> lk(mu_);
          cv_.wait(lk, [&] { return gen_.load() != seen || stop_.load(); });
        }
      }
      if (stop_.load()) return;
      seen = gen_.load(std::memory_order_acquire);
      grab();
      done_.fetch_add(1, std::memory_order_release);
    }
  }
  int n_;
  std::vector<std::thread> ts_;
  std::atomic<uint64_t> gen_{0};
  std::atomic<int> next_{0}, done_{0};
  std::atomic<bool> stop_{false};
  int items_ = 0;
  const std::function<void(int)>* fn_ = nullptr;
  std::mutex mu_;
  std::condition_variable cv_;
};

// The pool this thread's products may split over (none: one thread).
inline Pool*& tl_pool() {
  static thread_local Pool* p = nullptr;
  return p;
}

// -------------------------------------------------------- weight panels ---

// 16 weight rows per panel; per block 640 bytes: [8][16][4] int8, [16] f32
// dw, [16] i32 128·Σw (rows past the matrix are zero).
constexpr int kPanelCols = 16, kPanelBlock = 640;

struct Panels {
  std::vector<uint8_t> b;
  int nb = 0, np = 0;
};

inline void pack_panels(const Weight& w, Panels& P) {
  const int n = w.rows, nb = w.cols / QK, np = (n + 15) / 16;
  const long ld = long(nb) * Q8BYTES;
  P.nb = nb;
  P.np = np;
  P.b.assign(size_t(np) * nb * kPanelBlock, 0);
  for (int pi = 0; pi < np; pi++)
    for (int b = 0; b < nb; b++) {
      uint8_t* dst = P.b.data() + (size_t(pi) * nb + b) * kPanelBlock;
      for (int j = 0; j < 16; j++) {
        const int col = pi * 16 + j;
        if (col >= n) continue;
        const uint8_t* blk = w.q + col * ld + long(b) * Q8BYTES;
        int32_t s = 0;
        for (int g = 0; g < 8; g++)
          for (int i = 0; i < 4; i++) {
            dst[g * 64 + j * 4 + i] = blk[2 + 4 * g + i];
            s += int32_t(int8_t(blk[2 + 4 * g + i]));
          }
        const float d = f16_to_f32(uint16_t(blk[0] | blk[1] << 8));
        std::memcpy(dst + 512 + j * 4, &d, 4);
        const int32_t c = 128 * s;
        std::memcpy(dst + 576 + j * 4, &c, 4);
      }
    }
}

struct PanelSlot {
  std::once_flag once;
  Panels p;
};

// The weight's panels: packed once into its slot, or into `tmp` for a
// weight without one (a one-off product).
inline const Panels& panels_of(const Weight& w, Panels& tmp) {
  if (w.slot) {
    std::call_once(w.slot->once, [&] { pack_panels(w, w.slot->p); });
    return w.slot->p;
  }
  pack_panels(w, tmp);
  return tmp;
}

// ------------------------------------------------------- int8 products ---

// Rows r0..r0+rows-1 (rows ≤ 6) of C against panel pi: ua the unsigned
// activations (q + 128, k per row), da their scales (nb per row).
__attribute__((target("avx512f,avx512bw,avx512vl,avx512vnni"))) inline void q8_panel_vnni512(
    const Panels& P, int pi, const uint8_t* ua, const float* da, int rows, int k, float* c, int ldc, int cols) {
  const int nb = P.nb;
  __m512 acc[6];
  for (int r = 0; r < 6; r++) acc[r] = r < rows ? _mm512_maskz_loadu_ps(__mmask16((1u << cols) - 1), c + long(r) * ldc)
                                                 : _mm512_setzero_ps();
  const uint8_t* wp = P.b.data() + size_t(pi) * nb * kPanelBlock;
  for (int b = 0; b < nb; b++, wp += kPanelBlock) {
    __m512i s[6];
    for (int r = 0; r < 6; r++) s[r] = _mm512_setzero_si512();
    for (int g = 0; g < 8; g++) {
      const __m512i w = _mm512_loadu_si512(wp + g * 64);
      for (int r = 0; r < rows; r++) {
        int32_t a4;
        std::memcpy(&a4, ua + long(r) * k + b * QK + 4 * g, 4);
        s[r] = _mm512_dpbusd_epi32(s[r], _mm512_set1_epi32(a4), w);
      }
    }
    const __m512i corr = _mm512_loadu_si512(wp + 576);
    const __m512 dw = _mm512_loadu_ps(reinterpret_cast<const float*>(wp + 512));
    for (int r = 0; r < rows; r++) {
      const __m512 t = _mm512_mul_ps(_mm512_cvtepi32_ps(_mm512_sub_epi32(s[r], corr)), dw);
      acc[r] = _mm512_fmadd_ps(t, _mm512_set1_ps(da[long(r) * nb + b]), acc[r]);
    }
  }
  for (int r = 0; r < rows; r++) _mm512_mask_storeu_ps(c + long(r) * ldc, __mmask16((1u << cols) - 1), acc[r]);
}

// The same with 256-bit registers and no VNNI: each group of four bytes is
// widened to int16 and summed by vpmaddwd, exact in int32.
__attribute__((target("avx2,fma,f16c"))) inline void q8_panel_avx2(const Panels& P, int pi, const uint8_t* ua,
                                                                   const float* da, int rows, int k, float* c, int ldc,
                                                                   int cols) {
  const int nb = P.nb;
  for (int h = 0; h < 2; h++) {  // the panel's two halves of 8 rows
    const int c0 = h * 8, cn = std::min(8, cols - c0);
    if (cn <= 0) break;
    float tmp[6][8];
    __m256 acc[6];
    for (int r = 0; r < rows; r++) {
      for (int j = 0; j < 8; j++) tmp[r][j] = j < cn ? c[long(r) * ldc + c0 + j] : 0.f;
      acc[r] = _mm256_loadu_ps(tmp[r]);
    }
    const uint8_t* wp = P.b.data() + size_t(pi) * nb * kPanelBlock;
    for (int b = 0; b < nb; b++, wp += kPanelBlock) {
      __m256i s[6];
      for (int r = 0; r < 6; r++) s[r] = _mm256_setzero_si256();
      for (int g = 0; g < 8; g++) {
        // 8 rows × 4 bytes → two vectors of int16: bytes 0-1 and 2-3 of each row
        const __m256i w8 = _mm256_cvtepi8_epi16(_mm_loadu_si128(reinterpret_cast<const __m128i*>(wp + g * 64 + c0 * 4)));
        const __m256i w16 = _mm256_cvtepi8_epi16(
            _mm_loadu_si128(reinterpret_cast<const __m128i*>(wp + g * 64 + c0 * 4 + 16)));
        for (int r = 0; r < rows; r++) {
          const uint8_t* a = ua + long(r) * k + b * QK + 4 * g;
          const int32_t p01 = int32_t(a[0]) | int32_t(a[1]) << 16, p23 = int32_t(a[2]) | int32_t(a[3]) << 16;
          // w8 holds rows 0-3 (4 int16 each), w16 rows 4-7
          const __m256i av = _mm256_setr_epi32(p01, p23, p01, p23, p01, p23, p01, p23);
          const __m256i lo = _mm256_madd_epi16(w8, av), hi = _mm256_madd_epi16(w16, av);
          // lo: [r0 (01), r0 (23), r1 (01), r1 (23) | r2.., r3..]; pairwise add to rows
          const __m256i sum = _mm256_hadd_epi32(lo, hi);  // [r0 r1 r4 r5 | r2 r3 r6 r7]
          s[r] = _mm256_add_epi32(s[r], _mm256_permutevar8x32_epi32(sum, _mm256_setr_epi32(0, 1, 4, 5, 2, 3, 6, 7)));
        }
      }
      const __m256i corr = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(wp + 576 + c0 * 4));
      const __m256 dw = _mm256_loadu_ps(reinterpret_cast<const float*>(wp + 512 + c0 * 4));
      for (int r = 0; r < rows; r++) {
        const __m256 t = _mm256_mul_ps(_mm256_cvtepi32_ps(_mm256_sub_epi32(s[r], corr)), dw);
        acc[r] = _mm256_fmadd_ps(t, _mm256_set1_ps(da[long(r) * nb + b]), acc[r]);
      }
    }
    for (int r = 0; r < rows; r++) {
      _mm256_storeu_ps(tmp[r], acc[r]);
      for (int j = 0; j < cn; j++) c[long(r) * ldc + c0 + j] = tmp[r][j];
    }
  }
}

// matmulQ8Int with the fast kernels (same values as matmul_q8_int).
inline void matmul_q8_int_fast(float* c, int ldc, const float* a, int lda, int m, const Weight& w, const float* bias) {
  const int n = w.rows, k = w.cols, nb = k / QK;
  Panels tmp;
  const Panels& P = panels_of(w, tmp);
  std::vector<int8_t> q(size_t(m) * k);
  std::vector<uint8_t> ua(size_t(m) * k);
  std::vector<float> sa(size_t(m) * nb);
  for (int i = 0; i < m; i++) {
    quant_q8_act(q.data() + long(i) * k, sa.data() + long(i) * nb, a + long(i) * lda, nb);
    for (int t = 0; t < k; t++) ua[size_t(i) * k + t] = uint8_t(int(q[size_t(i) * k + t]) + 128);
    float* ci = c + long(i) * ldc;
    for (int j = 0; j < n; j++) ci[j] = bias ? bias[j] : 0.f;
  }
  const bool v512 = cpu_vnni512();
  auto panel = [&](int pi) {
    const int cols = std::min(16, n - pi * 16);
    for (int r0 = 0; r0 < m; r0 += 6) {
      const int rows = std::min(6, m - r0);
      float* cp = c + long(r0) * ldc + pi * 16;
      if (v512)
        q8_panel_vnni512(P, pi, ua.data() + long(r0) * k, sa.data() + long(r0) * nb, rows, k, cp, ldc, cols);
      else
        q8_panel_avx2(P, pi, ua.data() + long(r0) * k, sa.data() + long(r0) * nb, rows, k, cp, ldc, cols);
    }
  };
  Pool* pool = tl_pool();
  if (pool && pool->size() > 1) {
    const int items = std::min(P.np, 4 * pool->size());
    pool->run(items, [&](int it) {
      for (int pi = P.np * it / items; pi < P.np * (it + 1) / items; pi++) panel(pi);
    });
  } else {
    for (int pi = 0; pi < P.np; pi++) panel(pi);
  }
}

// ----------------------------------------------------- float-path dots ---

__attribute__((target("avx2,fma,f16c"))) inline float hsum8_v(__m256 a) {
  alignas(32) float t[8];
  _mm256_store_ps(t, a);
  return hsum8(t);
}

// Eight int8 values widened to float (VPMOVSXBD + VCVTDQ2PS, exact).
__attribute__((target("avx2,fma,f16c"))) inline __m256 ld8_q(const uint8_t* p) {
  int64_t v;
  std::memcpy(&v, p, 8);
  return _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_cvtsi64_si128(v)));
}

// dot4q8avx for one row (same values as dot_q8_avx_row).
__attribute__((target("avx2,fma,f16c"))) inline float dot_q8_row_v(const float* x, const uint8_t* q, int nb) {
  __m256 acc = _mm256_setzero_ps();
  for (int b = 0; b < nb; b++) {
    const uint8_t* blk = q + long(b) * Q8BYTES;
    const float* xs = x + b * QK;
    __m256 y = _mm256_mul_ps(ld8_q(blk + 2), _mm256_loadu_ps(xs));
    y = _mm256_fmadd_ps(ld8_q(blk + 10), _mm256_loadu_ps(xs + 8), y);
    y = _mm256_fmadd_ps(ld8_q(blk + 18), _mm256_loadu_ps(xs + 16), y);
    y = _mm256_fmadd_ps(ld8_q(blk + 26), _mm256_loadu_ps(xs + 24), y);
    const float d = f16_to_f32(uint16_t(blk[0] | blk[1] << 8));
    acc = _mm256_fmadd_ps(y, _mm256_set1_ps(d), acc);
  }
  return hsum8_v(acc);
}

// dot4f32avx for one row over k (a multiple of 16).
__attribute__((target("avx2,fma,f16c"))) inline float dot_f32_row_v(const float* x, const float* w, int k) {
  __m256 a = _mm256_setzero_ps(), b = _mm256_setzero_ps();
  for (int c = 0; c < k; c += 16) {
    a = _mm256_fmadd_ps(_mm256_loadu_ps(x + c), _mm256_loadu_ps(w + c), a);
    b = _mm256_fmadd_ps(_mm256_loadu_ps(x + c + 8), _mm256_loadu_ps(w + c + 8), b);
  }
  return hsum8_v(_mm256_add_ps(a, b));
}

// dot4f16avx for one row over k (a multiple of 16).
__attribute__((target("avx2,fma,f16c"))) inline float dot_f16_row_v(const float* x, const uint16_t* w, int k) {
  __m256 a = _mm256_setzero_ps(), b = _mm256_setzero_ps();
  for (int c = 0; c < k; c += 16) {
    const __m256 w0 = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(w + c)));
    const __m256 w1 = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(w + c + 8)));
    a = _mm256_fmadd_ps(_mm256_loadu_ps(x + c), w0, a);
    b = _mm256_fmadd_ps(_mm256_loadu_ps(x + c + 8), w1, b);
  }
  return hsum8_v(_mm256_add_ps(a, b));
}

// gemvRows for one row of A (same values as gemv_rows), groups of four
// weight rows split over the pool.
inline void gemv_rows_fast(float* y, const float* x, const Weight& w, const float* bias) {
  const int n = w.rows, k = w.cols, groups = (n + 3) / 4;
  auto group = [&](int gi) {
    const int j = gi * 4;
    if (j + 4 <= n) {
      for (int r = 0; r < 4; r++) {
        const int jj = j + r;
        float v;
        switch (w.type) {
          case F16: {
            const int kk = k & ~15;
            v = kk > 0 ? dot_f16_row_v(x, w.h + long(jj) * k, kk) : 0.f;
            if (kk < k) v += dot_f16_go(x + kk, w.h + long(jj) * k + kk, k - kk);
            break;
          }
          case Q8_0:
            v = dot_q8_row_v(x, w.q + long(jj) * (k / QK) * Q8BYTES, k / QK);
            break;
          default: {
            const int kk = k & ~15;
            v = kk > 0 ? dot_f32_row_v(x, w.f + long(jj) * k, kk) : 0.f;
            if (kk < k) v += dot_f32_go(x + kk, w.f + long(jj) * k + kk, k - kk);
          }
        }
        y[jj] = v;
      }
    } else {
      for (int jj = j; jj < n; jj++) {
        switch (w.type) {
          case F16:
            y[jj] = dot_f16_go(x, w.h + long(jj) * k, k);
            break;
          case Q8_0:
            y[jj] = dot_q8_go(x, w.q + long(jj) * (k / QK) * Q8BYTES, k);
            break;
          default:
            y[jj] = dot_f32_go(x, w.f + long(jj) * k, k);
        }
      }
    }
    if (bias)
      for (int jj = j; jj < std::min(j + 4, n); jj++) y[jj] += bias[jj];
  };
  Pool* pool = tl_pool();
  if (pool && pool->size() > 1 && groups >= 16) {
    const int items = std::min(groups, 4 * pool->size());
    pool->run(items, [&](int it) {
      for (int gi = groups * it / items; gi < groups * (it + 1) / items; gi++) group(gi);
    });
  } else {
    for (int gi = 0; gi < groups; gi++) group(gi);
  }
}

inline bool gemv_rows_fast_ok(float* y, const float* x, const Weight& w, const float* bias) {
  if (!cpu_avx2()) return false;
  gemv_rows_fast(y, x, w, bias);
  return true;
}

// whisper/gemm.go:124-209's packed product for rows below m/6·6 (same
// values as matmul_whisper): per output c = bias (or 0), then for each
// 256-deep pass c += the fused chain over that pass; lanes run 16 outputs'
// chains side by side, the weight panel widened to float32 once per pass.
__attribute__((target("avx2,fma,f16c"))) inline void mw_panel(float* c, int ldc, const float* a, int lda, int mfull,
                                                               int n, int k, const Weight& b, int p, float* bt) {
  constexpr int KC = 256;
  const int col0 = p * 16, cols = std::min(16, n - col0);
  for (int k0 = 0; k0 < k; k0 += KC) {
    const int kn = std::min(KC, k - k0);
    for (int kk = 0; kk < kn; kk++)
      for (int j = 0; j < 16; j++) {
        const int col = col0 + j;
        bt[kk * 16 + j] = j < cols ? (b.type == F16 ? f16_to_f32(b.h[long(col) * k + k0 + kk]) : b.f[long(col) * k + k0 + kk])
                                   : 0.f;
      }
    for (int i = 0; i < mfull; i++) {
      const float* ai = a + long(i) * lda + k0;
      __m256 lo = _mm256_setzero_ps(), hi = _mm256_setzero_ps();
      for (int kk = 0; kk < kn; kk++) {
        const __m256 av = _mm256_set1_ps(ai[kk]);
        lo = _mm256_fmadd_ps(av, _mm256_loadu_ps(bt + kk * 16), lo);
        hi = _mm256_fmadd_ps(av, _mm256_loadu_ps(bt + kk * 16 + 8), hi);
      }
      alignas(32) float acc[16];
      _mm256_store_ps(acc, lo);
      _mm256_store_ps(acc + 8, hi);
      float* ci = c + long(i) * ldc + col0;
      for (int j = 0; j < cols; j++) ci[j] = ci[j] + acc[j];
    }
  }
}

inline bool matmul_whisper_fast(float* c, int ldc, const float* a, int lda, int m, int n, int k, const Weight& b,
                                const float* bias) {
  if (!cpu_avx2() || m < 6 || !(b.type == F16 || b.type == F32)) return false;
  const int mfull = m / 6 * 6, np = (n + 15) / 16;
  for (int i = 0; i < mfull; i++)
    for (int j = 0; j < n; j++) c[long(i) * ldc + j] = bias ? bias[j] : 0.f;
  Pool* pool = tl_pool();
  auto run = [&](int p0, int p1) {
    std::vector<float> bt(256 * 16);
    for (int p = p0; p < p1; p++) mw_panel(c, ldc, a, lda, mfull, n, k, b, p, bt.data());
  };
  if (pool && pool->size() > 1 && np > 1) {
    const int items = std::min(np, 4 * pool->size());
    pool->run(items, [&](int it) { run(np * it / items, np * (it + 1) / items); });
  } else {
    run(0, np);
  }
  for (int i = mfull; i < m; i++) gemv_rows_fast(c + long(i) * ldc, a + long(i) * lda, b, bias);
  return true;
}

// kern.Linear with the fast kernels (the dispatch of kern.go:185-201).
inline bool linear_fast(float* dst, const float* x, int m, const Weight& w, const float* bias) {
  if (!cpu_avx2()) return false;
  if (m == 0 || w.rows == 0) return true;
  if (w.type == Q8_0 && (w.dropped || m >= 2)) {
    matmul_q8_int_fast(dst, w.rows, x, w.cols, m, w, bias);
    return true;
  }
  for (int i = 0; i < m; i++) gemv_rows_fast(dst + long(i) * w.rows, x + long(i) * w.cols, w, bias);
  return true;
}

// ------------------------------------------------- exp and activations ---

// EXP8 (same values as exp_avx, lane by lane).
__attribute__((target("avx2,fma,f16c"))) inline __m256 exp8_v(__m256 x) {
  const __m256 log2e = _mm256_set1_ps(bits_f32(0x3fb8aa3b)), ln2hi = _mm256_set1_ps(bits_f32(0x3f317200)),
               ln2lo = _mm256_set1_ps(bits_f32(0x35bfbe8e));
  x = _mm256_max_ps(x, _mm256_set1_ps(-87.f));
  x = _mm256_min_ps(x, _mm256_set1_ps(88.f));
  const __m256 n = _mm256_round_ps(_mm256_mul_ps(x, log2e), _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
  __m256 r = _mm256_fnmadd_ps(n, ln2hi, x);
  r = _mm256_fnmadd_ps(n, ln2lo, r);
  __m256 p = _mm256_fmadd_ps(_mm256_set1_ps(bits_f32(0x3ab60b61)), r, _mm256_set1_ps(bits_f32(0x3c088889)));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(bits_f32(0x3d2aaaab)));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(bits_f32(0x3e2aaaab)));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(0.5f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(1.f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(1.f));
  const __m256i e = _mm256_slli_epi32(_mm256_add_epi32(_mm256_cvttps_epi32(n), _mm256_set1_epi32(127)), 23);
  return _mm256_mul_ps(p, _mm256_castsi256_ps(e));
}

// geluVec (same values as gelu_vec).
__attribute__((target("avx2,fma,f16c"))) inline void gelu_vec_v(float* x, int len) {
  const int n = len & ~7;
  for (int i = 0; i < n; i += 8) {
    const __m256 v = _mm256_loadu_ps(x + i);
    __m256 u = _mm256_mul_ps(v, v);
    u = _mm256_fmadd_ps(_mm256_set1_ps(bits_f32(0x3d372713)), u, _mm256_set1_ps(1.f));
    u = _mm256_mul_ps(v, u);
    u = _mm256_mul_ps(_mm256_set1_ps(bits_f32(0x3f4c422a)), u);
    u = _mm256_min_ps(u, _mm256_set1_ps(9.f));
    u = _mm256_max_ps(u, _mm256_set1_ps(-9.f));
    __m256 e = exp8_v(_mm256_add_ps(u, u));
    e = _mm256_add_ps(e, _mm256_set1_ps(1.f));
    e = _mm256_div_ps(_mm256_set1_ps(2.f), e);
    e = _mm256_sub_ps(_mm256_set1_ps(1.f), e);
    e = _mm256_add_ps(e, _mm256_set1_ps(1.f));
    e = _mm256_mul_ps(e, v);
    _mm256_storeu_ps(x + i, _mm256_mul_ps(e, _mm256_set1_ps(0.5f)));
  }
  for (int i = n; i < len; i++) x[i] = gelu_go(x[i]);
}

// siluVec (same values as silu_vec).
__attribute__((target("avx2,fma,f16c"))) inline void silu_vec_v(float* x, int len) {
  const int n = len & ~7;
  for (int i = 0; i < n; i += 8) {
    const __m256 v = _mm256_loadu_ps(x + i);
    const __m256 e = exp8_v(_mm256_sub_ps(_mm256_setzero_ps(), v));
    _mm256_storeu_ps(x + i, _mm256_div_ps(v, _mm256_add_ps(e, _mm256_set1_ps(1.f))));
  }
  for (int i = n; i < len; i++) x[i] = silu_go(x[i]);
}

inline bool gelu_vec_fast(float* x, int len) {
  if (!cpu_avx2()) return false;
  gelu_vec_v(x, len);
  return true;
}
inline bool silu_vec_fast(float* x, int len) {
  if (!cpu_avx2()) return false;
  silu_vec_v(x, len);
  return true;
}

// expSub (same value and outputs as expsub_vec).
__attribute__((target("avx2,fma,f16c"))) inline float expsub_fast(float* x, int len, float mx) {
  const int n = len & ~7;
  float s = 0.f;
  if (n > 0) {
    __m256 acc = _mm256_setzero_ps();
    const __m256 m = _mm256_set1_ps(mx);
    for (int c = 0; c < n; c += 8) {
      const __m256 e = exp8_v(_mm256_sub_ps(_mm256_loadu_ps(x + c), m));
      _mm256_storeu_ps(x + c, e);
      acc = _mm256_add_ps(acc, e);
    }
    s = hsum8_v(acc);
  }
  float t = 0.f;
  for (int i = n; i < len; i++) {
    const float e = expf_go(x[i] - mx);
    x[i] = e;
    t += e;
  }
  return s + t;
}

// attend_one with the fast kernels (same values), heads split over the pool.
__attribute__((target("avx2,fma,f16c"))) inline void attend_head_fast(float* out, const float* q, const float* kc,
                                                                       const float* vc, int nk, int d, int hd, int h,
                                                                       float scale, float* sc) {
  const float* qh = q + h * hd;
  const int kk = hd & ~15;
  for (int j = 0; j < nk; j++) {
    const float* kj = kc + long(j) * d + h * hd;
    if ((j & ~3) + 4 <= nk) {  // a key of a group of four: dotF32x4
      float v = kk > 0 ? dot_f32_row_v(qh, kj, kk) : 0.f;
      if (kk < hd) v += dot_f32_go(qh + kk, kj + kk, hd - kk);
      sc[j] = v;
    } else {
      sc[j] = dot_f32_go(qh, kj, hd);
    }
  }
  float mx = -INFINITY;
  for (int j = 0; j < nk; j++) {
    sc[j] *= scale;
    mx = std::max(mx, sc[j]);
  }
  const float inv = 1.f / expsub_fast(sc, nk, mx);
  for (int j = 0; j < nk; j++) sc[j] *= inv;
  float* o = out + h * hd;
  if (hd % 8 == 0) {
    __m256 acc[16];
    const int nv = hd / 8;
    for (int i = 0; i < nv && i < 16; i++) acc[i] = _mm256_setzero_ps();
    if (nv <= 16) {
      for (int j = 0; j < nk; j++) {
        const float w = sc[j];
        if (w == 0) continue;
        const __m256 wv = _mm256_set1_ps(w);
        const float* vj = vc + long(j) * d + h * hd;
        for (int i = 0; i < nv; i++) acc[i] = _mm256_fmadd_ps(wv, _mm256_loadu_ps(vj + 8 * i), acc[i]);
      }
      for (int i = 0; i < nv; i++) _mm256_storeu_ps(o + 8 * i, acc[i]);
      return;
    }
  }
  for (int i = 0; i < hd; i++) o[i] = 0;
  for (int j = 0; j < nk; j++) {
    const float w = sc[j];
    if (w != 0) {
      const float* vj = vc + long(j) * d + h * hd;
      for (int i = 0; i < hd; i++) o[i] = std::fma(w, vj[i], o[i]);
    }
  }
}

inline bool attend_one_fast(float* out, const float* q, const float* kc, const float* vc, int nk, int d, int heads) {
  if (!cpu_avx2()) return false;
  const int hd = d / heads;
  const float scale = float(1 / std::sqrt(double(hd)));
  Pool* pool = tl_pool();
  if (pool && pool->size() > 1) {
    pool->run(heads, [&](int h) {
      std::vector<float> sc(size_t(nk) + 8);
      attend_head_fast(out, q, kc, vc, nk, d, hd, h, scale, sc.data());
    });
  } else {
    std::vector<float> sc(size_t(nk) + 8);
    for (int h = 0; h < heads; h++) attend_head_fast(out, q, kc, vc, nk, d, hd, h, scale, sc.data());
  }
  return true;
}

}  // namespace orc
