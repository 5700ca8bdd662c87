// TEST INFRASTRUCTURE — the CPU oracle of the Whisper text decoder's token
// loop (whisper/decoder.go, encoder.go:120-140, transcribe.go:370-494) and
// of the audio encoder (encoder.go:10-118).
// Only tests, the smoke check and the benchmark's CPU baseline use it.
//
// Restated from the reference operation by operation on the kernels of
// kern.h, which whisper/kernels_amd64.s repeats (dot4f16avx, dot4f32avx,
// EXP8, geluAVX are the same instruction sequences):
//  * weights are float16 in memory (model.go:424-447): a Q8_0 block widens
//    as f32toF16(float(int8 q) · f16tab[d]) (model.go:486-490, f16.go:36-71);
//  * matmul (gemm.go:124-209): fewer than 6 rows → gemv per row (dotF16x4
//    per four weight rows, dotF16Go for the rest, then + bias); 6 or more →
//    the packed kernel: C starts at the bias, and per 256-deep pass gets
//    += the fused chain over that pass (k6x16avx, kernels_amd64.s:5-86);
//  * layerNorm (mathx.go:55-75): float64 sums, mean and 1/sd cast to
//    float32, ((v − mean)·inv)·w + b in float32;
//  * softmax (mathx.go:78-90): EXP8 lanes for the first len&~7 values, Go
//    expf for the rest, × (1/Σ);
//  * decode (decoder.go:33-140), cross K/V (encoder.go:120-140), process
//    and sample at temperature 0 (transcribe.go:370-520).
#pragma once

#include <cmath>
#include <limits>
#include <string>
#include <vector>

#include "kern.h"

namespace orc {

// Q8_0 block → float16 values, model.go:486-490 then f32toF16.
inline void q8_to_f16(const uint8_t* blocks, long n, uint16_t* out) {
  for (long b = 0; b < n / QK; b++) {
    const uint8_t* blk = blocks + b * Q8BYTES;
    const float dd = f16_to_f32(uint16_t(blk[0] | blk[1] << 8));
    for (int j = 0; j < QK; j++) out[b * QK + j] = f32_to_f16(float(int8_t(blk[2 + j])) * dd);
  }
}

// layerNorm, whisper/mathx.go:55-75.
inline void ln_whisper(float* y, const float* x, int n, const float* w, const float* b) {
  double sum = 0;
  for (int i = 0; i < n; i++) sum += double(x[i]);
  const float mean = float(sum / double(n));
  double vs = 0;
  for (int i = 0; i < n; i++) {
    const double d = double(x[i] - mean);
    vs += d * d;
  }
  const float inv = float(1.0 / std::sqrt(vs / double(n) + 1e-5));
  for (int i = 0; i < n; i++) y[i] = (x[i] - mean) * inv * w[i] + b[i];
}

// softmax, whisper/mathx.go:78-90.
inline void softmax_whisper(float* x, int n) {
  float mx = -std::numeric_limits<float>::infinity();
  for (int i = 0; i < n; i++)
    if (x[i] > mx) mx = x[i];
  const float s = expsub_vec(x, n, mx);
  const float inv = 1.f / s;
  for (int i = 0; i < n; i++) x[i] *= inv;
}

// matmul, whisper/gemm.go:124-209: C[m][n] = A[m][k]·Bᵀ + bias, B F16 or F32.
inline bool matmul_whisper_fast(float* c, int ldc, const float* a, int lda, int m, int n, int k, const Weight& b,
                                const float* bias);

inline void matmul_whisper(float* c, int ldc, const float* a, int lda, int m, int n, int k, const Weight& b,
                           const float* bias) {
  if (fast_on() && matmul_whisper_fast(c, ldc, a, lda, m, n, k, b, bias)) return;
  const int MR = 6, NR = 16, KC = 256;
  auto brow = [&](int col, int kk) { return b.type == F16 ? f16_to_f32(b.h[long(col) * k + kk]) : b.f[long(col) * k + kk]; };
  if (m < MR) {
    for (int i = 0; i < m; i++) gemv_rows(c + long(i) * ldc, a + long(i) * lda, b, bias);
    return;
  }
  const int mfull = m / MR * MR;
  for (int i = 0; i < mfull; i++)
    for (int j = 0; j < n; j++) c[long(i) * ldc + j] = bias ? bias[j] : 0.f;
  for (int k0 = 0; k0 < k; k0 += KC) {
    const int kn = std::min(KC, k - k0);
    for (int p = 0; p * NR < n; p++)
      for (int i = 0; i < mfull; i++)
        for (int j = 0; j < NR; j++) {
          const int col = p * NR + j;
          float acc = 0.f;
          for (int kk = 0; kk < kn; kk++)
            acc = std::fma(a[long(i) * lda + k0 + kk], col < n ? brow(col, k0 + kk) : 0.f, acc);
          if (col < n) c[long(i) * ldc + col] = c[long(i) * ldc + col] + acc;
        }
  }
  for (int i = mfull; i < m; i++) gemv_rows(c + long(i) * ldc, a + long(i) * lda, b, bias);
}

struct WLayer {
  const float *attn_ln_w = nullptr, *attn_ln_b = nullptr;
  Weight q, k, v, o;
  const float *qb = nullptr, *vb = nullptr, *ob = nullptr;
  const float *x_ln_w = nullptr, *x_ln_b = nullptr;
  Weight xq, xk, xv, xo;
  const float *xqb = nullptr, *xvb = nullptr, *xob = nullptr;
  const float *mlp_ln_w = nullptr, *mlp_ln_b = nullptr;
  Weight fc1, fc2;
  const float *fc1b = nullptr, *fc2b = nullptr;
};

// The vocabulary's special tokens (vocab.go:19-43).
struct WVocab {
  int n = 0, n_lang = 0, eot = 0, sot = 0, translate = 0, transcribe = 0, solm = 0, prev = 0, nosp = 0, not_ = 0,
      beg = 0, space = -1;
  std::vector<int> suppress;  // vocab.suppressed(), vocab.go:103-118
  void init(int n_vocab) {
    n = n_vocab;
    eot = 50256, sot = 50257;
    translate = 50357, transcribe = 50358, solm = 50359, prev = 50360, nosp = 50361, not_ = 50362, beg = 50363;
    if (n_vocab >= 51865) {
      n_lang = n_vocab - 51765 - 1;
      const int dt = n_lang - 98;
      eot++, sot++;
      translate += dt, transcribe += dt, solm += dt, prev += dt, nosp += dt, not_ += dt, beg += dt;
    }
  }
};

// An encoder block (model.go:360-372).
struct WEncLayer {
  const float *attn_ln_w = nullptr, *attn_ln_b = nullptr;
  Weight q, k, v, o;
  const float *qb = nullptr, *vb = nullptr, *ob = nullptr;
  const float *mlp_ln_w = nullptr, *mlp_ln_b = nullptr;
  Weight fc1, fc2;
  const float *fc1b = nullptr, *fc2b = nullptr;
};

struct Whisper {
  int n_vocab = 0, n_audio_ctx = 1500, n_text_ctx = 0, n_state = 0, n_head = 0;
  // the audio encoder (model.go:352-372), when bound
  int n_mels = 0, n_audio_head = 0;
  Weight conv1, conv2;  // [state][n_mels·3], [state][state·3] F16
  const float *conv1b = nullptr, *conv2b = nullptr, *enc_pos = nullptr, *enc_ln_w = nullptr, *enc_ln_b = nullptr;
  std::vector<WEncLayer> enc;
  const float* dec_pos = nullptr;  // [n_text_ctx][n_state]
  Weight tok_emb;                  // [n_vocab][n_state] F16
  const float *ln_w = nullptr, *ln_b = nullptr;
  std::vector<WLayer> layers;
  WVocab voc;
};

// One decoding sequence: self-attention cache and this window's cross K/V.
struct WSeq {
  std::vector<std::vector<float>> sk, sv;  // [layer][n_text_ctx·n_state]
  int n = 0;
  std::vector<std::vector<float>> ck, cv;  // [layer][heads·ctx·hd] (V transposed per head)
  void init(const Whisper& m) {
    sk.assign(m.layers.size(), std::vector<float>(size_t(m.n_text_ctx) * m.n_state, 0.f));
    sv = sk;
    ck.assign(m.layers.size(), std::vector<float>(size_t(m.n_audio_ctx) * m.n_state, 0.f));
    cv = ck;
    n = 0;
  }
};

// parGelu, encoder.go:147-151: geluVec over chunks of 2^14 values.
inline void par_gelu(float* x, long n) {
  const long chunk = 1 << 14;
  for (long o = 0; o < n; o += chunk) gelu_vec(x + o, int(std::min(chunk, n - o)));
}

// encode, whisper/encoder.go:10-118: a window's log-mel [n_mels][3000]
// (channel-major) → the encoder output [n_audio_ctx][state]. max_blocks ≥ 0
// runs only that many blocks (for timing a bounded sample).
inline void whisper_encode(const Whisper& m, const float* mel, float* out, int max_blocks = -1) {
  const int st = m.n_state, nmel = m.n_mels, W = 3000, ctx = m.n_audio_ctx;
  // conv1: 3 taps, stride 1, padding 1; a row is (channel, tap) → c·3 + k
  const int cols1 = nmel * 3;
  std::vector<float> x1(size_t(W) * cols1, 0.f), h1(size_t(W) * st);
  for (int t = 0; t < W; t++)
    for (int c = 0; c < nmel; c++)
      for (int k = 0; k < 3; k++)
        if (t + k - 1 >= 0 && t + k - 1 < W) x1[size_t(t) * cols1 + c * 3 + k] = mel[size_t(c) * W + t + k - 1];
  matmul_whisper(h1.data(), st, x1.data(), cols1, W, st, cols1, m.conv1, m.conv1b);
  par_gelu(h1.data(), long(h1.size()));
  // conv2: 3 taps, stride 2, padding 1, down to ctx positions
  const int cols2 = st * 3;
  std::vector<float> x2(size_t(ctx) * cols2, 0.f), x(size_t(ctx) * st);
  for (int t = 0; t < ctx; t++)
    for (int k = 0; k < 3; k++) {
      const int i = 2 * t + k - 1;
      if (i < 0 || i >= W) continue;
      for (int c = 0; c < st; c++) x2[size_t(t) * cols2 + c * 3 + k] = h1[size_t(i) * st + c];
    }
  matmul_whisper(x.data(), st, x2.data(), cols2, ctx, st, cols2, m.conv2, m.conv2b);
  par_gelu(x.data(), long(x.size()));
  for (size_t i = 0; i < x.size(); i++) x[i] += m.enc_pos[i];
  const int nh = m.n_audio_head, hd = st / nh;
  const float sc = float(1 / std::sqrt(double(hd)));
  std::vector<float> cur(x.size()), q(x.size()), k(x.size()), v(x.size()), att(x.size()), ff(size_t(ctx) * 4 * st);
  std::vector<float> qh(size_t(ctx) * hd), kh(size_t(ctx) * hd), vt(size_t(hd) * ctx), oh(size_t(ctx) * hd);
  std::vector<float> scores(size_t(ctx) * ctx);
  Weight wk, wv;
  wk.type = wv.type = F32;
  wk.rows = ctx, wk.cols = hd, wk.f = kh.data();
  wv.rows = hd, wv.cols = ctx, wv.f = vt.data();
  auto ln_rows = [&](float* y, const float* src, const float* w, const float* b) {
    for (int t = 0; t < ctx; t++) ln_whisper(y + size_t(t) * st, src + size_t(t) * st, st, w, b);
  };
  int nb = 0;
  for (const WEncLayer& L : m.enc) {
    if (max_blocks >= 0 && nb++ >= max_blocks) break;  // a timing sample only
    ln_rows(cur.data(), x.data(), L.attn_ln_w, L.attn_ln_b);
    matmul_whisper(q.data(), st, cur.data(), st, ctx, st, st, L.q, L.qb);
    matmul_whisper(k.data(), st, cur.data(), st, ctx, st, st, L.k, nullptr);
    matmul_whisper(v.data(), st, cur.data(), st, ctx, st, st, L.v, L.vb);
    for (int h = 0; h < nh; h++) {
      for (int t = 0; t < ctx; t++)
        for (int d = 0; d < hd; d++) {
          qh[size_t(t) * hd + d] = q[size_t(t) * st + h * hd + d] * sc;  // copy, then scale(qh, sc)
          kh[size_t(t) * hd + d] = k[size_t(t) * st + h * hd + d];
          vt[size_t(d) * ctx + t] = v[size_t(t) * st + h * hd + d];
        }
      matmul_whisper(scores.data(), ctx, qh.data(), hd, ctx, ctx, hd, wk, nullptr);
      for (int t = 0; t < ctx; t++) softmax_whisper(scores.data() + size_t(t) * ctx, ctx);
      matmul_whisper(oh.data(), hd, scores.data(), ctx, ctx, hd, ctx, wv, nullptr);
      for (int t = 0; t < ctx; t++)
        for (int d = 0; d < hd; d++) att[size_t(t) * st + h * hd + d] = oh[size_t(t) * hd + d];
    }
    matmul_whisper(cur.data(), st, att.data(), st, ctx, st, st, L.o, L.ob);
    for (size_t i = 0; i < x.size(); i++) x[i] += cur[i];
    ln_rows(cur.data(), x.data(), L.mlp_ln_w, L.mlp_ln_b);
    matmul_whisper(ff.data(), 4 * st, cur.data(), st, ctx, 4 * st, st, L.fc1, L.fc1b);
    par_gelu(ff.data(), long(ff.size()));
    matmul_whisper(cur.data(), st, ff.data(), 4 * st, ctx, st, 4 * st, L.fc2, L.fc2b);
    for (size_t i = 0; i < x.size(); i++) x[i] += cur[i];
  }
  ln_rows(out, x.data(), m.enc_ln_w, m.enc_ln_b);
}

// encoder.go:120-140: cross keys (scaled by 1/√hd) and values from the
// encoder output enc [ctx][state].
inline void whisper_cross_kv(const Whisper& m, WSeq& s, const float* enc) {
  const int st = m.n_state, ctx = m.n_audio_ctx, nh = m.n_head, hd = st / nh;
  const float tsc = float(1 / std::sqrt(double(hd)));
  std::vector<float> k(size_t(ctx) * st), v(size_t(ctx) * st);
  for (size_t li = 0; li < m.layers.size(); li++) {
    const WLayer& L = m.layers[li];
    matmul_whisper(k.data(), st, enc, st, ctx, st, st, L.xk, nullptr);
    matmul_whisper(v.data(), st, enc, st, ctx, st, st, L.xv, L.xvb);
    for (int h = 0; h < nh; h++)
      for (int t = 0; t < ctx; t++)
        for (int d = 0; d < hd; d++) {
          s.ck[li][size_t(h) * ctx * hd + size_t(t) * hd + d] = k[size_t(t) * st + h * hd + d] * tsc;
          s.cv[li][size_t(h) * ctx * hd + size_t(d) * ctx + t] = v[size_t(t) * st + h * hd + d];
        }
  }
}

// decode, decoder.go:33-140: runs tokens after the cache's positions;
// logits of the rows listed in want. Returns false if the context is full.
inline bool whisper_decode(const Whisper& m, WSeq& s, const int* tokens, int nt, const int* want, int nwant,
                           float* logits_out) {
  const int st = m.n_state, nh = m.n_head, hd = st / nh, ctx = m.n_audio_ctx, pos0 = s.n;
  if (pos0 + nt > m.n_text_ctx) return false;
  const float sc = float(1 / std::sqrt(double(hd)));
  std::vector<float> x(size_t(nt) * st), cur(x.size()), q(x.size()), att(x.size()), kn(x.size()), vn(x.size()),
      ff(size_t(nt) * 4 * st), sbuf(size_t(std::max(ctx, pos0 + nt)));
  for (int i = 0; i < nt; i++)
    for (int j = 0; j < st; j++)
      x[size_t(i) * st + j] =
          f16_to_f32(m.tok_emb.h[size_t(tokens[i]) * st + j]) + m.dec_pos[size_t(pos0 + i) * st + j];
  for (size_t li = 0; li < m.layers.size(); li++) {
    const WLayer& L = m.layers[li];
    for (int i = 0; i < nt; i++) ln_whisper(&cur[size_t(i) * st], &x[size_t(i) * st], st, L.attn_ln_w, L.attn_ln_b);
    matmul_whisper(q.data(), st, cur.data(), st, nt, st, st, L.q, L.qb);
    matmul_whisper(kn.data(), st, cur.data(), st, nt, st, st, L.k, nullptr);
    matmul_whisper(vn.data(), st, cur.data(), st, nt, st, st, L.v, L.vb);
    float* ck = s.sk[li].data();
    float* cvv = s.sv[li].data();
    std::copy(kn.begin(), kn.end(), ck + size_t(pos0) * st);
    std::copy(vn.begin(), vn.end(), cvv + size_t(pos0) * st);
    for (int i = 0; i < nt; i++)
      for (int h = 0; h < nh; h++) {
        const int n = pos0 + i + 1;
        float* sc_ = sbuf.data();
        const float* qi = &q[size_t(i) * st + h * hd];
        for (int j = 0; j < n; j++) sc_[j] = dot_f32_go(qi, ck + size_t(j) * st + h * hd, hd) * sc;
        softmax_whisper(sc_, n);
        float* out = &att[size_t(i) * st + h * hd];
        for (int d = 0; d < hd; d++) out[d] = 0.f;
        for (int j = 0; j < n; j++) {
          const float* vj = cvv + size_t(j) * st + h * hd;
          for (int d = 0; d < hd; d++) out[d] += sc_[j] * vj[d];
        }
      }
    matmul_whisper(cur.data(), st, att.data(), st, nt, st, st, L.o, L.ob);
    add_to(x.data(), cur.data(), nt * st);
    // cross-attention
    for (int i = 0; i < nt; i++) ln_whisper(&cur[size_t(i) * st], &x[size_t(i) * st], st, L.x_ln_w, L.x_ln_b);
    matmul_whisper(q.data(), st, cur.data(), st, nt, st, st, L.xq, L.xqb);
    for (int i = 0; i < nt; i++)
      for (int h = 0; h < nh; h++) {
        const float* kd = &s.ck[li][size_t(h) * ctx * hd];
        const float* vd = &s.cv[li][size_t(h) * ctx * hd];
        const float* qi = &q[size_t(i) * st + h * hd];
        float* sc_ = sbuf.data();
        float o4[4];
        int j = 0;
        for (; j + 4 <= ctx; j += 4) {
          dot_f32x4(qi, kd + size_t(j) * hd, hd, hd, o4);
          for (int r = 0; r < 4; r++) sc_[j + r] = o4[r];
        }
        for (; j < ctx; j++) sc_[j] = dot_f32_go(qi, kd + size_t(j) * hd, hd);
        softmax_whisper(sc_, ctx);
        float* out = &att[size_t(i) * st + h * hd];
        int d = 0;
        for (; d + 4 <= hd; d += 4) {
          dot_f32x4(sc_, vd + size_t(d) * ctx, ctx, ctx, o4);
          for (int r = 0; r < 4; r++) out[d + r] = o4[r];
        }
        for (; d < hd; d++) out[d] = dot_f32_go(sc_, vd + size_t(d) * ctx, ctx);
      }
    matmul_whisper(cur.data(), st, att.data(), st, nt, st, st, L.xo, L.xob);
    add_to(x.data(), cur.data(), nt * st);
    // feed-forward
    for (int i = 0; i < nt; i++) ln_whisper(&cur[size_t(i) * st], &x[size_t(i) * st], st, L.mlp_ln_w, L.mlp_ln_b);
    matmul_whisper(ff.data(), 4 * st, cur.data(), st, nt, 4 * st, st, L.fc1, L.fc1b);
    gelu_vec(ff.data(), nt * 4 * st);
    matmul_whisper(cur.data(), st, ff.data(), 4 * st, nt, st, 4 * st, L.fc2, L.fc2b);
    add_to(x.data(), cur.data(), nt * st);
  }
  s.n = pos0 + nt;
  std::vector<float> row((size_t)st);
  for (int w = 0; w < nwant; w++) {
    ln_whisper(row.data(), &x[size_t(want[w]) * st], st, m.ln_w, m.ln_b);
    gemv_rows(logits_out + size_t(w) * m.n_vocab, row.data(), m.tok_emb, nullptr);
  }
  return true;
}

// A sequence's sampling state (transcribe.go:56-64): what process needs.
struct WSampleState {
  int nt = 0;                 // tokens sampled so far
  int last = -1, penult = -1;  // the last two of them
  bool has_ts = false;
  int seek_delta = 3000;  // winFrames
};

struct WToken {
  int id, tid;
  float p, plog;
};

// logSoftmax, transcribe.go:496-515.
inline void log_softmax_w(float* dst, const float* x, int n) {
  const float ninf = -std::numeric_limits<float>::infinity();
  float mx = ninf;
  for (int i = 0; i < n; i++) mx = std::max(mx, x[i]);
  float s = 0.f;
  for (int i = 0; i < n; i++)
    if (x[i] > ninf) s += expf_go(x[i] - mx);
  const float ls = float(std::log(double(s))) + mx;
  for (int i = 0; i < n; i++) dst[i] = x[i] > ninf ? x[i] - ls : ninf;
}

// softmaxInf, transcribe.go:517-535.
inline void softmax_inf(float* x, int n) {
  const float ninf = -std::numeric_limits<float>::infinity();
  float mx = ninf;
  for (int i = 0; i < n; i++) mx = std::max(mx, x[i]);
  float s = 0.f;
  for (int i = 0; i < n; i++) {
    if (x[i] > ninf) {
      const float e = expf_go(x[i] - mx);
      x[i] = e;
      s += e;
    } else {
      x[i] = 0.f;
    }
  }
  for (int i = 0; i < n; i++) x[i] /= s;
}

// process then sample at temperature 0 (transcribe.go:370-494): the rules
// on lg (modified in place), then the most likely token and timestamp.
inline WToken whisper_process_sample(const Whisper& m, const WSampleState& q, float* lg) {
  const WVocab& v = m.voc;
  const int n = m.n_vocab;
  const float ninf = -std::numeric_limits<float>::infinity();
  const bool initial = q.nt == 0;
  if (initial) {
    lg[v.eot] = ninf;
    if (v.space >= 0) lg[v.space] = ninf;
  }
  lg[v.not_] = ninf;
  lg[v.sot] = lg[v.nosp] = lg[v.solm] = ninf;
  lg[v.translate] = lg[v.transcribe] = lg[v.prev] = ninf;
  for (int i = 0; i < v.n_lang; i++) lg[v.sot + 1 + i] = ninf;
  for (int t : v.suppress) lg[t] = ninf;
  const bool last = q.nt > 0 && q.last >= v.beg;
  const bool penult = q.nt < 2 || q.penult >= v.beg;
  if (last) {
    if (penult)
      for (int i = v.beg; i < n; i++) lg[i] = ninf;
    else
      for (int i = 0; i < v.eot; i++) lg[i] = ninf;
  }
  if (initial) {
    const double prec = 30.0 / double(m.n_audio_ctx);
    const int tid0 = int(std::round(1.0 / prec));
    for (int i = v.beg + tid0 + 1; i < n; i++) lg[i] = ninf;
  }
  if (q.has_ts)
    for (int i = v.beg; i < v.beg + q.seek_delta / 2 && i < n; i++) lg[i] = ninf;
  std::vector<float> logprobs((size_t)n), probs((size_t)n);
  log_softmax_w(logprobs.data(), lg, n);
  float ts_max = ninf;
  for (int i = v.beg; i < n; i++) ts_max = std::max(ts_max, logprobs[size_t(i)]);
  if (ts_max > ninf) {
    float sum = 0.f;
    for (int i = v.beg; i < n; i++)
      if (logprobs[size_t(i)] > ninf) sum += expf_go(logprobs[size_t(i)] - ts_max);
    const float ts_lp = float(std::log(double(sum))) + ts_max;
    float text_max = ninf;
    for (int i = 0; i < v.beg; i++) text_max = std::max(text_max, logprobs[size_t(i)]);
    if (ts_lp > text_max)
      for (int i = 0; i < v.beg; i++) lg[i] = logprobs[size_t(i)] = ninf;
  }
  for (int i = 0; i < n; i++) probs[size_t(i)] = lg[i];
  softmax_inf(probs.data(), n);
  int id = 0;
  for (int i = 0; i < n; i++)
    if (probs[size_t(i)] > probs[size_t(id)]) id = i;
  int tid = v.beg;
  for (int i = v.beg; i < n; i++)
    if (probs[size_t(i)] > probs[size_t(tid)]) tid = i;
  if (id >= v.beg) tid = id;
  return {id, tid, probs[size_t(id)], logprobs[size_t(id)]};
}

// The window loop's bookkeeping after a sampled token (transcribe.go:
// 218-224) that process depends on.
inline void whisper_after_sample(const Whisper& m, WSampleState& q, const WToken& t, int i) {
  q.penult = q.last;
  q.last = t.id;
  q.nt++;
  if (t.id > m.voc.beg) {
    q.seek_delta = 2 * (t.id - m.voc.beg);
    q.has_ts = true;
  }
  (void)i;
}

// A fixed-length greedy run (the C2 benchmark loop): decode the prompt,
// keep the no-speech probability of row sot_at, then `steps` rounds of
// process/sample → decode of the sampled token. Returns the tokens (the
// window's stop rules are the caller's; this loop does not stop).
inline std::vector<WToken> whisper_greedy(const Whisper& m, WSeq& s, const int* prompt, int np, int sot_at, int steps,
                                          float* no_speech) {
  std::vector<float> lg(size_t(2) * m.n_vocab);
  const int want[2] = {sot_at, np - 1};
  std::vector<WToken> out;
  if (!whisper_decode(m, s, prompt, np, want, 2, lg.data())) return out;
  {
    std::vector<float> p(lg.begin(), lg.begin() + m.n_vocab);
    softmax_whisper(p.data(), m.n_vocab);
    if (no_speech) *no_speech = p[size_t(m.voc.nosp)];
  }
  WSampleState q;
  std::vector<float> cur(lg.begin() + m.n_vocab, lg.end());
  for (int i = 0; i < steps; i++) {
    const WToken t = whisper_process_sample(m, q, cur.data());
    out.push_back(t);
    whisper_after_sample(m, q, t, i);
    if (i + 1 == steps) break;
    const int want0 = 0;
    if (!whisper_decode(m, s, &t.id, 1, &want0, 1, cur.data())) break;
  }
  return out;
}

}  // namespace orc
