// TEST INFRASTRUCTURE ONLY: the CPU oracle of the FastConformer encoder
// (conformer/encoder.go:41-480, model.go:350-410) for the offline case —
// "regular" attention over all frames, centred depthwise convolution,
// non-causal subsampling — restated operation by operation on kern.h and
// flowlm.h. Only tests/ and the benchmark's CPU baseline use it. Checked
// against a float64 encoder; parity against reference outputs unpinned (the
// reference's encoder tests need model dumps that are not in the tree).
// The position table's sin/cos are glibc's where the reference calls Go's
// math package: the same to the last float64 ulp or nearly, not pinned.
#pragma once
#include <cmath>
#include <limits>
#include <vector>

#include "flowlm.h"
#include "whisper.h"

namespace orc {

// The Conformer's weights (model.go:48-76) as the loader leaves them: every
// matrix packed with its rows dropped (so the int8 path), the 1×1
// convolutions rounded to Q8_0 by ToQ8 when the file keeps them float16,
// the taps of the subsampling and depthwise convolutions transposed to
// [taps][channels], batch norm folded into a scale and bias.
struct CFF {
  const float *norm_w = nullptr, *norm_b = nullptr;
  Weight w1, w2;
  const float *b1 = nullptr, *b2 = nullptr;
};

struct CBlock {
  CFF ff1, ff2;
  const float *norm_att_w = nullptr, *norm_att_b = nullptr;
  Weight q, k, v, out, pos;
  const float *qb = nullptr, *kb = nullptr, *vb = nullptr, *outb = nullptr;
  const float *pos_u = nullptr, *pos_v = nullptr;
  const float *norm_conv_w = nullptr, *norm_conv_b = nullptr;
  Weight pw1, pw2;
  const float *pw1b = nullptr, *pw2b = nullptr;
  std::vector<float> dw;  // [kernel][d]
  const float* dwb = nullptr;
  std::vector<float> cn_w, cn_b;
  const float *norm_out_w = nullptr, *norm_out_b = nullptr;
};

struct Conformer {
  int d = 0, heads = 0, dff = 0, kernel = 0, sub_c = 0, n_mels = 0;
  bool xscaling = false, ln_conv = false;
  std::vector<float> w0, w2, w5;  // [9][c]
  const float *b0 = nullptr, *b2 = nullptr, *b5 = nullptr, *b3 = nullptr, *b6 = nullptr, *outb = nullptr;
  Weight w3, w6, out;
  std::vector<CBlock> blocks;
};

// subOut (encoder.go:32-39), non-causal.
inline int sub_out(int n) { return (n - 1) / 2 + 1; }

// AddScaled → axpy (kernels_amd64.go:252-262): fused for the first len&~7
// values (axpyAVX), Go's unfused dst += s·src for the rest.
inline void axpy_vec(float* dst, const float* src, int len, float s) {
  const int n = len & ~7;
  for (int i = 0; i < n; i++) dst[i] = std::fma(src[i], s, dst[i]);
  for (int i = n; i < len; i++) dst[i] += s * src[i];
}

// reluVec: max(v, 0) keeping −0 and NaN (VMAXPS with the value second;
// Go's v < 0 → 0).
inline void relu_vec(float* x, long len) {
  for (long i = 0; i < len; i++)
    if (x[i] < 0) x[i] = 0.f;
}

inline void mask_rows(float* x, int rows, int valid, long width) {
  for (long i = long(std::max(valid, 0)) * width; i < long(rows) * width; i++) x[i] = 0.f;
}

// conv0 (encoder.go:41-75): one plane [T][F] to c channels [T1][F1][c].
inline std::vector<float> conv0(const float* in, int T, int F, const std::vector<float>& w, const float* b, int c,
                                int* T1o, int* F1o) {
  const int T1 = sub_out(T), F1 = sub_out(F);
  std::vector<float> out(size_t(T1) * F1 * c);
  for (int t = 0; t < T1; t++)
    for (int f = 0; f < F1; f++) {
      float taps[9];
      for (int kt = 0; kt < 3; kt++)
        for (int kf = 0; kf < 3; kf++) {
          const int ti = 2 * t + kt - 1, fi = 2 * f + kf - 1;
          taps[kt * 3 + kf] = ti >= 0 && ti < T && fi >= 0 && fi < F ? in[size_t(ti) * F + fi] : 0.f;
        }
      float* o = &out[(size_t(t) * F1 + f) * c];
      std::copy(b, b + c, o);
      for (int j = 0; j < 9; j++)
        if (taps[j] != 0) axpy_vec(o, &w[size_t(j) * c], c, taps[j]);
    }
  *T1o = T1, *F1o = F1;
  return out;
}

// dwConv2 (encoder.go:77-111): depthwise 3×3 stride 2 on [T][F][c].
inline std::vector<float> dw_conv2(const float* in, int T, int F, int c, const std::vector<float>& w, const float* b,
                                   int* T1o, int* F1o) {
  const int T1 = sub_out(T), F1 = sub_out(F);
  std::vector<float> out(size_t(T1) * F1 * c);
  for (int t = 0; t < T1; t++)
    for (int f = 0; f < F1; f++) {
      float* o = &out[(size_t(t) * F1 + f) * c];
      std::copy(b, b + c, o);
      for (int kt = 0; kt < 3; kt++) {
        const int ti = 2 * t + kt - 1;
        if (ti < 0 || ti >= T) continue;
        for (int kf = 0; kf < 3; kf++) {
          const int fi = 2 * f + kf - 1;
          if (fi < 0 || fi >= F) continue;
          const float* x = &in[(size_t(ti) * F + fi) * c];
          const float* wk = &w[size_t(kt * 3 + kf) * c];
          for (int i = 0; i < c; i++) o[i] += wk[i] * x[i];
        }
      }
    }
  *T1o = T1, *F1o = F1;
  return out;
}

inline void lin(float* dst, const float* x, int m, const Weight& w, const float* bias) {
  Weight d = w;
  d.dropped = true;
  linear(dst, x, m, d, bias);
}

// subsample (encoder.go:123-168): log-mel [mels][frames] (the first valid
// real) → [T][d] and its valid length.
inline std::vector<float> conformer_subsample(const Conformer& m, const float* mel, int frames, int valid, int* To,
                                              int* Lo) {
  const int nm = m.n_mels, c = m.sub_c;
  std::vector<float> in(size_t(frames) * nm, 0.f);
  for (int f = 0; f < nm; f++)
    for (int t = 0; t < std::min(frames, valid); t++) in[size_t(t) * nm + f] = mel[size_t(f) * frames + t];
  int T, F, L = valid;
  std::vector<float> x = conv0(in.data(), frames, nm, m.w0, m.b0, c, &T, &F);
  L = sub_out(L);
  mask_rows(x.data(), T, L, long(F) * c);
  relu_vec(x.data(), long(x.size()));
  x = dw_conv2(x.data(), T, F, c, m.w2, m.b2, &T, &F);
  L = sub_out(L);
  mask_rows(x.data(), T, L, long(F) * c);
  std::vector<float> y(x.size());
  lin(y.data(), x.data(), T * F, m.w3, m.b3);
  mask_rows(y.data(), T, L, long(F) * c);
  relu_vec(y.data(), long(y.size()));
  x = dw_conv2(y.data(), T, F, c, m.w5, m.b5, &T, &F);
  L = sub_out(L);
  mask_rows(x.data(), T, L, long(F) * c);
  y.assign(x.size(), 0.f);
  lin(y.data(), x.data(), T * F, m.w6, m.b6);
  mask_rows(y.data(), T, L, long(F) * c);
  relu_vec(y.data(), long(y.size()));
  std::vector<float> flat(size_t(T) * c * F);
  for (int t = 0; t < T; t++)
    for (int f = 0; f < F; f++)
      for (int ch = 0; ch < c; ch++) flat[size_t(t) * c * F + size_t(ch) * F + f] = y[(size_t(t) * F + f) * c + ch];
  std::vector<float> out(size_t(T) * m.d);
  lin(out.data(), flat.data(), T, m.out, m.outb);
  *To = T;
  *Lo = std::max(0, std::min(L, T));
  return out;
}

// relPosEmb (encoder.go:171-194): rows for positions n−1 down to −(n−1).
inline std::vector<float> rel_pos_emb(int n, int d) {
  std::vector<float> out(size_t(2 * n - 1) * d);
  for (int i = 0; i < 2 * n - 1; i++) {
    const double pos = double(n - 1 - i);
    float* row = &out[size_t(i) * d];
    for (int j = 0; j < d; j += 2) {
      const float div = float(std::exp(double(j) * -(std::log(10000.0) / double(d))));
      const double a = double(float(pos) * div);
      row[j] = float(std::sin(a));
      if (j + 1 < d) row[j + 1] = float(std::cos(a));
    }
  }
  return out;
}

inline void ln_rows_kern(float* y, const float* x, int rows, int n, const float* w, const float* b) {
  for (int r = 0; r < rows; r++) ln_whisper(y + size_t(r) * n, x + size_t(r) * n, n, w, b);
}

// feedForward (encoder.go:244-250).
inline void conformer_ff(const Conformer& m, float* x, int T, const CFF& w, std::vector<float>& ln,
                         std::vector<float>& ff, std::vector<float>& tmp) {
  const int D = m.d;
  ln_rows_kern(ln.data(), x, T, D, w.norm_w, w.norm_b);
  lin(ff.data(), ln.data(), T, w.w1, w.b1);
  silu_vec(ff.data(), T * w.w1.rows);
  lin(tmp.data(), ff.data(), T, w.w2, w.b2);
  axpy_vec(x, tmp.data(), T * D, 0.5f);
}

// attention (encoder.go:259-331), offline: query q < L sees keys [0, L);
// queries in blocks of 32; each block's scores and position terms are two
// MatMulF32 products, the values a third.
inline void conformer_attention(const Conformer& m, const CBlock& b, float* x, const float* ln, int T, int L,
                                const float* pp) {
  const int D = m.d, H = m.heads, hd = D / H, bl = 32;
  std::vector<float> q(size_t(T) * D), k(size_t(T) * D), v(size_t(T) * D), qu(q.size()), qv(q.size()), vt(q.size());
  std::vector<float> glu(q.size(), 0.f), att(q.size());
  lin(q.data(), ln, T, b.q, b.qb);
  lin(k.data(), ln, T, b.k, b.kb);
  lin(v.data(), ln, T, b.v, b.vb);
  for (int t = 0; t < T; t++)
    for (int h = 0; h < H; h++)
      for (int j = 0; j < hd; j++) {
        const size_t o = size_t(t) * D + h * hd + j;
        qu[o] = q[o] + b.pos_u[h * hd + j];
        qv[o] = q[o] + b.pos_v[h * hd + j];
      }
  for (int t = 0; t < T; t++)
    for (int c = 0; c < D; c++) vt[size_t(c) * T + t] = v[size_t(t) * D + c];
  const float scale = float(1 / std::sqrt(double(hd)));
  const int nb = (T + bl - 1) / bl;
  auto keys = [&](int qq, int* lo, int* hi) {
    if (qq >= L) {
      *lo = *hi = 0;
    } else {
      *lo = 0, *hi = L;
    }
  };
  for (int h = 0; h < H; h++)
    for (int blk = 0; blk < nb; blk++) {
      const int q0 = blk * bl, q1 = std::min(T, (blk + 1) * bl), nq = q1 - q0;
      int k0 = T, k1 = 0;
      for (int qq = q0; qq < q1; qq++) {
        int lo, hi;
        keys(qq, &lo, &hi);
        k0 = std::min(k0, lo), k1 = std::max(k1, hi);
      }
      const int nk = k1 - k0;
      if (nk <= 0) {
        for (size_t i = size_t(q0) * D; i < size_t(q1) * D; i++) glu[i] = 0.f;
        continue;
      }
      const int np = nq + nk - 1, jlo = T - 1 - (q1 - 1) + k0;
      std::vector<float> sc(size_t(nq) * nk), bd(size_t(nq) * np);
      matmul_kern_f32(sc.data(), nk, qu.data() + size_t(q0) * D + h * hd, D, k.data() + size_t(k0) * D + h * hd, D, nq,
                      nk, hd);
      matmul_kern_f32(bd.data(), np, qv.data() + size_t(q0) * D + h * hd, D, pp + size_t(jlo) * D + h * hd, D, nq, np,
                      hd);
      for (int i = 0; i < nq; i++) {
        float* row = &sc[size_t(i) * nk];
        const float* brow = &bd[size_t(i) * np + nq - 1 - i];
        int lo, hi;
        keys(q0 + i, &lo, &hi);
        float mx = -std::numeric_limits<float>::infinity();
        for (int kk = 0; kk < nk; kk++) {
          const int kq = k0 + kk;
          if (kq < lo || kq >= hi) {
            row[kk] = -std::numeric_limits<float>::infinity();
            continue;
          }
          const float val = (row[kk] + brow[kk]) * scale;
          row[kk] = val;
          mx = std::max(mx, val);
        }
        if (std::isinf(mx) && mx < 0) {
          for (int kk = 0; kk < nk; kk++) row[kk] = 0.f;
          continue;
        }
        const float sum = expsub_vec(row, nk, mx);
        const float inv = 1.f / sum;
        for (int kk = 0; kk < nk; kk++) row[kk] *= inv;
      }
      matmul_kern_f32(glu.data() + size_t(q0) * D + h * hd, D, sc.data(), nk, vt.data() + size_t(h) * hd * T + k0, T,
                      nq, hd, nk);
    }
  lin(att.data(), glu.data(), T, b.out, b.outb);
  for (size_t i = 0; i < size_t(T) * D; i++) x[i] += att[i];
}

// convModule (encoder.go:343-397), offline (no carried frames).
inline void conformer_conv(const Conformer& m, const CBlock& b, float* x, const float* ln, int T, int L) {
  const int D = m.d, K = m.kernel, padL = (K - 1) / 2;
  std::vector<float> conv(size_t(T) * 2 * D), g(size_t(T) * D), dw(size_t(T) * D);
  lin(conv.data(), ln, T, b.pw1, b.pw1b);
  for (int t = 0; t < T; t++)
    for (int c = 0; c < D; c++) {
      const float* a = &conv[size_t(t) * 2 * D];
      g[size_t(t) * D + c] = t >= L ? 0.f : a[c] * sigmoid_go(a[D + c]);
    }
  for (int t = 0; t < T; t++) {
    float* o = &dw[size_t(t) * D];
    for (int c = 0; c < D; c++) o[c] = b.dwb ? b.dwb[c] : 0.f;
    for (int j = 0; j < K; j++) {
      const int ti = t + j - padL;
      if (ti < 0 || ti >= T) continue;
      const float* src = &g[size_t(ti) * D];
      const float* w = &b.dw[size_t(j) * D];
      for (int c = 0; c < D; c++) o[c] += w[c] * src[c];
    }
  }
  if (m.ln_conv) {
    std::vector<float> tmp(dw);
    ln_rows_kern(dw.data(), tmp.data(), T, D, b.cn_w.data(), b.cn_b.data());
  } else {
    for (int t = 0; t < T; t++)
      for (int c = 0; c < D; c++) dw[size_t(t) * D + c] = dw[size_t(t) * D + c] * b.cn_w[c] + b.cn_b[c];
  }
  silu_vec(dw.data(), T * D);
  lin(conv.data(), dw.data(), T, b.pw2, b.pw2b);
  for (size_t i = 0; i < size_t(T) * D; i++) x[i] += conv[i];
}

// Model.encode (encoder.go:436-489) without a language prompt or speaker
// kernels: log-mel [mels][frames] → [L][d] rows; returns L (*T the rows
// before trimming).
inline std::vector<float> conformer_encode(const Conformer& m, const float* mel, int frames, int valid, int* Lo,
                                           int max_blocks = -1) {
  int T, L;
  std::vector<float> x = conformer_subsample(m, mel, frames, valid, &T, &L);
  const int D = m.d;
  if (m.xscaling) {
    const float s = float(std::sqrt(double(D)));
    for (float& v : x) v *= s;
  }
  std::vector<float> pos = rel_pos_emb(T, D), pp(pos.size());
  std::vector<float> ln(size_t(T) * D), ff(size_t(T) * m.dff), tmp(size_t(T) * D);
  int nbk = 0;
  for (const CBlock& b : m.blocks) {
    if (max_blocks >= 0 && nbk++ >= max_blocks) break;  // a timing sample only
    lin(pp.data(), pos.data(), 2 * T - 1, b.pos, nullptr);
    conformer_ff(m, x.data(), T, b.ff1, ln, ff, tmp);
    ln_rows_kern(ln.data(), x.data(), T, D, b.norm_att_w, b.norm_att_b);
    conformer_attention(m, b, x.data(), ln.data(), T, L, pp.data());
    ln_rows_kern(ln.data(), x.data(), T, D, b.norm_conv_w, b.norm_conv_b);
    conformer_conv(m, b, x.data(), ln.data(), T, L);
    conformer_ff(m, x.data(), T, b.ff2, ln, ff, tmp);
    ln_rows_kern(tmp.data(), x.data(), T, D, b.norm_out_w, b.norm_out_b);
    std::copy(tmp.begin(), tmp.end(), x.begin());
  }
  x.resize(size_t(L) * D);
  *Lo = L;
  return x;
}

}  // namespace orc
