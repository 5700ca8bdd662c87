// TEST INFRASTRUCTURE ONLY: the CPU oracle for the Pocket TTS FlowLM token
// loop (pockettts/lm.go, pockettts/nn.go, pockettts/speak.go), restated in
// C++ on top of kern.h. Used by tests/, smoke() and the CPU baseline only.
#pragma once
#include <map>
#include <string>

#include "kern.h"

namespace orc {

// layerNorm, pockettts/nn.go:27-49: float64 mean and biased variance,
// output rounded to float32 and then (if w) o·w + b in float32.
inline void layer_norm_pt(float* dst, const float* src, int rows, int n, const float* w, const float* b, double eps) {
  for (int r = 0; r < rows; r++) {
    const float* x = src + long(r) * n;
    float* y = dst + long(r) * n;
    double s = 0;
    for (int i = 0; i < n; i++) s += double(x[i]);
    double mean = s / double(n);
    double q = 0;
    for (int i = 0; i < n; i++) {
      double d = double(x[i]) - mean;
      q += d * d;
    }
    double inv = 1.0 / std::sqrt(q / double(n) + eps);
    for (int i = 0; i < n; i++) {
      float o = float((double(x[i]) - mean) * inv);
      if (w) o = o * w[i] + b[i];
      y[i] = o;
    }
  }
}

// ropeFreqs, pockettts/nn.go:69-76.
inline std::vector<float> rope_freqs(int head_dim, double period) {
  float c = float(-std::log(period) * 2 / double(head_dim));
  std::vector<float> f((size_t)(head_dim / 2));
  for (size_t i = 0; i < f.size(); i++) f[i] = float(std::exp(double(float(i) * c)));
  return f;
}

// The cos/sin applyRope takes for pair i at position pos (nn.go:84-85).
inline void rope_cs(float f, int pos, float* c, float* s) {
  double a = double(f * float(pos));
  *c = float(std::cos(a));
  *s = float(std::sin(a));
}

// applyRope, pockettts/nn.go:80-93.
inline void apply_rope(float* x, int heads, const std::vector<float>& freqs, int pos) {
  int hd = int(freqs.size()) * 2;
  for (size_t i = 0; i < freqs.size(); i++) {
    float c, s;
    rope_cs(freqs[i], pos, &c, &s);
    for (int h = 0; h < heads; h++) {
      int j = h * hd + 2 * int(i);
      float r = x[j], im = x[j + 1];
      x[j] = r * c - im * s;
      x[j + 1] = r * s + im * c;
    }
  }
}

struct FlowLMLayer {
  const float *norm1w, *norm1b, *norm2w, *norm2b;
  Weight qkv, out, ff1, ff2;
};

struct ResBlock {
  const float *normw, *normb, *b1, *b2, *adab;
  Weight fc1, fc2, ada;
};

struct TimeEmbed {
  const float *freqs, *b1, *b2, *alpha;
  int half;
  Weight fc1, fc2;
};

struct FlowLM {
  int d, heads, ff, ldim, fd;
  std::vector<FlowLMLayer> layers;
  std::vector<float> freqs;
  Weight input, eosw, cond, finput, final_ada, fout;
  Weight embed;  // lm.embed [tokens + 1][d] (rows 0 when the model has none)
  Weight speaker;  // lm.speaker_proj [d][ldim] float32 (rows 0 when the model has none)
  const float* bosv = nullptr;  // lm.bos_voice [d]
  const float *bos, *outw, *outb, *mean, *stdv, *condb, *finputb, *final_adab, *foutb;
  float eosb;
  TimeEmbed time[2];
  std::vector<ResBlock> res;
};

// One stream's transformer state (tstate, nn.go:120-123): per layer the
// rotated keys and the values, a row of d per position.
struct Stream {
  std::vector<std::vector<float>> k, v;
  int pos = 0;
};

// timeEmbed.embed, pockettts/lm.go:62-89.
inline std::vector<float> time_embed(const TimeEmbed& e, float t) {
  int half = e.half;
  std::vector<float> in((size_t)(2 * half));
  for (int i = 0; i < half; i++) {
    double a = double(t * e.freqs[i]);
    in[size_t(i)] = float(std::cos(a));
    in[size_t(half + i)] = float(std::sin(a));
  }
  std::vector<float> h((size_t)(e.fc1.rows)), y((size_t)(e.fc2.rows));
  linear(h.data(), in.data(), 1, e.fc1, e.b1);
  silu_vec(h.data(), e.fc1.rows);
  linear(y.data(), h.data(), 1, e.fc2, e.b2);
  double s = 0;
  for (float v : y) s += double(v);
  double mean = s / double(y.size());
  double q = 0;
  for (float v : y) q += (double(v) - mean) * (double(v) - mean);
  float inv = float(1.0 / std::sqrt(q / double(y.size() - 1) + 1e-5));
  for (size_t i = 0; i < y.size(); i++) y[i] *= e.alpha[i] * inv;
  return y;
}

// flowHead.timeConds, pockettts/lm.go:93-104.
inline std::vector<std::vector<float>> time_conds(const FlowLM& m, int steps) {
  std::vector<std::vector<float>> out;
  for (int i = 0; i < steps; i++) {
    auto s = time_embed(m.time[0], float(double(i) / double(steps)));
    auto t = time_embed(m.time[1], float(double(i + 1) / double(steps)));
    for (size_t j = 0; j < s.size(); j++) s[j] = (s[j] + t[j]) / 2;
    out.push_back(s);
  }
  return out;
}

// transformer.attend for one query (T = 1, no context window),
// pockettts/nn.go:200-243: scores by gemvRows (dotF32x4 per group of four
// keys, dotF32Go for the last nk%4), scaled, max, expSub, scaled by 1/Σ,
// then the values added with AddScaled (axpy, one fused step per key).
inline bool attend_one_fast(float* out, const float* q, const float* kc, const float* vc, int nk, int d, int heads);

inline void attend_one(float* out, const float* q, const float* kc, const float* vc, int nk, int d, int heads) {
  if (fast_on() && attend_one_fast(out, q, kc, vc, nk, d, heads)) return;
  int hd = d / heads;
  float scale = float(1 / std::sqrt(double(hd)));
  std::vector<float> sc((size_t)(nk));
  for (int h = 0; h < heads; h++) {
    const float* qh = q + h * hd;
    for (int j = 0; j < nk; j += 4) {
      if (j + 4 <= nk) {
        float o4[4];
        dot_f32x4(qh, kc + long(j) * d + h * hd, d, hd, o4);
        for (int r = 0; r < 4; r++) sc[size_t(j + r)] = o4[r];
      } else {
        for (int jj = j; jj < nk; jj++) sc[size_t(jj)] = dot_f32_go(qh, kc + long(jj) * d + h * hd, hd);
      }
    }
    float mx = -INFINITY;
    for (int j = 0; j < nk; j++) {
      sc[size_t(j)] *= scale;
      mx = std::max(mx, sc[size_t(j)]);
    }
    float inv = 1.f / expsub_vec(sc.data(), nk, mx);
    for (int j = 0; j < nk; j++) sc[size_t(j)] *= inv;
    float* o = out + h * hd;
    for (int i = 0; i < hd; i++) o[i] = 0;
    for (int j = 0; j < nk; j++) {
      float w = sc[size_t(j)];
      if (w != 0) {
        const float* vj = vc + long(j) * d + h * hd;
        for (int i = 0; i < hd; i++) o[i] = std::fma(w, vj[i], o[i]);
      }
    }
  }
}

// Scratch for one step; Trace holds the intermediates tests compare.
struct Trace {
  std::vector<float> x_in;                      // input projection
  std::vector<std::vector<float>> x_after;      // residual stream after each layer
  std::vector<std::vector<float>> q_rot, att;   // per layer: rotated q, attention output
  std::vector<float> lm_out;                    // after out_norm
  float eos = 0;
};

// transformer.forward for one row (nn.go:142-182, T = 1, no layer scale,
// context 0), followed by out_norm (lm.go:164-170).
inline void transformer_step(const FlowLM& m, float* x, Stream& st, float* lm_out, Trace* tr) {
  int d = m.d;
  std::vector<float> h((size_t)(d)), qkv((size_t)(3 * d)), att((size_t)(d)), ff((size_t)(m.ff));
  for (size_t li = 0; li < m.layers.size(); li++) {
    const FlowLMLayer& l = m.layers[li];
    layer_norm_pt(h.data(), x, 1, d, l.norm1w, l.norm1b, 1e-5);
    linear(qkv.data(), h.data(), 1, l.qkv, nullptr);
    apply_rope(qkv.data(), m.heads, m.freqs, st.pos);
    apply_rope(qkv.data() + d, m.heads, m.freqs, st.pos);
    st.k[li].insert(st.k[li].end(), qkv.begin() + d, qkv.begin() + 2 * d);
    st.v[li].insert(st.v[li].end(), qkv.begin() + 2 * d, qkv.end());
    int nk = int(st.k[li].size() / size_t(d));
    attend_one(att.data(), qkv.data(), st.k[li].data(), st.v[li].data(), nk, d, m.heads);
    if (tr) {
      tr->q_rot.emplace_back(qkv.begin(), qkv.begin() + d);
      tr->att.push_back(att);
    }
    linear(h.data(), att.data(), 1, l.out, nullptr);
    add_to(x, h.data(), d);
    layer_norm_pt(h.data(), x, 1, d, l.norm2w, l.norm2b, 1e-5);
    linear(ff.data(), h.data(), 1, l.ff1, nullptr);
    gelu_vec(ff.data(), m.ff);
    linear(h.data(), ff.data(), 1, l.ff2, nullptr);
    add_to(x, h.data(), d);
    if (tr) tr->x_after.emplace_back(x, x + d);
  }
  st.pos += 1;
  layer_norm_pt(lm_out, x, 1, d, m.outw, m.outb, 1e-5);
}

// kern.MatMulF32 (kern.go:205-211 → gemm.go:116-185) with a float32 B of
// row stride ldb, no bias: up to 16 rows of A take gemvRows (dotF32x4 per
// group of four B rows, dotF32Go for the rest); more rows take the packed
// kernel for the first m/6·6 (C starts at 0 and each 256-deep pass adds
// its fused chain, k6x16avx) and gemvRows for the others.
inline void matmul_kern_f32(float* c, int ldc, const float* a, int lda, const float* b, int ldb, int m, int n, int k) {
  auto gemv_row = [&](float* y, const float* x) {
    for (int j = 0; j < n; j += 4) {
      if (j + 4 <= n) {
        float o4[4];
        dot_f32x4(x, b + long(j) * ldb, ldb, k, o4);
        for (int r = 0; r < 4; r++) y[j + r] = o4[r];
      } else {
        for (int jj = j; jj < n; jj++) y[jj] = dot_f32_go(x, b + long(jj) * ldb, k);
      }
    }
  };
  if (m <= 16) {
    for (int i = 0; i < m; i++) gemv_row(c + long(i) * ldc, a + long(i) * lda);
    return;
  }
  const int mfull = m / 6 * 6;
  for (int i = 0; i < mfull; i++)
    for (int j = 0; j < n; j++) c[long(i) * ldc + j] = 0.f;
  for (int k0 = 0; k0 < k; k0 += 256) {
    const int kn = std::min(256, k - k0);
    for (int i = 0; i < mfull; i++)
      for (int j = 0; j < n; j++) {
        float acc = 0.f;
        for (int kk = 0; kk < kn; kk++) acc = std::fma(a[long(i) * lda + k0 + kk], b[long(j) * ldb + k0 + kk], acc);
        c[long(i) * ldc + j] = c[long(i) * ldc + j] + acc;
      }
  }
  for (int i = mfull; i < m; i++) gemv_row(c + long(i) * ldc, a + long(i) * lda);
}

// transformer.attend for T queries at positions pos0.. (nn.go:200-243, no
// context window): per head the scores of all T queries against the nk =
// pos0 + T keys are one MatMulF32; each query's visible scores are scaled,
// softmaxed (expSub, × 1/Σ) and the rest cleared; the values are added key
// by key (AddScaled) for T < 4, else one MatMulF32 against the head's
// transposed values.
inline void attend_rows(float* out, const float* qkv, int T, const float* kc, const float* vc, int pos0, int d,
                        int heads) {
  const int hd = d / heads, nk = pos0 + T;
  const float scale = float(1 / std::sqrt(double(hd)));
  std::vector<float> sc(size_t(T) * nk), vt(size_t(hd) * nk);
  for (int h = 0; h < heads; h++) {
    matmul_kern_f32(sc.data(), nk, qkv + h * hd, 3 * d, kc + h * hd, d, T, nk, hd);
    for (int r = 0; r < T; r++) {
      const int p = pos0 + r;
      float* row = sc.data() + size_t(r) * nk;
      float mx = -INFINITY;
      for (int j = 0; j <= p; j++) {
        row[j] *= scale;
        mx = std::max(mx, row[j]);
      }
      const float inv = 1.f / expsub_vec(row, p + 1, mx);
      for (int j = 0; j <= p; j++) row[j] *= inv;
      for (int j = p + 1; j < nk; j++) row[j] = 0.f;
    }
    if (T < 4) {
      for (int r = 0; r < T; r++) {
        float* o = out + long(r) * d + h * hd;
        for (int i = 0; i < hd; i++) o[i] = 0.f;
        for (int j = 0; j < nk; j++) {
          const float w = sc[size_t(r) * nk + j];
          if (w != 0) {
            const float* vj = vc + long(j) * d + h * hd;
            for (int i = 0; i < hd; i++) o[i] = std::fma(w, vj[i], o[i]);
          }
        }
      }
      continue;
    }
    for (int j = 0; j < nk; j++)
      for (int i = 0; i < hd; i++) vt[size_t(i) * nk + j] = vc[long(j) * d + h * hd + i];
    matmul_kern_f32(out + h * hd, d, sc.data(), nk, vt.data(), nk, T, hd, nk);
  }
}

// transformer.forward for T rows (nn.go:142-182, no layer scale, context
// 0): every layer's products take all T rows at once (int8 path for T ≥ 2),
// RoPE at positions pos.., the T keys and values appended before
// attending. Then out_norm of the last row (lm.go:164-170) into lm_out.
inline void transformer_rows(const FlowLM& m, float* x, int T, Stream& st, float* lm_out) {
  const int d = m.d;
  std::vector<float> h(size_t(T) * d), qkv(size_t(T) * 3 * d), att(size_t(T) * d), ff(size_t(T) * m.ff);
  for (size_t li = 0; li < m.layers.size(); li++) {
    const FlowLMLayer& l = m.layers[li];
    layer_norm_pt(h.data(), x, T, d, l.norm1w, l.norm1b, 1e-5);
    linear(qkv.data(), h.data(), T, l.qkv, nullptr);
    for (int r = 0; r < T; r++) {
      float* row = qkv.data() + size_t(r) * 3 * d;
      apply_rope(row, m.heads, m.freqs, st.pos + r);
      apply_rope(row + d, m.heads, m.freqs, st.pos + r);
    }
    for (int r = 0; r < T; r++) {
      const float* row = qkv.data() + size_t(r) * 3 * d;
      st.k[li].insert(st.k[li].end(), row + d, row + 2 * d);
      st.v[li].insert(st.v[li].end(), row + 2 * d, row + 3 * d);
    }
    attend_rows(att.data(), qkv.data(), T, st.k[li].data(), st.v[li].data(), st.pos, d, m.heads);
    linear(h.data(), att.data(), T, l.out, nullptr);
    add_to(x, h.data(), T * d);
    layer_norm_pt(h.data(), x, T, d, l.norm2w, l.norm2b, 1e-5);
    linear(ff.data(), h.data(), T, l.ff1, nullptr);
    gelu_vec(ff.data(), T * m.ff);
    linear(h.data(), ff.data(), T, l.ff2, nullptr);
    add_to(x, h.data(), T * d);
  }
  st.pos += T;
  if (lm_out) layer_norm_pt(lm_out, x + size_t(T - 1) * d, 1, d, m.outw, m.outb, 1e-5);
}

// Weight.Row for the embedding (kern.go:116-122): float32 rows are copied,
// Q8_0 rows dequantised (dequantQ8: float(q)·d, exact).
inline void weight_row(const Weight& w, int j, float* dst) {
  if (w.type == Q8_0) {
    const int nb = w.cols / QK;
    const uint8_t* blk = w.q + long(j) * nb * Q8BYTES;
    for (int b = 0; b < nb; b++, blk += Q8BYTES) {
      const float dd = f16_to_f32(uint16_t(blk[0] | blk[1] << 8));
      for (int i = 0; i < QK; i++) dst[b * QK + i] = float(int8_t(blk[2 + i])) * dd;
    }
    return;
  }
  for (int i = 0; i < w.cols; i++) dst[i] = w.f[long(j) * w.cols + i];
}

// flowLM.text, pockettts/lm.go:172-181: the tokens' embedding rows through
// the transformer; lm_out gets the output at the last token.
inline void flowlm_text(const FlowLM& m, const int* ids, int T, Stream& st, float* lm_out) {
  std::vector<float> x(size_t(T) * m.d);
  for (int i = 0; i < T; i++) weight_row(m.embed, ids[i], x.data() + size_t(i) * m.d);
  transformer_rows(m, x.data(), T, st, lm_out);
}

// The flow-LM half of Model.CloneVoice (voice.go:94-106, cloneCond :113-127
// after Mimi's encoder): cond = kern.Linear(latents, lm.speaker_proj)
// (float32 weight: MatMul's gemvRows up to 16 rows, the packed kernel
// beyond), then [bos_voice; cond] through the transformer from an empty
// state, whose caches are the voice.
inline void flowlm_voice_latents(const FlowLM& m, const float* lat, int n, Stream& st) {
  const int d = m.d;
  std::vector<float> x(size_t(n + 1) * d);
  std::copy(m.bosv, m.bosv + d, x.begin());
  matmul_kern_f32(x.data() + d, d, lat, m.speaker.cols, m.speaker.f, m.speaker.cols, n, d, m.speaker.cols);
  st.k.assign(m.layers.size(), {});
  st.v.assign(m.layers.size(), {});
  st.pos = 0;
  transformer_rows(m, x.data(), n + 1, st, nullptr);
}

// flowLM.step, pockettts/lm.go:185-195. latent == nullptr is the first
// frame (bos).
inline float flowlm_step(const FlowLM& m, const float* latent, Stream& st, float* lm_out, Trace* tr) {
  std::vector<float> x((size_t)(m.d));
  linear(x.data(), latent ? latent : m.bos, 1, m.input, nullptr);
  if (tr) tr->x_in = x;
  transformer_step(m, x.data(), st, lm_out, tr);
  float e;
  linear(&e, lm_out, 1, m.eosw, nullptr);
  float eos = e + m.eosb;
  if (tr) {
    tr->lm_out.assign(lm_out, lm_out + m.d);
    tr->eos = eos;
  }
  return eos;
}

// flowHead.net, pockettts/lm.go:126-160.
inline std::vector<float> flow_net(const FlowLM& m, const float* y, const float* x) {
  int D = m.fd;
  std::vector<float> h((size_t)(D)), sy(y, y + D), mod((size_t)(3 * D)), n((size_t)(D)), mm((size_t)(D));
  linear(h.data(), x, 1, m.finput, m.finputb);
  silu_vec(sy.data(), D);
  for (const ResBlock& r : m.res) {
    linear(mod.data(), sy.data(), 1, r.ada, r.adab);
    const float *shift = mod.data(), *scale = mod.data() + D, *gate = mod.data() + 2 * D;
    layer_norm_pt(n.data(), h.data(), 1, D, r.normw, r.normb, 1e-6);
    for (int j = 0; j < D; j++) n[size_t(j)] = n[size_t(j)] * (1 + scale[j]) + shift[j];
    linear(mm.data(), n.data(), 1, r.fc1, r.b1);
    silu_vec(mm.data(), D);
    linear(n.data(), mm.data(), 1, r.fc2, r.b2);
    for (int j = 0; j < D; j++) h[size_t(j)] += gate[j] * n[size_t(j)];
  }
  linear(mod.data(), sy.data(), 1, m.final_ada, m.final_adab);
  const float *shift = mod.data(), *scale = mod.data() + D;
  layer_norm_pt(n.data(), h.data(), 1, D, nullptr, nullptr, 1e-6);
  for (int j = 0; j < D; j++) n[size_t(j)] = n[size_t(j)] * (1 + scale[j]) + shift[j];
  std::vector<float> out((size_t)(m.ldim));
  linear(out.data(), n.data(), 1, m.fout, m.foutb);
  return out;
}

// flowHead.sample, pockettts/lm.go:108-124.
inline void flow_sample(const FlowLM& m, const float* c, const float* x0, const std::vector<std::vector<float>>& tc,
                        float* latent) {
  int D = m.fd;
  std::vector<float> y((size_t)(D)), yi((size_t)(D));
  linear(y.data(), c, 1, m.cond, m.condb);
  std::vector<float> cur(x0, x0 + m.ldim);
  for (const auto& t : tc) {
    for (int j = 0; j < D; j++) yi[size_t(j)] = y[size_t(j)] + t[size_t(j)];
    auto v = flow_net(m, yi.data(), cur.data());
    float n = float(tc.size());
    for (int j = 0; j < m.ldim; j++) cur[size_t(j)] += v[size_t(j)] / n;
  }
  std::memcpy(latent, cur.data(), sizeof(float) * size_t(m.ldim));
}

}  // namespace orc
