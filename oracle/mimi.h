// TEST INFRASTRUCTURE ONLY: the CPU oracle of Mimi's decoder as Pocket TTS
// runs it (pockettts/mimi.go:24-150, nn.go:52-64 and 258-327,
// speak.go:177-190) and of its encoder as CloneVoice runs it (mimi.go:152-
// 179, voice.go:113-124), restated on kern.h and flowlm.h. Only tests/ use it.
// Checked by the reference's model-free streaming tests (pockettts/
// nn_test.go:37-153, restated in tests/) and a float64 decoder; parity
// against reference outputs unpinned (the tree has none for Mimi).
#pragma once
#include <algorithm>
#include <cstring>
#include <vector>

#include "flowlm.h"

namespace orc {

// kern.Linear for the decoder's weights (kern.go:185-201). Its Q8_0 weights
// are packed with their rows dropped at load (model.go:324-366), so every
// product takes the int8 path; float32 ones take MatMul's float path:
// gemvRows up to 16 rows (dots, then + bias), else the packed kernel for
// the first m/6·6 rows (C starts at the bias, each 256-deep pass adds its
// fused chain) and gemvRows for the rest.
inline void linear_mimi(float* dst, const float* x, int m, const Weight& w, const float* bias) {
  if (w.type == Q8_0) {
    Weight d = w;
    d.dropped = true;
    linear(dst, x, m, d, bias);
    return;
  }
  const int n = w.rows, k = w.cols;
  if (m <= 16) {
    for (int i = 0; i < m; i++) gemv_rows(dst + long(i) * n, x + long(i) * k, w, bias);
    return;
  }
  const int mfull = m / 6 * 6;
  for (int i = 0; i < mfull; i++)
    for (int j = 0; j < n; j++) dst[long(i) * n + j] = bias ? bias[j] : 0.f;
  for (int k0 = 0; k0 < k; k0 += 256) {
    const int kn = std::min(256, k - k0);
    for (int i = 0; i < mfull; i++)
      for (int j = 0; j < n; j++) {
        float acc = 0.f;
        for (int kk = 0; kk < kn; kk++) acc = std::fma(x[long(i) * k + k0 + kk], w.f[long(j) * k + k0 + kk], acc);
        dst[long(i) * n + j] = dst[long(i) * n + j] + acc;
      }
  }
  for (int i = mfull; i < m; i++) gemv_rows(dst + long(i) * n, x + long(i) * k, w, bias);
}

// elu, nn.go:52-64: per 512-value chunk t = min(v, 0), ExpSub(t, 0) (EXP8
// lanes for the chunk's first len&~7 values, Go's expf for the rest), then
// max(v, 0) + (t − 1).
inline void elu_vec(float* x, long len) {
  float t[512];
  for (long o = 0; o < len; o += 512) {
    const int c = int(std::min(512L, len - o));
    for (int i = 0; i < c; i++) t[i] = x[o + i] < 0.f ? x[o + i] : 0.f;
    expsub_vec(t, c, 0.f);
    for (int i = 0; i < c; i++) x[o + i] = (x[o + i] > 0.f ? x[o + i] : 0.f) + (t[i] - 1.f);
  }
}

// A transformer layer with the layer scales Mimi's have (ls1, ls2).
struct MLayer {
  const float *norm1w, *norm1b, *norm2w, *norm2b, *ls1, *ls2;
  Weight qkv, out, ff1, ff2;
};

struct MTransformer {
  int d = 0, heads = 0, ff = 0, context = 0;
  std::vector<MLayer> layers;
  std::vector<float> freqs;
};

// attend for T queries with a context window (nn.go:200-243): the keys
// from lo0 = max(start, pos0 − context + 1) — the caches here keep every
// row, and the reference's trimming never drops one a query can still see —
// are one MatMulF32 for the scores; query p sees [max(lo0, p − context + 1), p].
inline void attend_window(float* out, const float* qkv, int T, const float* kc, const float* vc, int pos0, int d,
                          int heads, int context) {
  const int hd = d / heads, lo0 = context > 0 ? std::max(0, pos0 - context + 1) : 0, nk = pos0 + T - lo0;
  const float scale = float(1 / std::sqrt(double(hd)));
  std::vector<float> sc(size_t(T) * nk), vt(size_t(hd) * nk);
  const float* k0 = kc + long(lo0) * d;
  const float* v0 = vc + long(lo0) * d;
  for (int h = 0; h < heads; h++) {
    matmul_kern_f32(sc.data(), nk, qkv + h * hd, 3 * d, k0 + h * hd, d, T, nk, hd);
    for (int r = 0; r < T; r++) {
      const int p = pos0 + r, lo = context > 0 ? std::max(lo0, p - context + 1) : lo0;
      float* row = sc.data() + size_t(r) * nk;
      float* s = row + (lo - lo0);
      const int ns = p + 1 - lo;
      float mx = -INFINITY;
      for (int j = 0; j < ns; j++) {
        s[j] *= scale;
        mx = std::max(mx, s[j]);
      }
      const float inv = 1.f / expsub_vec(s, ns, mx);
      for (int j = 0; j < ns; j++) s[j] *= inv;
      for (int j = 0; j < lo - lo0; j++) row[j] = 0.f;
      for (int j = p + 1 - lo0; j < nk; j++) row[j] = 0.f;
    }
    if (T < 4) {
      for (int r = 0; r < T; r++) {
        float* o = out + long(r) * d + h * hd;
        for (int i = 0; i < hd; i++) o[i] = 0.f;
        for (int j = 0; j < nk; j++) {
          const float w = sc[size_t(r) * nk + j];
          if (w != 0) {
            const float* vj = v0 + long(j) * d + h * hd;
            for (int i = 0; i < hd; i++) o[i] = std::fma(w, vj[i], o[i]);
          }
        }
      }
      continue;
    }
    for (int j = 0; j < nk; j++)
      for (int i = 0; i < hd; i++) vt[size_t(i) * nk + j] = v0[long(j) * d + h * hd + i];
    matmul_kern_f32(out + h * hd, d, sc.data(), nk, vt.data(), nk, T, hd, nk);
  }
}

// transformer.forward (nn.go:142-182) with the window and layer scales:
// x += ls·y as addScaled does (unfused).
inline void mtransformer_rows(const MTransformer& t, float* x, int T, Stream& st) {
  const int d = t.d;
  std::vector<float> h(size_t(T) * d), qkv(size_t(T) * 3 * d), att(size_t(T) * d), ff(size_t(T) * t.ff);
  auto add_scaled = [&](const float* y, const float* s) {
    for (long i = 0; i < long(T) * d; i++) x[i] += s[i % d] * y[i];
  };
  for (size_t li = 0; li < t.layers.size(); li++) {
    const MLayer& l = t.layers[li];
    layer_norm_pt(h.data(), x, T, d, l.norm1w, l.norm1b, 1e-5);
    linear_mimi(qkv.data(), h.data(), T, l.qkv, nullptr);
    for (int r = 0; r < T; r++) {
      float* row = qkv.data() + size_t(r) * 3 * d;
      apply_rope(row, t.heads, t.freqs, st.pos + r);
      apply_rope(row + d, t.heads, t.freqs, st.pos + r);
    }
    for (int r = 0; r < T; r++) {
      const float* row = qkv.data() + size_t(r) * 3 * d;
      st.k[li].insert(st.k[li].end(), row + d, row + 2 * d);
      st.v[li].insert(st.v[li].end(), row + 2 * d, row + 3 * d);
    }
    attend_window(att.data(), qkv.data(), T, st.k[li].data(), st.v[li].data(), st.pos, d, t.heads, t.context);
    linear_mimi(h.data(), att.data(), T, l.out, nullptr);
    add_scaled(h.data(), l.ls1);
    layer_norm_pt(h.data(), x, T, d, l.norm2w, l.norm2b, 1e-5);
    linear_mimi(ff.data(), h.data(), T, l.ff1, nullptr);
    gelu_vec(ff.data(), T * t.ff);
    linear_mimi(h.data(), ff.data(), T, l.ff2, nullptr);
    add_scaled(h.data(), l.ls2);
  }
  st.pos += T;
}

// conv (nn.go:258-300): causal Conv1d over [prev rows; x], weight [cout][k·cin].
struct MConv {
  Weight w;
  const float* b = nullptr;
  int cin = 0, cout = 0, k = 1, stride = 1, dil = 1;
  int past() const { return (k - 1) * dil + 1 - stride; }
};

inline void conv_run(const MConv& c, std::vector<float>& prev, const float* x, int T, float* y) {
  const int P = c.past(), cin = c.cin, To = T / c.stride;
  if (c.k == 1 && c.stride == 1) {
    linear_mimi(y, x, T, c.w, c.b);
    return;
  }
  std::vector<float> buf(size_t(P + T) * cin), col(size_t(To) * c.k * cin);
  std::copy(prev.begin(), prev.end(), buf.begin());
  std::copy(x, x + long(T) * cin, buf.begin() + long(P) * cin);
  for (int t = 0; t < To; t++)
    for (int j = 0; j < c.k; j++) {
      const long s = long(t * c.stride + j * c.dil) * cin;
      std::copy(buf.begin() + s, buf.begin() + s + cin, col.begin() + (long(t) * c.k + j) * cin);
    }
  linear_mimi(y, col.data(), To, c.w, c.b);
  std::copy(buf.begin() + long(T) * cin, buf.end(), prev.begin());
}

// convtr (nn.go:302-327): ConvTranspose1d, weight [k·cout][cin]; the k taps
// of every input row added over the bias in input order, then the partial
// carried from the last call; the new partial is the tail less the bias.
struct MConvTr {
  Weight w;
  const float* b = nullptr;
  int cin = 0, cout = 0, k = 1, stride = 1;
};

inline void convtr_run(const MConvTr& c, std::vector<float>& partial, const float* x, int T, float* y) {
  const int co = c.cout, S = c.stride, L = (T - 1) * S + c.k, PT = c.k - S;
  std::vector<float> z(size_t(T) * c.k * co), full(size_t(L) * co);
  linear_mimi(z.data(), x, T, c.w, nullptr);
  for (int i = 0; i < L; i++) std::copy(c.b, c.b + co, full.begin() + long(i) * co);
  for (int t = 0; t < T; t++)
    for (int j = 0; j < c.k; j++)
      for (int i = 0; i < co; i++) full[size_t(t * S + j) * co + i] += z[(size_t(t) * c.k + j) * co + i];
  for (int i = 0; i < PT * co; i++) full[size_t(i)] += partial[size_t(i)];
  for (int i = 0; i < PT * co; i++) partial[size_t(i)] = full[size_t(L - PT) * co + i] - c.b[i % co];
  std::copy(full.begin(), full.begin() + long(T) * S * co, y);
}

// A SEANet step (mimi.go:14-21): a conv, a transposed conv or a residual
// block (x + conv1x1(ELU(conv(ELU(x))))), with an ELU before it or not.
struct MStep {
  int kind = 0;  // 0 conv, 1 convtr, 2 residual block
  bool elu = false;
  MConv c, ra, rb;
  MConvTr t;
};

struct MimiDecoder {
  Weight quant;  // [d][ldim]
  const float* up = nullptr;  // [d][2·upS] depthwise
  int upS = 1, ldim = 0, frame = 0, sample_rate = 0;
  MTransformer tf;
  std::vector<MStep> steps;
};

// decState (mimi.go:108-124) plus speakChunk's started flag.
struct MimiState {
  Stream tf;
  std::vector<float> up_part;
  std::vector<std::vector<float>> prev;  // per step (a residual block has two)
  bool started = false;
};

// newSeaState (mimi.go:34-52): each step's carried rows (a residual block
// has two slots).
inline std::vector<std::vector<float>> sea_state(const std::vector<MStep>& steps) {
  std::vector<std::vector<float>> prev;
  for (const MStep& st : steps) {
    if (st.kind == 0) prev.emplace_back(size_t(st.c.past()) * st.c.cin, 0.f);
    if (st.kind == 1) prev.emplace_back(size_t(st.t.k - st.t.stride) * st.t.cout, 0.f);
    if (st.kind == 2) {
      prev.emplace_back(size_t(st.ra.past()) * st.ra.cin, 0.f);
      prev.emplace_back(size_t(st.rb.past()) * st.rb.cin, 0.f);
    }
  }
  return prev;
}

inline MimiState mimi_state(const MimiDecoder& m) {
  MimiState s;
  s.tf.k.assign(m.tf.layers.size(), {});
  s.tf.v.assign(m.tf.layers.size(), {});
  s.up_part.assign(size_t(m.upS) * m.tf.d, 0.f);
  s.prev = sea_state(m.steps);
  return s;
}

// runSea (mimi.go:61-106): T rows of Cc values through the steps, the
// carried rows in prev; x, T and Cc become the output's.
inline void run_sea(const std::vector<MStep>& steps, std::vector<std::vector<float>>& prev, std::vector<float>& x,
                    int& T, int& Cc) {
  size_t pi = 0;
  for (const MStep& st : steps) {
    if (st.elu) elu_vec(x.data(), long(T) * Cc);
    if (st.kind == 0) {
      std::vector<float> y(size_t(T / st.c.stride) * st.c.cout);
      conv_run(st.c, prev[pi++], x.data(), T, y.data());
      T /= st.c.stride;
      Cc = st.c.cout;
      x.swap(y);
    } else if (st.kind == 1) {
      std::vector<float> y(size_t(T) * st.t.stride * st.t.cout);
      convtr_run(st.t, prev[pi++], x.data(), T, y.data());
      T *= st.t.stride;
      Cc = st.t.cout;
      x.swap(y);
    } else {
      std::vector<float> v(x), h(size_t(T) * st.ra.cout), o(size_t(T) * Cc);
      elu_vec(v.data(), long(T) * Cc);
      conv_run(st.ra, prev[pi], v.data(), T, h.data());
      elu_vec(h.data(), long(T) * st.ra.cout);
      conv_run(st.rb, prev[pi + 1], h.data(), T, o.data());
      for (size_t i = 0; i < x.size(); i++) x[i] = x[i] + o[i];
      pi += 2;
    }
  }
}

// mimiDecoder.decode for one latent (mimi.go:126-150, runSea :45-98), then
// speakChunk's fade-in on the first frame (speak.go:185-190). pcm gets the
// frame's samples.
inline void mimi_decode(const MimiDecoder& m, MimiState& s, const float* lat, float* pcm) {
  const int C = m.tf.d, S = m.upS, K = 2 * S;
  std::vector<float> z((size_t(C))), full(size_t(K) * C, 0.f);
  linear_mimi(z.data(), lat, 1, m.quant, nullptr);
  for (int c = 0; c < C; c++)
    for (int j = 0; j < K; j++) full[size_t(j) * C + c] += z[size_t(c)] * m.up[size_t(c) * K + j];
  for (int i = 0; i < S * C; i++) full[size_t(i)] += s.up_part[size_t(i)];
  std::copy(full.begin() + long(S) * C, full.end(), s.up_part.begin());
  int T = S, Cc = C;
  std::vector<float> x(full.begin(), full.begin() + long(S) * C);
  mtransformer_rows(m.tf, x.data(), T, s.tf);
  run_sea(m.steps, s.prev, x, T, Cc);
  std::copy(x.begin(), x.begin() + long(T) * Cc, pcm);
  if (!s.started) {
    const int fade = m.sample_rate / 200, n = std::min(fade, T * Cc);
    for (int i = 0; i < n; i++) pcm[i] *= float(i) / float(fade - 1);
    s.started = true;
  }
}

// mimiEncoder (mimi.go:30-34, model.go:181-200, 308-313): the SEANet
// encoder's steps, the transformer and the downsampling conv to 12.5 Hz
// (weight [ldim][2·up·d], no bias, its first call padded with copies of
// the first row: "replicate").
struct MimiEncoder {
  std::vector<MStep> steps;
  MTransformer tf;
  MConv down;
  std::vector<float> down_b;
};

// encState (mimi.go:152-162).
struct MimiEncState {
  std::vector<std::vector<float>> sea;
  Stream tf;
  std::vector<float> down;
  bool first = true;
};

inline MimiEncState mimi_enc_state(const MimiEncoder& e) {
  MimiEncState s;
  s.sea = sea_state(e.steps);
  s.tf.k.assign(e.tf.layers.size(), {});
  s.tf.v.assign(e.tf.layers.size(), {});
  s.down.assign(size_t(e.down.past()) * e.down.cin, 0.f);
  return s;
}

// encode (mimi.go:164-179): n samples (a multiple of the hop) → latents.
inline std::vector<float> mimi_encode(const MimiEncoder& e, MimiEncState& st, const float* pcm, int n) {
  std::vector<float> x(pcm, pcm + n);
  int T = n, C = 1;
  run_sea(e.steps, st.sea, x, T, C);
  mtransformer_rows(e.tf, x.data(), T, st.tf);
  if (st.first) {
    for (int i = 0; i < e.down.past(); i++) std::copy(x.begin(), x.begin() + C, st.down.begin() + long(i) * C);
    st.first = false;
  }
  std::vector<float> out(size_t(T / e.down.stride) * e.down.cout);
  conv_run(e.down, st.down, x.data(), T, out.data());
  return out;
}

// cloneCond's encoding (voice.go:113-124): x (24 kHz, after end_on_pause)
// padded with zeros to whole frames, encoded twelve frames at a time with
// one state. Returns the latents [frames][ldim].
inline std::vector<float> mimi_clone_latents(const MimiEncoder& e, const float* x, int n, int frame) {
  std::vector<float> buf(x, x + n);
  buf.resize(size_t(n + (frame - n % frame) % frame), 0.f);
  MimiEncState st = mimi_enc_state(e);
  std::vector<float> lat;
  const int piece = 12 * frame;
  for (size_t i = 0; i < buf.size(); i += size_t(piece)) {
    const int len = int(std::min(buf.size() - i, size_t(piece)));
    std::vector<float> y = mimi_encode(e, st, buf.data() + i, len);
    lat.insert(lat.end(), y.begin(), y.end());
  }
  return lat;
}

}  // namespace orc
