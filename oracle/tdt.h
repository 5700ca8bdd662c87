// TEST INFRASTRUCTURE — the CPU oracle of the greedy RNN-T / TDT decode loop
// (conformer/rnnt.go). Only tests, the smoke check and the benchmark's CPU
// baseline use it; the product never links it.
//
// Restated from the reference, operation by operation, on the kernels of
// kern.h (the amd64 float path for the m=1 products, the int8 path for the
// encoder projection):
//  * predict (rnnt.go:46-68): per LSTM layer gates = Wx·x + b, then
//    gates += Wh·h (two products, then kern.Add); i, f, o = sigmoid
//    (conformer/encoder.go:13: 1/(1+Expf(-v))), g = tanh32 (float64 tanh,
//    rnnt.go:42), c = f·c' + i·g and h = o·tanh32(c), unfused (Go, amd64 v1);
//  * joint (rnnt.go:91-106): predProj = jPred·pred + b, hidden =
//    act(encProj + predProj), logits = jOut·hidden + b;
//  * Decode (rnnt.go:111-173): encProj for all frames by one int8-path
//    product, then the loop with its argmaxes (strict '>', first wins,
//    rnnt.go:70-78), softmaxAt (float64 sum, :80-89), frame skipping and
//    max_symbols rule, at most 16·T + 1024 iterations.
// Go's math.Tanh / math.Exp are not under the reference tree; glibc's tanh and
// exp stand in for them (both within an ulp of float64, invisible after the
// float32 cast in practice, not pinned).
#pragma once

#include <cmath>
#include <vector>

#include "kern.h"

namespace orc {

enum JointAct { ACT_RELU = 0, ACT_SIGMOID = 1, ACT_TANH = 2 };

struct TDTLayer {
  Weight wx, wh;
  const float* b = nullptr;
};

struct TDT {
  int H = 0, V = 0, J = 0, blank = 0, max_symbols = 10;
  bool tdt = true;
  int act = ACT_RELU;
  std::vector<int> durations;
  const float* embed = nullptr;  // [V][H], F32
  std::vector<TDTLayer> lstm;
  Weight jenc, jpred, jout;
  const float *jencb = nullptr, *jpredb = nullptr, *joutb = nullptr;
};

// DecoderState (rnnt.go:19-24).
struct TDTState {
  std::vector<std::vector<float>> h, c;
  int last = -1;
  void init(const TDT& m) {
    h.assign(m.lstm.size(), std::vector<float>(size_t(m.H), 0.f));
    c.assign(m.lstm.size(), std::vector<float>(size_t(m.H), 0.f));
    last = -1;
  }
};

struct TDTToken {
  int id, frame, duration;
  float p;
};

inline float tanh32(float x) { return float(std::tanh(double(x))); }

// predict, rnnt.go:46-68: one step from st (fed st.last) into next; returns
// the top layer's h (a row of next).
inline const float* tdt_predict(const TDT& m, const TDTState& st, TDTState& next, std::vector<float>& gates,
                                std::vector<float>& tmp) {
  const int H = m.H;
  std::vector<float> x0((size_t)H, 0.f);
  if (st.last >= 0 && st.last != m.blank)
    for (int j = 0; j < H; j++) x0[size_t(j)] = m.embed[size_t(st.last) * H + j];
  const float* x = x0.data();
  for (size_t l = 0; l < m.lstm.size(); l++) {
    const TDTLayer& ly = m.lstm[l];
    linear(gates.data(), x, 1, ly.wx, ly.b);
    linear(tmp.data(), st.h[l].data(), 1, ly.wh, nullptr);
    add_to(gates.data(), tmp.data(), 4 * H);
    float* h = next.h[l].data();
    float* c = next.c[l].data();
    const float* cp = st.c[l].data();
    for (int j = 0; j < H; j++) {
      const float i = sigmoid_go(gates[size_t(j)]);
      const float f = sigmoid_go(gates[size_t(H + j)]);
      const float g = tanh32(gates[size_t(2 * H + j)]);
      const float o = sigmoid_go(gates[size_t(3 * H + j)]);
      c[j] = f * cp[j] + i * g;
      h[j] = o * tanh32(c[j]);
    }
    x = h;
  }
  return x;
}

// softmaxAt, rnnt.go:80-89.
inline float softmax_at(const float* v, int n, int i) {
  const float mx = v[argmax(v, n)];
  double s = 0;
  for (int k = 0; k < n; k++) s += std::exp(double(v[k] - mx));
  return float(std::exp(double(v[i] - mx)) / s);
}

// Go's builtin max(v, 0) for float32: NaN stays NaN, -0 gives +0.
inline float relu_go(float v) { return v != v ? v : (v > 0.f ? v : 0.f); }

// joint, rnnt.go:91-106.
inline void tdt_joint(const TDT& m, const float* enc_proj, const float* pred, float* hidden, float* pred_proj,
                      float* logits) {
  linear(pred_proj, pred, 1, m.jpred, m.jpredb);
  for (int i = 0; i < m.J; i++) {
    float v = enc_proj[i] + pred_proj[i];
    switch (m.act) {
      case ACT_SIGMOID:
        v = sigmoid_go(v);
        break;
      case ACT_TANH:
        v = tanh32(v);
        break;
      default:
        v = relu_go(v);
    }
    hidden[i] = v;
  }
  linear(logits, hidden, 1, m.jout, m.joutb);
}

// Decode, rnnt.go:111-173. st is read and left at the state after the last
// iteration (the reference's deferred copyFrom). Returns the tokens;
// *iters gets the loop's iteration count and *emits the prediction steps.
inline std::vector<TDTToken> tdt_decode(const TDT& m, const float* enc, int T, TDTState& st, int frame_offset,
                                        long* iters = nullptr, long* preds = nullptr) {
  std::vector<TDTToken> out;
  if (T == 0) return out;
  const int J = m.J, H = m.H;
  TDTState cur = st, next;
  next.init(m);
  std::vector<float> enc_proj((size_t)T * J);
  linear(enc_proj.data(), enc, T, m.jenc, m.jencb);
  std::vector<float> gates((size_t)4 * H), tmp((size_t)4 * H), hidden((size_t)J), pred_proj((size_t)J),
      logits((size_t)m.jout.rows);
  const int ntok = m.V, nd = int(m.durations.size());
  std::vector<float> pred((size_t)H);
  bool dirty = true;
  int step = 0, new_symbols = 0;
  const int max_iters = 16 * T + 1024;
  long it = 0, np = 0;
  for (int iter = 0; step < T && iter < max_iters; iter++) {
    it++;
    if (dirty) {
      const float* p = tdt_predict(m, cur, next, gates, tmp);
      std::copy(p, p + H, pred.begin());
      dirty = false;
      np++;
    }
    tdt_joint(m, enc_proj.data() + size_t(step) * J, pred.data(), hidden.data(), pred_proj.data(), logits.data());
    const int tok = argmax(logits.data(), ntok);
    const bool blank = tok == m.blank;
    int duration = 1;
    if (m.tdt) duration = m.durations[size_t(argmax(logits.data() + ntok, nd))];
    if (!blank) {
      out.push_back({tok, frame_offset + step, duration, softmax_at(logits.data(), ntok, tok)});
      next.last = tok;
      std::swap(cur, next);
      dirty = true;
    }
    if (!m.tdt) {
      if (blank) {
        step++;
        new_symbols = 0;
      } else if (++new_symbols, m.max_symbols > 0 && new_symbols >= m.max_symbols) {
        step++;
        new_symbols = 0;
      }
      continue;
    }
    step += duration;
    new_symbols++;
    if (duration != 0) {
      new_symbols = 0;
    } else if (m.max_symbols > 0 && new_symbols >= m.max_symbols) {
      step++;
      new_symbols = 0;
    }
  }
  st = cur;
  if (iters) *iters = it;
  if (preds) *preds = np;
  return out;
}

}  // namespace orc
