// TEST INFRASTRUCTURE ONLY: C entry points of the CPU oracle, loaded by
// tests/ (ctypes), __graft_entry__.smoke() and bench.py's CPU-baseline leg.
// The product (gorelaxor_b200/csrc) never links or loads this library.
//
// Parity status: the kernel layer is pinned against the reference's own
// known answers and converter fixtures (tests/golden, made by
// tests/golden/make_golden.py from tools/convert_nemo.py); the model-level
// restatement follows the reference line by line but no reference tensor
// dumps exist to pin it end to end (the reference ships none).
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <thread>

#include "conformer.h"
#include "fast.h"
#include "flowlm.h"
#include "mimi.h"
#include "tdt.h"
#include "whisper.h"

using namespace orc;

namespace {

struct OFlowLM {
  FlowLM m;
  std::map<std::string, Weight> w;
  std::map<std::string, const float*> v;
  std::vector<std::vector<float>> tc;
  int decode_steps = 1;
  std::string err;
};

Weight get_w(OFlowLM* o, const std::string& name) {
  auto it = o->w.find(name);
  if (it == o->w.end()) {
    o->err = "missing " + name;
    return Weight{};
  }
  return it->second;
}

const float* get_v(OFlowLM* o, const std::string& name) {
  auto it = o->v.find(name);
  if (it == o->v.end()) {
    o->err = "missing " + name;
    return nullptr;
  }
  return it->second;
}

}  // namespace

extern "C" {

// ---- kernel layer -------------------------------------------------------

// The fast mode (fast.h) on or off for every later call; returns which
// kernels it runs on this processor: 2 AVX-512 VNNI, 1 AVX2, 0 none (the
// exact mode then runs).
int orc_set_fast(int on) {
  fast_flag().store(on ? 1 : 0);
  return cpu_vnni512() ? 2 : cpu_avx2() ? 1 : 0;
}

// A pool of `threads` threads over which the calling thread's products and
// attention heads split (a single stream's work, as the reference's
// Options.Threads); threads <= 1 removes it.
void orc_set_pool(int threads) {
  static std::unique_ptr<Pool> pool;
  tl_pool() = nullptr;
  pool.reset();
  if (threads > 1) {
    pool = std::make_unique<Pool>(threads);
    tl_pool() = pool.get();
  }
}

float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
float orc_expf_go(float x) { return expf_go(x); }
float orc_exp_avx(float x) { return exp_avx(x); }
float orc_gelu_go(float x) { return gelu_go(x); }
float orc_gelu_avx(float x) { return gelu_avx(x); }
float orc_silu_go(float x) { return silu_go(x); }
float orc_silu_avx(float x) { return silu_avx(x); }
float orc_expsub(float* x, int n, float mx) { return expsub_vec(x, n, mx); }
void orc_gelu_vec(float* x, int n) { gelu_vec(x, n); }
void orc_silu_vec(float* x, int n) { silu_vec(x, n); }

void orc_quant_act(int8_t* q, float* sc, const float* x, int nb) { quant_q8_act(q, sc, x, nb); }
void orc_to_q8(uint8_t* out, const float* v, int rows, int cols) { to_q8(out, v, rows, cols); }

// kern.Linear with the reference's dispatch. type: 0 F32, 1 F16, 2 Q8_0.
void orc_linear(float* dst, const float* x, int m, int type, const void* w, int rows, int cols, int dropped,
                const float* bias) {
  Weight wt;
  wt.rows = rows;
  wt.cols = cols;
  wt.type = WType(type);
  if (wt.type == Q8_0) wt.slot = std::make_shared<PanelSlot>();
  wt.f = (const float*)w;
  wt.h = (const uint16_t*)w;
  wt.q = (const uint8_t*)w;
  wt.dropped = dropped != 0;
  linear(dst, x, m, wt, bias);
}

void orc_layer_norm_pt(float* dst, const float* src, int rows, int n, const float* w, const float* b, double eps) {
  layer_norm_pt(dst, src, rows, n, w, b, eps);
}

void orc_rope_table(float* cs, int head_dim, double period, int positions) {
  auto f = rope_freqs(head_dim, period);
  int nf = int(f.size());
  for (int p = 0; p < positions; p++)
    for (int i = 0; i < nf; i++) rope_cs(f[size_t(i)], p, cs + (long(p) * nf + i) * 2, cs + (long(p) * nf + i) * 2 + 1);
}

void orc_attend_one(float* out, const float* q, const float* kc, const float* vc, int nk, int d, int heads) {
  attend_one(out, q, kc, vc, nk, d, heads);
}

// ---- FlowLM -------------------------------------------------------------

void* orc_flowlm_new(int d, int heads, int ff, int layers, int ldim, int fd, int depth, double period) {
  auto* o = new OFlowLM();
  o->m.d = d;
  o->m.heads = heads;
  o->m.ff = ff;
  o->m.ldim = ldim;
  o->m.fd = fd;
  o->m.layers.resize(size_t(layers));
  o->m.res.resize(size_t(depth));
  o->m.freqs = rope_freqs(d / heads, period);
  return o;
}

void orc_flowlm_free(void* h) { delete (OFlowLM*)h; }

// Registers one tensor (the caller keeps the memory alive). Matrices are
// [rows][cols]; Q8_0 rows are 34-byte blocks.
void orc_flowlm_tensor(void* h, const char* name, int type, int rows, int cols, const void* p) {
  auto* o = (OFlowLM*)h;
  Weight w;
  w.rows = rows;
  w.cols = cols;
  w.type = WType(type);
  if (w.type == Q8_0) w.slot = std::make_shared<PanelSlot>();
  w.f = (const float*)p;
  w.q = (const uint8_t*)p;
  o->w[name] = w;
  o->v[name] = (const float*)p;
}

// Binds the registered tensors (pockettts/model.go:240-278) and computes
// the time conditions once (speak.go:57). Returns 0 or -1 (see orc_error).
int orc_flowlm_ready(void* h, int decode_steps) {
  auto* o = (OFlowLM*)h;
  FlowLM& m = o->m;
  char b[128];
  for (size_t i = 0; i < m.layers.size(); i++) {
    std::snprintf(b, sizeof b, "lm.blk.%zu.", i);
    std::string p = b;
    FlowLMLayer& l = m.layers[i];
    l.norm1w = get_v(o, p + "norm1.weight");
    l.norm1b = get_v(o, p + "norm1.bias");
    l.norm2w = get_v(o, p + "norm2.weight");
    l.norm2b = get_v(o, p + "norm2.bias");
    l.qkv = get_w(o, p + "attn_qkv.weight");
    l.out = get_w(o, p + "attn_out.weight");
    l.ff1 = get_w(o, p + "ff1.weight");
    l.ff2 = get_w(o, p + "ff2.weight");
    // pack() drops the transformer's Q8_0 rows (model.go:331-366).
    for (Weight* w : {&l.qkv, &l.out, &l.ff1, &l.ff2}) w->dropped = w->type == Q8_0;
  }
  m.input = get_w(o, "lm.input.weight");
  m.bos = get_v(o, "lm.bos");
  m.outw = get_v(o, "lm.out_norm.weight");
  m.outb = get_v(o, "lm.out_norm.bias");
  m.eosw = get_w(o, "lm.eos.weight");
  const float* eb = get_v(o, "lm.eos.bias");
  m.eosb = eb ? eb[0] : 0;
  m.mean = get_v(o, "lm.emb_mean");
  m.stdv = get_v(o, "lm.emb_std");
  m.cond = get_w(o, "flow.cond.weight");
  m.condb = get_v(o, "flow.cond.bias");
  m.finput = get_w(o, "flow.input.weight");
  m.finputb = get_v(o, "flow.input.bias");
  for (int k = 0; k < 2; k++) {
    std::snprintf(b, sizeof b, "flow.time.%d.", k);
    std::string p = b;
    TimeEmbed& t = m.time[k];
    t.freqs = get_v(o, p + "freqs");
    t.half = 128;
    t.fc1 = get_w(o, p + "fc1.weight");
    t.b1 = get_v(o, p + "fc1.bias");
    t.fc2 = get_w(o, p + "fc2.weight");
    t.b2 = get_v(o, p + "fc2.bias");
    t.alpha = get_v(o, p + "norm.alpha");
  }
  for (size_t i = 0; i < m.res.size(); i++) {
    std::snprintf(b, sizeof b, "flow.res.%zu.", i);
    std::string p = b;
    ResBlock& r = m.res[i];
    r.normw = get_v(o, p + "norm.weight");
    r.normb = get_v(o, p + "norm.bias");
    r.fc1 = get_w(o, p + "fc1.weight");
    r.b1 = get_v(o, p + "fc1.bias");
    r.fc2 = get_w(o, p + "fc2.weight");
    r.b2 = get_v(o, p + "fc2.bias");
    r.ada = get_w(o, p + "ada.weight");
    r.adab = get_v(o, p + "ada.bias");
  }
  m.final_ada = get_w(o, "flow.final.ada.weight");
  m.final_adab = get_v(o, "flow.final.ada.bias");
  m.fout = get_w(o, "flow.final.out.weight");
  m.foutb = get_v(o, "flow.final.out.bias");
  if (o->w.count("lm.embed")) m.embed = get_w(o, "lm.embed");  // optional: text prefill only
  if (o->w.count("lm.speaker_proj") && o->v.count("lm.bos_voice")) {  // optional: voice conditioning only
    m.speaker = get_w(o, "lm.speaker_proj");
    m.bosv = get_v(o, "lm.bos_voice");
  }
  if (!o->err.empty()) return -1;
  o->decode_steps = decode_steps;
  o->tc = time_conds(m, decode_steps);
  return 0;
}

const char* orc_error(void* h) { return ((OFlowLM*)h)->err.c_str(); }

// The time conditions (fd values per decode step).
void orc_flowlm_time_conds(void* h, float* out) {
  auto* o = (OFlowLM*)h;
  for (size_t i = 0; i < o->tc.size(); i++)
    std::memcpy(out + i * size_t(o->m.fd), o->tc[i].data(), sizeof(float) * size_t(o->m.fd));
}

// A stream whose caches hold a voice prompt: kv is [layers][2][n][d]
// (voice.go:40-62, keys already rotated).
void* orc_stream_new(void* h, int n, const float* kv) {
  auto* o = (OFlowLM*)h;
  int L = int(o->m.layers.size()), d = o->m.d;
  auto* s = new Stream();
  s->k.resize(size_t(L));
  s->v.resize(size_t(L));
  for (int l = 0; l < L; l++) {
    const float* kp = kv + (long(l) * 2 + 0) * n * d;
    const float* vp = kv + (long(l) * 2 + 1) * n * d;
    s->k[size_t(l)].assign(kp, kp + long(n) * d);
    s->v[size_t(l)].assign(vp, vp + long(n) * d);
  }
  s->pos = n;
  return s;
}

void orc_stream_free(void* s) { delete (Stream*)s; }

// The voice a clip's Mimi latents [n][ldim] make (voice.go:94-106 after
// the encoder): kv_out gets [layers][2][n + 1][d]. -1 without
// lm.speaker_proj (float32) and lm.bos_voice.
int orc_flowlm_voice_latents(void* h, const float* lat, int n, float* kv_out) {
  auto* o = (OFlowLM*)h;
  const FlowLM& m = o->m;
  if (m.speaker.rows != m.d || m.speaker.type != F32 || !m.bosv || n < 1) return -1;
  Stream st;
  flowlm_voice_latents(m, lat, n, st);
  const size_t rows = size_t(n + 1) * m.d;
  for (size_t l = 0; l < m.layers.size(); l++) {
    std::copy(st.k[l].begin(), st.k[l].end(), kv_out + (l * 2 + 0) * rows);
    std::copy(st.v[l].begin(), st.v[l].end(), kv_out + (l * 2 + 1) * rows);
  }
  return 0;
}

// flowLM.text (lm.go:172-181) on one stream: T token ids appended to its
// caches; lm_out (may be NULL) gets the output at the last token. Returns
// -1 if the model has no lm.embed or an id is out of range.
int orc_flowlm_text(void* h, void* sp, const int* ids, int T, float* lm_out) {
  auto* o = (OFlowLM*)h;
  if (o->m.embed.rows == 0 || T < 1) return -1;
  for (int i = 0; i < T; i++)
    if (ids[i] < 0 || ids[i] >= o->m.embed.rows) return -1;
  flowlm_text(o->m, ids, T, *(Stream*)sp, lm_out);
  return 0;
}
int orc_stream_pos(void* s) { return ((Stream*)s)->pos; }

// One frame of speakChunk's loop (speak.go:146-174) with the noise given:
// step, flow head, scaled latent. latent_in == NULL is the first frame.
// Outputs may be NULL, except latent_out. trace (may be NULL) gets, per
// layer, the residual stream after the layer [L][d], then the input
// projection [d].
float orc_flowlm_frame(void* h, void* sp, const float* latent_in, const float* noise, float* lm_out, float* latent_out,
                       float* scaled_out, float* trace) {
  auto* o = (OFlowLM*)h;
  const FlowLM& m = o->m;
  auto* s = (Stream*)sp;
  std::vector<float> out((size_t)(m.d));
  Trace tr;
  float eos = flowlm_step(m, latent_in, *s, out.data(), trace ? &tr : nullptr);
  if (lm_out) std::memcpy(lm_out, out.data(), sizeof(float) * size_t(m.d));
  flow_sample(m, out.data(), noise, o->tc, latent_out);
  if (scaled_out)
    for (int i = 0; i < m.ldim; i++) scaled_out[i] = latent_out[i] * m.stdv[i] + m.mean[i];
  if (trace) {
    size_t L = m.layers.size();
    for (size_t l = 0; l < L; l++) std::memcpy(trace + l * size_t(m.d), tr.x_after[l].data(), sizeof(float) * size_t(m.d));
    std::memcpy(trace + L * size_t(m.d), tr.x_in.data(), sizeof(float) * size_t(m.d));
  }
  return eos;
}

// `frames` frames for each of n streams, the first from bos, each next one
// from the previous latent. noise is [frames][n][ldim]; latents_out
// [frames][n][ldim], eos_out [frames][n], lm_out (may be NULL)
// [frames][n][d]. Streams run on `threads` threads, one stream at a time
// per thread (independent streams).
void orc_flowlm_run(void* h, int n, void** streams, int frames, const float* noise, float* latents_out, float* eos_out,
                    float* lm_out, int threads) {
  auto* o = (OFlowLM*)h;
  int ld = o->m.ldim, d = o->m.d;
  std::atomic<int> next{0};
  auto work = [&]() {
    for (;;) {
      int i = next.fetch_add(1);
      if (i >= n) return;
      std::vector<float> lat((size_t)ld), prev((size_t)ld);
      for (int f = 0; f < frames; f++) {
        const float* nz = noise + (long(f) * n + i) * ld;
        float* lmo = lm_out ? lm_out + (long(f) * n + i) * d : nullptr;
        float e = orc_flowlm_frame(h, streams[i], f == 0 ? nullptr : prev.data(), nz, lmo, lat.data(), nullptr, nullptr);
        std::memcpy(latents_out + (long(f) * n + i) * ld, lat.data(), sizeof(float) * size_t(ld));
        eos_out[long(f) * n + i] = e;
        prev = lat;
      }
    }
  };
  if (fast_on() && n == 1 && threads > 1) {
    // One stream: its products and attention heads split over the threads,
    // as the reference's Speak runs with Options.Threads (speak.go:100-102).
    Pool pool(threads);
    tl_pool() = &pool;
    work();
    tl_pool() = nullptr;
    return;
  }
  threads = std::max(1, std::min(threads, n));
  std::vector<std::thread> ts;
  for (int t = 1; t < threads; t++) ts.emplace_back(work);
  work();
  for (auto& t : ts) t.join();
}

// ---------------------------------------------------------------- TDT ---
// The greedy RNN-T / TDT decoder of conformer/rnnt.go (see tdt.h).

struct OTDT {
  TDT m;
  std::map<std::string, Weight> w;
  std::map<std::string, const float*> v;
  std::string err;
};

void* orc_tdt_new(int H, int layers, int V, int J, int blank, int max_symbols, int tdt, int act, const int* durations,
                  int nd) {
  auto* o = new OTDT();
  o->m.H = H;
  o->m.V = V;
  o->m.J = J;
  o->m.blank = blank;
  o->m.max_symbols = max_symbols;
  o->m.tdt = tdt != 0;
  o->m.act = act;
  o->m.durations.assign(durations, durations + nd);
  o->m.lstm.resize(size_t(layers));
  return o;
}

void orc_tdt_free(void* h) { delete (OTDT*)h; }

const char* orc_tdt_error(void* h) { return ((OTDT*)h)->err.c_str(); }

void orc_tdt_tensor(void* h, const char* name, int type, int rows, int cols, const void* p) {
  auto* o = (OTDT*)h;
  Weight w;
  w.rows = rows;
  w.cols = cols;
  w.type = WType(type);
  if (w.type == Q8_0) w.slot = std::make_shared<PanelSlot>();
  w.f = (const float*)p;
  w.q = (const uint8_t*)p;
  o->w[name] = w;
  o->v[name] = (const float*)p;
}

// Binds the decoder tensors (conformer/model.go:306-314).
int orc_tdt_ready(void* h) {
  auto* o = (OTDT*)h;
  auto W = [&](const std::string& n) {
    auto it = o->w.find(n);
    if (it == o->w.end()) {
      o->err = "missing " + n;
      return Weight{};
    }
    return it->second;
  };
  auto Vv = [&](const std::string& n) -> const float* {
    auto it = o->v.find(n);
    if (it == o->v.end()) {
      o->err = "missing " + n;
      return nullptr;
    }
    return it->second;
  };
  TDT& m = o->m;
  m.embed = Vv("pred.embed.weight");
  for (size_t i = 0; i < m.lstm.size(); i++) {
    const std::string p = "pred.lstm." + std::to_string(i) + ".";
    m.lstm[i].wx = W(p + "Wx");
    m.lstm[i].wh = W(p + "Wh");
    m.lstm[i].b = Vv(p + "bias");
  }
  m.jenc = W("joint.enc.weight");
  m.jencb = Vv("joint.enc.bias");
  m.jpred = W("joint.pred.weight");
  m.jpredb = Vv("joint.pred.bias");
  m.jout = W("joint.out.weight");
  m.joutb = Vv("joint.out.bias");
  return o->err.empty() ? 0 : -1;
}

// Decode (rnnt.go:111) of one stream. h, c: [layers][H] and *last, the
// DecoderState, read and updated. tokens: [cap][4] (id, frame, duration,
// p as float bits). Returns the token count (all of them, even past cap).
int orc_tdt_decode(void* hm, const float* enc, int T, int frame_offset, float* h, float* c, int* last, int* tokens,
                   int cap, long* iters, long* preds) {
  const TDT& m = ((OTDT*)hm)->m;
  TDTState st;
  st.init(m);
  for (size_t l = 0; l < m.lstm.size(); l++) {
    std::memcpy(st.h[l].data(), h + l * size_t(m.H), sizeof(float) * size_t(m.H));
    std::memcpy(st.c[l].data(), c + l * size_t(m.H), sizeof(float) * size_t(m.H));
  }
  st.last = *last;
  std::vector<TDTToken> out = tdt_decode(m, enc, T, st, frame_offset, iters, preds);
  for (size_t l = 0; l < m.lstm.size(); l++) {
    std::memcpy(h + l * size_t(m.H), st.h[l].data(), sizeof(float) * size_t(m.H));
    std::memcpy(c + l * size_t(m.H), st.c[l].data(), sizeof(float) * size_t(m.H));
  }
  *last = st.last;
  for (size_t i = 0; i < out.size() && int(i) < cap; i++) {
    tokens[4 * i] = out[i].id;
    tokens[4 * i + 1] = out[i].frame;
    tokens[4 * i + 2] = out[i].duration;
    std::memcpy(&tokens[4 * i + 3], &out[i].p, 4);
  }
  return int(out.size());
}

// n independent fresh decodes on `threads` host threads (the CPU baseline):
// enc [n][T][D]; counts [n]; tokens [n][cap][4].
void orc_tdt_run(void* hm, int n, const float* enc, int T, int D, int* tokens, int cap, int* counts, long* iters,
                 int threads) {
  const TDT& m = ((OTDT*)hm)->m;
  std::atomic<int> next{0};
  std::atomic<long> it_total{0};
  auto work = [&]() {
    for (;;) {
      const int i = next.fetch_add(1);
      if (i >= n) return;
      std::vector<float> h(m.lstm.size() * size_t(m.H), 0.f), c(h.size(), 0.f);
      int last = -1;
      long it = 0;
      counts[i] = orc_tdt_decode(hm, enc + size_t(i) * T * D, T, 0, h.data(), c.data(), &last,
                                 tokens + size_t(i) * cap * 4, cap, &it, nullptr);
      it_total += it;
    }
  };
  threads = std::max(1, std::min(threads, n));
  std::vector<std::thread> ts;
  for (int t = 1; t < threads; t++) ts.emplace_back(work);
  work();
  for (auto& t : ts) t.join();
  if (iters) *iters = it_total.load();
}

// ------------------------------------------------------------ Whisper ---
// The text decoder's token loop (whisper/decoder.go, transcribe.go; see
// whisper.h). Matrices are registered as float16 (the reference's memory
// form); orc_q8_to_f16 widens Q8_0 blocks the way the reference loads them.

struct OWhisper {
  Whisper m;
  std::map<std::string, Weight> w;
  std::map<std::string, const float*> v;
  std::string err;
};

void orc_q8_to_f16(const uint8_t* blocks, long n, uint16_t* out) { q8_to_f16(blocks, n, out); }

void* orc_whisper_new(int n_vocab, int n_text_ctx, int n_state, int n_head, int n_layer) {
  auto* o = new OWhisper();
  o->m.n_vocab = n_vocab;
  o->m.n_text_ctx = n_text_ctx;
  o->m.n_state = n_state;
  o->m.n_head = n_head;
  o->m.layers.resize(size_t(n_layer));
  o->m.voc.init(n_vocab);
  return o;
}

void orc_whisper_free(void* h) { delete (OWhisper*)h; }

const char* orc_whisper_error(void* h) { return ((OWhisper*)h)->err.c_str(); }

// type 0: float32 (vectors or matrices), 1: float16 matrix [rows][cols].
void orc_whisper_tensor(void* h, const char* name, int type, int rows, int cols, const void* p) {
  auto* o = (OWhisper*)h;
  Weight w;
  w.rows = rows;
  w.cols = cols;
  w.type = WType(type);
  if (w.type == Q8_0) w.slot = std::make_shared<PanelSlot>();
  w.f = (const float*)p;
  w.h = (const uint16_t*)p;
  o->w[name] = w;
  o->v[name] = (const float*)p;
}

// The vocabulary's words (lengths[i] bytes each, concatenated): the " "
// token and vocab.suppressed() (vocab.go:96-118): the non-speech marks and
// their " "-prefixed forms below eot, then " -" and " '".
void orc_whisper_vocab(void* h, const char* bytes, const int* lengths, int nwords) {
  auto* o = (OWhisper*)h;
  std::map<std::string, int> to_id;
  long off = 0;
  for (int i = 0; i < nwords; i++) {
    std::string w(bytes + off, size_t(lengths[i]));
    off += lengths[i];
    to_id.emplace(w, i);
  }
  WVocab& v = o->m.voc;
  auto it = to_id.find(" ");
  v.space = it == to_id.end() ? -1 : it->second;
  static const char* marks[] = {"\"", "#", "(", ")", "*", "+", "/", ":", ";", "<", "=", ">", "@", "[", "\\", "]", "^",
                                "_", "`", "{", "|", "}", "~", "「", "」", "『", "』", "<<", ">>", "<<<", ">>>", "--",
                                "---", "-(", "-[", "('", "(\"", "((", "))", "(((", ")))", "[[", "]]", "{{", "}}",
                                "♪♪", "♪♪♪", "♩", "♪", "♫", "♬", "♭", "♮", "♯"};
  v.suppress.clear();
  for (const char* t : marks)
    for (const std::string& s : {std::string(t), " " + std::string(t)}) {
      auto f = to_id.find(s);
      if (f != to_id.end() && f->second < v.eot) v.suppress.push_back(f->second);
    }
  for (const char* s : {" -", " '"}) {
    auto f = to_id.find(s);
    if (f != to_id.end()) v.suppress.push_back(f->second);
  }
}

int orc_whisper_suppress(void* h, int* out, int cap) {
  const auto& s = ((OWhisper*)h)->m.voc.suppress;
  for (size_t i = 0; i < s.size() && int(i) < cap; i++) out[i] = s[i];
  return int(s.size());
}

// Binds the decoder tensors (whisper/model.go:464-484).
int orc_whisper_ready(void* h) {
  auto* o = (OWhisper*)h;
  auto W = [&](const std::string& n) {
    auto it = o->w.find(n);
    if (it == o->w.end()) {
      o->err = "missing " + n;
      return Weight{};
    }
    return it->second;
  };
  auto V = [&](const std::string& n) -> const float* {
    auto it = o->v.find(n);
    if (it == o->v.end()) {
      o->err = "missing " + n;
      return nullptr;
    }
    return it->second;
  };
  Whisper& m = o->m;
  m.dec_pos = V("decoder.positional_embedding");
  m.tok_emb = W("decoder.token_embedding.weight");
  m.ln_w = V("decoder.ln.weight");
  m.ln_b = V("decoder.ln.bias");
  for (size_t i = 0; i < m.layers.size(); i++) {
    const std::string p = "decoder.blocks." + std::to_string(i) + ".";
    WLayer& L = m.layers[i];
    L.attn_ln_w = V(p + "attn_ln.weight");
    L.attn_ln_b = V(p + "attn_ln.bias");
    L.q = W(p + "attn.query.weight");
    L.qb = V(p + "attn.query.bias");
    L.k = W(p + "attn.key.weight");
    L.v = W(p + "attn.value.weight");
    L.vb = V(p + "attn.value.bias");
    L.o = W(p + "attn.out.weight");
    L.ob = V(p + "attn.out.bias");
    L.x_ln_w = V(p + "cross_attn_ln.weight");
    L.x_ln_b = V(p + "cross_attn_ln.bias");
    L.xq = W(p + "cross_attn.query.weight");
    L.xqb = V(p + "cross_attn.query.bias");
    L.xk = W(p + "cross_attn.key.weight");
    L.xv = W(p + "cross_attn.value.weight");
    L.xvb = V(p + "cross_attn.value.bias");
    L.xo = W(p + "cross_attn.out.weight");
    L.xob = V(p + "cross_attn.out.bias");
    L.mlp_ln_w = V(p + "mlp_ln.weight");
    L.mlp_ln_b = V(p + "mlp_ln.bias");
    L.fc1 = W(p + "mlp.0.weight");
    L.fc1b = V(p + "mlp.0.bias");
    L.fc2 = W(p + "mlp.2.weight");
    L.fc2b = V(p + "mlp.2.bias");
  }
  if (m.n_mels > 0) {  // the audio encoder (model.go:352-372)
    m.enc_pos = V("encoder.positional_embedding");
    m.conv1 = W("encoder.conv1.weight");
    m.conv1b = V("encoder.conv1.bias");
    m.conv2 = W("encoder.conv2.weight");
    m.conv2b = V("encoder.conv2.bias");
    m.enc_ln_w = V("encoder.ln_post.weight");
    m.enc_ln_b = V("encoder.ln_post.bias");
    for (size_t i = 0; i < m.enc.size(); i++) {
      const std::string p = "encoder.blocks." + std::to_string(i) + ".";
      WEncLayer& L = m.enc[i];
      L.attn_ln_w = V(p + "attn_ln.weight");
      L.attn_ln_b = V(p + "attn_ln.bias");
      L.q = W(p + "attn.query.weight");
      L.qb = V(p + "attn.query.bias");
      L.k = W(p + "attn.key.weight");
      L.v = W(p + "attn.value.weight");
      L.vb = V(p + "attn.value.bias");
      L.o = W(p + "attn.out.weight");
      L.ob = V(p + "attn.out.bias");
      L.mlp_ln_w = V(p + "mlp_ln.weight");
      L.mlp_ln_b = V(p + "mlp_ln.bias");
      L.fc1 = W(p + "mlp.0.weight");
      L.fc1b = V(p + "mlp.0.bias");
      L.fc2 = W(p + "mlp.2.weight");
      L.fc2b = V(p + "mlp.2.bias");
    }
  }
  return o->err.empty() ? 0 : -1;
}

// Declares the audio encoder's shape; its tensors are then bound by
// orc_whisper_ready.
void orc_whisper_encoder(void* h, int n_mels, int n_audio_head, int n_audio_layer) {
  Whisper& m = ((OWhisper*)h)->m;
  m.n_mels = n_mels;
  m.n_audio_head = n_audio_head;
  m.enc.resize(size_t(n_audio_layer));
}

// encode of one window: mel [n_mels][3000] → out [1500][state].
void orc_whisper_encode(void* h, const float* mel, float* out) { whisper_encode(((OWhisper*)h)->m, mel, out); }
// The front end and the first `blocks` blocks only (a timing sample).
void orc_whisper_encode_blocks(void* h, const float* mel, float* out, int blocks) {
  whisper_encode(((OWhisper*)h)->m, mel, out, blocks);
}

void* orc_wseq_new(void* h) {
  auto* s = new WSeq();
  s->init(((OWhisper*)h)->m);
  return s;
}

void orc_wseq_free(void* s) { delete (WSeq*)s; }

void orc_whisper_cross_kv(void* h, void* s, const float* enc) { whisper_cross_kv(((OWhisper*)h)->m, *(WSeq*)s, enc); }

// The sequence's cross K ([heads][ctx][hd], pre-scaled) and V ([heads][hd][ctx]) of a layer.
void orc_wseq_cross(void* s, int layer, float* k, float* v) {
  auto* q = (WSeq*)s;
  std::copy(q->ck[size_t(layer)].begin(), q->ck[size_t(layer)].end(), k);
  std::copy(q->cv[size_t(layer)].begin(), q->cv[size_t(layer)].end(), v);
}

int orc_whisper_decode(void* h, void* s, const int* tokens, int nt, const int* want, int nwant, float* logits) {
  return whisper_decode(((OWhisper*)h)->m, *(WSeq*)s, tokens, nt, want, nwant, logits) ? 0 : -1;
}

// The packed or per-row matmul of whisper/gemm.go (tests of its order).
void orc_whisper_matmul(float* c, const float* a, int m, int n, int k, int type, const void* b, const float* bias) {
  Weight w;
  w.rows = n;
  w.cols = k;
  w.type = WType(type);
  if (w.type == Q8_0) w.slot = std::make_shared<PanelSlot>();
  w.f = (const float*)b;
  w.h = (const uint16_t*)b;
  matmul_whisper(c, n, a, k, m, n, k, w, bias);
}

// process + sample at temperature 0 for a sequence in state st = {nt,
// last, penult, has_ts, seek_delta}; lg is modified as process does.
// out = {id, tid, p bits, plog bits}.
void orc_whisper_process_sample(void* h, const int* st, float* lg, int* out) {
  WSampleState q;
  q.nt = st[0], q.last = st[1], q.penult = st[2], q.has_ts = st[3] != 0, q.seek_delta = st[4];
  const WToken t = whisper_process_sample(((OWhisper*)h)->m, q, lg);
  out[0] = t.id;
  out[1] = t.tid;
  std::memcpy(&out[2], &t.p, 4);
  std::memcpy(&out[3], &t.plog, 4);
}

// whisper_greedy (see whisper.h). tokens [steps][4]; returns the count.
int orc_whisper_greedy(void* h, void* s, const int* prompt, int np, int sot_at, int steps, int* tokens,
                       float* no_speech) {
  const std::vector<WToken> out = whisper_greedy(((OWhisper*)h)->m, *(WSeq*)s, prompt, np, sot_at, steps, no_speech);
  for (size_t i = 0; i < out.size(); i++) {
    tokens[4 * i] = out[i].id;
    tokens[4 * i + 1] = out[i].tid;
    std::memcpy(&tokens[4 * i + 2], &out[i].p, 4);
    std::memcpy(&tokens[4 * i + 3], &out[i].plog, 4);
  }
  return int(out.size());
}

// n independent streams on host threads (the CPU baseline): each takes its
// encoder output enc + i·ctx·state, the cross K/V, then the greedy run.
void orc_whisper_run(void* h, int n, const float* enc, const int* prompt, int np, int sot_at, int steps, int* tokens,
                     int threads) {
  const Whisper& m = ((OWhisper*)h)->m;
  std::atomic<int> next{0};
  auto work = [&]() {
    for (;;) {
      const int i = next.fetch_add(1);
      if (i >= n) return;
      WSeq s;
      s.init(m);
      whisper_cross_kv(m, s, enc + size_t(i) * m.n_audio_ctx * m.n_state);
      const std::vector<WToken> out = whisper_greedy(m, s, prompt, np, sot_at, steps, nullptr);
      for (size_t k = 0; k < out.size(); k++) tokens[(size_t(i) * steps + k)] = out[k].id;
    }
  };
  if (fast_on() && n == 1 && threads > 1) {
    // One stream: its products and attention heads split over the threads,
    // as the reference's Speak runs with Options.Threads (speak.go:100-102).
    Pool pool(threads);
    tl_pool() = &pool;
    work();
    tl_pool() = nullptr;
    return;
  }
  threads = std::max(1, std::min(threads, n));
  std::vector<std::thread> ts;
  for (int t = 1; t < threads; t++) ts.emplace_back(work);
  work();
  for (auto& t : ts) t.join();
}


// ---- Mimi decoder ---------------------------------------------------------

struct OMimi {
  MimiDecoder m;
  MimiEncoder enc;
  bool has_enc = false;
  std::vector<float> zeros;
  std::map<std::string, Weight> w;
  std::map<std::string, const float*> v;
  std::string err;
  std::vector<int> ratios;
  int nf = 0, kk = 0, resk = 0, lastk = 0, dil = 0, comp = 0, nres = 0;
};

// Config as the loader reads it (model.go:280-300): d, heads, ff, context,
// max period, upsample; SEANet ratios, n_filters, kernel sizes, dilation
// base, compress, residual layers; latent dim and sample rate.
void* orc_mimi_new(int d, int heads, int ff, int context, double period, int up, const int* ratios, int nratios,
                   int nf, int k, int resk, int lastk, int dil, int comp, int nres, int ldim, int sample_rate) {
  auto* o = new OMimi();
  o->m.tf.d = d;
  o->m.tf.heads = heads;
  o->m.tf.ff = ff;
  o->m.tf.context = context;
  o->m.tf.freqs = rope_freqs(d / heads, period);
  o->m.upS = up;
  o->m.ldim = ldim;
  o->m.sample_rate = sample_rate;
  o->ratios.assign(ratios, ratios + nratios);
  o->nf = nf, o->kk = k, o->resk = resk, o->lastk = lastk, o->dil = dil, o->comp = comp, o->nres = nres;
  int hop = 1;
  for (int r : o->ratios) hop *= r;
  o->m.frame = hop * up;
  return o;
}
void orc_mimi_free(void* h) { delete (OMimi*)h; }
void orc_mimi_tensor(void* h, const char* name, int type, int rows, int cols, const void* p) {
  auto* o = (OMimi*)h;
  Weight w;
  w.rows = rows;
  w.cols = cols;
  w.type = WType(type);
  if (w.type == Q8_0) w.slot = std::make_shared<PanelSlot>();
  w.f = (const float*)p;
  w.q = (const uint8_t*)p;
  o->w[name] = w;
  o->v[name] = (const float*)p;
}
const char* orc_mimi_error(void* h) { return ((OMimi*)h)->err.c_str(); }

// Binds the tensors the way model.go:102-200 names them.
int orc_mimi_ready(void* h) {
  auto* o = (OMimi*)h;
  MimiDecoder& m = o->m;
  auto W = [&](const std::string& n) {
    auto it = o->w.find(n);
    if (it == o->w.end()) {
      if (o->err.empty()) o->err = "missing " + n;
      return Weight{};
    }
    return it->second;
  };
  auto V = [&](const std::string& n) -> const float* {
    auto it = o->v.find(n);
    if (it == o->v.end()) {
      if (o->err.empty()) o->err = "missing " + n;
      return nullptr;
    }
    return it->second;
  };
  m.quant = W("mimi.quant");
  m.up = V("mimi.up");
  for (int i = 0;; i++) {
    const std::string p = "mimi.dec_tf." + std::to_string(i) + ".";
    if (!o->w.count(p + "attn_qkv.weight")) break;
    MLayer l;
    l.norm1w = V(p + "norm1.weight");
    l.norm1b = V(p + "norm1.bias");
    l.norm2w = V(p + "norm2.weight");
    l.norm2b = V(p + "norm2.bias");
    l.ls1 = V(p + "ls1");
    l.ls2 = V(p + "ls2");
    l.qkv = W(p + "attn_qkv.weight");
    l.out = W(p + "attn_out.weight");
    l.ff1 = W(p + "ff1.weight");
    l.ff2 = W(p + "ff2.weight");
    m.tf.layers.push_back(l);
  }
  auto conv = [&](const std::string& n, int cin, int cout, int k, int stride, int dl) {
    MConv c;
    c.w = W(n + ".weight");
    c.b = V(n + ".bias");
    c.cin = cin, c.cout = cout, c.k = k, c.stride = stride, c.dil = dl;
    return c;
  };
  int mult = 1 << o->ratios.size();
  MStep first;
  first.kind = 0;
  first.c = conv("mimi.dec.0", m.tf.d, mult * o->nf, o->kk, 1, 1);
  m.steps.push_back(first);
  int idx = 1;
  for (int r : o->ratios) {
    idx++;
    MStep t;
    t.kind = 1;
    t.elu = true;
    const std::string n = "mimi.dec." + std::to_string(idx);
    t.t.w = W(n + ".weight");
    t.t.b = V(n + ".bias");
    t.t.cin = mult * o->nf, t.t.cout = mult * o->nf / 2, t.t.k = 2 * r, t.t.stride = r;
    m.steps.push_back(t);
    idx++;
    const int dim = mult * o->nf / 2;
    for (int j = 0, dl = 1; j < o->nres; j++, dl *= o->dil) {
      const std::string p = "mimi.dec." + std::to_string(idx) + ".";
      MStep rb;
      rb.kind = 2;
      rb.ra = conv(p + "1", dim, dim / o->comp, o->resk, 1, dl);
      rb.rb = conv(p + "3", dim / o->comp, dim, 1, 1, 1);
      m.steps.push_back(rb);
      idx++;
    }
    mult /= 2;
  }
  idx++;
  MStep last;
  last.kind = 0;
  last.elu = true;
  last.c = conv("mimi.dec." + std::to_string(idx), o->nf, 1, o->lastk, 1, 1);
  m.steps.push_back(last);
  // the encoder (model.go:181-200, 308-313), when the tensors are there
  if (o->w.count("mimi.enc.0.weight")) {
    o->has_enc = true;
    MimiEncoder& e = o->enc;
    e.tf.d = m.tf.d, e.tf.heads = m.tf.heads, e.tf.ff = m.tf.ff, e.tf.context = m.tf.context;
    e.tf.freqs = m.tf.freqs;
    for (int i = 0;; i++) {
      const std::string p = "mimi.enc_tf." + std::to_string(i) + ".";
      if (!o->w.count(p + "attn_qkv.weight")) break;
      MLayer l;
      l.norm1w = V(p + "norm1.weight");
      l.norm1b = V(p + "norm1.bias");
      l.norm2w = V(p + "norm2.weight");
      l.norm2b = V(p + "norm2.bias");
      l.ls1 = V(p + "ls1");
      l.ls2 = V(p + "ls2");
      l.qkv = W(p + "attn_qkv.weight");
      l.out = W(p + "attn_out.weight");
      l.ff1 = W(p + "ff1.weight");
      l.ff2 = W(p + "ff2.weight");
      e.tf.layers.push_back(l);
    }
    MStep first;
    first.c = conv("mimi.enc.0", 1, o->nf, o->kk, 1, 1);
    e.steps.push_back(first);
    int eidx = 1, emult = 1;
    for (int ri = int(o->ratios.size()) - 1; ri >= 0; ri--) {
      const int r = o->ratios[size_t(ri)], dim = emult * o->nf;
      for (int j = 0, dl = 1; j < o->nres; j++, dl *= o->dil) {
        const std::string p = "mimi.enc." + std::to_string(eidx) + ".";
        MStep rb;
        rb.kind = 2;
        rb.ra = conv(p + "1", dim, dim / o->comp, o->resk, 1, dl);
        rb.rb = conv(p + "3", dim / o->comp, dim, 1, 1, 1);
        e.steps.push_back(rb);
        eidx++;
      }
      eidx++;  // ELU
      MStep cv;
      cv.elu = true;
      cv.c = conv("mimi.enc." + std::to_string(eidx), dim, 2 * dim, 2 * r, r, 1);
      e.steps.push_back(cv);
      eidx++;
      emult *= 2;
    }
    eidx++;
    MStep elast;
    elast.elu = true;
    elast.c = conv("mimi.enc." + std::to_string(eidx), emult * o->nf, m.tf.d, o->lastk, 1, 1);
    e.steps.push_back(elast);
    o->zeros.assign(size_t(m.ldim), 0.f);
    e.down.w = W("mimi.down");
    e.down.b = o->zeros.data();
    e.down.cin = m.tf.d, e.down.cout = m.ldim, e.down.k = 2 * m.upS, e.down.stride = m.upS, e.down.dil = 1;
  }
  return o->err.empty() ? 0 : -1;
}

// cloneCond's Mimi encoding of n samples (24 kHz): the latents [frames][ldim]
// into out (room for (n + frame − 1)/frame rows); returns the row count, or
// −1 without an encoder.
int orc_mimi_clone_latents(void* h, const float* x, int n, float* out) {
  auto* o = (OMimi*)h;
  if (!o->has_enc) return -1;
  const std::vector<float> lat = mimi_clone_latents(o->enc, x, n, o->m.frame);
  std::copy(lat.begin(), lat.end(), out);
  return int(lat.size() / size_t(o->m.ldim));
}

void* orc_mimi_state(void* h) { return new MimiState(mimi_state(((OMimi*)h)->m)); }
void orc_mimi_state_free(void* s) { delete (MimiState*)s; }
// One latent [ldim] → one frame of samples.
void orc_mimi_decode(void* h, void* s, const float* lat, float* pcm) {
  mimi_decode(((OMimi*)h)->m, *(MimiState*)s, lat, pcm);
}
int orc_mimi_frame(void* h) { return ((OMimi*)h)->m.frame; }
void orc_elu(float* x, long n) { elu_vec(x, n); }

// The streaming pieces alone, for the reference's model-free checks
// (pockettts/nn_test.go:37-153): conv.run, convtr.run and attend with a
// context window, float32 weights.
void orc_mimi_conv_run(const float* w, const float* b, int cin, int cout, int k, int stride, int dil, float* prev,
                       const float* x, int T, float* y) {
  MConv c;
  c.w.type = F32, c.w.rows = cout, c.w.cols = k * cin, c.w.f = w;
  c.b = b, c.cin = cin, c.cout = cout, c.k = k, c.stride = stride, c.dil = dil;
  std::vector<float> pv(prev, prev + size_t(c.past()) * cin);
  conv_run(c, pv, x, T, y);
  std::copy(pv.begin(), pv.end(), prev);
}
void orc_mimi_convtr_run(const float* w, const float* b, int cin, int cout, int k, int S, float* partial,
                         const float* x, int T, float* y) {
  MConvTr c;
  c.w.type = F32, c.w.rows = k * cout, c.w.cols = cin, c.w.f = w;
  c.b = b, c.cin = cin, c.cout = cout, c.k = k, c.stride = S;
  std::vector<float> pt(partial, partial + size_t(k - S) * cout);
  convtr_run(c, pt, x, T, y);
  std::copy(pt.begin(), pt.end(), partial);
}
void orc_attend_window(float* out, const float* qkv, int T, const float* kc, const float* vc, int pos0, int d,
                       int heads, int context) {
  attend_window(out, qkv, T, kc, vc, pos0, d, heads, context);
}

// ---- the FastConformer encoder (conformer.h) ----

struct OConf {
  Conformer m;
  std::map<std::string, Weight> w;
  std::map<std::string, const float*> v;
  std::map<std::string, std::pair<int, int>> shape;
  std::vector<std::vector<uint8_t>> own;  // Q8_0 blocks made by ToQ8
  std::string err;
};

void* orc_fconf_new(int d, int heads, int layers, int dff, int kernel, int sub_c, int n_mels, int xscaling,
                    int ln_conv) {
  auto* o = new OConf();
  Conformer& m = o->m;
  m.d = d, m.heads = heads, m.dff = dff, m.kernel = kernel, m.sub_c = sub_c, m.n_mels = n_mels;
  m.xscaling = xscaling != 0, m.ln_conv = ln_conv != 0;
  m.blocks.resize(size_t(layers));
  return o;
}
void orc_fconf_free(void* h) { delete (OConf*)h; }
const char* orc_fconf_error(void* h) { return ((OConf*)h)->err.c_str(); }

// type 0: float32 values, 1: float16 bits (a matrix), 2: Q8_0 blocks.
void orc_fconf_tensor(void* h, const char* name, int type, int rows, int cols, const void* p) {
  auto* o = (OConf*)h;
  Weight w;
  w.rows = rows, w.cols = cols;
  w.type = type == 2 ? Q8_0 : type == 1 ? F16 : F32;
  w.f = (const float*)p;
  w.h = (const uint16_t*)p;
  w.q = (const uint8_t*)p;
  o->w[name] = w;
  o->v[name] = (const float*)p;
  o->shape[name] = {rows, cols};
}

// loadEncoder, model.go:357-410.
int orc_fconf_ready(void* h) {
  auto* o = (OConf*)h;
  Conformer& m = o->m;
  auto V = [&](const std::string& n) -> const float* {
    auto it = o->v.find(n);
    if (it == o->v.end()) {
      if (o->err.empty()) o->err = "missing " + n;
      return nullptr;
    }
    return it->second;
  };
  auto Vopt = [&](const std::string& n) -> const float* {
    auto it = o->v.find(n);
    return it == o->v.end() ? nullptr : it->second;
  };
  auto W = [&](const std::string& n) -> Weight {
    auto it = o->w.find(n);
    if (it == o->w.end()) {
      if (o->err.empty()) o->err = "missing " + n;
      return Weight{};
    }
    Weight w = it->second;
    if (w.type == F16 && w.cols % QK == 0) {  // ToQ8 (kern.go:139-170) from the widened values
      std::vector<float> f(size_t(w.rows) * w.cols);
      for (size_t i = 0; i < f.size(); i++) f[i] = f16_to_f32(w.h[i]);
      o->own.emplace_back(size_t(w.rows) * (w.cols / QK) * Q8BYTES);
      to_q8(o->own.back().data(), f.data(), w.rows, w.cols);
      w.type = Q8_0;
      w.q = o->own.back().data();
      w.slot = std::make_shared<PanelSlot>();
    }
    return w;
  };
  auto taps = [&](const std::string& n, int c, int ntaps) {  // transposeTaps: [c][taps] → [taps][c]
    std::vector<float> out(size_t(c) * ntaps);
    const float* src = V(n);
    if (src)
      for (int i = 0; i < c; i++)
        for (int j = 0; j < ntaps; j++) out[size_t(j) * c + i] = src[size_t(i) * ntaps + j];
    return out;
  };
  const std::string pe = "enc.pre_encode.";
  const int c = m.sub_c, d = m.d;
  m.w0 = taps(pe + "conv.0.weight", c, 9);
  m.b0 = V(pe + "conv.0.bias");
  m.w2 = taps(pe + "conv.2.weight", c, 9);
  m.b2 = V(pe + "conv.2.bias");
  m.w3 = W(pe + "conv.3.weight");
  m.b3 = V(pe + "conv.3.bias");
  m.w5 = taps(pe + "conv.5.weight", c, 9);
  m.b5 = V(pe + "conv.5.bias");
  m.w6 = W(pe + "conv.6.weight");
  m.b6 = V(pe + "conv.6.bias");
  m.out = W(pe + "out.weight");
  m.outb = V(pe + "out.bias");
  for (size_t i = 0; i < m.blocks.size(); i++) {
    const std::string p = "enc.blocks." + std::to_string(i) + ".";
    CBlock& b = m.blocks[i];
    auto ff = [&](const std::string& n) {
      CFF f;
      f.norm_w = V(p + "norm_" + n + ".weight");
      f.norm_b = V(p + "norm_" + n + ".bias");
      f.w1 = W(p + n + ".linear1.weight");
      f.b1 = Vopt(p + n + ".linear1.bias");
      f.w2 = W(p + n + ".linear2.weight");
      f.b2 = Vopt(p + n + ".linear2.bias");
      return f;
    };
    b.ff1 = ff("ff1");
    b.ff2 = ff("ff2");
    b.norm_att_w = V(p + "norm_attn.weight");
    b.norm_att_b = V(p + "norm_attn.bias");
    b.q = W(p + "attn.linear_q.weight");
    b.qb = Vopt(p + "attn.linear_q.bias");
    b.k = W(p + "attn.linear_k.weight");
    b.kb = Vopt(p + "attn.linear_k.bias");
    b.v = W(p + "attn.linear_v.weight");
    b.vb = Vopt(p + "attn.linear_v.bias");
    b.out = W(p + "attn.linear_out.weight");
    b.outb = Vopt(p + "attn.linear_out.bias");
    b.pos = W(p + "attn.linear_pos.weight");
    b.pos_u = V(p + "attn.pos_bias_u");
    b.pos_v = V(p + "attn.pos_bias_v");
    b.norm_conv_w = V(p + "norm_conv.weight");
    b.norm_conv_b = V(p + "norm_conv.bias");
    b.pw1 = W(p + "conv.pointwise1.weight");
    b.pw1b = Vopt(p + "conv.pointwise1.bias");
    b.pw2 = W(p + "conv.pointwise2.weight");
    b.pw2b = Vopt(p + "conv.pointwise2.bias");
    b.dw = taps(p + "conv.depthwise.weight", d, m.kernel);
    b.dwb = Vopt(p + "conv.depthwise.bias");
    b.norm_out_w = V(p + "norm_out.weight");
    b.norm_out_b = V(p + "norm_out.bias");
    const float *gw = V(p + "conv.bn.weight"), *gb = V(p + "conv.bn.bias");
    if (m.ln_conv) {
      if (gw && gb) b.cn_w.assign(gw, gw + d), b.cn_b.assign(gb, gb + d);
    } else {
      const float *mean = V(p + "conv.bn.running_mean"), *vr = V(p + "conv.bn.running_var");
      if (gw && gb && mean && vr) {
        b.cn_w.resize(size_t(d));
        b.cn_b.resize(size_t(d));
        for (int j = 0; j < d; j++) {
          const float sc = float(double(gw[j]) / std::sqrt(double(vr[j]) + 1e-5));
          b.cn_w[size_t(j)] = sc;
          b.cn_b[size_t(j)] = gb[j] - mean[j] * sc;
        }
      }
    }
  }
  return o->err.empty() ? 0 : -1;
}

// Model.encode of one utterance: mel [n_mels][frames], the first valid real;
// out gets [L][d] (room for sub_out³(frames) rows); returns L. max_blocks ≥ 0
// runs that many blocks only (a timing sample).
int orc_fconf_encode(void* h, const float* mel, int frames, int valid, float* out, int max_blocks) {
  int L = 0;
  std::vector<float> x = conformer_encode(((OConf*)h)->m, mel, frames, valid, &L, max_blocks);
  std::copy(x.begin(), x.end(), out);
  return L;
}

}  // extern "C"
