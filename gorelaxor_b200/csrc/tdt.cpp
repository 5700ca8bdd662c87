// The C ABI of the TDT / RNN-T decoder (include/grx.h): the decoder part of
// conformer.FromGGUF (conformer/model.go:190-236, 306-314) and
// Model.Decode (conformer/rnnt.go:111-173) for a batch of streams, with
// the loop on the device (k_tdt.cu): one round of kernels per iteration,
// replayed from a CUDA graph, the host only polling for the end.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/grx.h"
#include "gguf.h"
#include "host.h"
#include "kernels.h"

using namespace grx;

struct grx_tdt {
  Arena ar;
  int dev = 0;
  int H = 0, layers = 0, V = 0, J = 0, D = 0, nout = 0, blank = 0, max_symbols = 10, tdt = 1, act = 0;
  std::vector<int> durations;
  float* embed = nullptr;
  std::vector<DQ8> wx, wh;
  std::vector<float*> lb;
  DQ8 jenc, jpred, jout;
  float *jenc_b = nullptr, *jpred_b = nullptr, *jout_b = nullptr;
};

struct grx_tdt_batch {
  Arena ar;
  grx_tdt* m = nullptr;
  int n = 0, max_t = 0, cap = 0;
  cudaStream_t st = nullptr;
  TdtArgs a;
  // encoder projection: the rows rounded to Q8_0 and the product
  int8_t* eq = nullptr;
  float2* es = nullptr;
  float* enc_proj = nullptr;
  float* enc_row = nullptr;  // [n][J]: the float-path product of row 0 (streams with T = 1)
  float* d_enc = nullptr;    // [n][max_t][D] staging for host input
  int* d_T = nullptr;
  int* d_off = nullptr;
  int* tokens = nullptr;  // [n][cap][4] staging for host output
  int* h_count = nullptr; // pinned [2]: the active count after a replay
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaGraphExec_t exec = nullptr;
  int per_replay = 0;  // iterations per graph replay
  int64_t launches = 0, iterations = 0;
  ~grx_tdt_batch() {
    cudaSetDevice(ar.dev);
    if (exec) cudaGraphExecDestroy(exec);
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
    if (h_count) cudaFreeHost(h_count);
    if (st) cudaStreamDestroy(st);
  }
};

namespace {

constexpr int kRoundsPerReplay = 8;  // loop iterations per graph replay (even: the parity returns to 0)

int launches_per_iteration(const grx_tdt* m) { return m->layers + 3; }

}  // namespace

extern "C" {

int grx_tdt_load(const void* bytes, size_t len, int device, grx_tdt** out) {
  if (!bytes || !out) return fail(GRX_EINVAL, "grx_tdt_load: null argument");
  int rc = device_init(device);
  if (rc) return rc;
  GGUF f;
  if (!f.parse(bytes, len)) return fail(GRX_EFORMAT, f.err);
  const std::string arch = f.get_string("general.architecture", "");
  if (arch != "parakeet") return fail(GRX_EFORMAT, "conformer: architecture \"" + arch + "\" is not a FastConformer transducer");
  auto m = std::make_unique<grx_tdt>();
  m->ar.dev = m->dev = device;
  const std::string p = "stt.parakeet.";
  // readHParams, model.go:190-236 (decoder settings)
  const std::string head = f.get_string(p + "head_kind", "rnnt");
  m->H = int(f.get_int(p + "predictor.hidden", 0));
  m->layers = int(f.get_int(p + "predictor.n_layers", 0));
  m->V = int(f.get_int(p + "predictor.vocab", 0));
  m->J = int(f.get_int(p + "joint.hidden", 0));
  m->D = int(f.get_int(p + "encoder.d_model", 0));
  const std::string act = f.get_string(p + "joint.activation", "relu");
  m->act = act == "sigmoid" ? 1 : act == "tanh" ? 2 : 0;
  m->blank = int(f.get_int("tokenizer.ggml.blank_token_id", -1));
  if (head == "rnnt") {
    m->tdt = 0;
    m->max_symbols = 10;
  } else if (head == "tdt") {
    m->tdt = 1;
    auto it = f.kv.find(p + "tdt.durations");
    if (it != f.kv.end() && it->second.kind == GValue::ARR)
      for (const GValue& v : it->second.a) m->durations.push_back(int(v.kind == GValue::FLOAT ? int64_t(v.f) : v.i));
    if (m->durations.empty()) return fail(GRX_EFORMAT, "conformer: a TDT model needs its durations");
    m->max_symbols = int(f.get_int(p + "tdt.max_symbols", 10));
    if (m->max_symbols < 1 || m->max_symbols > 100)
      return fail(GRX_EFORMAT, "conformer: tdt.max_symbols " + std::to_string(m->max_symbols) + " is out of range");
  } else {
    return fail(GRX_EFORMAT, "conformer: \"" + head + "\" models are not supported (only RNN-T and TDT)");
  }
  if (m->V < 2 || m->H <= 0 || m->layers <= 0 || m->J <= 0 || m->D <= 0)
    return fail(GRX_EFORMAT, "conformer: the model file is missing its decoder settings");
  if (m->blank < 0) m->blank = m->V - 1;  // model.go:337-339
  // what the kernels take
  if (m->H % 32 || m->J % 32 || m->D % 128 || m->H > 1024 || m->J > 1024 || m->layers > TDT_MAX_LAYERS ||
      int(m->durations.size()) > TDT_MAX_DURATIONS || m->blank >= m->V)
    return fail(GRX_EINVAL, "conformer: decoder dimensions outside what the kernels take");
  m->nout = m->V + (m->tdt ? int(m->durations.size()) : 0);

  std::string err;
  auto shape_ok = [&](const std::string& name, int64_t rows, int64_t cols) -> const GTensor* {
    if (!err.empty()) return nullptr;
    int64_t r, c;
    if (!f.matrix_shape(name, &r, &c)) {
      err = "conformer: the model has no " + name;
      return nullptr;
    }
    if (r != rows || c != cols) {
      err = "conformer: " + name + " is " + std::to_string(r) + "x" + std::to_string(c) + ", want " +
            std::to_string(rows) + "x" + std::to_string(cols);
      return nullptr;
    }
    return &f.tensors.at(name);
  };
  auto q8 = [&](const std::string& name, int64_t rows, int64_t cols) -> DQ8 {
    const GTensor* t = shape_ok(name, rows, cols);
    if (!t) return DQ8{};
    if (t->type != G_Q8_0) {
      err = "conformer: " + name + " is not Q8_0 (this build runs Q8_0 decoders)";
      return DQ8{};
    }
    return upload_q8(m->ar, t->data, int(rows), int(cols), &rc);
  };
  auto vec = [&](const std::string& name, int64_t n) -> float* {
    if (!err.empty()) return nullptr;
    std::vector<float> v;
    auto it = f.tensors.find(name);
    if (it == f.tensors.end() || it->second.elems() != n || !f.float32(name, v)) {
      err = "conformer: no " + std::to_string(n) + "-value " + name;
      return nullptr;
    }
    return m->ar.upload(v.data(), v.size(), &rc);
  };
  const int H = m->H, J = m->J;
  m->embed = vec("pred.embed.weight", int64_t(m->V) * H);
  for (int i = 0; i < m->layers; i++) {
    const std::string lp = "pred.lstm." + std::to_string(i) + ".";
    m->wx.push_back(q8(lp + "Wx", 4 * H, H));
    m->wh.push_back(q8(lp + "Wh", 4 * H, H));
    m->lb.push_back(vec(lp + "bias", 4 * H));
  }
  m->jenc = q8("joint.enc.weight", J, m->D);
  m->jenc_b = vec("joint.enc.bias", J);
  m->jpred = q8("joint.pred.weight", J, H);
  m->jpred_b = vec("joint.pred.bias", J);
  m->jout = q8("joint.out.weight", m->nout, J);
  m->jout_b = vec("joint.out.bias", m->nout);
  if (!err.empty()) return fail(GRX_EFORMAT, err);
  if (rc) return rc;
  *out = m.release();
  return GRX_OK;
}

void grx_tdt_free(grx_tdt* m) { delete m; }

int grx_tdt_dims(const grx_tdt* m, int* hidden, int* layers, int* vocab, int* joint, int* d_enc, int* n_durations,
                 int* blank, int* is_tdt) {
  if (!m) return fail(GRX_EINVAL, "null model");
  if (hidden) *hidden = m->H;
  if (layers) *layers = m->layers;
  if (vocab) *vocab = m->V;
  if (joint) *joint = m->J;
  if (d_enc) *d_enc = m->D;
  if (n_durations) *n_durations = int(m->durations.size());
  if (blank) *blank = m->blank;
  if (is_tdt) *is_tdt = m->tdt;
  return GRX_OK;
}

int grx_tdt_batch_create(grx_tdt* m, int n, int max_t, int cap, grx_tdt_batch** out) {
  if (!m || !out || n <= 0 || max_t <= 0 || cap <= 0) return fail(GRX_EINVAL, "grx_tdt_batch_create: bad argument");
  CK(cudaSetDevice(m->dev));
  auto b = std::make_unique<grx_tdt_batch>();
  b->ar.dev = m->dev;
  b->m = m;
  b->n = n;
  b->max_t = max_t;
  b->cap = cap;
  CK(cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking));
  CK(cudaMallocHost(&b->h_count, 2 * sizeof(int)));
  for (cudaEvent_t& e : b->ev) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  int rc = 0;
  const size_t rows = size_t(n) * max_t;
  b->eq = b->ar.alloc<int8_t>(rows * m->D, &rc);
  b->es = b->ar.alloc<float2>(rows * (m->D / 32), &rc);
  b->enc_proj = b->ar.alloc<float>(rows * m->J, &rc);
  b->enc_row = b->ar.alloc<float>(size_t(n) * m->J, &rc);
  b->d_enc = b->ar.alloc<float>(rows * m->D, &rc);
  b->d_T = b->ar.alloc<int>(n, &rc);
  b->d_off = b->ar.alloc<int>(n, &rc);
  b->tokens = b->ar.alloc<int>(size_t(n) * cap * 4, &rc);
  TdtArgs& a = b->a;
  a.n = n;
  a.H = m->H;
  a.layers = m->layers;
  a.V = m->V;
  a.J = m->J;
  a.nout = m->nout;
  a.ndur = int(m->durations.size());
  a.blank = m->blank;
  a.max_symbols = m->max_symbols;
  a.tdt = m->tdt;
  a.act = m->act;
  a.max_t = max_t;
  a.cap = cap;
  for (int i = 0; i < a.ndur; i++) a.durations[i] = m->durations[size_t(i)];
  a.embed = m->embed;
  for (int l = 0; l < m->layers; l++) {
    a.lstm_wx[l] = m->wx[size_t(l)];
    a.lstm_wh[l] = m->wh[size_t(l)];
    a.lstm_b[l] = m->lb[size_t(l)];
  }
  a.jpred = m->jpred;
  a.jout = m->jout;
  a.jpred_b = m->jpred_b;
  a.jout_b = m->jout_b;
  a.enc_proj = b->enc_proj;
  a.pred_proj = b->ar.alloc<float>(size_t(n) * m->J, &rc);
  a.logits = b->ar.alloc<float>(size_t(n) * m->nout, &rc);
  const size_t hs = size_t(2) * m->layers * n * m->H;
  a.h = b->ar.alloc<float>(hs, &rc);
  a.c = b->ar.alloc<float>(hs, &rc);
  a.cur = b->ar.alloc<int>(n, &rc);
  a.last = b->ar.alloc<int>(n, &rc);
  a.step = b->ar.alloc<int>(n, &rc);
  a.nsym = b->ar.alloc<int>(n, &rc);
  a.iter = b->ar.alloc<int>(n, &rc);
  a.ntok = b->ar.alloc<int>(n, &rc);
  a.T = b->d_T;
  a.frame_offset = b->d_off;
  a.tokens = b->tokens;
  a.active = b->ar.alloc<int>(size_t(2) * n, &rc);
  a.dirty = b->ar.alloc<int>(size_t(2) * n, &rc);
  a.counts = b->ar.alloc<int>(4, &rc);
  if (rc) return rc;
  *out = b.release();
  return grx_tdt_batch_reset(*out);
}

void grx_tdt_batch_free(grx_tdt_batch* b) { delete b; }

int grx_tdt_batch_reset(grx_tdt_batch* b) {
  if (!b) return fail(GRX_EINVAL, "null batch");
  CK(cudaSetDevice(b->ar.dev));
  const TdtArgs& a = b->a;
  const size_t hs = size_t(2) * a.layers * a.n * a.H * sizeof(float);
  CK(cudaMemsetAsync(a.h, 0, hs, b->st));
  CK(cudaMemsetAsync(a.c, 0, hs, b->st));
  CK(cudaMemsetAsync(a.cur, 0, size_t(a.n) * sizeof(int), b->st));
  CK(cudaMemsetAsync(a.last, 0xff, size_t(a.n) * sizeof(int), b->st));  // -1
  CK(cudaStreamSynchronize(b->st));
  return GRX_OK;
}

int grx_tdt_state_get(grx_tdt_batch* b, int i, float* h, float* c, int* last) {
  if (!b || i < 0 || i >= b->n) return fail(GRX_EINVAL, "grx_tdt_state_get: bad argument");
  CK(cudaSetDevice(b->ar.dev));
  const TdtArgs& a = b->a;
  int cur = 0;
  CK(cudaMemcpyAsync(&cur, a.cur + i, sizeof(int), cudaMemcpyDeviceToHost, b->st));
  if (last) CK(cudaMemcpyAsync(last, a.last + i, sizeof(int), cudaMemcpyDeviceToHost, b->st));
  CK(cudaStreamSynchronize(b->st));
  for (int l = 0; l < a.layers; l++) {
    const size_t o = ((size_t(cur) * a.layers + l) * a.n + i) * a.H;
    if (h) CK(cudaMemcpyAsync(h + size_t(l) * a.H, a.h + o, a.H * sizeof(float), cudaMemcpyDeviceToHost, b->st));
    if (c) CK(cudaMemcpyAsync(c + size_t(l) * a.H, a.c + o, a.H * sizeof(float), cudaMemcpyDeviceToHost, b->st));
  }
  CK(cudaStreamSynchronize(b->st));
  return GRX_OK;
}

int grx_tdt_state_set(grx_tdt_batch* b, int i, const float* h, const float* c, int last) {
  if (!b || i < 0 || i >= b->n || !h || !c) return fail(GRX_EINVAL, "grx_tdt_state_set: bad argument");
  if (last < -1 || last >= b->a.V) return fail(GRX_EINVAL, "grx_tdt_state_set: last token out of range");
  CK(cudaSetDevice(b->ar.dev));
  const TdtArgs& a = b->a;
  int cur = 0;
  CK(cudaMemcpyAsync(&cur, a.cur + i, sizeof(int), cudaMemcpyDeviceToHost, b->st));
  CK(cudaStreamSynchronize(b->st));
  for (int l = 0; l < a.layers; l++) {
    const size_t o = ((size_t(cur) * a.layers + l) * a.n + i) * a.H;
    CK(cudaMemcpyAsync(a.h + o, h + size_t(l) * a.H, a.H * sizeof(float), cudaMemcpyHostToDevice, b->st));
    CK(cudaMemcpyAsync(a.c + o, c + size_t(l) * a.H, a.H * sizeof(float), cudaMemcpyHostToDevice, b->st));
  }
  CK(cudaMemcpyAsync(a.last + i, &last, sizeof(int), cudaMemcpyHostToDevice, b->st));
  CK(cudaStreamSynchronize(b->st));
  return GRX_OK;
}

}  // extern "C"

namespace {

// The loop body graph: kRoundsPerReplay iterations, parities 0, 1, 0, ...
int build_graph(grx_tdt_batch* b) {
  if (b->exec) return GRX_OK;
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal));
  for (int r = 0; r < kRoundsPerReplay; r++) launch_tdt_iteration(b->a, r & 1, b->st);
  cudaError_t e = cudaStreamEndCapture(b->st, &g);
  if (e != cudaSuccess) return fail(GRX_ECUDA, std::string("TDT loop capture: ") + cudaGetErrorString(e));
  e = cudaGraphInstantiate(&b->exec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(GRX_ECUDA, std::string("TDT loop graph: ") + cudaGetErrorString(e));
  b->per_replay = kRoundsPerReplay;
  return GRX_OK;
}

// Decode of encoder output d_enc [n][max_t][D] (device). The loop writes
// the batch's token buffer; they are copied to d_tokens [n][cap][4] when
// that is another buffer, and the counts to d_counts (may be NULL).
int decode(grx_tdt_batch* b, const float* d_enc, const int* T, const int* frame_offset, int* d_tokens, int* d_counts) {
  grx_tdt* m = b->m;
  const int n = b->n;
  std::vector<int> Th(T, T + n), off(size_t(n), 0);
  int maxT = 0;
  bool any_one = false;
  for (int i = 0; i < n; i++) {
    if (Th[size_t(i)] < 0 || Th[size_t(i)] > b->max_t) return fail(GRX_EINVAL, "grx_tdt_decode: T out of range");
    maxT = std::max(maxT, Th[size_t(i)]);
    any_one |= Th[size_t(i)] == 1;
    if (frame_offset) off[size_t(i)] = frame_offset[i];
  }
  int rc = build_graph(b);
  if (rc) return rc;
  CK(cudaMemcpyAsync(b->d_T, Th.data(), sizeof(int) * size_t(n), cudaMemcpyHostToDevice, b->st));
  CK(cudaMemcpyAsync(b->d_off, off.data(), sizeof(int) * size_t(n), cudaMemcpyHostToDevice, b->st));
  if (maxT > 0) {
    // encProj = jEnc·enc + b for every stream's frames (rnnt.go:124): the
    // int8 path, as Linear takes it for T ≥ 2 rows ...
    const int rows = n * b->max_t;
    launch_quant(d_enc, rows, m->D, b->eq, b->es, b->st);
    EpiArgs e;
    e.epi = EPI_STORE;
    e.y = b->enc_proj;
    e.ldy = m->J;
    e.bias = m->jenc_b;
    launch_q8_product(b->eq, b->es, rows, m->jenc, e, b->st);
    b->launches += 2;
    if (any_one) {
      // ... and the float path for a stream of a single frame (kern.go:189)
      FArgs fa;
      fa.epi = FE_BIAS;
      fa.x = d_enc;
      fa.ldx = b->max_t * m->D;
      fa.wq = m->jenc.q;
      fa.wd = m->jenc.d;
      fa.N = m->J;
      fa.K = m->D;
      fa.bias = m->jenc_b;
      fa.y = b->enc_row;
      fa.ldy = m->J;
      launch_flin(fa, n, b->st);
      b->launches++;
      for (int i = 0; i < n; i++)
        if (Th[size_t(i)] == 1)
          CK(cudaMemcpyAsync(b->enc_proj + size_t(i) * b->max_t * m->J, b->enc_row + size_t(i) * m->J,
                             sizeof(float) * size_t(m->J), cudaMemcpyDeviceToDevice, b->st));
    }
  }
  launch_tdt_begin(b->a, b->st);
  CK(cudaGetLastError());
  // The loop: graph replays until no stream is left. Replay k+1 is queued
  // before the host reads the active count left by replay k, so the device
  // does not wait for the host; the replay after the end finds empty lists.
  const int64_t max_iters = 16 * int64_t(maxT) + 1024;
  int64_t replays = 0;
  bool finished = maxT == 0;
  while (!finished) {
    CK(cudaGraphLaunch(b->exec, b->st));
    CK(cudaMemcpyAsync(b->h_count + (replays & 1), b->a.counts, sizeof(int), cudaMemcpyDeviceToHost, b->st));
    CK(cudaEventRecord(b->ev[replays & 1], b->st));
    replays++;
    if (replays >= 2) {
      CK(cudaEventSynchronize(b->ev[replays & 1]));  // the replay before the one just queued
      finished = b->h_count[replays & 1] == 0;
    }
    finished |= replays * b->per_replay >= max_iters;
  }
  CK(cudaStreamSynchronize(b->st));
  b->launches += replays * b->per_replay * launches_per_iteration(m) + 2;
  b->iterations += replays * b->per_replay;
  if (d_tokens != b->tokens)
    CK(cudaMemcpyAsync(d_tokens, b->tokens, sizeof(int) * 4 * size_t(n) * b->cap, cudaMemcpyDeviceToDevice, b->st));
  if (d_counts) CK(cudaMemcpyAsync(d_counts, b->a.ntok, sizeof(int) * size_t(n), cudaMemcpyDeviceToDevice, b->st));
  CK(cudaGetLastError());
  return GRX_OK;
}

}  // namespace

extern "C" {

int grx_tdt_decode(grx_tdt_batch* b, const float* enc, const int* T, const int* frame_offset, grx_tdt_token* tokens,
                   int* counts) {
  if (!b || !enc || !T || !tokens || !counts) return fail(GRX_EINVAL, "grx_tdt_decode: null argument");
  CK(cudaSetDevice(b->ar.dev));
  const size_t elems = size_t(b->n) * b->max_t * b->m->D;
  CK(cudaMemcpyAsync(b->d_enc, enc, elems * sizeof(float), cudaMemcpyHostToDevice, b->st));
  int rc = decode(b, b->d_enc, T, frame_offset, b->tokens, nullptr);
  if (rc) return rc;
  CK(cudaMemcpyAsync(counts, b->a.ntok, sizeof(int) * size_t(b->n), cudaMemcpyDeviceToHost, b->st));
  CK(cudaMemcpyAsync(tokens, b->tokens, sizeof(grx_tdt_token) * size_t(b->n) * b->cap, cudaMemcpyDeviceToHost, b->st));
  CK(cudaStreamSynchronize(b->st));
  return GRX_OK;
}

int grx_tdt_decode_device(grx_tdt_batch* b, const float* d_enc, const int* T, const int* frame_offset,
                          grx_tdt_token* d_tokens, int* d_counts) {
  if (!b || !d_enc || !T || !d_tokens || !d_counts) return fail(GRX_EINVAL, "grx_tdt_decode_device: null argument");
  CK(cudaSetDevice(b->ar.dev));
  int rc = decode(b, d_enc, T, frame_offset, reinterpret_cast<int*>(d_tokens), d_counts);
  if (rc) return rc;
  CK(cudaStreamSynchronize(b->st));
  return GRX_OK;
}

void* grx_tdt_batch_cuda_stream(const grx_tdt_batch* b) { return b ? (void*)b->st : nullptr; }

int64_t grx_tdt_batch_launches(const grx_tdt_batch* b) { return b ? b->launches : -1; }

int64_t grx_tdt_batch_iterations(const grx_tdt_batch* b) { return b ? b->iterations : -1; }

int64_t grx_tdt_batch_stream_iterations(grx_tdt_batch* b) {
  if (!b) return fail(GRX_EINVAL, "null batch");
  CK(cudaSetDevice(b->ar.dev));
  std::vector<int> it(size_t(b->n));
  CK(cudaMemcpyAsync(it.data(), b->a.iter, sizeof(int) * size_t(b->n), cudaMemcpyDeviceToHost, b->st));
  CK(cudaStreamSynchronize(b->st));
  int64_t t = 0;
  for (int v : it) t += v;
  return t;
}

}  // extern "C"
