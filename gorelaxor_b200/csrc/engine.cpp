// The host side of libgrx: the C ABI of include/grx.h over the kernels.
//
// What it mirrors (paths in the gorelaxor tree):
//  * kern.Weight / kern.Linear (internal/kern/kern.go:41-201) — grx_weight_*,
//    grx_linear, with the reference's dispatch between the int8 and float
//    paths (kern.go:189);
//  * pockettts.Load / LoadVoice (pockettts/model.go:202-322,
//    voice.go:26-63) — grx_flowlm_load, grx_voice_load: the same tensor
//    names, shape checks and settings, the Q8_0 weights uploaded to HBM;
//  * the per-frame loop of speakChunk (speak.go:146-175) for a batch of
//    independent streams — grx_streams_*: the KV caches stay in HBM, one
//    frame is one CUDA graph replay of the kernel sequence below, the raw
//    latent is fed back on the device.
// Errors are codes plus a per-thread message; nothing here aborts.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/grx.h"
#include "gguf.h"
#include "host.h"
#include "kernels.h"

using namespace grx;

// ------------------------------------------------------------ handles ----

struct grx_gguf {
  GGUF f;
};

struct grx_weight {
  Arena ar;
  int type = 0;  // 0 F32, 2 Q8_0
  int rows = 0, cols = 0;
  bool dropped = false;
  DQ8 q8;
  float* f = nullptr;
};

struct Layer {
  float *n1w, *n1b, *n2w, *n2b;
  DQ8 qkv, out, ff1, ff2;
};

struct Res {
  float *nw, *nb, *b1, *b2, *adab;
  DQ8 fc1, fc2, ada;
};

struct grx_flowlm {
  Arena ar;
  int dev = 0;
  int d = 0, heads = 0, ff = 0, L = 0, ldim = 0, fd = 0, depth = 0, steps = 1;
  double period = 1e4;
  std::string sha;
  std::vector<Layer> layers;
  std::vector<Res> res;
  float *win = nullptr, *bos = nullptr, *outw = nullptr, *outb = nullptr, *eosw = nullptr;
  float eosb = 0;
  float *mean = nullptr, *stdv = nullptr;
  DQ8 cond, fada;
  float *condb = nullptr, *fin = nullptr, *finb = nullptr, *fadab = nullptr, *fout = nullptr, *foutb = nullptr;
  float* tc = nullptr;  // [steps][fd] time conditions
  std::vector<float> freqs;
  float* embed = nullptr;  // lm.embed widened to float32 [embed_rows][d], if the file has it
  int embed_rows = 0;
  float* speaker = nullptr;  // lm.speaker_proj [d][ldim] float32, and lm.bos_voice [d], if the file has them
  float* bosv = nullptr;
};

struct grx_voice {
  int positions = 0;
  std::vector<float> kv;  // [L][2][positions][d]
  std::string model;
};

// Bytes of a set's FrameIO before its noise rows in their shared device block.
constexpr size_t kIoPad = 256;

struct grx_streams {
  Arena ar;
  grx_flowlm* m = nullptr;
  int n = 0, cap = 0;
  cudaStream_t st = nullptr;
  float* kv = nullptr;
  int *pos = nullptr, *pos0 = nullptr;
  float *x = nullptr, *q = nullptr, *lm_out = nullptr, *eos = nullptr, *lat = nullptr, *rope = nullptr;
  int8_t *xq = nullptr, *xqf = nullptr;
  float2 *xs = nullptr, *xsf = nullptr;
  float *y0 = nullptr, *sy = nullptr, *h = nullptr, *mod = nullptr, *mod2 = nullptr, *nrm = nullptr, *mm = nullptr,
        *cur = nullptr;
  float *noise1 = nullptr, *lat1 = nullptr, *scaled1 = nullptr, *eos1 = nullptr;
  FrameIO* io = nullptr;
  cudaGraphExec_t exec = nullptr;  // one frame
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec_n = nullptr;  // kGraphFrames frames, for device-resident runs
  cudaGraph_t graph_n = nullptr;
  int64_t launches = 0;
  int per_frame = 0;
  // A large set runs as parts, each with its own CUDA stream and frame graph,
  // so that one part's memory-bound attention overlaps the other's
  // latency-bound products; the parent's stream forks to and joins them.
  std::vector<std::unique_ptr<grx_streams>> parts;
  int row0 = 0;  // a part's first stream within its parent
  cudaEvent_t ev = nullptr;
  // One stream runs its frames in the persistent kernel (k_frame1.cu) when
  // the model and the device suit it: its arguments in device memory, the
  // launch shape, the grid barrier counter and the watchdog's error word.
  bool b1 = false;
  Frame1Args* f1 = nullptr;
  size_t f1_smem = 0;
  uint32_t f1_slot = 0;
  int f1_grid = 0;
  unsigned* f1_bar = nullptr;
  int* f1_err = nullptr;
  // the error word as a launch left it, copied on the stream into pinned
  // memory, so a check after the stream's synchronisation needs no copy of
  // its own (f1_err_copied: such a copy was queued since the last check)
  int* f1_err_h = nullptr;
  bool f1_err_copied = false;
  // grx_streams_step's traffic, one copy each way: the frame's FrameIO and
  // noise rows are one device block (io, then noise1 kIoPad bytes in),
  // filled from in1_h; the latent, scaled and eos rows and then the
  // persistent kernel's error word are another (out1), read into out1_h
  uint8_t* in1_h = nullptr;
  size_t in1_bytes = 0;
  float *out1 = nullptr, *out1_h = nullptr;
  size_t out1_floats = 0;
  ~grx_streams() {
    parts.clear();
    cudaSetDevice(ar.dev);
    if (f1_err_h) cudaFreeHost(f1_err_h);
    if (in1_h) cudaFreeHost(in1_h);
    if (out1_h) cudaFreeHost(out1_h);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (exec_n) cudaGraphExecDestroy(exec_n);
    if (graph_n) cudaGraphDestroy(graph_n);
    if (ev) cudaEventDestroy(ev);
    if (st) cudaStreamDestroy(st);
  }
};

namespace {

// A stream set runs as up to stream_parts_max() parts of at least this many
// streams each.
constexpr int kMinPart = 64;

// Two parts unless GRX_STREAM_PARTS (1 to 8) says otherwise.
int stream_parts_max() {
  const char* v = getenv("GRX_STREAM_PARTS");
  const int p = v ? atoi(v) : 2;
  return p < 1 ? 1 : p > 8 ? 8 : p;
}

// The kernel sequence of one frame for all streams (see grx.h): flowLM.step
// (lm.go:185-195 → nn.go:142-182) then flowHead.sample (lm.go:108-160).
// Returns the number of kernels launched.
int enqueue_frame(grx_streams* s) {
  grx_flowlm* m = s->m;
  const int M = s->n, d = m->d, fd = m->fd;
  cudaStream_t st = s->st;
  int k = 0;
  // x = lm.input · latent (F32 weight, dot4f32avx order; bos at frame 0).
  {
    FArgs a;
    a.epi = FE_BIAS;
    a.x = s->lat;
    a.ldx = m->ldim;
    a.wf = m->win;
    a.N = d;
    a.K = m->ldim;
    a.y = s->x;
    a.ldy = d;
    launch_flin(a, M, st);
    k++;
  }
  for (int l = 0; l < m->L; l++) {
    const Layer& ly = m->layers[size_t(l)];
    LnArgs ln;
    ln.x = s->x;
    ln.w = ly.n1w;
    ln.b = ly.n1b;
    ln.eps = 1e-5;
    ln.mode = LN_Q8;
    ln.q8 = s->xq;
    ln.q8s = s->xs;
    launch_ln(ln, M, d, st);
    EpiArgs e;
    e.epi = EPI_ROPE_KV;
    e.kv.q = s->q;
    e.kv.kv = s->kv;
    e.kv.pos = s->pos;
    e.kv.rope = s->rope;
    e.kv.layer = l;
    e.kv.layers = m->L;
    e.kv.heads = m->heads;
    e.kv.cap = s->cap;
    e.kv.d = d;
    launch_q8_product(s->xq, s->xs, M, ly.qkv, e, st);
    AttnArgs at;
    at.q = s->q;
    at.kv = s->kv;
    at.pos = s->pos;
    at.q8 = s->xq;
    at.q8s = s->xs;
    at.layer = l;
    at.layers = m->L;
    at.heads = m->heads;
    at.cap = s->cap;
    at.d = d;
    at.io = s->io;
    launch_attn(at, M, st);
    EpiArgs r;
    r.epi = EPI_RESID;
    r.y = s->x;
    r.ldy = d;
    launch_q8_product(s->xq, s->xs, M, ly.out, r, st);
    ln.w = ly.n2w;
    ln.b = ly.n2b;
    launch_ln(ln, M, d, st);
    EpiArgs g;
    g.epi = EPI_GELU_Q8;
    g.q8 = s->xqf;
    g.q8s = s->xsf;
    launch_q8_product(s->xq, s->xs, M, ly.ff1, g, st);
    launch_q8_product(s->xqf, s->xsf, M, ly.ff2, r, st);
    k += 7;
  }
  {  // out_norm → lm_out; eos; position += 1
    LnArgs ln;
    ln.x = s->x;
    ln.w = m->outw;
    ln.b = m->outb;
    ln.eps = 1e-5;
    ln.mode = LN_F32;
    ln.y = s->lm_out;
    ln.eosw = m->eosw;
    ln.eosb = m->eosb;
    ln.eos = s->eos;
    ln.io = s->io;
    ln.pos = s->pos;
    launch_ln(ln, M, d, st);
    k += 1;
  }
  // Flow head. y = cond·lm_out + b; per step: sy = silu(y + tc_i), net.
  const bool one = m->steps == 1;
  {
    FArgs a;
    a.epi = one ? FE_COND : FE_BIAS;
    a.x = s->lm_out;
    a.ldx = d;
    a.wq = m->cond.q;
    a.wd = m->cond.d;
    a.N = fd;
    a.K = d;
    a.bias = m->condb;
    a.y = one ? s->sy : s->y0;
    a.ldy = fd;
    a.aux = m->tc;
    launch_flin(a, M, st);
    k++;
  }
  for (int step = 0; step < m->steps; step++) {
    if (!one) {
      launch_cond_step(s->y0, m->tc + size_t(step) * fd, s->sy, M, fd, st);
      k++;
    }
    {  // h = input·cur + b (cur = the noise at the first step)
      FArgs a;
      a.epi = FE_BIAS;
      a.x = s->cur;
      a.ldx = m->ldim;
      a.io = s->io;
      a.x_noise = step == 0;
      a.wf = m->fin;
      a.N = fd;
      a.K = m->ldim;
      a.bias = m->finb;
      a.y = s->h;
      a.ldy = fd;
      launch_flin(a, M, st);
      k++;
    }
    for (const Res& r : m->res) {
      FArgs a;
      a.epi = FE_BIAS;
      a.x = s->sy;
      a.ldx = fd;
      a.wq = r.ada.q;
      a.wd = r.ada.d;
      a.N = 3 * fd;
      a.K = fd;
      a.bias = r.adab;
      a.y = s->mod;
      a.ldy = 3 * fd;
      launch_flin(a, M, st);
      LnArgs ln;
      ln.x = s->h;
      ln.w = r.nw;
      ln.b = r.nb;
      ln.eps = 1e-6;
      ln.mode = LN_MOD;
      ln.y = s->nrm;
      ln.mod = s->mod;
      ln.ldmod = 3 * fd;
      ln.shift = 0;
      ln.scale = fd;
      launch_ln(ln, M, fd, st);
      FArgs f1;
      f1.epi = FE_SILU;
      f1.x = s->nrm;
      f1.ldx = fd;
      f1.wq = r.fc1.q;
      f1.wd = r.fc1.d;
      f1.N = fd;
      f1.K = fd;
      f1.bias = r.b1;
      f1.y = s->mm;
      f1.ldy = fd;
      launch_flin(f1, M, st);
      FArgs f2 = f1;
      f2.epi = FE_GATE;
      f2.x = s->mm;
      f2.wq = r.fc2.q;
      f2.wd = r.fc2.d;
      f2.bias = r.b2;
      f2.y = s->h;
      f2.aux = s->mod + 2 * fd;
      f2.ldaux = 3 * fd;
      launch_flin(f2, M, st);
      k += 4;
    }
    {
      FArgs a;
      a.epi = FE_BIAS;
      a.x = s->sy;
      a.ldx = fd;
      a.wq = m->fada.q;
      a.wd = m->fada.d;
      a.N = 2 * fd;
      a.K = fd;
      a.bias = m->fadab;
      a.y = s->mod2;
      a.ldy = 2 * fd;
      launch_flin(a, M, st);
      LnArgs ln;
      ln.x = s->h;
      ln.eps = 1e-6;
      ln.mode = LN_MOD;
      ln.y = s->nrm;
      ln.mod = s->mod2;
      ln.ldmod = 2 * fd;
      ln.shift = 0;
      ln.scale = fd;
      launch_ln(ln, M, fd, st);
      FArgs o;
      const bool last = step + 1 == m->steps;
      o.epi = FE_LATENT;
      o.x = s->nrm;
      o.ldx = fd;
      o.wf = m->fout;
      o.N = m->ldim;
      o.K = fd;
      o.bias = m->foutb;
      o.y = last ? s->lat : s->cur;  // the last step's latent feeds the next frame
      o.ldy = m->ldim;
      o.aux = s->cur;  // cur before this step: the noise at the first step
      o.ldaux = m->ldim;
      o.aux_noise = step == 0;
      o.io = s->io;
      o.io_out = last;
      o.steps = float(m->steps);
      o.mean = m->mean;
      o.stdv = m->stdv;
      if (last) {
        o.out2 = s->lat1;
        o.out3 = s->scaled1;
      }
      launch_flin(o, M, st);
      k += 3;
    }
  }
  launch_tick(s->io, st);
  k++;
  return k;
}

// Sets up the persistent one-stream kernel for a set of one stream whose
// model has one decode step (GRX_FRAME1=0 keeps the per-kernel graph path).
// Leaves b1 false when the model or the device does not suit it.
int frame1_setup(grx_streams* s) {
  const char* env = getenv("GRX_FRAME1");
  grx_flowlm* m = s->m;
  if ((env && env[0] == '0') || s->n != 1 || m->steps != 1 || m->L > F1_MAX_LAYERS || m->depth > F1_MAX_DEPTH ||
      m->depth < 1)
    return GRX_OK;
  int G = 0, coop = 0;
  CK(cudaDeviceGetAttribute(&G, cudaDevAttrMultiProcessorCount, s->ar.dev));
  CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, s->ar.dev));
  if (!coop) return GRX_OK;
  Frame1Args A;
  A.d = m->d;
  A.heads = m->heads;
  A.ff = m->ff;
  A.L = m->L;
  A.ldim = m->ldim;
  A.fd = m->fd;
  A.depth = m->depth;
  A.cap = s->cap;
  for (int l = 0; l < m->L; l++) {
    const Layer& ly = m->layers[size_t(l)];
    A.layers[l].n1w = ly.n1w;
    A.layers[l].n1b = ly.n1b;
    A.layers[l].n2w = ly.n2w;
    A.layers[l].n2b = ly.n2b;
    A.layers[l].qkv = ly.qkv;
    A.layers[l].out = ly.out;
    A.layers[l].ff1 = ly.ff1;
    A.layers[l].ff2 = ly.ff2;
  }
  for (int k = 0; k < m->depth; k++) {
    const Res& r = m->res[size_t(k)];
    A.res[k].nw = r.nw;
    A.res[k].nb = r.nb;
    A.res[k].b1 = r.b1;
    A.res[k].b2 = r.b2;
    A.res[k].adab = r.adab;
    A.res[k].fc1 = r.fc1;
    A.res[k].fc2 = r.fc2;
    A.res[k].ada = r.ada;
  }
  A.win = m->win;
  A.outw = m->outw;
  A.outb = m->outb;
  A.eosw = m->eosw;
  A.eosb = m->eosb;
  A.mean = m->mean;
  A.stdv = m->stdv;
  A.cond = m->cond;
  A.fada = m->fada;
  A.condb = m->condb;
  A.fin = m->fin;
  A.finb = m->finb;
  A.fadab = m->fadab;
  A.fout = m->fout;
  A.foutb = m->foutb;
  A.tc = m->tc;
  A.kv = s->kv;
  A.pos = s->pos;
  A.rope = s->rope;
  A.x = s->x;
  A.q = s->q;
  A.lm_out = s->lm_out;
  A.eos = s->eos;
  A.lat = s->lat;
  A.sy = s->sy;
  A.h = s->h;
  A.mod2 = s->mod2;
  A.mm = s->mm;
  A.io = s->io;
  size_t smem = 0;
  uint32_t slot = 0;
  if (!frame1_suits(A, &smem, &slot, G) || frame1_max_active(smem) < 1) {
    cudaGetLastError();
    return GRX_OK;
  }
  int rc = 0;
  A.att = s->ar.alloc<float>(size_t(m->d), &rc);
  A.ffq = s->ar.alloc<int8_t>(size_t(m->ff), &rc);
  A.ffs = s->ar.alloc<float>(size_t(m->ff / 32), &rc);
  A.mod = s->ar.alloc<float>(size_t(m->depth) * 3 * m->fd, &rc);
  A.bar = s->ar.alloc<unsigned>(1, &rc);
  A.err = reinterpret_cast<int*>(s->out1 + s->out1_floats - 1);  // read back with the step's outputs
  if (rc) return rc;
  CK(cudaMemset(A.err, 0, sizeof(int)));
  CK(cudaHostAlloc(&s->f1_err_h, sizeof(int), cudaHostAllocDefault));
  s->f1 = s->ar.upload(&A, 1, &rc);
  if (rc) return rc;
  s->f1_smem = smem;
  s->f1_slot = slot;
  s->f1_grid = G;
  s->f1_bar = A.bar;
  s->f1_err = A.err;
  s->b1 = true;
  return GRX_OK;
}

// Queues `frames` frames of a persistent-kernel set, then (copy_err) the
// copy of its error word that frame1_check reads.
int frame1_run(grx_streams* s, int frames, int stall = 0, bool copy_err = true) {
  if (frames <= 0) return GRX_OK;
  CK(cudaMemsetAsync(s->f1_bar, 0, sizeof(unsigned), s->st));
  CK(launch_frame1(s->f1, s->f1_smem, s->f1_slot, s->f1_grid, frames, stall, s->st));
  if (copy_err) CK(cudaMemcpyAsync(s->f1_err_h, s->f1_err, sizeof(int), cudaMemcpyDeviceToHost, s->st));
  s->f1_err_copied = copy_err;
  s->launches += 1;
  return GRX_OK;
}

// The persistent kernel's error word as the host read it.
int frame1_error(int e) {
  if (e)
    return fail(GRX_ETIMEDOUT, std::string("the persistent frame kernel gave up on a ") +
                                   (e == 1 ? "grid barrier" : "weight copy") + " after its one-second limit");
  return GRX_OK;
}

// After the set's stream is synchronised: GRX_ETIMEDOUT if a bounded wait of
// the persistent kernel ran out (the set's state is then undefined until a
// reset).
int frame1_check(grx_streams* s) {
  if (!s->b1) return GRX_OK;
  int e = 0;
  if (s->f1_err_copied) {
    e = *s->f1_err_h;
    s->f1_err_copied = false;
  } else {
    CK(cudaMemcpy(&e, s->f1_err, sizeof e, cudaMemcpyDeviceToHost));
  }
  return frame1_error(e);
}

// A device-resident run replays kGraphFrames frames per graph launch (the
// frame counter in FrameIO moves on inside the graph), which spares most of
// the gaps between graph launches; the step-by-step path replays one frame.
constexpr int kGraphFrames = 8;

int build_graph(grx_streams* s) {
  for (int n : {1, kGraphFrames}) {
    CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    int k = 0;
    for (int f = 0; f < n; f++) k = enqueue_frame(s);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(s->st, &g);
    if (e != cudaSuccess) return fail(GRX_ECUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    if (n == 1) {
      s->graph = g;
      CK(cudaGraphInstantiate(&s->exec, g, 0));
      s->per_frame = k;
    } else {
      s->graph_n = g;
      CK(cudaGraphInstantiate(&s->exec_n, g, 0));
    }
  }
  return GRX_OK;
}

// Queues `frames` frames of one set (or part) on its stream.
int replay_frames(grx_streams* s, int frames) {
  int f = 0;
  for (; f + kGraphFrames <= frames; f += kGraphFrames) CK(cudaGraphLaunch(s->exec_n, s->st));
  for (; f < frames; f++) CK(cudaGraphLaunch(s->exec, s->st));
  return GRX_OK;
}

std::vector<float> rope_freqs(int hd, double period) {
  float c = float(-std::log(period) * 2 / double(hd));
  std::vector<float> f(size_t(hd / 2));
  for (size_t i = 0; i < f.size(); i++) f[i] = float(std::exp(double(float(i) * c)));
  return f;
}

}  // namespace

// ================================================================ C ABI ==

extern "C" {

int grx_last_error(char* buf, size_t len) {
  const std::string& e = last_error_message();
  if (buf && len) {
    size_t n = std::min(len - 1, e.size());
    std::memcpy(buf, e.data(), n);
    buf[n] = 0;
  }
  return int(e.size());
}

int grx_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

// ---- GGUF ----

int grx_gguf_open(const void* bytes, size_t len, grx_gguf** out) {
  if (!bytes || !out) return fail(GRX_EINVAL, "grx_gguf_open: null argument");
  auto f = std::make_unique<grx_gguf>();
  if (!f->f.parse(bytes, len)) return fail(GRX_EFORMAT, f->f.err);
  *out = f.release();
  return GRX_OK;
}

void grx_gguf_close(grx_gguf* f) { delete f; }

int64_t grx_gguf_int(const grx_gguf* f, const char* key, int64_t def) { return f ? f->f.get_int(key, def) : def; }

double grx_gguf_float(const grx_gguf* f, const char* key, double def) { return f ? f->f.get_float(key, def) : def; }

int grx_gguf_string(const grx_gguf* f, const char* key, char* buf, size_t len) {
  if (!f) return fail(GRX_EINVAL, "null file");
  auto it = f->f.kv.find(key);
  if (it == f->f.kv.end() || it->second.kind != GValue::STR) return fail(GRX_EINVAL, std::string("no string ") + key);
  const std::string& s = it->second.s;
  if (buf && len) {
    size_t n = std::min(len - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return int(s.size());
}

int grx_gguf_tensor(const grx_gguf* f, const char* name, int* type, int64_t dims[4]) {
  if (!f) return fail(GRX_EINVAL, "null file");
  auto it = f->f.tensors.find(name);
  if (it == f->f.tensors.end()) return fail(GRX_EINVAL, std::string("no tensor ") + name);
  if (type) *type = it->second.type;
  for (size_t i = 0; i < 4; i++) dims[i] = i < it->second.dims.size() ? it->second.dims[i] : 1;
  return int(it->second.dims.size());
}

int grx_gguf_float32(const grx_gguf* f, const char* name, float* dst, size_t n) {
  if (!f || !dst) return fail(GRX_EINVAL, "null argument");
  std::vector<float> v;
  if (!f->f.float32(name, v)) return fail(GRX_EINVAL, std::string("no tensor ") + name);
  if (v.size() != n) return fail(GRX_EINVAL, "wrong size for " + std::string(name));
  std::memcpy(dst, v.data(), n * 4);
  return GRX_OK;
}

// ---- operator ----

int grx_weight_q8(int device, const void* blocks, int rows, int cols, grx_weight** out) {
  if (!blocks || !out || rows <= 0 || cols <= 0 || cols % 32 != 0)
    return fail(GRX_EINVAL, "kern: Q8_0 rows must be a multiple of 32 values");
  int rc = device_init(device);
  if (rc) return rc;
  auto w = std::make_unique<grx_weight>();
  w->ar.dev = device;
  w->type = 2;
  w->rows = rows;
  w->cols = cols;
  w->q8 = upload_q8(w->ar, (const uint8_t*)blocks, rows, cols, &rc);
  if (rc) return rc;
  *out = w.release();
  return GRX_OK;
}

int grx_weight_f32(int device, const float* v, int rows, int cols, grx_weight** out) {
  if (!v || !out || rows <= 0 || cols <= 0) return fail(GRX_EINVAL, "bad F32 weight");
  int rc = device_init(device);
  if (rc) return rc;
  auto w = std::make_unique<grx_weight>();
  w->ar.dev = device;
  w->type = 0;
  w->rows = rows;
  w->cols = cols;
  w->f = w->ar.upload(v, size_t(rows) * cols, &rc);
  if (rc) return rc;
  *out = w.release();
  return GRX_OK;
}

int grx_weight_drop_rows(grx_weight* w) {
  if (!w) return fail(GRX_EINVAL, "null weight");
  if (w->type == 2) w->dropped = true;
  return GRX_OK;
}

void grx_weight_free(grx_weight* w) { delete w; }

int grx_linear(const grx_weight* w, const float* x, int m, const float* bias, float* dst) {
  if (!w || !x || !dst || m < 0) return fail(GRX_EINVAL, "grx_linear: bad argument");
  if (m == 0) return GRX_OK;
  CK(cudaSetDevice(w->ar.dev));
  const int n = w->rows, k = w->cols;
  const bool int8 = w->type == 2 && (w->dropped || m >= 2);
  if (!int8 && m > 16) return fail(GRX_EINVAL, "grx_linear: float-path products take at most 16 rows");
  if (int8 && m > 8 && k % 64 != 0) return fail(GRX_EINVAL, "grx_linear: int8 products of more than 8 rows need K % 64 == 0");
  if (int8 && m <= 8 && n % 32 != 0) return fail(GRX_EINVAL, "grx_linear: int8 products of up to 8 rows need N % 32 == 0");
  int rc = 0;
  Arena ar;
  ar.dev = w->ar.dev;
  float* dx = ar.upload(x, size_t(m) * k, &rc);
  float* db = bias ? ar.upload(bias, size_t(n), &rc) : nullptr;
  float* dy = ar.alloc<float>(size_t(m) * n, &rc);
  if (rc) return rc;
  if (int8) {
    int8_t* q = ar.alloc<int8_t>(size_t(m) * k, &rc);
    float2* s = ar.alloc<float2>(size_t(m) * (k / 32), &rc);
    if (rc) return rc;
    launch_quant(dx, m, k, q, s, 0);
    EpiArgs e;
    e.epi = EPI_STORE;
    e.y = dy;
    e.ldy = n;
    e.bias = db;
    launch_q8_product(q, s, m, w->q8, e, 0);
  } else {
    if (w->type == 2 ? k % 32 : k % 16) return fail(GRX_EINVAL, "grx_linear: K must be whole blocks");
    const int kmax = w->type == 2 ? flin_max_k_q8() : flin_max_k();
    if (k > kmax) return fail(GRX_EINVAL, "grx_linear: float-path K above " + std::to_string(kmax));
    FArgs a;
    a.epi = FE_BIAS;
    a.x = dx;
    a.ldx = k;
    a.wq = w->type == 2 ? w->q8.q : nullptr;
    a.wd = w->type == 2 ? w->q8.d : nullptr;
    a.wf = w->type == 0 ? w->f : nullptr;
    a.N = n;
    a.K = k;
    a.bias = db;
    a.y = dy;
    a.ldy = n;
    launch_flin(a, m, 0);
  }
  CK(cudaGetLastError());
  CK(cudaMemcpy(dst, dy, size_t(m) * n * 4, cudaMemcpyDeviceToHost));
  return GRX_OK;
}

// ---- FlowLM ----

int grx_flowlm_load(const void* bytes, size_t len, int device, grx_flowlm** out) {
  if (!bytes || !out) return fail(GRX_EINVAL, "grx_flowlm_load: null argument");
  int rc = device_init(device);
  if (rc) return rc;
  GGUF f;
  if (!f.parse(bytes, len)) return fail(GRX_EFORMAT, f.err);
  if (f.get_string("general.architecture", "") != "pockettts")
    return fail(GRX_EFORMAT, "pockettts: the file isn't a Pocket TTS model");
  auto m = std::make_unique<grx_flowlm>();
  m->ar.dev = device;
  m->dev = device;
  m->sha = f.get_string("general.source.sha256", "");
  if (m->sha.empty()) return fail(GRX_EFORMAT, "pockettts: the file doesn't name its source");
  std::string err;
  // loader.num, model.go:93-100.
  auto num = [&](const char* key) -> int {
    int64_t v = f.get_int(key, -1);
    if (v < 1 || v > (1 << 16)) {
      if (err.empty()) err = std::string("pockettts: the setting ") + key + " is " + std::to_string(v);
      return 1;
    }
    return int(v);
  };
  // loader.mat / loader.vec with shape checks, model.go:61-91.
  auto vec = [&](const std::string& name, int64_t n) -> float* {
    if (!err.empty()) return nullptr;
    std::vector<float> v;
    auto it = f.tensors.find(name);
    if (it == f.tensors.end() || it->second.elems() != n || !f.float32(name, v)) {
      err = "pockettts: no " + std::to_string(n) + "-value " + name;
      return nullptr;
    }
    return m->ar.upload(v.data(), v.size(), &rc);
  };
  auto shape_ok = [&](const std::string& name, int64_t rows, int64_t cols) -> const GTensor* {
    if (!err.empty()) return nullptr;
    int64_t r, c;
    if (!f.matrix_shape(name, &r, &c)) {
      err = "pockettts: no tensor " + name;
      return nullptr;
    }
    if (r != rows || c != cols) {
      err = "pockettts: " + name + " is " + std::to_string(r) + "x" + std::to_string(c) + ", want " +
            std::to_string(rows) + "x" + std::to_string(cols);
      return nullptr;
    }
    return &f.tensors.at(name);
  };
  auto q8 = [&](const std::string& name, int64_t rows, int64_t cols) -> DQ8 {
    const GTensor* t = shape_ok(name, rows, cols);
    if (!t) return DQ8{};
    if (t->type != G_Q8_0) {
      // A float tensor where Q8_0 is expected: round it the way ToQ8 does
      // is not what the reference's loader does; refuse.
      err = "pockettts: " + name + " is not Q8_0";
      return DQ8{};
    }
    return upload_q8(m->ar, t->data, int(rows), int(cols), &rc);
  };
  auto f32m = [&](const std::string& name, int64_t rows, int64_t cols) -> float* {
    const GTensor* t = shape_ok(name, rows, cols);
    if (!t) return nullptr;
    std::vector<float> v;
    f.float32(name, v);
    if (t->type == G_Q8_0) {
      err = "pockettts: " + name + " is Q8_0 where float32 is expected";
      return nullptr;
    }
    return m->ar.upload(v.data(), v.size(), &rc);
  };
  m->ldim = num("pockettts.latent_dim");
  m->d = num("pockettts.lm.d_model");
  m->heads = num("pockettts.lm.heads");
  m->ff = num("pockettts.lm.ff");
  m->L = num("pockettts.lm.layers");
  m->fd = num("pockettts.flow.dim");
  m->depth = num("pockettts.flow.depth");
  m->steps = num("pockettts.decode_steps");
  m->period = f.get_float("pockettts.lm.max_period", 1e4);
  if (!err.empty()) return fail(GRX_EFORMAT, err);
  const int d = m->d, ff = m->ff, fd = m->fd, ld = m->ldim;
  if (d % m->heads != 0 || d / m->heads != 64)
    return fail(GRX_EINVAL, "pockettts: heads of " + std::to_string(d / m->heads) + " values (this build runs 64)");
  if (d % 128 || ff % 128 || fd % 128 || ld % 16 || d > 4096 || fd > 4096)
    return fail(GRX_EINVAL, "pockettts: model dimensions outside what the kernels take");
  for (int i = 0;; i++) {
    std::string p = "lm.blk." + std::to_string(i) + ".";
    if (!f.has(p + "norm1.weight")) break;
    Layer ly;
    ly.n1w = vec(p + "norm1.weight", d);
    ly.n1b = vec(p + "norm1.bias", d);
    ly.n2w = vec(p + "norm2.weight", d);
    ly.n2b = vec(p + "norm2.bias", d);
    ly.qkv = q8(p + "attn_qkv.weight", 3 * d, d);
    ly.out = q8(p + "attn_out.weight", d, d);
    ly.ff1 = q8(p + "ff1.weight", ff, d);
    ly.ff2 = q8(p + "ff2.weight", d, ff);
    m->layers.push_back(ly);
  }
  if (err.empty() && int(m->layers.size()) != m->L)
    err = "pockettts: the flow LM has " + std::to_string(m->layers.size()) + " layers";
  m->win = f32m("lm.input.weight", d, ld);
  m->bos = vec("lm.bos", ld);
  m->outw = vec("lm.out_norm.weight", d);
  m->outb = vec("lm.out_norm.bias", d);
  m->eosw = f32m("lm.eos.weight", 1, d);
  {
    std::vector<float> b;
    if (err.empty() && (!f.float32("lm.eos.bias", b) || b.size() != 1)) err = "pockettts: no 1-value lm.eos.bias";
    if (!b.empty()) m->eosb = b[0];
  }
  m->mean = vec("lm.emb_mean", ld);
  m->stdv = vec("lm.emb_std", ld);
  m->cond = q8("flow.cond.weight", fd, d);
  m->condb = vec("flow.cond.bias", fd);
  m->fin = f32m("flow.input.weight", fd, ld);
  m->finb = vec("flow.input.bias", fd);
  if (err.empty() && f.has("lm.embed")) {  // the text embedding (model.go:246): text prefill only
    int64_t r = 0, c = 0;
    std::vector<float> v;
    if (!f.matrix_shape("lm.embed", &r, &c) || c != d || r < 1 || r > (1 << 24) || !f.float32("lm.embed", v)) {
      err = "pockettts: lm.embed is not a [tokens + 1][" + std::to_string(d) + "] matrix";
    } else {
      m->embed = m->ar.upload(v.data(), v.size(), &rc);
      m->embed_rows = int(r);
    }
  }
  if (err.empty() && f.has("lm.speaker_proj") && f.has("lm.bos_voice")) {  // voice cloning (model.go:309-316)
    m->speaker = f32m("lm.speaker_proj", d, ld);
    m->bosv = vec("lm.bos_voice", d);
  }
  DQ8 tfc1[2], tfc2[2];
  float *tb1[2], *tb2[2], *alpha[2];
  std::vector<float> freqs[2];
  for (int k = 0; k < 2; k++) {
    std::string p = "flow.time." + std::to_string(k) + ".";
    if (err.empty() && (!f.float32(p + "freqs", freqs[k]) || freqs[k].size() != 128))
      err = "pockettts: no 128-value " + p + "freqs";
    tfc1[k] = q8(p + "fc1.weight", fd, 256);
    tb1[k] = vec(p + "fc1.bias", fd);
    tfc2[k] = q8(p + "fc2.weight", fd, fd);
    tb2[k] = vec(p + "fc2.bias", fd);
    alpha[k] = vec(p + "norm.alpha", fd);
  }
  for (int i = 0; i < m->depth; i++) {
    std::string p = "flow.res." + std::to_string(i) + ".";
    Res r;
    r.nw = vec(p + "norm.weight", fd);
    r.nb = vec(p + "norm.bias", fd);
    r.fc1 = q8(p + "fc1.weight", fd, fd);
    r.b1 = vec(p + "fc1.bias", fd);
    r.fc2 = q8(p + "fc2.weight", fd, fd);
    r.b2 = vec(p + "fc2.bias", fd);
    r.ada = q8(p + "ada.weight", 3 * fd, fd);
    r.adab = vec(p + "ada.bias", 3 * fd);
    m->res.push_back(r);
  }
  m->fada = q8("flow.final.ada.weight", 2 * fd, fd);
  m->fadab = vec("flow.final.ada.bias", 2 * fd);
  m->fout = f32m("flow.final.out.weight", ld, fd);
  m->foutb = vec("flow.final.out.bias", ld);
  if (!err.empty()) return fail(GRX_EFORMAT, err);
  if (rc) return rc;
  m->freqs = rope_freqs(64, m->period);

  // The time conditions, once (Speak, speak.go:57 → lm.go:62-104): the
  // embedders' [cos, sin] inputs in float64 on the host, the MLPs and the
  // normalization on the device with the same kernels as the frame.
  {
    const int S = m->steps;
    std::vector<float> in[2];
    for (int k = 0; k < 2; k++) {
      in[k].resize(size_t(S) * 256);
      for (int s = 0; s < S; s++) {
        float t = float(double(s + k) / double(S));
        for (int i = 0; i < 128; i++) {
          double a = double(t * freqs[k][size_t(i)]);
          in[k][size_t(s) * 256 + i] = float(std::cos(a));
          in[k][size_t(s) * 256 + 128 + i] = float(std::sin(a));
        }
      }
    }
    Arena tmp;
    tmp.dev = device;
    float* y[2];
    for (int k = 0; k < 2; k++) {
      float* din = tmp.upload(in[k].data(), in[k].size(), &rc);
      float* hh = tmp.alloc<float>(size_t(S) * fd, &rc);
      y[k] = tmp.alloc<float>(size_t(S) * fd, &rc);
      if (rc) return rc;
      FArgs a;
      a.epi = FE_SILU;
      a.x = din;
      a.ldx = 256;
      a.wq = tfc1[k].q;
      a.wd = tfc1[k].d;
      a.N = fd;
      a.K = 256;
      a.bias = tb1[k];
      a.y = hh;
      a.ldy = fd;
      launch_flin(a, S, 0);
      FArgs b = a;
      b.epi = FE_BIAS;
      b.x = hh;
      b.ldx = fd;
      b.wq = tfc2[k].q;
      b.wd = tfc2[k].d;
      b.K = fd;
      b.bias = tb2[k];
      b.y = y[k];
      launch_flin(b, S, 0);
    }
    m->tc = m->ar.alloc<float>(size_t(S) * fd, &rc);
    if (rc) return rc;
    launch_time_norm(y[0], y[1], alpha[0], alpha[1], fd, S, m->tc, 0);
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
  }
  *out = m.release();
  return GRX_OK;
}

void grx_flowlm_free(grx_flowlm* m) { delete m; }

int grx_flowlm_dims(const grx_flowlm* m, int* d, int* heads, int* ff, int* layers, int* ldim, int* fdim, int* depth,
                    int* steps) {
  if (!m) return fail(GRX_EINVAL, "null model");
  if (d) *d = m->d;
  if (heads) *heads = m->heads;
  if (ff) *ff = m->ff;
  if (layers) *layers = m->L;
  if (ldim) *ldim = m->ldim;
  if (fdim) *fdim = m->fd;
  if (depth) *depth = m->depth;
  if (steps) *steps = m->steps;
  return GRX_OK;
}

int grx_voice_kv(const grx_voice* v, int* positions, float* kv) {
  if (!v) return fail(GRX_EINVAL, "grx_voice_kv: null voice");
  if (positions) *positions = v->positions;
  if (kv) std::memcpy(kv, v->kv.data(), sizeof(float) * v->kv.size());
  return GRX_OK;
}

int grx_voice_raw(grx_flowlm* m, int positions, const float* kv, grx_voice** out) {
  if (!m || !kv || !out) return fail(GRX_EINVAL, "grx_voice_raw: null argument");
  if (positions < 1 || positions > 4096) return fail(GRX_EINVAL, "pockettts: a voice of " + std::to_string(positions) + " positions");
  auto v = std::make_unique<grx_voice>();
  v->positions = positions;
  size_t n = size_t(m->L) * 2 * positions * m->d;
  v->kv.assign(kv, kv + n);
  for (float x : v->kv)
    if (!std::isfinite(x)) return fail(GRX_EFORMAT, "pockettts: the voice has values that aren't numbers");
  v->model = m->sha;
  *out = v.release();
  return GRX_OK;
}

int grx_voice_load(grx_flowlm* m, const void* bytes, size_t len, grx_voice** out) {
  if (!m || !bytes || !out) return fail(GRX_EINVAL, "grx_voice_load: null argument");
  GGUF f;
  if (!f.parse(bytes, len)) return fail(GRX_EFORMAT, f.err);
  if (f.get_string("general.architecture", "") != "pockettts-voice")
    return fail(GRX_EFORMAT, "pockettts: the file isn't a Pocket TTS voice");
  if (f.get_string("pockettts.voice.model.sha256", "") != m->sha)
    return fail(GRX_EFORMAT, "pockettts: the voice was made for a different model file");
  int64_t nl = f.get_int("pockettts.voice.layers", 0), n = f.get_int("pockettts.voice.positions", 0);
  if (nl != m->L || n < 1 || n > 4096)
    return fail(GRX_EFORMAT, "pockettts: the voice holds " + std::to_string(nl) + " layers of " + std::to_string(n) + " positions");
  std::vector<float> kv(size_t(m->L) * 2 * size_t(n) * m->d);
  for (int i = 0; i < m->L; i++)
    for (int j = 0; j < 2; j++) {
      std::string name = "voice." + std::to_string(i) + "." + "kv"[j];
      auto it = f.tensors.find(name);
      if (it == f.tensors.end() || it->second.dims.size() != 2 || it->second.dims[0] != m->d || it->second.dims[1] != n)
        return fail(GRX_EFORMAT, "pockettts: the voice has no " + std::to_string(n) + "x" + std::to_string(m->d) + " " + name);
      std::vector<float> v;
      if (!f.float32(name, v)) return fail(GRX_EFORMAT, "pockettts: unreadable " + name);
      std::memcpy(&kv[(size_t(i) * 2 + j) * size_t(n) * m->d], v.data(), v.size() * 4);
    }
  return grx_voice_raw(m, int(n), kv.data(), out);
}

void grx_voice_free(grx_voice* v) { delete v; }

int grx_streams_reset(grx_streams* s) {
  if (!s) return fail(GRX_EINVAL, "null streams");
  for (auto& p : s->parts) {
    int rc = grx_streams_reset(p.get());
    if (rc) return rc;
  }
  if (!s->parts.empty()) return GRX_OK;
  grx_flowlm* m = s->m;
  CK(cudaSetDevice(s->ar.dev));
  CK(cudaMemcpyAsync(s->pos, s->pos0, sizeof(int) * size_t(s->n), cudaMemcpyDeviceToDevice, s->st));
  if (s->b1) CK(cudaMemsetAsync(s->f1_err, 0, sizeof(int), s->st));
  for (int i = 0; i < s->n; i++)
    CK(cudaMemcpyAsync(s->lat + size_t(i) * m->ldim, m->bos, sizeof(float) * size_t(m->ldim), cudaMemcpyDeviceToDevice,
                       s->st));
  CK(cudaStreamSynchronize(s->st));
  s->f1_err_copied = false;  // the reset cleared the word; a copy queued before it is stale
  return GRX_OK;
}

// flowLM.text (lm.go:172-181) for the streams of one set or part: stream i's
// tokens are ids[off[i] .. off[i+1]) (off relative to the caller's array).
// All streams' token rows go through each layer together; rows r of stream
// i sit at positions pos[i] + r and write its cache.
static int streams_text_one(grx_streams* q, const int* ids, const int* off, float* out, const float* d_xin = nullptr) {
  grx_flowlm* m = q->m;
  const int n = q->n, d = m->d, ff = m->ff;
  std::vector<int> pos((size_t(n)));
  CK(cudaMemcpyAsync(pos.data(), q->pos, sizeof(int) * size_t(n), cudaMemcpyDeviceToHost, q->st));
  CK(cudaStreamSynchronize(q->st));
  std::vector<int> row_id, row_slot, row_pos, c_row0, c_T, c_pos0, c_slot, last_row;
  int tmax = 0;
  for (int i = 0; i < n; i++) {
    const int T = off[i + 1] - off[i];
    if (T == 0) continue;
    if (pos[size_t(i)] + T > q->cap)
      return fail(GRX_ERANGE, "grx_streams_text: stream " + std::to_string(q->row0 + i) + " holds " +
                                  std::to_string(pos[size_t(i)]) + " positions; " + std::to_string(T) +
                                  " tokens pass the " + std::to_string(q->cap) + " it was made for");
    c_row0.push_back(int(row_id.size()));
    c_T.push_back(T);
    c_pos0.push_back(pos[size_t(i)]);
    c_slot.push_back(i);
    for (int r = 0; r < T; r++) {
      row_id.push_back(ids ? ids[off[i] - off[0] + r] : 0);
      row_slot.push_back(i);
      row_pos.push_back(pos[size_t(i)] + r);
    }
    last_row.push_back(int(row_id.size()) - 1);
    tmax = std::max(tmax, T);
  }
  const int R = int(row_id.size()), ns = int(c_T.size());
  if (R == 0) return GRX_OK;
  int rc = 0;
  Arena ar;
  ar.dev = q->ar.dev;
  float* x = ar.alloc<float>(size_t(R) * d, &rc);
  float* qb = ar.alloc<float>(size_t(R) * d, &rc);
  int8_t* xq = ar.alloc<int8_t>(size_t(R) * d, &rc);
  float2* xs = ar.alloc<float2>(size_t(R) * (d / 32), &rc);  // a scale per 32-value block
  int8_t* fq = ar.alloc<int8_t>(size_t(R) * ff, &rc);
  float2* fs = ar.alloc<float2>(size_t(R) * (ff / 32), &rc);
  int* dint = ar.alloc<int>(size_t(3) * R + size_t(5) * ns, &rc);
  float* lo = out ? ar.alloc<float>(size_t(ns) * d, &rc) : nullptr;
  float* lrow = out ? ar.alloc<float>(size_t(ns) * d, &rc) : nullptr;
  if (rc) return rc;
  std::vector<int> hint;
  for (const auto* v : {&row_id, &row_slot, &row_pos, &c_row0, &c_T, &c_pos0, &c_slot, &last_row})
    hint.insert(hint.end(), v->begin(), v->end());
  CK(cudaMemcpyAsync(dint, hint.data(), sizeof(int) * hint.size(), cudaMemcpyHostToDevice, q->st));
  const int *d_id = dint, *d_slot = dint + R, *d_pos = dint + 2 * R, *d_row0 = dint + 3 * R, *d_T = d_row0 + ns,
            *d_pos0 = d_T + ns, *d_cslot = d_pos0 + ns, *d_last = d_cslot + ns;
  cudaStream_t st = q->st;
  if (d_xin)  // the rows themselves (voice conditioning), in row order
    CK(cudaMemcpyAsync(x, d_xin, sizeof(float) * size_t(R) * d, cudaMemcpyDeviceToDevice, st));
  else
    launch_embed_rows(x, m->embed, d_id, R, d, st);
  for (int l = 0; l < m->L; l++) {
    const Layer& ly = m->layers[size_t(l)];
    LnArgs ln;
    ln.x = x;
    ln.w = ly.n1w;
    ln.b = ly.n1b;
    ln.eps = 1e-5;
    ln.mode = LN_Q8;
    ln.q8 = xq;
    ln.q8s = xs;
    launch_ln(ln, R, d, st);
    EpiArgs e;
    e.epi = EPI_ROPE_KV;
    e.kv.q = qb;
    e.kv.kv = q->kv;
    e.kv.pos = d_pos;
    e.kv.row_stream = d_slot;
    e.kv.rope = q->rope;
    e.kv.layer = l;
    e.kv.layers = m->L;
    e.kv.heads = m->heads;
    e.kv.cap = q->cap;
    e.kv.d = d;
    launch_q8_product(xq, xs, R, ly.qkv, e, st);
    AttnRowsArgs at;
    at.q = qb;
    at.kv = q->kv;
    at.row0 = d_row0;
    at.T = d_T;
    at.pos0 = d_pos0;
    at.slot = d_cslot;
    at.q8 = xq;
    at.q8s = xs;
    at.layer = l;
    at.layers = m->L;
    at.heads = m->heads;
    at.cap = q->cap;
    at.d = d;
    launch_attn_rows(at, ns, tmax, st);
    EpiArgs r;
    r.epi = EPI_RESID;
    r.y = x;
    r.ldy = d;
    launch_q8_product(xq, xs, R, ly.out, r, st);
    ln.w = ly.n2w;
    ln.b = ly.n2b;
    launch_ln(ln, R, d, st);
    EpiArgs g;
    g.epi = EPI_GELU_Q8;
    g.q8 = fq;
    g.q8s = fs;
    launch_q8_product(xq, xs, R, ly.ff1, g, st);
    launch_q8_product(fq, fs, R, ly.ff2, r, st);
  }
  for (size_t i = 0; i < c_T.size(); i++) pos[size_t(c_slot[i])] += c_T[i];
  CK(cudaMemcpyAsync(q->pos, pos.data(), sizeof(int) * size_t(n), cudaMemcpyHostToDevice, st));
  if (out) {
    // out_norm of each stream's last token row (lm.go:164-170)
    launch_embed_rows(lrow, x, d_last, ns, d, st);
    LnArgs on;
    on.x = lrow;
    on.w = m->outw;
    on.b = m->outb;
    on.eps = 1e-5;
    on.mode = LN_F32;
    on.y = lo;
    launch_ln(on, ns, d, st);
    std::vector<float> h((size_t(ns) * d));
    CK(cudaMemcpyAsync(h.data(), lo, sizeof(float) * h.size(), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    for (int i = 0; i < ns; i++)
      std::memcpy(out + size_t(c_slot[size_t(i)]) * d, h.data() + size_t(i) * d, sizeof(float) * size_t(d));
  }
  CK(cudaStreamSynchronize(st));
  CK(cudaGetLastError());
  return GRX_OK;
}

int grx_streams_text(grx_streams* s, const int* ids, const int* offsets, float* out) {
  if (!s || !offsets || (!ids && offsets[s->n] > 0)) return fail(GRX_EINVAL, "grx_streams_text: null argument");
  grx_flowlm* m = s->m;
  if (!m->embed) return fail(GRX_EINVAL, "grx_streams_text: the model has no lm.embed");
  if (offsets[0] != 0) return fail(GRX_EINVAL, "grx_streams_text: offsets[0] must be 0");
  for (int i = 0; i < s->n; i++)
    if (offsets[i + 1] < offsets[i]) return fail(GRX_EINVAL, "grx_streams_text: offsets must not decrease");
  for (int j = 0; j < offsets[s->n]; j++)
    if (ids[j] < 0 || ids[j] >= m->embed_rows)
      return fail(GRX_EINVAL, "grx_streams_text: token id " + std::to_string(ids[j]) + " outside the " +
                                  std::to_string(m->embed_rows) + "-row embedding");
  CK(cudaSetDevice(s->ar.dev));
  if (s->parts.empty()) return streams_text_one(s, ids, offsets, out);
  for (auto& p : s->parts) {
    int rc = streams_text_one(p.get(), ids + offsets[p->row0], offsets + p->row0, out ? out + size_t(p->row0) * m->d : nullptr);
    if (rc) return rc;
  }
  return GRX_OK;
}

// The flow-LM half of Model.CloneVoice (voice.go:94-106; cloneCond :113-127
// after Mimi's encoder): cond = kern.Linear(latents, lm.speaker_proj), a
// float32 weight, so MatMul's float path — gemvRows up to 16 rows, else the
// packed kernel for the first n/6·6 rows and gemvRows for the rest — then
// [bos_voice; cond] through the transformer from an empty state (lm.run with
// n + 1 rows); the caches are the voice.
static int streams_create_one(grx_flowlm* m, int n, const grx_voice* const* voices, int max_frames,
                              std::unique_ptr<grx_streams>* out);

int grx_voice_from_latents(grx_flowlm* m, const float* latents, int n, grx_voice** out) {
  if (!m || !latents || !out) return fail(GRX_EINVAL, "grx_voice_from_latents: null argument");
  if (!m->speaker || !m->bosv) return fail(GRX_EINVAL, "pockettts: this model file has no voice cloning");
  if (n < 1 || n > 4095) return fail(GRX_EINVAL, "pockettts: " + std::to_string(n) + " latent frames");
  int rc = device_init(m->dev);
  if (rc) return rc;
  const int d = m->d, ld = m->ldim, L = m->L, H = m->heads, hd = 64;
  grx_voice empty;
  empty.model = m->sha;
  const grx_voice* vp = &empty;
  std::unique_ptr<grx_streams> s;
  rc = streams_create_one(m, 1, &vp, n + 1, &s);
  if (rc) return rc;
  Arena ar;
  ar.dev = m->dev;
  float* dl = ar.upload(latents, size_t(n) * ld, &rc);
  float* rows = ar.alloc<float>(size_t(n + 1) * d, &rc);
  if (rc) return rc;
  cudaStream_t st = s->st;
  CK(cudaMemcpyAsync(rows, m->bosv, sizeof(float) * d, cudaMemcpyDeviceToDevice, st));
  const int packed = n > 16 ? n / 6 * 6 : 0;  // rows through the packed kernel
  if (packed > 0) {
    WmmArgs w;
    w.a = dl;
    w.lda = ld;
    w.m = packed;
    w.w.f = m->speaker;
    w.w.rows = d;
    w.w.cols = ld;
    w.mode = WM_STORE;
    w.c = rows + d;
    w.ldc = d;
    launch_wmm(w, 1, st);
  }
  if (packed < n) {
    FArgs a;
    a.epi = FE_BIAS;
    a.x = dl + size_t(packed) * ld;
    a.ldx = ld;
    a.wf = m->speaker;
    a.N = d;
    a.K = ld;
    a.y = rows + size_t(1 + packed) * d;
    a.ldy = d;
    launch_flin(a, n - packed, st);
  }
  std::vector<int> off = {0, n + 1};
  rc = streams_text_one(s.get(), nullptr, off.data(), nullptr, rows);
  if (rc) return rc;
  // the cache [layer][k|v][head][position][64] → the voice's [layer][k|v][position][d]
  std::vector<float> c(size_t(L) * 2 * H * s->cap * hd);
  CK(cudaMemcpy(c.data(), s->kv, sizeof(float) * c.size(), cudaMemcpyDeviceToHost));
  auto v = std::make_unique<grx_voice>();
  v->positions = n + 1;
  v->model = m->sha;
  v->kv.resize(size_t(L) * 2 * (n + 1) * d);
  for (int l = 0; l < L; l++)
    for (int k = 0; k < 2; k++)
      for (int h = 0; h < H; h++)
        for (int p = 0; p <= n; p++)
          std::memcpy(&v->kv[((size_t(l) * 2 + k) * (n + 1) + p) * d + size_t(h) * hd],
                      &c[(((size_t(l) * 2 + k) * H + h) * s->cap + p) * hd], sizeof(float) * hd);
  *out = v.release();
  return GRX_OK;
}

static int streams_create_one(grx_flowlm* m, int n, const grx_voice* const* voices, int max_frames,
                              std::unique_ptr<grx_streams>* out);

int grx_streams_create(grx_flowlm* m, int n, const grx_voice* const* voices, int max_frames, grx_streams** out) {
  if (!m || !voices || !out || n < 1 || max_frames < 1) return fail(GRX_EINVAL, "grx_streams_create: bad argument");
  int rc = device_init(m->dev);
  if (rc) return rc;
  const int nparts = std::max(1, std::min(stream_parts_max(), n / kMinPart));
  if (nparts == 1) {
    std::unique_ptr<grx_streams> s;
    rc = streams_create_one(m, n, voices, max_frames, &s);
    if (rc) return rc;
    *out = s.release();
    return GRX_OK;
  }
  auto s = std::make_unique<grx_streams>();
  s->ar.dev = m->dev;
  s->m = m;
  s->n = n;
  CK(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
  CK(cudaEventCreateWithFlags(&s->ev, cudaEventDisableTiming));
  for (int i = 0, r0 = 0; i < nparts; i++) {
    const int ni = n / nparts + (i < n % nparts ? 1 : 0);
    std::unique_ptr<grx_streams> p;
    rc = streams_create_one(m, ni, voices + r0, max_frames, &p);
    if (rc) return rc;
    p->row0 = r0;
    CK(cudaEventCreateWithFlags(&p->ev, cudaEventDisableTiming));
    s->cap = p->cap;
    s->per_frame += p->per_frame;
    s->parts.push_back(std::move(p));
    r0 += ni;
  }
  *out = s.release();
  return GRX_OK;
}

static int streams_create_one(grx_flowlm* m, int n, const grx_voice* const* voices, int max_frames,
                              std::unique_ptr<grx_streams>* out) {
  int rc = 0;
  int maxp = 0;
  for (int i = 0; i < n; i++) {
    if (!voices[i]) return fail(GRX_EINVAL, "null voice");
    if (voices[i]->model != m->sha) return fail(GRX_EINVAL, "pockettts: the voice was made for a different model");
    maxp = std::max(maxp, voices[i]->positions);
  }
  auto s = std::make_unique<grx_streams>();
  s->ar.dev = m->dev;
  s->m = m;
  s->n = n;
  s->cap = maxp + max_frames;
  const int d = m->d, fd = m->fd, ld = m->ldim, H = m->heads, L = m->L, hd = 64;
  const size_t per_stream = size_t(L) * 2 * H * s->cap * hd;
  CK(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
  s->kv = s->ar.alloc<float>(per_stream * n, &rc);
  s->pos = s->ar.alloc<int>(size_t(n), &rc);
  s->pos0 = s->ar.alloc<int>(size_t(n), &rc);
  s->x = s->ar.alloc<float>(size_t(n) * d, &rc);
  s->q = s->ar.alloc<float>(size_t(n) * d, &rc);
  s->lm_out = s->ar.alloc<float>(size_t(n) * d, &rc);
  s->eos = s->ar.alloc<float>(size_t(n), &rc);
  s->lat = s->ar.alloc<float>(size_t(n) * ld, &rc);
  s->xq = s->ar.alloc<int8_t>(size_t(n) * d, &rc);
  s->xs = s->ar.alloc<float2>(size_t(n) * d / 32, &rc);
  s->xqf = s->ar.alloc<int8_t>(size_t(n) * m->ff, &rc);
  s->xsf = s->ar.alloc<float2>(size_t(n) * m->ff / 32, &rc);
  s->y0 = s->ar.alloc<float>(size_t(n) * fd, &rc);
  s->sy = s->ar.alloc<float>(size_t(n) * fd, &rc);
  s->h = s->ar.alloc<float>(size_t(n) * fd, &rc);
  s->mod = s->ar.alloc<float>(size_t(n) * 3 * fd, &rc);
  s->mod2 = s->ar.alloc<float>(size_t(n) * 2 * fd, &rc);
  s->nrm = s->ar.alloc<float>(size_t(n) * fd, &rc);
  s->mm = s->ar.alloc<float>(size_t(n) * fd, &rc);
  s->cur = s->ar.alloc<float>(size_t(n) * ld, &rc);
  {
    static_assert(sizeof(FrameIO) <= kIoPad, "the noise rows follow the FrameIO");
    s->in1_bytes = kIoPad + size_t(n) * ld * 4;
    uint8_t* in1 = s->ar.alloc<uint8_t>(s->in1_bytes, &rc);
    s->io = reinterpret_cast<FrameIO*>(in1);
    s->noise1 = reinterpret_cast<float*>(in1 + kIoPad);
    s->out1_floats = 2 * size_t(n) * ld + size_t(n) + 1;
    s->out1 = s->ar.alloc<float>(s->out1_floats, &rc);
    s->lat1 = s->out1;
    s->scaled1 = s->out1 + size_t(n) * ld;
    s->eos1 = s->out1 + 2 * size_t(n) * ld;
  }
  if (rc) return rc;
  CK(cudaHostAlloc(&s->in1_h, s->in1_bytes, cudaHostAllocDefault));
  CK(cudaHostAlloc(&s->out1_h, s->out1_floats * 4, cudaHostAllocDefault));
  // RoPE cos/sin for every position the streams can reach (nn.go:84-85).
  {
    std::vector<float> t(size_t(s->cap) * hd);
    for (int p = 0; p < s->cap; p++)
      for (int i = 0; i < hd / 2; i++) {
        double a = double(m->freqs[size_t(i)] * float(p));
        t[(size_t(p) * (hd / 2) + i) * 2] = float(std::cos(a));
        t[(size_t(p) * (hd / 2) + i) * 2 + 1] = float(std::sin(a));
      }
    s->rope = s->ar.upload(t.data(), t.size(), &rc);
  }
  // The voices' caches, into the per-head layout; streams sharing a voice
  // copy the first one's device rows.
  std::vector<int> p0((size_t)n);
  std::vector<float> lay;
  for (int i = 0; i < n; i++) {
    const grx_voice* v = voices[i];
    p0[size_t(i)] = v->positions;
    float* dst = s->kv + per_stream * size_t(i);
    int first = -1;
    for (int j = 0; j < i; j++)
      if (voices[j] == v) {
        first = j;
        break;
      }
    if (first >= 0) {
      CK(cudaMemcpy(dst, s->kv + per_stream * size_t(first), per_stream * 4, cudaMemcpyDeviceToDevice));
      continue;
    }
    const int P = v->positions;
    lay.assign(size_t(H) * P * hd, 0.f);
    for (int l = 0; l < L; l++)
      for (int kvi = 0; kvi < 2; kvi++) {
        const float* src = &v->kv[(size_t(l) * 2 + kvi) * size_t(P) * d];
        for (int p = 0; p < P; p++)
          for (int h = 0; h < H; h++)
            std::memcpy(&lay[(size_t(h) * P + p) * hd], src + size_t(p) * d + h * hd, hd * 4);
        for (int h = 0; h < H; h++) {
          float* hp = dst + ((size_t(l) * 2 + kvi) * H + h) * size_t(s->cap) * hd;
          CK(cudaMemcpy(hp, &lay[size_t(h) * P * hd], size_t(P) * hd * 4, cudaMemcpyHostToDevice));
        }
      }
  }
  CK(cudaMemcpy(s->pos0, p0.data(), sizeof(int) * size_t(n), cudaMemcpyHostToDevice));
  rc = frame1_setup(s.get());
  if (rc) return rc;
  rc = grx_streams_reset(s.get());
  if (rc) return rc;
  rc = build_graph(s.get());
  if (rc) return rc;
  *out = std::move(s);
  return GRX_OK;
}

void grx_streams_free(grx_streams* s) { delete s; }

int grx_streams_pos(const grx_streams* s, int i) {
  if (!s || i < 0 || i >= s->n) return fail(GRX_EINVAL, "bad stream index");
  for (const auto& p : s->parts)
    if (i < p->row0 + p->n) return grx_streams_pos(p.get(), i - p->row0);
  int p = 0;
  cudaSetDevice(s->ar.dev);
  if (cudaMemcpy(&p, s->pos + i, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return fail(GRX_ECUDA, "read pos");
  return p;
}

int64_t grx_streams_launches(const grx_streams* s) {
  if (!s) return 0;
  int64_t l = s->launches;
  for (const auto& p : s->parts) l += p->launches;
  return l;
}

void* grx_streams_cuda_stream(const grx_streams* s) { return s ? (void*)s->st : nullptr; }

int grx_streams_parts(const grx_streams* s) {
  if (!s) return fail(GRX_EINVAL, "null streams");
  return s->parts.empty() ? 1 : int(s->parts.size());
}

// Checks that `frames` more frames fit the caches (positions are equal for
// streams that started from voices of equal length; the longest decides).
static int check_room(grx_streams* s, int frames) {
  for (auto& p : s->parts) {
    int rc = check_room(p.get(), frames);
    if (rc) return rc;
  }
  if (!s->parts.empty()) return GRX_OK;
  int maxp = 0;
  std::vector<int> p(size_t(s->n));
  CK(cudaMemcpyAsync(p.data(), s->pos, sizeof(int) * size_t(s->n), cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));
  for (int v : p) maxp = std::max(maxp, v);
  if (maxp + frames > s->cap)
    return fail(GRX_ERANGE, "the streams hold " + std::to_string(maxp) + " positions; " + std::to_string(frames) +
                                " more frames pass the " + std::to_string(s->cap) + " they were made for");
  return GRX_OK;
}

int grx_streams_step(grx_streams* s, const float* noise, float* lm_out, float* eos, float* latent, float* scaled) {
  if (!s || !noise) return fail(GRX_EINVAL, "grx_streams_step: null argument");
  CK(cudaSetDevice(s->ar.dev));
  int rc = check_room(s, 1);
  if (rc) return rc;
  // each part (or the set itself) queues its frame on its own stream
  std::vector<grx_streams*> sets;
  if (s->parts.empty()) sets.push_back(s);
  for (auto& p : s->parts) sets.push_back(p.get());
  const int ld = s->m->ldim, d = s->m->d;
  for (grx_streams* q : sets) {
    const size_t r0 = size_t(q->row0), nl = size_t(q->n) * ld;
    FrameIO io{q->noise1, nullptr, nullptr, q->eos1, 0, nullptr, q->n, 0, 0, 1};
    if (q->b1) {
      io.latent = q->lat1;
      io.scaled = q->scaled1;
    }
    // the FrameIO and the noise rows in one copy
    std::memcpy(q->in1_h, &io, sizeof io);
    std::memcpy(q->in1_h + kIoPad, noise + r0 * ld, nl * 4);
    CK(cudaMemcpyAsync(q->io, q->in1_h, q->in1_bytes, cudaMemcpyHostToDevice, q->st));
    if (q->b1) {
      rc = frame1_run(q, 1, 0, false);  // its error word comes back with the outputs
      if (rc) return rc;
    } else {
      CK(cudaGraphLaunch(q->exec, q->st));
      q->launches += q->per_frame;
    }
  }
  // the copies out after every part's frame is queued: a copy to pageable
  // host memory returns only when it is done, and would otherwise hold back
  // the next part's launch
  for (grx_streams* q : sets) {
    const size_t r0 = size_t(q->row0);
    if (lm_out) CK(cudaMemcpyAsync(lm_out + r0 * d, q->lm_out, size_t(q->n) * d * 4, cudaMemcpyDeviceToHost, q->st));
    // latent, scaled, eos and the error word in one copy
    CK(cudaMemcpyAsync(q->out1_h, q->out1, q->out1_floats * 4, cudaMemcpyDeviceToHost, q->st));
  }
  for (grx_streams* q : sets) CK(cudaStreamSynchronize(q->st));
  for (grx_streams* q : sets) {
    const size_t r0 = size_t(q->row0), nl = size_t(q->n) * ld;
    const float* o = q->out1_h;
    if (latent) std::memcpy(latent + r0 * ld, o, nl * 4);
    if (scaled) std::memcpy(scaled + r0 * ld, o + nl, nl * 4);
    if (eos) std::memcpy(eos + r0, o + 2 * nl, size_t(q->n) * 4);
    if (q->b1) {
      int e = 0;
      std::memcpy(&e, o + q->out1_floats - 1, sizeof e);
      rc = frame1_error(e);
      if (rc) return rc;
    }
  }
  return GRX_OK;
}

int grx_streams_run_device(grx_streams* s, int frames, const float* d_noise, float* d_latent, float* d_eos) {
  return grx_streams_run_device_timed(s, frames, d_noise, d_latent, d_eos, nullptr);
}

int grx_streams_run_device_timed(grx_streams* s, int frames, const float* d_noise, float* d_latent, float* d_eos,
                                 unsigned long long* d_attn_ts) {
  if (!s || !d_noise || frames < 0) return fail(GRX_EINVAL, "grx_streams_run_device: bad argument");
  CK(cudaSetDevice(s->ar.dev));
  int rc = check_room(s, frames);
  if (rc) return rc;
  if (s->parts.empty()) {
    FrameIO io{d_noise, d_latent, nullptr, d_eos, 0, d_attn_ts, s->n, 0, 0, 1};
    CK(cudaMemcpyAsync(s->io, &io, sizeof io, cudaMemcpyHostToDevice, s->st));
    if (s->b1) return frame1_run(s, frames);
    int rc2 = replay_frames(s, frames);
    if (rc2) return rc2;
    s->launches += int64_t(frames) * s->per_frame;
    return GRX_OK;
  }
  // fork: the parts wait for what was queued on the parent's stream
  CK(cudaEventRecord(s->ev, s->st));
  for (size_t i = 0; i < s->parts.size(); i++) {
    auto& p = s->parts[i];
    CK(cudaStreamWaitEvent(p->st, s->ev, 0));
    FrameIO io{d_noise, d_latent, nullptr, d_eos, 0, d_attn_ts, s->n, p->row0, int(i), int(s->parts.size())};
    CK(cudaMemcpyAsync(p->io, &io, sizeof io, cudaMemcpyHostToDevice, p->st));
  }
  for (int f = 0; f < frames; f += kGraphFrames)
    for (auto& p : s->parts) {
      int rc2 = replay_frames(p.get(), std::min(kGraphFrames, frames - f));
      if (rc2) return rc2;
    }
  // join: the parent's stream waits for every part
  for (auto& p : s->parts) {
    p->launches += int64_t(frames) * p->per_frame;
    CK(cudaEventRecord(p->ev, p->st));
    CK(cudaStreamWaitEvent(s->st, p->ev, 0));
  }
  return GRX_OK;
}

int grx_streams_sync(grx_streams* s) {
  if (!s) return fail(GRX_EINVAL, "null streams");
  CK(cudaSetDevice(s->ar.dev));
  CK(cudaStreamSynchronize(s->st));
  CK(cudaGetLastError());
  return frame1_check(s);
}

int grx_streams_persistent(const grx_streams* s) {
  if (!s) return fail(GRX_EINVAL, "null streams");
  return s->b1 ? 1 : 0;
}

int grx_streams_watchdog_test(grx_streams* s) {
  if (!s) return fail(GRX_EINVAL, "null streams");
  if (!s->b1) return fail(GRX_EINVAL, "grx_streams_watchdog_test: the set does not run the persistent kernel");
  CK(cudaSetDevice(s->ar.dev));
  int rc = check_room(s, 1);
  if (rc) return rc;
  FrameIO io{s->noise1, s->lat1, s->scaled1, s->eos1, 0, nullptr, s->n, 0, 0, 1};
  CK(cudaMemsetAsync(s->noise1, 0, sizeof(float) * size_t(s->m->ldim), s->st));
  CK(cudaMemcpyAsync(s->io, &io, sizeof io, cudaMemcpyHostToDevice, s->st));
  rc = frame1_run(s, 1, 1);
  if (rc) return rc;
  CK(cudaStreamSynchronize(s->st));
  CK(cudaGetLastError());
  return frame1_check(s);
}

}  // extern "C"

// Accessors for entry points defined in other files.
namespace grx {

int set_error(int code, const char* msg) { return fail(code, msg); }

int weight_device(const grx_weight* w) { return w->ar.dev; }

bool weight_q8(const grx_weight* w, const DQ8** q8, bool* dropped) {
  if (w->type != 2) return false;
  *q8 = &w->q8;
  *dropped = w->dropped;
  return true;
}

}  // namespace grx
