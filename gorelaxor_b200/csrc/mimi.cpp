// Mimi's decoder on the device (grx_mimi_*): the half of pockettts.Load
// that binds it (pockettts/model.go:102-178, 280-307) and
// mimiDecoder.decode (mimi.go:126-150) with runSea (:45-98) and
// speakChunk's fade-in (speak.go:177-190), for n independent streams that
// each decode one latent per call.
//
// One call runs every stream's rows through each step together: the
// products take all n·T rows at once where the reference's order does not
// depend on the call's row count (the int8 path, the float path up to 16
// rows), and per stream (grid z) where it does (the packed kernel of a
// float32 weight beyond 16 rows). The transformer's caches are rings of
// context + S − 1 positions per layer and stream, enough for every key a
// windowed query can see; the carried rows of the convolutions and of the
// upsampling alternate between two buffers, so a call reads the last call's
// and writes the next one's.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/grx.h"
#include "gguf.h"
#include "host.h"
#include "kernels.h"

using namespace grx;

namespace {

// A decoder weight as the reference holds it after pack(): Q8_0 (always the
// int8 path) or float32 (MatMul's float path).
struct MW {
  bool q8 = false;
  DQ8 q;
  float* f = nullptr;
  int rows = 0, cols = 0;
};

struct MConv {
  MW w;
  float* b = nullptr;
  int cin = 0, cout = 0, k = 1, stride = 1, dil = 1;
  int past() const { return (k - 1) * dil + 1 - stride; }
};

struct MStep {
  int kind = 0;  // 0 conv, 1 transposed conv (in c), 2 residual block (ra, rb)
  bool elu = false;
  MConv c, ra, rb;
};

struct MLayer {
  float *n1w, *n1b, *n2w, *n2b, *ls1, *ls2;
  DQ8 qkv, out, ff1, ff2;
};

std::vector<float> rope_freqs(int hd, double period) {
  float c = float(-std::log(period) * 2 / double(hd));
  std::vector<float> f(size_t(hd / 2));
  for (size_t i = 0; i < f.size(); i++) f[i] = float(std::exp(double(float(i) * c)));
  return f;
}

}  // namespace

struct grx_mimi {
  Arena ar;
  int dev = 0;
  int d = 0, heads = 0, ff = 0, context = 0, S = 0, ldim = 0, frame = 0, sample_rate = 0;
  std::vector<float> freqs;
  MW quant;
  float* up = nullptr;  // [d][2S]
  std::vector<MLayer> layers;
  std::vector<MStep> steps;
  // the encoder, when the file has one (model.go:181-200, 308-313)
  bool has_enc = false;
  int hop = 0;  // samples per encoder transformer row
  std::vector<MLayer> enc_layers;
  std::vector<MStep> enc_steps;
  MConv down;  // to the latent rate, no bias (down.b zeros), first call padded by replication
};

struct grx_mimi_streams {
  Arena ar;
  grx_mimi* m = nullptr;
  // the network a set runs: the decoder's (S = upsample rows per call) or
  // the encoder's (S = transformer rows of a full piece)
  const std::vector<MLayer>* layers = nullptr;
  const std::vector<MStep>* steps = nullptr;
  int S = 0;
  int n = 0, max_frames = 0, ring = 0, frames = 0;  // frames decoded since the last reset (all streams)
  cudaStream_t st = nullptr;
  float* kv = nullptr;  // [n][layers][2][heads][ring][64]
  float* rope = nullptr;
  int *pos = nullptr, *rowpos = nullptr, *rowslot = nullptr, *crow0 = nullptr, *cT = nullptr, *cslot = nullptr;
  int* started = nullptr;
  float *lat = nullptr, *z = nullptr, *x = nullptr, *qb = nullptr, *pcm = nullptr;
  float* up_part[2] = {nullptr, nullptr};
  int8_t *xq = nullptr, *fq = nullptr, *aq = nullptr;
  float2 *xs = nullptr, *fs = nullptr, *as = nullptr;
  // per carried-rows slot (steps in order; a residual block has two), two buffers
  std::vector<float*> carry[2];
  std::vector<size_t> carry_n;  // values per stream
  float *sa = nullptr, *sb = nullptr, *se = nullptr, *stage = nullptr, *col = nullptr, *zt = nullptr, *sh = nullptr;
  int par = 0;
  // encoder sets: the padded clips [n][max_samples], the latents of a piece,
  // the row count the row tables were last written for
  float *clip = nullptr, *piece_lat = nullptr;
  int max_samples = 0, rows_for = -1;
  int64_t launches = 0;
  // A decoder set's call as CUDA graphs, one per carried-buffer parity,
  // captured on first use with the set's own latent and sample buffers
  // (graph_tried: capture was attempted; graph_launches: kernels per call).
  cudaGraphExec_t graph[2] = {nullptr, nullptr};
  bool graph_tried = false;
  int64_t graph_launches = 0;
  // An encoder set's pieces as CUDA graphs, by piece length, carried-buffer
  // parity and whether the piece is the clip's first (null exec: capture
  // failed, the piece is launched directly).
  struct PieceGraph {
    int T0, par;
    bool first;
    cudaGraphExec_t exec;
    int64_t launches;
  };
  std::vector<PieceGraph> piece_graphs;
  ~grx_mimi_streams() {
    cudaSetDevice(ar.dev);
    for (cudaGraphExec_t g : graph)
      if (g) cudaGraphExecDestroy(g);
    for (const PieceGraph& pg : piece_graphs)
      if (pg.exec) cudaGraphExecDestroy(pg.exec);
    if (st) cudaStreamDestroy(st);
  }
};

namespace {

// The largest per-stream sizes one call needs, from the step plan (floats,
// except qk: the int8 path's rounded activations, values).
struct MimiSizes {
  size_t act = 0, stage = 0, col = 0, zt = 0, h = 0, qk = 0;
};

// A convolution of stride 1 and dilation 1 reads its window from staged rows.
bool staged(const MConv& c) { return c.k > 1 && c.stride == 1 && c.dil == 1; }

MimiSizes mimi_sizes(const grx_mimi* m) {
  MimiSizes s;
  int T = m->S, C = m->d;
  s.act = size_t(T) * C;
  s.qk = size_t(T) * std::max(m->d, m->ff);
  auto prod = [&](const MW& w, int rows) { s.qk = std::max(s.qk, size_t(rows) * w.cols); };
  prod(m->quant, 1);
  auto conv = [&](const MConv& c, int t) {
    const int To = t / c.stride;
    if (staged(c))
      s.stage = std::max(s.stage, size_t(c.past() + t) * c.cin);
    else if (!(c.k == 1 && c.stride == 1))
      s.col = std::max(s.col, size_t(To) * c.k * c.cin);
    prod(c.w, To);
    return To;
  };
  for (const MStep& st : m->steps) {
    s.act = std::max(s.act, size_t(T) * C);
    if (st.kind == 0) {
      T = conv(st.c, T);
      C = st.c.cout;
    } else if (st.kind == 1) {
      s.zt = std::max(s.zt, size_t(T) * st.c.k * st.c.cout);
      prod(st.c.w, T);
      T *= st.c.stride;
      C = st.c.cout;
    } else {
      conv(st.ra, T);
      s.h = std::max(s.h, size_t(T) * st.ra.cout);
      conv(st.rb, T);
    }
    s.act = std::max(s.act, size_t(T) * C);
  }
  return s;
}

// The same for an encoder set: pieces of T0 samples through the SEANet
// encoder, the transformer's rows, the downsampling convolution.
MimiSizes enc_sizes(const grx_mimi* m, int T0) {
  MimiSizes s;
  int T = T0, C = 1;
  auto prod = [&](const MW& w, int rows) { s.qk = std::max(s.qk, size_t(rows) * w.cols); };
  auto conv = [&](const MConv& c, int t) {
    const int To = t / c.stride;
    if (staged(c))
      s.stage = std::max(s.stage, size_t(c.past() + t) * c.cin);
    else if (!(c.k == 1 && c.stride == 1))
      s.col = std::max(s.col, size_t(To) * c.k * c.cin);
    prod(c.w, To);
    return To;
  };
  for (const MStep& st : m->enc_steps) {
    s.act = std::max(s.act, size_t(T) * C);
    if (st.kind == 0) {
      T = conv(st.c, T);
      C = st.c.cout;
    } else {
      conv(st.ra, T);
      s.h = std::max(s.h, size_t(T) * st.ra.cout);
      conv(st.rb, T);
    }
    s.act = std::max(s.act, size_t(T) * C);
  }
  conv(m->down, T);
  s.qk = std::max(s.qk, size_t(T) * std::max(m->d, m->ff));
  return s;
}

// A product's input: T rows per stream, row t of stream s the K values at
// x + (s·sstride + t)·ldx (ldx < K: a staged convolution window), through the
// ELU first when elu_len (the per-stream array length; x dense, Q8_0 only).
struct MIn {
  const float* x;
  int ldx, sstride, K, elu_len;
};

// y[n·T][N] = (or, resid, +=) the input times Wᵀ (+ bias), with the
// reference's order for a call of T rows per stream (kern.Linear,
// kern.go:185-201): the int8 path for a Q8_0 weight; for a float32 one
// gemvRows up to 16 rows, else the packed kernel for each stream's first
// T/6·6 rows and gemvRows for the rest.
void mimi_product(grx_mimi_streams* s, const MW& w, const MIn& in, int T, const float* bias, float* y, bool resid) {
  const int n = s->n, N = w.rows, K = w.cols, M = n * T;
  cudaStream_t st = s->st;
  if (w.q8) {
    launch_mimi_quant(in.x, in.ldx, in.sstride, n, T, K, in.elu_len, s->aq, s->as, st);
    s->launches++;
    EpiArgs e;
    e.epi = resid ? EPI_RESID : EPI_STORE;
    e.bias = bias;
    e.ldy = N;
    if (M <= 8 || K % 64 == 0) {
      e.y = y;
      launch_q8_product(s->aq, s->as, M, w.q, e, st);
      s->launches++;
      return;
    }
    // odd block counts: the up-to-8-row kernel, which takes any
    for (int r = 0; r < M; r += 8) {
      e.y = y + size_t(r) * N;
      launch_q8_product(s->aq + size_t(r) * K, s->as + size_t(r) * (K / 32), std::min(8, M - r), w.q, e, st);
      s->launches++;
    }
    return;
  }
  const int mf = T > 16 ? T / 6 * 6 : 0;  // rows per stream through the packed kernel
  if (mf > 0) {
    if (mimi_fconv_fits(in.ldx, K, N)) {
      FconvArgs f;
      f.x = in.x;
      f.sstride = in.sstride;
      f.cin = in.ldx;
      f.K = K;
      f.T = T;
      f.mf = mf;
      f.w = w.f;
      f.bias = bias;
      f.N = N;
      f.y = y;
      f.resid = resid;
      launch_mimi_fconv(f, n, st);
    } else {
      WmmArgs p;
      p.a = in.x;
      p.lda = in.ldx;
      p.a_zs = size_t(in.sstride) * in.ldx;
      p.m = mf;
      p.w.f = w.f;
      p.w.rows = N;
      p.w.cols = K;
      p.bias = bias;
      p.mode = resid ? WM_RESID : WM_STORE;
      p.c = y;
      p.ldc = N;
      p.c_zs = size_t(T) * N;
      launch_wmm(p, n, st);
    }
    s->launches++;
  }
  if (mf < T && K % 4) {  // K < 16: dotF32Go alone
    launch_mimi_gemv_small(in.x, in.ldx, in.sstride, T, mf, w.f, N, K, bias, y, resid, n, st);
    s->launches++;
  } else if (mf < T) {
    FArgs a;
    a.epi = resid ? FE_RESID : FE_BIAS;
    a.x = in.x;
    a.ldx = in.ldx;
    a.wf = w.f;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.y = y;
    a.ldy = N;
    a.rg_len = T - mf;
    a.rg_stride = in.sstride;
    a.rg_off = mf;
    a.ry_stride = T;
    a.ry_off = mf;
    launch_flin(a, n * (T - mf), st);
    s->launches++;
  }
}

// conv.run (nn.go:275-300) for the T rows per stream of x (dense
// [n][T][cin]), through the ELU first when elu; carried rows in slot ci.
void mimi_conv(grx_mimi_streams* s, const MConv& c, int ci, const float* x, int T, bool elu, float* y, bool resid) {
  const int n = s->n, cin = c.cin;
  cudaStream_t st = s->st;
  const bool window = staged(c) || (c.k == 1 && c.stride == 1);
  if (window && !c.w.q8 && T > 16 && T % 6 == 0 && mimi_fconv_fits(cin, c.k * cin, c.cout)) {
    // every row through the packed kernel: the window read in place from x
    // (carried rows, ELU) by the product itself
    FconvArgs f;
    f.x = x;
    f.cin = cin;
    f.K = c.k * cin;
    f.T = T;
    f.mf = T;
    f.w = c.w.f;
    f.bias = c.b;
    f.N = c.cout;
    f.y = y;
    f.resid = resid;
    f.virt = 1;
    f.P = c.k == 1 ? 0 : c.past();
    f.elu = elu;
    f.carry_in = s->carry[s->par][size_t(ci)];
    f.carry_out = s->carry[s->par ^ 1][size_t(ci)];
    launch_mimi_fconv(f, n, st);
    s->launches++;
    return;
  }
  if (c.k == 1 && c.stride == 1) {
    if (elu && !c.w.q8) {
      launch_mimi_elu(x, s->se, n, T * cin, st);
      s->launches++;
      x = s->se;
      elu = false;
    }
    mimi_product(s, c.w, MIn{x, cin, T, cin, elu ? T * cin : 0}, T, c.b, y, resid);
    return;
  }
  const int P = c.past();
  float* cin_ = s->carry[s->par][size_t(ci)];
  float* cout_ = s->carry[s->par ^ 1][size_t(ci)];
  if (staged(c)) {
    launch_mimi_stage(x, cin_, cout_, s->stage, n, T, cin, P, elu, st);
    s->launches++;
    mimi_product(s, c.w, MIn{s->stage, cin, P + T, c.k * cin, 0}, T, c.b, y, resid);
    return;
  }
  if (elu) {
    launch_mimi_elu(x, s->se, n, T * cin, st);
    s->launches++;
    x = s->se;
  }
  launch_mimi_im2col(x, cin_, cout_, s->col, n, T, cin, c.k, c.stride, c.dil, P, st);
  s->launches++;
  const int To = T / c.stride;
  mimi_product(s, c.w, MIn{s->col, c.k * cin, To, c.k * cin, 0}, To, c.b, y, resid);
}

// transformer.forward (nn.go:142-182) with the window and layer scales for
// the S rows of every stream in s->x.
void mimi_transformer(grx_mimi_streams* s, int S) {
  grx_mimi* m = s->m;
  const int n = s->n, R = n * S, d = m->d, L = int(s->layers->size());
  cudaStream_t st = s->st;
  launch_mimi_rows(s->pos, S, R, s->rowpos, st);
  s->launches++;
  for (int l = 0; l < L; l++) {
    const MLayer& ly = (*s->layers)[size_t(l)];
    LnArgs ln;
    ln.x = s->x;
    ln.w = ly.n1w;
    ln.b = ly.n1b;
    ln.eps = 1e-5;
    ln.mode = LN_Q8;
    ln.q8 = s->xq;
    ln.q8s = s->xs;
    launch_ln(ln, R, d, st);
    EpiArgs e;
    e.epi = EPI_ROPE_KV;
    e.kv.q = s->qb;
    e.kv.kv = s->kv;
    e.kv.pos = s->rowpos;
    e.kv.row_stream = s->rowslot;
    e.kv.rope = s->rope;
    e.kv.layer = l;
    e.kv.layers = L;
    e.kv.heads = m->heads;
    e.kv.cap = s->ring;
    e.kv.d = d;
    e.kv.ring = s->ring;
    launch_q8_product(s->xq, s->xs, R, ly.qkv, e, st);
    AttnRowsArgs at;
    at.q = s->qb;
    at.kv = s->kv;
    at.row0 = s->crow0;
    at.T = s->cT;
    at.pos0 = s->pos;
    at.slot = s->cslot;
    at.q8 = s->xq;
    at.q8s = s->xs;
    at.layer = l;
    at.layers = L;
    at.heads = m->heads;
    at.cap = s->ring;
    at.d = d;
    at.context = m->context;
    at.ring = s->ring;
    launch_attn_rows(at, n, S, st);
    EpiArgs r;
    r.epi = EPI_RESID;
    r.y = s->x;
    r.ldy = d;
    r.ls = ly.ls1;
    launch_q8_product(s->xq, s->xs, R, ly.out, r, st);
    ln.w = ly.n2w;
    ln.b = ly.n2b;
    launch_ln(ln, R, d, st);
    EpiArgs g;
    g.epi = EPI_GELU_Q8;
    g.q8 = s->fq;
    g.q8s = s->fs;
    launch_q8_product(s->xq, s->xs, R, ly.ff1, g, st);
    r.ls = ly.ls2;
    launch_q8_product(s->fq, s->fs, R, ly.ff2, r, st);
    s->launches += 7;
  }
  launch_mimi_advance(s->pos, S, n, st);
  s->launches++;
}

// One latent per stream (d_lat [n][ldim]) → one frame per stream
// (d_pcm [n][frame]), queued on the set's stream.
void mimi_enqueue(grx_mimi_streams* s, const float* d_lat, float* d_pcm) {
  grx_mimi* m = s->m;
  const int n = s->n, C = m->d, S = m->S;
  cudaStream_t st = s->st;
  mimi_product(s, m->quant, MIn{d_lat, m->ldim, 1, m->ldim, 0}, 1, nullptr, s->z, false);
  launch_mimi_up(s->z, m->up, s->up_part[s->par], s->x, s->up_part[s->par ^ 1], n, S, C, st);
  s->launches++;
  mimi_transformer(s, S);
  float* x = s->x;
  int T = S, Cc = C;
  size_t ci = 0;
  auto other = [&](const float* p) { return p == s->sa ? s->sb : s->sa; };
  for (const MStep& stp : m->steps) {
    if (stp.kind == 0) {
      float* y = &stp == &m->steps.back() && stp.c.cout == 1 && stp.c.stride == 1 ? d_pcm : other(x);
      mimi_conv(s, stp.c, int(ci++), x, T, stp.elu, y, false);
      T /= stp.c.stride;
      Cc = stp.c.cout;
      x = y;
    } else if (stp.kind == 1) {
      const MConv& c = stp.c;
      const float* in = x;
      int elu_len = 0;
      if (stp.elu && c.w.q8) {
        elu_len = T * Cc;
      } else if (stp.elu) {
        launch_mimi_elu(x, s->se, n, T * Cc, st);
        s->launches++;
        in = s->se;
      }
      mimi_product(s, c.w, MIn{in, Cc, T, Cc, elu_len}, T, nullptr, s->zt, false);
      float* y = other(x);
      launch_mimi_convtr(s->zt, c.b, s->carry[s->par][ci], y, s->carry[s->par ^ 1][ci], n, T, c.cout, c.k, c.stride,
                         st);
      s->launches++;
      ci++;
      T *= c.stride;
      Cc = c.cout;
      x = y;
    } else {
      // x + conv1x1(ELU(conv(ELU(x)))), the sum added into x in place
      mimi_conv(s, stp.ra, int(ci), x, T, true, s->sh, false);
      mimi_conv(s, stp.rb, int(ci + 1), s->sh, T, true, x, true);
      ci += 2;
    }
  }
  if (x != d_pcm)  // a decoder that does not end in the one-channel conv
    cudaMemcpyAsync(d_pcm, x, sizeof(float) * size_t(n) * T * Cc, cudaMemcpyDeviceToDevice, st);
  launch_mimi_fade(d_pcm, s->started, n, m->frame, m->sample_rate / 200, st);
  s->launches++;
  s->par ^= 1;
}

// One decode call of every stream (latents d_lat in, samples d_pcm out):
// the captured graph of the call's parity when there is one (the latents
// and samples pass through the set's own buffers), else the launches.
void mimi_decode_frame(grx_mimi_streams* s, const float* d_lat, float* d_pcm) {
  grx_mimi* m = s->m;
  cudaStream_t st = s->st;
  if (!s->graph_tried) {
    s->graph_tried = true;
    const int par0 = s->par;
    const int64_t l0 = s->launches;
    bool ok = true;
    for (int p = 0; p < 2 && ok; p++) {
      s->par = p;
      cudaGraph_t g = nullptr;
      ok = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
      if (ok) mimi_enqueue(s, s->lat, s->pcm);
      ok = cudaStreamEndCapture(st, &g) == cudaSuccess && ok && g;
      if (ok) ok = cudaGraphInstantiate(&s->graph[p], g, 0) == cudaSuccess;
      if (g) cudaGraphDestroy(g);
    }
    s->graph_launches = (s->launches - l0) / 2;
    s->launches = l0;
    s->par = par0;
    if (!ok) {
      cudaGetLastError();
      for (cudaGraphExec_t& g : s->graph)
        if (g) cudaGraphExecDestroy(g), g = nullptr;
    }
  }
  if (!s->graph[0] || !s->graph[1]) {
    mimi_enqueue(s, d_lat, d_pcm);
    return;
  }
  if (d_lat != s->lat)
    cudaMemcpyAsync(s->lat, d_lat, sizeof(float) * size_t(s->n) * m->ldim, cudaMemcpyDeviceToDevice, st);
  cudaGraphLaunch(s->graph[s->par], st);
  s->par ^= 1;
  s->launches += s->graph_launches;
  if (d_pcm != s->pcm)
    cudaMemcpyAsync(d_pcm, s->pcm, sizeof(float) * size_t(s->n) * m->frame, cudaMemcpyDeviceToDevice, st);
}

int mimi_reset(grx_mimi_streams* s) {
  grx_mimi* m = s->m;
  const int n = s->n;
  CK(cudaSetDevice(s->ar.dev));
  CK(cudaMemsetAsync(s->pos, 0, sizeof(int) * size_t(n), s->st));
  CK(cudaMemsetAsync(s->started, 0, sizeof(int) * size_t(n), s->st));
  for (int b = 0; b < 2; b++) {
    if (s->up_part[b]) CK(cudaMemsetAsync(s->up_part[b], 0, sizeof(float) * size_t(n) * m->S * m->d, s->st));
    for (size_t i = 0; i < s->carry_n.size(); i++)
      if (s->carry_n[i]) CK(cudaMemsetAsync(s->carry[b][i], 0, sizeof(float) * size_t(n) * s->carry_n[i], s->st));
  }
  CK(cudaStreamSynchronize(s->st));
  s->frames = 0;
  s->par = 0;
  return GRX_OK;
}

// What every set holds, for s->layers, s->steps and s->S rows per
// transformer call: the transformer's caches (rings of s->ring positions)
// and activations, the step buffers sized by z, the carried rows of every
// step (and of `extra`, a last convolution), the row tables for S rows and
// the RoPE table of `positions` positions.
int set_init(grx_mimi_streams* s, const MimiSizes& z, size_t positions, const MConv* extra) {
  grx_mimi* m = s->m;
  const int S = s->S, d = m->d, L = int(s->layers->size()), H = m->heads, hd = 64;
  const size_t N = size_t(s->n), R = N * S;
  int rc = 0;
  s->kv = s->ar.alloc<float>(N * L * 2 * H * s->ring * hd, &rc);
  s->pos = s->ar.alloc<int>(N, &rc);
  s->started = s->ar.alloc<int>(N, &rc);
  s->rowpos = s->ar.alloc<int>(R, &rc);
  int* stat = s->ar.alloc<int>(R + 3 * N, &rc);
  s->x = s->ar.alloc<float>(R * d, &rc);
  s->qb = s->ar.alloc<float>(R * d, &rc);
  s->xq = s->ar.alloc<int8_t>(R * d, &rc);
  s->xs = s->ar.alloc<float2>(R * d / 32, &rc);
  s->fq = s->ar.alloc<int8_t>(R * m->ff, &rc);
  s->fs = s->ar.alloc<float2>(R * m->ff / 32, &rc);
  s->aq = s->ar.alloc<int8_t>(N * z.qk, &rc);
  s->as = s->ar.alloc<float2>(N * z.qk / 32 + 1, &rc);
  s->sa = s->ar.alloc<float>(N * z.act, &rc);
  s->sb = s->ar.alloc<float>(N * z.act, &rc);
  s->se = s->ar.alloc<float>(N * z.act, &rc);
  s->stage = s->ar.alloc<float>(N * z.stage, &rc);
  s->col = s->ar.alloc<float>(N * z.col, &rc);
  s->zt = s->ar.alloc<float>(N * z.zt, &rc);
  s->sh = s->ar.alloc<float>(N * z.h, &rc);
  for (const MStep& st : *s->steps) {
    if (st.kind == 0) s->carry_n.push_back(size_t(st.c.past()) * st.c.cin);
    if (st.kind == 1) s->carry_n.push_back(size_t(st.c.k - st.c.stride) * st.c.cout);
    if (st.kind == 2) {
      s->carry_n.push_back(size_t(st.ra.past()) * st.ra.cin);
      s->carry_n.push_back(size_t(st.rb.past()) * st.rb.cin);
    }
  }
  if (extra) s->carry_n.push_back(size_t(extra->past()) * extra->cin);
  for (int b = 0; b < 2; b++)
    for (size_t c : s->carry_n) s->carry[b].push_back(s->ar.alloc<float>(N * std::max<size_t>(c, 1), &rc));
  if (rc) return rc;
  // static row tables: row r is stream r / S; call-stream i is rows i·S ..
  {
    std::vector<int> h(R + 3 * N);
    for (size_t r = 0; r < R; r++) h[r] = int(r / S);
    for (size_t i = 0; i < N; i++) {
      h[R + i] = int(i) * S;
      h[R + N + i] = S;
      h[R + 2 * N + i] = int(i);
    }
    CK(cudaMemcpy(stat, h.data(), sizeof(int) * h.size(), cudaMemcpyHostToDevice));
    s->rowslot = stat;
    s->crow0 = stat + R;
    s->cT = stat + R + N;
    s->cslot = stat + R + 2 * N;
    s->rows_for = S;
  }
  // RoPE cos/sin for every position the streams can reach (nn.go:84-85)
  {
    std::vector<float> t(positions * hd);
    for (size_t p = 0; p < positions; p++)
      for (int i = 0; i < hd / 2; i++) {
        double a = double(m->freqs[size_t(i)] * float(p));
        t[(p * (hd / 2) + i) * 2] = float(std::cos(a));
        t[(p * (hd / 2) + i) * 2 + 1] = float(std::sin(a));
      }
    s->rope = s->ar.upload(t.data(), t.size(), &rc);
  }
  return rc;
}

int check_frames(grx_mimi_streams* s, int frames) {
  if (frames < 0) return fail(GRX_EINVAL, "grx_mimi: a negative frame count");
  if (s->frames + frames > s->max_frames)
    return fail(GRX_ERANGE, "grx_mimi: the streams hold " + std::to_string(s->frames) + " frames; " +
                                std::to_string(frames) + " more pass the " + std::to_string(s->max_frames) +
                                " they were made for");
  return GRX_OK;
}

// encode (mimi.go:164-179) as cloneCond runs it (voice.go:113-124), for
// every clip of the set: the clips (d_pcm [n][samples]) padded with zeros
// to whole frames, then twelve frames at a time through the SEANet
// encoder, the transformer and the downsampling convolution with one state
// per clip; d_lat [n][frames][ldim]. Queued on the set's stream.
int enc_run(grx_mimi_streams* s, int samples, const float* d_pcm, float* d_lat) {
  grx_mimi* m = s->m;
  const int n = s->n, frame = m->frame, d = m->d, ldim = m->ldim, S = m->S, piece = 12 * frame;
  const int frames = (samples + frame - 1) / frame, padded = frames * frame;
  cudaStream_t st = s->st;
  int rc = mimi_reset(s);
  if (rc) return rc;
  CK(cudaMemsetAsync(s->clip, 0, sizeof(float) * size_t(n) * padded, st));
  CK(cudaMemcpy2DAsync(s->clip, sizeof(float) * padded, d_pcm, sizeof(float) * samples, sizeof(float) * samples, n,
                       cudaMemcpyDeviceToDevice, st));
  const size_t down_ci = s->carry_n.size() - 1;
  auto other = [&](const float* p) { return p == s->sa ? s->sb : s->sa; };
  // a piece from its samples in sa to its latents in piece_lat: SEANet's
  // encoder, the transformer on its T rows, the downsampling
  auto piece_kernels = [&](int T0, bool first) {
    float* x = s->sa;
    int T = T0;
    size_t ci = 0;
    for (const MStep& stp : m->enc_steps) {
      if (stp.kind == 0) {
        float* y = other(x);
        mimi_conv(s, stp.c, int(ci++), x, T, stp.elu, y, false);
        T /= stp.c.stride;
        x = y;
      } else {
        // x + conv1x1(ELU(conv(ELU(x)))), the sum added into x in place
        mimi_conv(s, stp.ra, int(ci), x, T, true, s->sh, false);
        mimi_conv(s, stp.rb, int(ci + 1), s->sh, T, true, x, true);
        ci += 2;
      }
    }
    cudaMemcpyAsync(s->x, x, sizeof(float) * size_t(n) * T * d, cudaMemcpyDeviceToDevice, st);
    mimi_transformer(s, T);
    if (first) {  // the first call's padding: copies of the first row
      launch_mimi_replicate(s->x, T, d, s->carry[s->par][down_ci], m->down.past(), n, st);
      s->launches++;
    }
    mimi_conv(s, m->down, int(down_ci), s->x, T, false, s->piece_lat, false);
  };
  for (int p0 = 0; p0 < padded; p0 += piece) {
    const int T0 = std::min(piece, padded - p0);
    const bool first = p0 == 0;
    CK(cudaMemcpy2DAsync(s->sa, sizeof(float) * T0, s->clip + p0, sizeof(float) * padded, sizeof(float) * T0, n,
                         cudaMemcpyDeviceToDevice, st));
    int T = T0;  // the transformer's rows: the encoder's strides applied
    for (const MStep& stp : m->enc_steps)
      if (stp.kind == 0) T /= stp.c.stride;
    if (T != s->rows_for) {
      launch_mimi_rowtab(T, n, s->rowslot, s->crow0, s->cT, s->cslot, st);
      s->launches++;
      s->rows_for = T;
    }
    // the piece's kernels from a graph captured the first time its shape
    // comes (same launches, same bits)
    grx_mimi_streams::PieceGraph* pg = nullptr;
    for (auto& e : s->piece_graphs)
      if (e.T0 == T0 && e.par == s->par && e.first == first) pg = &e;
    if (!pg) {
      grx_mimi_streams::PieceGraph e{T0, s->par, first, nullptr, 0};
      const int64_t l0 = s->launches;
      cudaGraph_t g = nullptr;
      bool ok = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
      if (ok) piece_kernels(T0, first);
      ok = cudaStreamEndCapture(st, &g) == cudaSuccess && ok && g;
      if (ok) ok = cudaGraphInstantiate(&e.exec, g, 0) == cudaSuccess;
      if (g) cudaGraphDestroy(g);
      if (!ok) {
        cudaGetLastError();
        e.exec = nullptr;
      }
      e.launches = s->launches - l0;
      s->launches = l0;
      s->piece_graphs.push_back(e);
      pg = &s->piece_graphs.back();
    }
    if (pg->exec) {
      CK(cudaGraphLaunch(pg->exec, st));
      s->launches += pg->launches;
    } else {
      piece_kernels(T0, first);
    }
    const int fr = T / S;
    CK(cudaMemcpy2DAsync(d_lat + size_t(p0 / frame) * ldim, sizeof(float) * frames * ldim, s->piece_lat,
                         sizeof(float) * fr * ldim, sizeof(float) * fr * ldim, n, cudaMemcpyDeviceToDevice, st));
    s->par ^= 1;
  }
  return GRX_OK;
}

}  // namespace

extern "C" {

int grx_mimi_load(const void* bytes, size_t len, int device, grx_mimi** out) {
  if (!bytes || !out) return fail(GRX_EINVAL, "grx_mimi_load: null argument");
  int rc = device_init(device);
  if (rc) return rc;
  GGUF f;
  if (!f.parse(bytes, len)) return fail(GRX_EFORMAT, f.err);
  if (f.get_string("general.architecture", "") != "pockettts")
    return fail(GRX_EFORMAT, "pockettts: the file isn't a Pocket TTS model");
  auto m = std::make_unique<grx_mimi>();
  m->ar.dev = device;
  m->dev = device;
  std::string err;
  auto num = [&](const char* key) -> int {  // loader.num, model.go:93-100
    int64_t v = f.get_int(key, -1);
    if (v < 1 || v > (1 << 16)) {
      if (err.empty()) err = std::string("pockettts: the setting ") + key + " is " + std::to_string(v);
      return 1;
    }
    return int(v);
  };
  auto vec = [&](const std::string& name, int64_t n) -> float* {  // loader.vec
    if (!err.empty()) return nullptr;
    std::vector<float> v;
    auto it = f.tensors.find(name);
    if (it == f.tensors.end() || it->second.elems() != n || !f.float32(name, v)) {
      err = "pockettts: no " + std::to_string(n) + "-value " + name;
      return nullptr;
    }
    return m->ar.upload(v.data(), v.size(), &rc);
  };
  auto mat = [&](const std::string& name, int64_t rows, int64_t cols) -> MW {  // loader.mat, then pack()
    MW w;
    if (!err.empty()) return w;
    int64_t r, c;
    if (!f.matrix_shape(name, &r, &c)) {
      err = "pockettts: no tensor " + name;
      return w;
    }
    if (r != rows || c != cols) {
      err = "pockettts: " + name + " is " + std::to_string(r) + "x" + std::to_string(c) + ", want " +
            std::to_string(rows) + "x" + std::to_string(cols);
      return w;
    }
    const GTensor& t = f.tensors.at(name);
    w.rows = int(rows);
    w.cols = int(cols);
    if (t.type == G_Q8_0) {
      if (rows % 32 || cols > kQ8GemvMaxK)
        err = "pockettts: " + name + " is a Q8_0 matrix outside what the kernels take (rows % 32, cols <= " +
              std::to_string(kQ8GemvMaxK) + ")";
      w.q8 = true;
      w.q = upload_q8(m->ar, t.data, w.rows, w.cols, &rc);
    } else if (t.type == G_F32) {
      if (cols % 4 && cols >= 16)
        err = "pockettts: " + name + " is a float32 matrix outside what the kernels take (cols % 4)";
      std::vector<float> v;
      f.float32(name, v);
      w.f = m->ar.upload(v.data(), v.size(), &rc);
    } else {
      err = "pockettts: " + name + " is neither Q8_0 nor float32 (the decoder's weights here are one or the other)";
    }
    return w;
  };
  // model.go:220-227, 280-305
  const int sr = num("pockettts.sample_rate");
  const double fr = f.get_float("pockettts.frame_rate", 0);
  m->sample_rate = sr;
  const int frame = fr > 0 ? int(double(sr) / fr) : 0;
  m->ldim = num("pockettts.latent_dim");
  m->d = num("pockettts.mimi.d_model");
  m->heads = num("pockettts.mimi.heads");
  m->ff = num("pockettts.mimi.ff");
  m->context = num("pockettts.mimi.context");
  const double period = f.get_float("pockettts.mimi.max_period", 1e4);
  m->S = num("pockettts.mimi.upsample");
  std::vector<int> ratios;
  {
    auto it = f.kv.find("pockettts.seanet.ratios");
    if (it != f.kv.end() && it->second.kind == GValue::ARR)
      for (const GValue& v : it->second.a) ratios.push_back(v.kind == GValue::INT ? int(v.i) : 0);
  }
  const int nf = num("pockettts.seanet.n_filters"), dim = num("pockettts.seanet.dimension");
  const int k = num("pockettts.seanet.kernel_size"), resk = num("pockettts.seanet.residual_kernel_size");
  const int lastk = num("pockettts.seanet.last_kernel_size"), dil = num("pockettts.seanet.dilation_base");
  const int comp = num("pockettts.seanet.compress"), nres = num("pockettts.seanet.n_residual_layers");
  int hop = 1;
  for (int r : ratios) {
    if (err.empty() && (r < 1 || r > 64)) err = "pockettts: a SEANet ratio of " + std::to_string(r);
    hop *= std::max(1, std::min(64, r));
  }
  if (err.empty() && (ratios.empty() || dim != m->d || hop * m->S != frame))
    err = "pockettts: SEANet's ratios don't make " + std::to_string(frame) + "-sample frames";
  if (!err.empty()) return fail(GRX_EFORMAT, err);
  m->frame = frame;
  const int d = m->d, ff = m->ff;
  if (d % m->heads || d / m->heads != 64)
    return fail(GRX_EINVAL, "pockettts: Mimi heads of " + std::to_string(d / m->heads) + " values (this build runs 64)");
  if (d % 128 || ff % 128 || d > 4096 || ff > 4096)
    return fail(GRX_EINVAL, "pockettts: Mimi dimensions outside what the kernels take");
  m->freqs = rope_freqs(64, period);
  m->quant = mat("mimi.quant", d, m->ldim);
  m->up = vec("mimi.up", int64_t(d) * 2 * m->S);
  // loader.transformer("mimi.dec_tf", ..., scale=true), model.go:102-128
  for (int i = 0;; i++) {
    const std::string p = "mimi.dec_tf." + std::to_string(i) + ".";
    if (!f.has(p + "norm1.weight")) break;
    MLayer ly;
    ly.n1w = vec(p + "norm1.weight", d);
    ly.n1b = vec(p + "norm1.bias", d);
    ly.n2w = vec(p + "norm2.weight", d);
    ly.n2b = vec(p + "norm2.bias", d);
    MW qkv = mat(p + "attn_qkv.weight", 3 * d, d), o = mat(p + "attn_out.weight", d, d);
    MW f1 = mat(p + "ff1.weight", ff, d), f2 = mat(p + "ff2.weight", d, ff);
    ly.ls1 = vec(p + "ls1", d);
    ly.ls2 = vec(p + "ls2", d);
    if (err.empty() && !(qkv.q8 && o.q8 && f1.q8 && f2.q8))
      err = "pockettts: " + p + "* are not all Q8_0 (this build runs the transformer's products on the int8 path)";
    ly.qkv = qkv.q;
    ly.out = o.q;
    ly.ff1 = f1.q;
    ly.ff2 = f2.q;
    m->layers.push_back(ly);
  }
  if (err.empty() && m->layers.empty()) err = "pockettts: no mimi.dec_tf layers";
  // loader.decoder, model.go:160-178
  auto conv = [&](const std::string& name, int cin, int cout, int kk, int stride, int dl) {
    MConv c;
    c.w = mat(name + ".weight", cout, int64_t(kk) * cin);
    c.b = vec(name + ".bias", cout);
    c.cin = cin, c.cout = cout, c.k = kk, c.stride = stride, c.dil = dl;
    return c;
  };
  int mult = 1 << ratios.size();
  {
    MStep first;
    first.c = conv("mimi.dec.0", d, mult * nf, k, 1, 1);
    m->steps.push_back(first);
  }
  int idx = 1;
  for (int r : ratios) {
    idx++;
    MStep t;
    t.kind = 1;
    t.elu = true;
    const std::string nm = "mimi.dec." + std::to_string(idx);
    t.c.w = mat(nm + ".weight", int64_t(2 * r) * (mult * nf / 2), mult * nf);
    t.c.b = vec(nm + ".bias", mult * nf / 2);
    t.c.cin = mult * nf, t.c.cout = mult * nf / 2, t.c.k = 2 * r, t.c.stride = r;
    m->steps.push_back(t);
    idx++;
    const int rdim = mult * nf / 2;
    for (int j = 0, dl = 1; j < nres; j++, dl *= dil) {
      const std::string p = "mimi.dec." + std::to_string(idx) + ".";
      MStep rb;
      rb.kind = 2;
      rb.ra = conv(p + "1", rdim, rdim / comp, resk, 1, dl);
      rb.rb = conv(p + "3", rdim / comp, rdim, 1, 1, 1);
      m->steps.push_back(rb);
      idx++;
    }
    mult /= 2;
  }
  idx++;
  {
    MStep last;
    last.elu = true;
    last.c = conv("mimi.dec." + std::to_string(idx), nf, 1, lastk, 1, 1);
    m->steps.push_back(last);
  }
  // the encoder (loader.encoder and the mimi.enc_tf transformer, model.go:
  // 181-200; mimi.down, 308-313), when the file has one
  if (f.has("mimi.enc.0.weight")) {
    m->has_enc = true;
    m->hop = hop;
    for (int i = 0;; i++) {
      const std::string p = "mimi.enc_tf." + std::to_string(i) + ".";
      if (!f.has(p + "norm1.weight")) break;
      MLayer ly;
      ly.n1w = vec(p + "norm1.weight", d);
      ly.n1b = vec(p + "norm1.bias", d);
      ly.n2w = vec(p + "norm2.weight", d);
      ly.n2b = vec(p + "norm2.bias", d);
      MW qkv = mat(p + "attn_qkv.weight", 3 * d, d), o = mat(p + "attn_out.weight", d, d);
      MW f1 = mat(p + "ff1.weight", ff, d), f2 = mat(p + "ff2.weight", d, ff);
      ly.ls1 = vec(p + "ls1", d);
      ly.ls2 = vec(p + "ls2", d);
      if (err.empty() && !(qkv.q8 && o.q8 && f1.q8 && f2.q8))
        err = "pockettts: " + p + "* are not all Q8_0 (this build runs the transformer's products on the int8 path)";
      ly.qkv = qkv.q;
      ly.out = o.q;
      ly.ff1 = f1.q;
      ly.ff2 = f2.q;
      m->enc_layers.push_back(ly);
    }
    if (err.empty() && m->enc_layers.empty()) err = "pockettts: no mimi.enc_tf layers";
    MStep first;
    first.c = conv("mimi.enc.0", 1, nf, k, 1, 1);
    m->enc_steps.push_back(first);
    int eidx = 1, emult = 1;
    for (int ri = int(ratios.size()) - 1; ri >= 0; ri--) {
      const int r = ratios[size_t(ri)], rdim = emult * nf;
      for (int j = 0, dl = 1; j < nres; j++, dl *= dil) {
        const std::string p = "mimi.enc." + std::to_string(eidx) + ".";
        MStep rb;
        rb.kind = 2;
        rb.ra = conv(p + "1", rdim, rdim / comp, resk, 1, dl);
        rb.rb = conv(p + "3", rdim / comp, rdim, 1, 1, 1);
        m->enc_steps.push_back(rb);
        eidx++;
      }
      eidx++;  // the ELU
      MStep cv;
      cv.elu = true;
      cv.c = conv("mimi.enc." + std::to_string(eidx), rdim, 2 * rdim, 2 * r, r, 1);
      m->enc_steps.push_back(cv);
      eidx++;
      emult *= 2;
    }
    eidx++;
    MStep elast;
    elast.elu = true;
    elast.c = conv("mimi.enc." + std::to_string(eidx), emult * nf, d, lastk, 1, 1);
    m->enc_steps.push_back(elast);
    m->down.w = mat("mimi.down", m->ldim, int64_t(2) * m->S * d);
    const std::vector<float> zeros(size_t(m->ldim), 0.f);  // no bias: gemvRows still adds one of zeros
    m->down.b = m->ar.upload(zeros.data(), zeros.size(), &rc);
    m->down.cin = d, m->down.cout = m->ldim, m->down.k = 2 * m->S, m->down.stride = m->S, m->down.dil = 1;
  }
  if (!err.empty()) return fail(GRX_EFORMAT, err);
  if (rc) return rc;
  *out = m.release();
  return GRX_OK;
}

void grx_mimi_free(grx_mimi* m) { delete m; }

int grx_mimi_dims(const grx_mimi* m, int* d, int* heads, int* layers, int* context, int* upsample, int* ldim,
                  int* frame, int* sample_rate) {
  if (!m) return fail(GRX_EINVAL, "null model");
  if (d) *d = m->d;
  if (heads) *heads = m->heads;
  if (layers) *layers = int(m->layers.size());
  if (context) *context = m->context;
  if (upsample) *upsample = m->S;
  if (ldim) *ldim = m->ldim;
  if (frame) *frame = m->frame;
  if (sample_rate) *sample_rate = m->sample_rate;
  return GRX_OK;
}

int grx_mimi_streams_create(grx_mimi* m, int n, int max_frames, grx_mimi_streams** out) {
  if (!m || !out || n < 1 || n > 65535 || max_frames < 1) return fail(GRX_EINVAL, "grx_mimi_streams_create: bad argument");
  const int S = m->S, d = m->d;
  if (int64_t(max_frames) * S > (int64_t(1) << 30)) return fail(GRX_ERANGE, "grx_mimi_streams_create: too many frames");
  int rc = device_init(m->dev);
  if (rc) return rc;
  CK(cudaSetDevice(m->dev));
  auto s = std::make_unique<grx_mimi_streams>();
  s->ar.dev = m->dev;
  s->m = m;
  s->layers = &m->layers;
  s->steps = &m->steps;
  s->S = S;
  s->n = n;
  s->max_frames = max_frames;
  s->ring = std::min(m->context + S - 1, max_frames * S);
  CK(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
  const size_t N = size_t(n);
  rc = set_init(s.get(), mimi_sizes(m), size_t(max_frames) * S, nullptr);
  s->lat = s->ar.alloc<float>(N * m->ldim, &rc);
  s->z = s->ar.alloc<float>(N * d, &rc);
  s->pcm = s->ar.alloc<float>(N * m->frame, &rc);
  for (int b = 0; b < 2; b++) s->up_part[b] = s->ar.alloc<float>(N * S * d, &rc);
  if (rc) return rc;
  rc = mimi_reset(s.get());
  if (rc) return rc;
  *out = s.release();
  return GRX_OK;
}

void grx_mimi_streams_free(grx_mimi_streams* s) { delete s; }

int grx_mimi_encoder_create(grx_mimi* m, int n, int max_samples, grx_mimi_streams** out) {
  if (!m || !out || n < 1 || n > 65535 || max_samples < 1)
    return fail(GRX_EINVAL, "grx_mimi_encoder_create: bad argument");
  if (!m->has_enc) return fail(GRX_EINVAL, "pockettts: this model file has no voice cloning");
  const int frame = m->frame, S = m->S;
  const int64_t frames = (int64_t(max_samples) + frame - 1) / frame;
  if (frames * frame * int64_t(n) > (int64_t(1) << 31)) return fail(GRX_ERANGE, "grx_mimi_encoder_create: too many samples");
  int rc = device_init(m->dev);
  if (rc) return rc;
  CK(cudaSetDevice(m->dev));
  auto s = std::make_unique<grx_mimi_streams>();
  s->ar.dev = m->dev;
  s->m = m;
  s->layers = &m->enc_layers;
  s->steps = &m->enc_steps;
  const int T0 = int(std::min<int64_t>(12 * frame, frames * frame));
  s->S = T0 / m->hop;  // transformer rows of the longest piece
  s->n = n;
  s->max_samples = max_samples;
  s->max_frames = int(frames);
  s->ring = int(std::min<int64_t>(m->context + s->S - 1, frames * S));
  CK(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
  rc = set_init(s.get(), enc_sizes(m, T0), size_t(frames) * S, &m->down);
  s->clip = s->ar.alloc<float>(size_t(n) * frames * frame, &rc);
  s->piece_lat = s->ar.alloc<float>(size_t(n) * 12 * m->ldim, &rc);
  if (rc) return rc;
  rc = mimi_reset(s.get());
  if (rc) return rc;
  *out = s.release();
  return GRX_OK;
}

int grx_mimi_encode_device(grx_mimi_streams* s, int samples, const float* d_pcm, float* d_latents) {
  if (!s || !d_pcm || !d_latents) return fail(GRX_EINVAL, "grx_mimi_encode_device: null argument");
  if (!s->clip) return fail(GRX_EINVAL, "grx_mimi_encode_device: not an encoder set");
  if (samples < 1 || samples > s->max_samples)
    return fail(GRX_ERANGE, "grx_mimi_encode: " + std::to_string(samples) + " samples for a set made for 1.." +
                                std::to_string(s->max_samples));
  CK(cudaSetDevice(s->ar.dev));
  int rc = enc_run(s, samples, d_pcm, d_latents);
  if (rc) return rc;
  CK(cudaGetLastError());
  return GRX_OK;
}

int grx_mimi_encode(grx_mimi_streams* s, int samples, const float* pcm, float* latents) {
  if (!s || !pcm || !latents) return fail(GRX_EINVAL, "grx_mimi_encode: null argument");
  if (!s->clip) return fail(GRX_EINVAL, "grx_mimi_encode: not an encoder set");
  if (samples < 1 || samples > s->max_samples)
    return fail(GRX_ERANGE, "grx_mimi_encode: " + std::to_string(samples) + " samples for a set made for 1.." +
                                std::to_string(s->max_samples));
  grx_mimi* m = s->m;
  const int frames = (samples + m->frame - 1) / m->frame;
  CK(cudaSetDevice(s->ar.dev));
  Arena tmp;
  tmp.dev = s->ar.dev;
  int rc = 0;
  float* d_pcm = tmp.alloc<float>(size_t(s->n) * samples, &rc);
  float* d_lat = tmp.alloc<float>(size_t(s->n) * frames * m->ldim, &rc);
  if (rc) return rc;
  CK(cudaMemcpyAsync(d_pcm, pcm, sizeof(float) * size_t(s->n) * samples, cudaMemcpyHostToDevice, s->st));
  rc = enc_run(s, samples, d_pcm, d_lat);
  if (rc) return rc;
  CK(cudaMemcpyAsync(latents, d_lat, sizeof(float) * size_t(s->n) * frames * m->ldim, cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));
  CK(cudaGetLastError());
  return GRX_OK;
}

int grx_mimi_clone_latents(grx_mimi* m, const float* pcm, int samples, float* latents, int* frames) {
  if (!m || !pcm || !latents || samples < 1) return fail(GRX_EINVAL, "grx_mimi_clone_latents: bad argument");
  grx_mimi_streams* s = nullptr;
  int rc = grx_mimi_encoder_create(m, 1, samples, &s);
  if (rc) return rc;
  rc = grx_mimi_encode(s, samples, pcm, latents);
  grx_mimi_streams_free(s);
  if (rc) return rc;
  if (frames) *frames = (samples + m->frame - 1) / m->frame;
  return GRX_OK;
}

int grx_voice_clone(grx_flowlm* lm, grx_mimi* m, const float* pcm, int samples, grx_voice** out) {
  if (!lm || !m || !pcm || !out || samples < 1) return fail(GRX_EINVAL, "grx_voice_clone: bad argument");
  const int frames = (samples + m->frame - 1) / m->frame;
  std::vector<float> lat(size_t(frames) * m->ldim);
  int rc = grx_mimi_clone_latents(m, pcm, samples, lat.data(), nullptr);
  if (rc) return rc;
  return grx_voice_from_latents(lm, lat.data(), frames, out);
}


int grx_mimi_streams_reset(grx_mimi_streams* s) {
  if (!s) return fail(GRX_EINVAL, "null stream set");
  return mimi_reset(s);
}

int grx_mimi_decode(grx_mimi_streams* s, const float* latents, float* pcm) {
  if (!s || !latents) return fail(GRX_EINVAL, "grx_mimi_decode: null argument");
  int rc = check_frames(s, 1);
  if (rc) return rc;
  grx_mimi* m = s->m;
  CK(cudaSetDevice(s->ar.dev));
  CK(cudaMemcpyAsync(s->lat, latents, sizeof(float) * size_t(s->n) * m->ldim, cudaMemcpyHostToDevice, s->st));
  mimi_decode_frame(s, s->lat, s->pcm);
  s->frames++;
  if (pcm)
    CK(cudaMemcpyAsync(pcm, s->pcm, sizeof(float) * size_t(s->n) * m->frame, cudaMemcpyDeviceToHost, s->st));
  CK(cudaStreamSynchronize(s->st));
  CK(cudaGetLastError());
  return GRX_OK;
}

int grx_mimi_decode_device(grx_mimi_streams* s, int frames, const float* d_latents, float* d_pcm) {
  if (!s || !d_latents || !d_pcm) return fail(GRX_EINVAL, "grx_mimi_decode_device: null argument");
  int rc = check_frames(s, frames);
  if (rc) return rc;
  grx_mimi* m = s->m;
  CK(cudaSetDevice(s->ar.dev));
  for (int f = 0; f < frames; f++) {
    mimi_decode_frame(s, d_latents + size_t(f) * s->n * m->ldim, d_pcm + size_t(f) * s->n * m->frame);
    s->frames++;
  }
  CK(cudaGetLastError());
  return GRX_OK;
}

int grx_mimi_sync(grx_mimi_streams* s) {
  if (!s) return fail(GRX_EINVAL, "null stream set");
  CK(cudaSetDevice(s->ar.dev));
  CK(cudaStreamSynchronize(s->st));
  CK(cudaGetLastError());
  return GRX_OK;
}

void* grx_mimi_cuda_stream(const grx_mimi_streams* s) { return s ? (void*)s->st : nullptr; }

int64_t grx_mimi_launches(const grx_mimi_streams* s) { return s ? s->launches : 0; }

int grx_mimi_frames(const grx_mimi_streams* s) {
  if (!s) return fail(GRX_EINVAL, "null stream set");
  return s->frames;
}

}  // extern "C"
