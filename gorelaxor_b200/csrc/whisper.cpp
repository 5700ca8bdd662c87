// The C ABI of the Whisper text decoder (include/grx.h): the decoder part of
// whisper.Load (whisper/model.go:94-223, 320-448, a whisper.cpp ggml file),
// the cross K/V of a window (encoder.go:120-140), and the greedy token loop
// at temperature 0 (decoder.go:33-140, transcribe.go:150-269, 370-520) for a
// batch of streams, one decode of every stream per CUDA-graph replay.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/grx.h"
#include "gguf.h"
#include "host.h"
#include "kernels.h"

using namespace grx;

namespace {

struct WLayerDev {
  float *attn_ln_w, *attn_ln_b, *x_ln_w, *x_ln_b, *mlp_ln_w, *mlp_ln_b;
  WMat q, k, v, o, xq, xk, xv, xo, fc1, fc2;
  float *qb, *vb, *ob, *xqb, *xvb, *xob, *fc1b, *fc2b;
  // q, k and v stacked into one matrix of 3·n_state rows, for one product
  // launch a decode step (rows 0 when their types differ)
  WMat qkv;
};

// A ggml tensor of the file: type, dims (fastest first), its bytes.
struct RawTensor {
  int type = 0;
  std::vector<int> ne;
  long n = 0;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
  bool used = false;
};

constexpr int T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8;

// typeBytes, model.go:262-273.
bool type_bytes(int t, long n, size_t* out) {
  if (t == T_F32) return *out = size_t(n) * 4, true;
  if (t == T_F16) return *out = size_t(n) * 2, true;
  int bs = t == T_Q4_0 ? 18 : t == T_Q4_1 ? 20 : t == T_Q5_0 ? 22 : t == T_Q5_1 ? 24 : t == T_Q8_0 ? 34 : 0;
  if (bs == 0 || n % 32 != 0) return false;
  *out = size_t(n) / 32 * bs;
  return true;
}

float h16(const uint8_t* p) { return f16_to_f32(uint16_t(p[0] | p[1] << 8)); }

// dequantBlock, model.go:449-492.
void dequant_block(int typ, const uint8_t* b, float* out) {
  switch (typ) {
    case T_Q4_0: {
      const float dd = h16(b);
      for (int j = 0; j < 16; j++) {
        out[j] = float(int(b[2 + j] & 0xF) - 8) * dd;
        out[j + 16] = float(int(b[2 + j] >> 4) - 8) * dd;
      }
      break;
    }
    case T_Q4_1: {
      const float dd = h16(b), mm = h16(b + 2);
      for (int j = 0; j < 16; j++) {
        out[j] = float(b[4 + j] & 0xF) * dd + mm;
        out[j + 16] = float(b[4 + j] >> 4) * dd + mm;
      }
      break;
    }
    case T_Q5_0: {
      const float dd = h16(b);
      uint32_t qh;
      std::memcpy(&qh, b + 2, 4);
      for (int j = 0; j < 16; j++) {
        const uint8_t xh0 = uint8_t(((qh >> j) << 4) & 0x10), xh1 = uint8_t((qh >> (j + 12)) & 0x10);
        out[j] = float(int((b[6 + j] & 0xF) | xh0) - 16) * dd;
        out[j + 16] = float(int((b[6 + j] >> 4) | xh1) - 16) * dd;
      }
      break;
    }
    case T_Q5_1: {
      const float dd = h16(b), mm = h16(b + 2);
      uint32_t qh;
      std::memcpy(&qh, b + 4, 4);
      for (int j = 0; j < 16; j++) {
        const uint8_t xh0 = uint8_t(((qh >> j) << 4) & 0x10), xh1 = uint8_t((qh >> (j + 12)) & 0x10);
        out[j] = float((b[8 + j] & 0xF) | xh0) * dd + mm;
        out[j + 16] = float((b[8 + j] >> 4) | xh1) * dd + mm;
      }
      break;
    }
    default: {  // Q8_0
      const float dd = h16(b);
      for (int j = 0; j < 32; j++) out[j] = float(int8_t(b[2 + j])) * dd;
    }
  }
}

// toF16, model.go:424-447: any tensor as float16 values.
std::vector<uint16_t> to_f16(const RawTensor& t) {
  std::vector<uint16_t> out(size_t(t.n));
  if (t.type == T_F16) {
    std::memcpy(out.data(), t.data, size_t(t.n) * 2);
  } else if (t.type == T_F32) {
    for (long i = 0; i < t.n; i++) {
      float f;
      std::memcpy(&f, t.data + i * 4, 4);
      out[size_t(i)] = f32_to_f16(f);
    }
  } else {
    size_t bs = 0;
    type_bytes(t.type, 32, &bs);
    float blk[32];
    for (long b = 0; b < t.n / 32; b++) {
      dequant_block(t.type, t.data + b * bs, blk);
      for (int j = 0; j < 32; j++) out[size_t(b * 32 + j)] = f32_to_f16(blk[j]);
    }
  }
  return out;
}

// toF32, model.go:408-422.
std::vector<float> to_f32(const RawTensor& t) {
  std::vector<float> out(size_t(t.n));
  if (t.type == T_F32) {
    std::memcpy(out.data(), t.data, size_t(t.n) * 4);
  } else {
    const std::vector<uint16_t> h = to_f16(t);
    for (size_t i = 0; i < h.size(); i++) out[i] = f16_to_f32(h[i]);
  }
  return out;
}

// Non-speech marks whose tokens are never sampled (vocab.go:96-101).
const char* const kNonSpeech[] = {"\"", "#", "(", ")", "*", "+", "/", ":", ";", "<", "=", ">", "@", "[", "\\", "]",
                                  "^", "_", "`", "{", "|", "}", "~", "「", "」", "『", "』", "<<", ">>", "<<<", ">>>",
                                  "--", "---", "-(", "-[", "('", "(\"", "((", "))", "(((", ")))", "[[", "]]", "{{",
                                  "}}", "♪♪", "♪♪♪", "♩", "♪", "♫", "♬", "♭", "♮", "♯"};

}  // namespace

// An audio encoder block (model.go:360-372).
struct WEncDev {
  float *attn_ln_w, *attn_ln_b, *mlp_ln_w, *mlp_ln_b;
  WMat q, k, v, o, fc1, fc2;
  float *qb, *vb, *ob, *fc1b, *fc2b;
};

struct grx_whisper {
  Arena ar;
  int dev = 0;
  int n_vocab = 0, n_audio_ctx = 0, n_state = 0, n_head = 0, n_text_layer = 0, n_text_ctx = 0, n_mels = 0;
  int n_audio_head = 0;
  // the audio encoder, when the file has its tensors (model.go:352-372)
  bool has_enc = false;
  WMat conv1, conv2;
  float *conv1b = nullptr, *conv2b = nullptr, *enc_pos = nullptr, *enc_ln_w = nullptr, *enc_ln_b = nullptr;
  std::vector<WEncDev> enc;
  std::vector<WLayerDev> layers;
  WMat tok_emb;
  float *dec_pos = nullptr, *ln_w = nullptr, *ln_b = nullptr;
  WVocabDev voc;
  std::vector<int> suppress;
  // float16 copies of the decoder's Q8_0 matrices, each value f16(q·d) as
  // the products widen it, made for the persistent one-stream kernel
  std::map<const int8_t*, uint16_t*> wide;
};

struct grx_whisper_batch {
  Arena ar;
  grx_whisper* m = nullptr;
  int n = 0;
  cudaStream_t st = nullptr;
  WRows rows;
  float *sk = nullptr, *sv = nullptr, *ck = nullptr, *cvt = nullptr;
  float *x = nullptr, *cur = nullptr, *q = nullptr, *att = nullptr, *ff = nullptr, *logits = nullptr, *scratch = nullptr;
  float *enc = nullptr, *no_speech = nullptr;
  // the audio encoder's work buffers, made at the first encode; its
  // attention runs enc_chunk streams at a time
  float *e_mel = nullptr, *e_x1 = nullptr, *e_h1 = nullptr, *e_x2 = nullptr, *e_x = nullptr, *e_cur = nullptr;
  float *e_q = nullptr, *e_k = nullptr, *e_v = nullptr, *e_att = nullptr, *e_ff = nullptr;
  float *e_qh = nullptr, *e_kh = nullptr, *e_vt = nullptr, *e_sc = nullptr;
  int enc_chunk = 0;
  int *row_stream = nullptr, *row_pos = nullptr, *row_tok = nullptr, *dst_row = nullptr, *out_step = nullptr;
  int* step = nullptr;
  WSample* state = nullptr;
  int* run_out = nullptr;  // [steps][n][4] of the current run (device)
  int run_cap = 0;
  int pos = 0;  // positions every stream holds (they all move together)
  // prompt rows [token][stream]: capacity in rows and the buffers
  int p_cap = 0;
  float *px = nullptr, *pcur = nullptr, *pq = nullptr, *patt = nullptr, *pff = nullptr;
  int *p_stream = nullptr, *p_pos = nullptr, *p_tok = nullptr, *p_dst = nullptr;
  cudaGraphExec_t g_decode = nullptr, g_step = nullptr;
  int per_decode = 0;
  int64_t launches = 0;
  // a batch of one stream runs its token loop in the persistent kernel
  // (k_wstep1): its arguments on the device, grid, barrier and error word
  bool ws1 = false;
  WStep1Args* ws1_args = nullptr;
  int ws1_grid = 0;
  size_t ws1_smem = 0;
  unsigned* ws1_bar = nullptr;
  int* ws1_err = nullptr;
  int* ws1_out = nullptr;  // the run_out the arguments hold
  ~grx_whisper_batch() {
    cudaSetDevice(ar.dev);
    if (g_decode) cudaGraphExecDestroy(g_decode);
    if (g_step) cudaGraphExecDestroy(g_step);
    if (st) cudaStreamDestroy(st);
  }
};

namespace {

size_t layer_stride_self(const grx_whisper* m, int n) { return size_t(n) * m->n_text_ctx * m->n_state; }
size_t layer_stride_cross(const grx_whisper* m, int n) { return size_t(n) * m->n_audio_ctx * m->n_state; }

void flin_w(const WMat& w, const float* x, int ldx, int rows, const float* bias, int epi, float* y, int ldy,
            const int* dst_row, cudaStream_t st) {
  FArgs a;
  a.epi = epi;
  a.x = x;
  a.ldx = ldx;
  a.wq = w.q;
  a.wd = w.d;
  a.wh = w.h;
  a.q8_as_f16 = w.q != nullptr;
  a.N = w.rows;
  a.K = w.cols;
  a.bias = bias;
  a.y = y;
  a.ldy = ldy;
  a.dst_row = dst_row;
  launch_flin(a, rows, st);
}

// One decode of every row (decoder.go:33-140 for one token per stream),
// then the positions move on. Returns the number of launches.
int enqueue_decode(grx_whisper_batch* b) {
  const grx_whisper* m = b->m;
  const int n = b->n, st = m->n_state;
  cudaStream_t s = b->st;
  int k = 0;
  launch_wembed(b->rows, m->tok_emb, m->dec_pos, b->x, s), k++;
  for (size_t l = 0; l < m->layers.size(); l++) {
    const WLayerDev& L = m->layers[l];
    float* skl = b->sk + l * layer_stride_self(m, n);
    float* svl = b->sv + l * layer_stride_self(m, n);
    const float* ckl = b->ck + l * layer_stride_cross(m, n);
    const float* cvl = b->cvt + l * layer_stride_cross(m, n);
    launch_wln(b->x, b->cur, L.attn_ln_w, L.attn_ln_b, n, st, s), k++;
    if (L.qkv.rows == 3 * st) {
      // q, k and v in one launch: the same products, three times the rows
      FArgs a;
      a.epi = FE_QKV;
      a.x = b->cur;
      a.ldx = st;
      a.wq = L.qkv.q;
      a.wd = L.qkv.d;
      a.wh = L.qkv.h;
      a.q8_as_f16 = L.qkv.q != nullptr;
      a.N = L.qkv.rows;
      a.K = L.qkv.cols;
      a.y = b->q;
      a.ldy = st;
      a.dst_row = b->dst_row;
      a.seg = st;
      a.qkv_bias[0] = L.qb;
      a.qkv_bias[2] = L.vb;
      a.qkv_y[0] = skl;
      a.qkv_y[1] = svl;
      launch_flin(a, n, s), k++;
    } else {
      flin_w(L.q, b->cur, st, n, L.qb, FE_BIAS, b->q, st, nullptr, s), k++;
      flin_w(L.k, b->cur, st, n, nullptr, FE_ROWPOS, skl, st, b->dst_row, s), k++;
      flin_w(L.v, b->cur, st, n, L.vb, FE_ROWPOS, svl, st, b->dst_row, s), k++;
    }
    launch_wself(b->rows, b->q, skl, svl, b->att, s), k++;
    flin_w(L.o, b->att, st, n, L.ob, FE_RESID, b->x, st, nullptr, s), k++;
    launch_wln(b->x, b->cur, L.x_ln_w, L.x_ln_b, n, st, s), k++;
    flin_w(L.xq, b->cur, st, n, L.xqb, FE_BIAS, b->q, st, nullptr, s), k++;
    launch_wcross(b->rows, b->q, ckl, cvl, b->att, b->scratch, size_t(n) * m->n_vocab, s), k++;
    flin_w(L.xo, b->att, st, n, L.xob, FE_RESID, b->x, st, nullptr, s), k++;
    launch_wln(b->x, b->cur, L.mlp_ln_w, L.mlp_ln_b, n, st, s), k++;
    flin_w(L.fc1, b->cur, st, n, L.fc1b, FE_GELU, b->ff, 4 * st, nullptr, s), k++;
    flin_w(L.fc2, b->ff, 4 * st, n, L.fc2b, FE_RESID, b->x, st, nullptr, s), k++;
  }
  launch_wln(b->x, b->cur, m->ln_w, m->ln_b, n, st, s), k++;
  flin_w(m->tok_emb, b->cur, st, n, nullptr, FE_BIAS, b->logits, m->n_vocab, nullptr, s), k++;
  launch_wtick(n, b->row_pos, b->dst_row, m->n_text_ctx, 1, nullptr, s), k++;
  return k;
}

int capture(grx_whisper_batch* b, bool with_sample, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal));
  int k = 0;
  if (with_sample) {
    launch_wproc(b->rows, b->logits, b->scratch, b->m->voc, b->state, b->run_out, b->step, b->row_tok, b->st), k++;
    launch_wtick(b->n, b->row_pos, b->dst_row, b->m->n_text_ctx, 0, b->step, b->st), k++;  // step += 1 only
  }
  k += enqueue_decode(b);
  cudaError_t e = cudaStreamEndCapture(b->st, &g);
  if (e != cudaSuccess) return fail(GRX_ECUDA, std::string("whisper graph capture: ") + cudaGetErrorString(e));
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(GRX_ECUDA, std::string("whisper graph: ") + cudaGetErrorString(e));
  b->per_decode = k;
  return GRX_OK;
}

// The persistent token loop for a batch of one stream when the model and the
// device suit it (GRX_WSTEP1=0 keeps the per-kernel graph): 64-value heads,
// K of every product a multiple of 64, Q8_0 or float16 matrices whose rows
// can be copied in 16-byte pieces, a cooperative launch of one CTA per SM
// with the weight buffers in shared memory.
int ws1_setup(grx_whisper_batch* b) {
  const char* env = getenv("GRX_WSTEP1");
  const grx_whisper* m = b->m;
  if ((env && env[0] == '0') || b->n != 1 || m->n_head * 64 != m->n_state || m->layers.empty() ||
      m->layers.size() > size_t(WS1_MAX_LAYERS) || m->n_vocab % 4 || m->n_audio_ctx % 4 || m->n_text_ctx % 4)
    return GRX_OK;
  auto al = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
  auto ok = [&](const WMat& w) {
    return w.f == nullptr && w.cols % 64 == 0 && (w.h ? al(w.h, 16) : w.q != nullptr && al(w.q, 16) && al(w.d, 4));
  };
  const int ff = m->layers[0].fc1.rows;
  if (!ok(m->tok_emb) || ff % 64 || !al(b->sv, 16) || !al(b->cvt, 16)) return GRX_OK;
  for (const WLayerDev& L : m->layers)
    if (!ok(L.q) || !ok(L.k) || !ok(L.v) || !ok(L.o) || !ok(L.xq) || !ok(L.xo) || !ok(L.fc1) || !ok(L.fc2) ||
        L.fc1.rows != ff)
      return GRX_OK;
  // the matrices as the kernel reads them: Q8_0 ones widened once into
  // float16 (the same values; its products then convert one value a term)
  grx_whisper* mw = b->m;
  int wrc = 0;
  auto wide = [&](WMat w) {
    if (w.h || !w.q) return w;
    uint16_t*& h = mw->wide[w.q];
    if (!h) {
      h = mw->ar.alloc<uint16_t>(size_t(w.rows) * w.cols, &wrc);
      if (!h) return w;
      launch_wwiden(w, h, nullptr);
    }
    WMat o = w;
    o.q = nullptr, o.d = nullptr, o.h = h;
    return o;
  };
  int G = 0, coop = 0;
  CK(cudaDeviceGetAttribute(&G, cudaDevAttrMultiProcessorCount, b->ar.dev));
  CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, b->ar.dev));
  if (!coop || G < 2 * m->n_head || G > WS1_MAX_GRID) return GRX_OK;
  WStep1Args A;
  A.st = m->n_state;
  A.nh = m->n_head;
  A.ctx = m->n_audio_ctx;
  A.text_ctx = m->n_text_ctx;
  A.ff = ff;
  A.L = int(m->layers.size());
  A.vocab = m->n_vocab;
  for (int l = 0; l < A.L; l++) {
    const WLayerDev& L = m->layers[size_t(l)];
    WS1Layer& Y = A.layers[l];
    Y.q = wide(L.q), Y.k = wide(L.k), Y.v = wide(L.v), Y.o = wide(L.o), Y.xq = wide(L.xq), Y.xo = wide(L.xo);
    Y.fc1 = wide(L.fc1), Y.fc2 = wide(L.fc2);
    Y.qb = L.qb, Y.vb = L.vb, Y.ob = L.ob, Y.xqb = L.xqb, Y.xob = L.xob, Y.fc1b = L.fc1b, Y.fc2b = L.fc2b;
    Y.ln1w = L.attn_ln_w, Y.ln1b = L.attn_ln_b, Y.ln2w = L.x_ln_w, Y.ln2b = L.x_ln_b, Y.ln3w = L.mlp_ln_w,
    Y.ln3b = L.mlp_ln_b;
    Y.sk = b->sk + size_t(l) * layer_stride_self(m, 1);
    Y.sv = b->sv + size_t(l) * layer_stride_self(m, 1);
    Y.ck = b->ck + size_t(l) * layer_stride_cross(m, 1);
    Y.cvt = b->cvt + size_t(l) * layer_stride_cross(m, 1);
  }
  A.emb = wide(m->tok_emb);
  if (wrc) {  // no room for the float16 copies: the per-kernel path
    cudaGetLastError();
    return GRX_OK;
  }
  CK(cudaDeviceSynchronize());
  A.dec_pos = m->dec_pos;
  A.lnw = m->ln_w;
  A.lnb = m->ln_b;
  A.voc = m->voc;
  A.state = b->state;
  A.row_tok = b->row_tok;
  A.row_pos = b->row_pos;
  A.dst_row = b->dst_row;
  A.step = b->step;
  A.logits = b->logits;
  A.scratch = b->scratch;
  // shared-memory plan: a weight buffer holds one layer's rows of this CTA
  // (at most ceil(n/G) rows of each product) or a chunk of logits rows
  const int R = (A.st + G - 1) / G, Rf = (ff + G - 1) / G;
  int wb = 0;
  for (const WS1Layer& Y : A.layers) {
    if (&Y - A.layers >= A.L) break;
    int lb = 0;
    for (int i = 0; i < 8; i++) lb += ws_slice_bytes(true, i == 6 ? Rf : R, i == 7 ? ff : A.st);
    wb = std::max(wb, lb);
  }
  A.lrows = std::min(64, (A.vocab + G - 1) / G);
  wb = std::max(wb, ws_slice_bytes(true, A.lrows, A.st));
  A.wb = (wb + 15) / 16 * 16;
  // CTAs a head in the self-attention and cross values: a power of two up
  // to 32 that fits G / heads, each with 64 / that outputs
  int per = 1;
  while (per * 2 <= std::min(32, G / A.nh)) per *= 2;
  A.so_nd = A.xo_nd = 64 / per;
  A.xv_floats = std::max(A.xo_nd * A.ctx, A.so_nd * A.text_ctx);
  {  // a CTA's key chunk of the cross scores, as k_wstep1 splits them
    const int ctx4 = A.ctx & ~3, ks = std::max(1, G / A.nh);
    A.xk_floats = ((ctx4 + ks - 1) / ks + 15) / 16 * 16 * 64;
  }
  const size_t smem = wstep1_smem(A);
  if (wstep1_max_active(smem) < 1) return GRX_OK;
  int rc = 0;
  A.x = b->ar.alloc<float>(size_t(A.st), &rc);
  A.q = b->ar.alloc<float>(size_t(A.st), &rc);
  A.att = b->ar.alloc<float>(size_t(A.st), &rc);
  A.ffb = b->ar.alloc<float>(size_t(ff), &rc);
  A.sg = b->ar.alloc<float>(size_t(A.nh) * A.ctx, &rc);
  A.mg = b->ar.alloc<float>(size_t(G), &rc);
  A.part = b->ar.alloc<float>(size_t(8) * G, &rc);
  A.partv = b->ar.alloc<int2>(size_t(2) * G, &rc);
  A.bar = b->ar.alloc<unsigned>(1, &rc);
  A.err = b->ar.alloc<int>(1, &rc);
  b->ws1_args = b->ar.alloc<WStep1Args>(1, &rc);
  if (rc) return rc;
  CK(cudaMemset(A.err, 0, sizeof(int)));
  CK(cudaMemcpy(b->ws1_args, &A, sizeof A, cudaMemcpyHostToDevice));
  b->ws1_bar = A.bar;
  b->ws1_err = A.err;
  b->ws1_grid = G;
  b->ws1_smem = smem;
  b->ws1 = true;
  return GRX_OK;
}

// GRX_ETIMEDOUT when the persistent kernel gave up on a wait (the word is
// cleared for the next run).
int ws1_check(grx_whisper_batch* b) {
  if (!b->ws1) return GRX_OK;
  int e = 0;
  CK(cudaMemcpy(&e, b->ws1_err, sizeof e, cudaMemcpyDeviceToHost));
  if (!e) return GRX_OK;
  CK(cudaMemset(b->ws1_err, 0, sizeof(int)));
  return fail(GRX_ETIMEDOUT, "the persistent Whisper step gave up on a grid barrier after its one-second limit");
}

}  // namespace

extern "C" {

int grx_whisper_load(const void* bytes, size_t len, int device, grx_whisper** out) {
  if (!bytes || !out) return fail(GRX_EINVAL, "grx_whisper_load: null argument");
  int rc = device_init(device);
  if (rc) return rc;
  const uint8_t* p = static_cast<const uint8_t*>(bytes);
  size_t off = 0;
  const std::string efmt = "not a Whisper model file in whisper.cpp (ggml) format";
  auto rd32 = [&](int32_t* v) {
    if (len - off < 4 || off > len) return false;
    std::memcpy(v, p + off, 4);
    off += 4;
    return true;
  };
  int32_t magic = 0;
  if (!rd32(&magic) || uint32_t(magic) != 0x67676d6c) return fail(GRX_EFORMAT, efmt);
  int32_t hv[11];
  for (int i = 0; i < 11; i++)
    if (!rd32(&hv[i])) return fail(GRX_EFORMAT, efmt);
  auto m = std::make_unique<grx_whisper>();
  m->ar.dev = m->dev = device;
  m->n_vocab = hv[0];
  m->n_audio_ctx = hv[1];
  const int n_audio_state = hv[2], n_audio_head = hv[3], n_audio_layer = hv[4];
  m->n_audio_head = n_audio_head;
  m->n_text_ctx = hv[5];
  m->n_state = hv[6];
  m->n_head = hv[7];
  m->n_text_layer = hv[8];
  m->n_mels = hv[9];
  // model.go:127-132
  if (n_audio_state != m->n_state || n_audio_state <= 0 || n_audio_head <= 0 || n_audio_state % n_audio_head != 0 ||
      m->n_head <= 0 || m->n_state % m->n_head != 0 || m->n_mels <= 0 || m->n_mels > 256 || m->n_audio_ctx != 1500 ||
      m->n_vocab < 51864 || m->n_vocab > 60000 || n_audio_layer <= 0 || n_audio_layer > 64 || m->n_text_layer <= 0 ||
      m->n_text_layer > 64 || m->n_text_ctx <= 0 || m->n_text_ctx > 4096)
    return fail(GRX_EFORMAT, "the model's dimensions aren't ones this program knows");
  if (m->n_state / m->n_head != 64 || m->n_state % 32 != 0)
    return fail(GRX_EINVAL, "whisper: heads of " + std::to_string(m->n_state / m->n_head) + " values (this build runs 64)");
  int32_t nmel = 0, nfft = 0;
  if (!rd32(&nmel) || !rd32(&nfft) || nmel != m->n_mels || nfft != 201) return fail(GRX_EFORMAT, efmt);
  const size_t melb = size_t(nmel) * size_t(nfft) * 4;
  if (len - off < melb) return fail(GRX_EFORMAT, efmt);
  off += melb;  // the mel filters belong to the front end
  int32_t nv = 0;
  if (!rd32(&nv) || nv <= 0 || nv > m->n_vocab) return fail(GRX_EFORMAT, efmt);
  std::map<std::string, int> to_id;
  for (int i = 0; i < nv; i++) {
    int32_t l = 0;
    if (!rd32(&l) || l < 0 || l > (1 << 16) || len - off < size_t(l)) return fail(GRX_EFORMAT, efmt);
    to_id.emplace(std::string(reinterpret_cast<const char*>(p + off), size_t(l)), i);
    off += size_t(l);
  }
  std::map<std::string, RawTensor> ts;
  while (off < len) {
    int32_t nd = 0, ln = 0, tt = 0;
    if (!rd32(&nd) || !rd32(&ln) || !rd32(&tt) || nd < 1 || nd > 4 || ln <= 0 || ln > 256)
      return fail(GRX_EFORMAT, efmt);
    RawTensor t;
    t.type = tt;
    long n = 1;
    for (int i = 0; i < nd; i++) {
      int32_t v = 0;
      if (!rd32(&v) || v <= 0 || long(v) > (1L << 31) / n) return fail(GRX_EFORMAT, efmt);
      t.ne.push_back(v);
      n *= v;
    }
    t.n = n;
    if (len - off < size_t(ln)) return fail(GRX_EFORMAT, efmt);
    const std::string name(reinterpret_cast<const char*>(p + off), size_t(ln));
    off += size_t(ln);
    if (!type_bytes(tt, n, &t.bytes))
      return fail(GRX_EFORMAT, "tensor " + name + " has a weight type (" + std::to_string(tt) + ") this program can't read");
    if (len - off < t.bytes) return fail(GRX_EFORMAT, "the model file is cut short");
    t.data = p + off;
    off += t.bytes;
    ts[name] = t;
  }
  // bind, model.go:320-402 (decoder part; the encoder's tensors are read
  // and left: its output is what the decoder is given)
  std::string err;
  const int st = m->n_state;
  auto get = [&](const std::string& name, std::vector<int> ne) -> RawTensor* {
    if (!err.empty()) return nullptr;
    auto it = ts.find(name);
    if (it == ts.end()) {
      err = "the model file has no tensor " + name;
      return nullptr;
    }
    long n = 1;
    for (int v : ne) n *= v;
    RawTensor& t = it->second;
    if (t.n != n || (t.ne.size() == ne.size() && t.ne[0] != ne[0])) {
      err = "tensor " + name + " has the wrong shape";
      return nullptr;
    }
    t.used = true;
    return &t;
  };
  auto as_f32 = [&](const std::string& name, const RawTensor& t) {
    // model.go:211-215: vectors, positional embeddings and [1]-wide
    // tensors load as float32; the rest through float16
    const bool f32 = t.ne.size() == 1 || t.ne[0] == 1 ||
                     (name.size() >= 20 && name.compare(name.size() - 20, 20, "positional_embedding") == 0);
    if (f32) return to_f32(t);
    const std::vector<uint16_t> h = to_f16(t);
    std::vector<float> out(h.size());
    for (size_t i = 0; i < h.size(); i++) out[i] = f16_to_f32(h[i]);
    return out;
  };
  auto vec = [&](const std::string& name, int n) -> float* {
    RawTensor* t = get(name, {n});
    if (!t) return nullptr;
    const std::vector<float> v = as_f32(name, *t);
    return m->ar.upload(v.data(), v.size(), &rc);
  };
  auto vec2 = [&](const std::string& name, int rows, int cols) -> float* {
    RawTensor* t = get(name, {cols, rows});
    if (!t) return nullptr;
    const std::vector<float> v = as_f32(name, *t);
    return m->ar.upload(v.data(), v.size(), &rc);
  };
  auto mat = [&](const std::string& name, int rows, int cols) -> WMat {
    WMat w;
    RawTensor* t = get(name, {cols, rows});
    if (!t) return w;
    w.rows = rows;
    w.cols = cols;
    const bool f32 = t->ne.size() == 1 || t->ne[0] == 1;
    if (t->type == T_Q8_0 && !f32 && cols % 32 == 0) {
      // Q8_0 stays in HBM; the kernels widen f16(q·d) as they read
      std::vector<int8_t> q(size_t(t->n));
      std::vector<uint16_t> d(size_t(t->n) / 32);
      for (long b = 0; b < t->n / 32; b++) {
        d[size_t(b)] = uint16_t(t->data[b * 34] | t->data[b * 34 + 1] << 8);
        std::memcpy(&q[size_t(b) * 32], t->data + b * 34 + 2, 32);
      }
      w.q = m->ar.upload(q.data(), q.size(), &rc);
      w.d = m->ar.upload(d.data(), d.size(), &rc);
    } else {
      std::vector<uint16_t> h;
      if (f32) {  // loaded as float32 first, then rounded (model.go:343-349)
        const std::vector<float> v = to_f32(*t);
        h.resize(v.size());
        for (size_t i = 0; i < v.size(); i++) h[i] = f32_to_f16(v[i]);
      } else {
        h = to_f16(*t);
      }
      w.h = m->ar.upload(h.data(), h.size(), &rc);
    }
    return w;
  };
  // three matrices of one type and width stacked by rows on the device
  auto stack3 = [&](const WMat& a, const WMat& b, const WMat& c) -> WMat {
    WMat w;
    const WMat* ms[3] = {&a, &b, &c};
    const bool q8 = a.q && b.q && c.q, h16 = a.h && b.h && c.h;
    if (rc || !(q8 || h16) || b.cols != a.cols || c.cols != a.cols) return w;
    w.rows = a.rows + b.rows + c.rows;
    w.cols = a.cols;
    if (q8) {
      int8_t* q = m->ar.alloc<int8_t>(size_t(w.rows) * w.cols, &rc);
      uint16_t* d = m->ar.alloc<uint16_t>(size_t(w.rows) * w.cols / 32, &rc);
      if (rc) return WMat{};
      for (int i = 0, r = 0; i < 3; r += ms[i]->rows, i++) {
        const size_t n = size_t(ms[i]->rows) * w.cols;
        if (cudaMemcpy(q + size_t(r) * w.cols, ms[i]->q, n, cudaMemcpyDeviceToDevice) != cudaSuccess ||
            cudaMemcpy(d + size_t(r) * w.cols / 32, ms[i]->d, n / 32 * 2, cudaMemcpyDeviceToDevice) != cudaSuccess)
          rc = fail(GRX_ECUDA, "stacking q, k and v failed");
      }
      w.q = q;
      w.d = d;
    } else {
      uint16_t* h = m->ar.alloc<uint16_t>(size_t(w.rows) * w.cols, &rc);
      if (rc) return WMat{};
      for (int i = 0, r = 0; i < 3; r += ms[i]->rows, i++)
        if (cudaMemcpy(h + size_t(r) * w.cols, ms[i]->h, size_t(ms[i]->rows) * w.cols * 2, cudaMemcpyDeviceToDevice) !=
            cudaSuccess)
          rc = fail(GRX_ECUDA, "stacking q, k and v failed");
      w.h = h;
    }
    return w;
  };
  m->dec_pos = vec2("decoder.positional_embedding", m->n_text_ctx, st);
  m->tok_emb = mat("decoder.token_embedding.weight", m->n_vocab, st);
  m->ln_w = vec("decoder.ln.weight", st);
  m->ln_b = vec("decoder.ln.bias", st);
  for (int i = 0; i < m->n_text_layer; i++) {
    const std::string lp = "decoder.blocks." + std::to_string(i) + ".";
    WLayerDev L;
    L.attn_ln_w = vec(lp + "attn_ln.weight", st);
    L.attn_ln_b = vec(lp + "attn_ln.bias", st);
    L.q = mat(lp + "attn.query.weight", st, st);
    L.qb = vec(lp + "attn.query.bias", st);
    L.k = mat(lp + "attn.key.weight", st, st);
    L.v = mat(lp + "attn.value.weight", st, st);
    L.vb = vec(lp + "attn.value.bias", st);
    L.o = mat(lp + "attn.out.weight", st, st);
    L.ob = vec(lp + "attn.out.bias", st);
    L.x_ln_w = vec(lp + "cross_attn_ln.weight", st);
    L.x_ln_b = vec(lp + "cross_attn_ln.bias", st);
    L.xq = mat(lp + "cross_attn.query.weight", st, st);
    L.xqb = vec(lp + "cross_attn.query.bias", st);
    L.xk = mat(lp + "cross_attn.key.weight", st, st);
    L.xv = mat(lp + "cross_attn.value.weight", st, st);
    L.xvb = vec(lp + "cross_attn.value.bias", st);
    L.xo = mat(lp + "cross_attn.out.weight", st, st);
    L.xob = vec(lp + "cross_attn.out.bias", st);
    L.mlp_ln_w = vec(lp + "mlp_ln.weight", st);
    L.mlp_ln_b = vec(lp + "mlp_ln.bias", st);
    L.fc1 = mat(lp + "mlp.0.weight", 4 * st, st);
    L.fc1b = vec(lp + "mlp.0.bias", 4 * st);
    L.fc2 = mat(lp + "mlp.2.weight", st, 4 * st);
    L.fc2b = vec(lp + "mlp.2.bias", st);
    L.qkv = stack3(L.q, L.k, L.v);
    m->layers.push_back(L);
  }
  // the audio encoder (model.go:352-372), bound when the file has it
  if (err.empty() && ts.count("encoder.conv1.weight")) {
    m->has_enc = true;
    m->enc_pos = vec2("encoder.positional_embedding", m->n_audio_ctx, st);
    m->conv1 = mat("encoder.conv1.weight", st, m->n_mels * 3);
    m->conv1b = vec("encoder.conv1.bias", st);
    m->conv2 = mat("encoder.conv2.weight", st, st * 3);
    m->conv2b = vec("encoder.conv2.bias", st);
    m->enc_ln_w = vec("encoder.ln_post.weight", st);
    m->enc_ln_b = vec("encoder.ln_post.bias", st);
    for (int i = 0; i < n_audio_layer; i++) {
      const std::string lp = "encoder.blocks." + std::to_string(i) + ".";
      WEncDev L;
      L.attn_ln_w = vec(lp + "attn_ln.weight", st);
      L.attn_ln_b = vec(lp + "attn_ln.bias", st);
      L.q = mat(lp + "attn.query.weight", st, st);
      L.qb = vec(lp + "attn.query.bias", st);
      L.k = mat(lp + "attn.key.weight", st, st);
      L.v = mat(lp + "attn.value.weight", st, st);
      L.vb = vec(lp + "attn.value.bias", st);
      L.o = mat(lp + "attn.out.weight", st, st);
      L.ob = vec(lp + "attn.out.bias", st);
      L.mlp_ln_w = vec(lp + "mlp_ln.weight", st);
      L.mlp_ln_b = vec(lp + "mlp_ln.bias", st);
      L.fc1 = mat(lp + "mlp.0.weight", 4 * st, st);
      L.fc1b = vec(lp + "mlp.0.bias", 4 * st);
      L.fc2 = mat(lp + "mlp.2.weight", st, 4 * st);
      L.fc2b = vec(lp + "mlp.2.bias", st);
      m->enc.push_back(L);
    }
  }
  if (!err.empty()) return fail(GRX_EFORMAT, err);
  for (const auto& kv : ts)
    if (!kv.second.used && kv.first.compare(0, 8, "encoder.") != 0)
      return fail(GRX_EFORMAT, "the model file has a tensor this program doesn't know: " + kv.first);
  if (rc) return rc;
  // the vocabulary's special tokens (vocab.go:19-43) and suppressed tokens
  WVocabDev& v = m->voc;
  v.n = m->n_vocab;
  v.eot = 50256, v.sot = 50257;
  v.translate = 50357, v.transcribe = 50358, v.solm = 50359, v.prev = 50360, v.nosp = 50361, v.not_ = 50362;
  v.beg = 50363;
  if (m->n_vocab >= 51865) {
    v.n_lang = m->n_vocab - 51765 - 1;
    const int dt = v.n_lang - 98;
    v.eot++, v.sot++;
    v.translate += dt, v.transcribe += dt, v.solm += dt, v.prev += dt, v.nosp += dt, v.not_ += dt, v.beg += dt;
  }
  auto sp = to_id.find(" ");
  v.space = sp == to_id.end() ? -1 : sp->second;
  for (const char* t : kNonSpeech)
    for (const std::string& s : {std::string(t), " " + std::string(t)}) {
      auto f = to_id.find(s);
      if (f != to_id.end() && f->second < v.eot) m->suppress.push_back(f->second);
    }
  for (const char* s : {" -", " '"}) {
    auto f = to_id.find(s);
    if (f != to_id.end()) m->suppress.push_back(f->second);
  }
  v.n_suppress = int(m->suppress.size());
  v.suppress = m->suppress.empty() ? nullptr : m->ar.upload(m->suppress.data(), m->suppress.size(), &rc);
  v.audio_ctx = m->n_audio_ctx;
  v.exact_rows = m->ar.alloc<unsigned long long>(1, &rc);
  if (rc) return rc;
  CK(cudaMemset(v.exact_rows, 0, sizeof(unsigned long long)));
  *out = m.release();
  return GRX_OK;
}

void grx_whisper_free(grx_whisper* m) { delete m; }

int64_t grx_whisper_exact_rows(const grx_whisper* m) {
  if (!m) return fail(GRX_EINVAL, "null model");
  unsigned long long v = 0;
  CK(cudaSetDevice(m->dev));
  CK(cudaMemcpy(&v, m->voc.exact_rows, sizeof v, cudaMemcpyDeviceToHost));
  return int64_t(v);
}

int grx_whisper_dims(const grx_whisper* m, int* n_vocab, int* n_audio_ctx, int* n_state, int* n_head,
                     int* n_text_layer, int* n_text_ctx) {
  if (!m) return fail(GRX_EINVAL, "null model");
  if (n_vocab) *n_vocab = m->n_vocab;
  if (n_audio_ctx) *n_audio_ctx = m->n_audio_ctx;
  if (n_state) *n_state = m->n_state;
  if (n_head) *n_head = m->n_head;
  if (n_text_layer) *n_text_layer = m->n_text_layer;
  if (n_text_ctx) *n_text_ctx = m->n_text_ctx;
  return GRX_OK;
}

int grx_whisper_tokens(const grx_whisper* m, int* eot, int* sot, int* prev, int* nosp, int* beg, int* n_lang) {
  if (!m) return fail(GRX_EINVAL, "null model");
  if (eot) *eot = m->voc.eot;
  if (sot) *sot = m->voc.sot;
  if (prev) *prev = m->voc.prev;
  if (nosp) *nosp = m->voc.nosp;
  if (beg) *beg = m->voc.beg;
  if (n_lang) *n_lang = m->voc.n_lang;
  return GRX_OK;
}

int grx_whisper_suppressed(const grx_whisper* m, int* out, int cap) {
  if (!m) return fail(GRX_EINVAL, "null model");
  for (size_t i = 0; i < m->suppress.size() && int(i) < cap; i++) out[i] = m->suppress[i];
  return int(m->suppress.size());
}

int grx_whisper_batch_create(grx_whisper* m, int n, grx_whisper_batch** out) {
  if (!m || !out || n <= 0) return fail(GRX_EINVAL, "grx_whisper_batch_create: bad argument");
  CK(cudaSetDevice(m->dev));
  auto b = std::make_unique<grx_whisper_batch>();
  b->ar.dev = m->dev;
  b->m = m;
  b->n = n;
  CK(cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking));
  wdecode_init();
  int rc = 0;
  const int st = m->n_state, L = m->n_text_layer;
  b->sk = b->ar.alloc<float>(size_t(L) * layer_stride_self(m, n), &rc);
  b->sv = b->ar.alloc<float>(size_t(L) * layer_stride_self(m, n), &rc);
  b->ck = b->ar.alloc<float>(size_t(L) * layer_stride_cross(m, n), &rc);
  b->cvt = b->ar.alloc<float>(size_t(L) * layer_stride_cross(m, n), &rc);
  b->x = b->ar.alloc<float>(size_t(n) * st, &rc);
  b->cur = b->ar.alloc<float>(size_t(n) * st, &rc);
  b->q = b->ar.alloc<float>(size_t(n) * st, &rc);
  b->att = b->ar.alloc<float>(size_t(n) * st, &rc);
  b->ff = b->ar.alloc<float>(size_t(n) * 4 * st, &rc);
  b->logits = b->ar.alloc<float>(size_t(n) * m->n_vocab, &rc);
  b->scratch = b->ar.alloc<float>(size_t(n) * m->n_vocab, &rc);
  b->enc = b->ar.alloc<float>(layer_stride_cross(m, n), &rc);
  b->no_speech = b->ar.alloc<float>(n, &rc);
  b->row_stream = b->ar.alloc<int>(n, &rc);
  b->row_pos = b->ar.alloc<int>(n, &rc);
  b->row_tok = b->ar.alloc<int>(n, &rc);
  b->dst_row = b->ar.alloc<int>(n, &rc);
  b->step = b->ar.alloc<int>(1, &rc);
  b->state = b->ar.alloc<WSample>(n, &rc);
  if (rc) return rc;
  std::vector<int> ids((size_t)n);
  for (int i = 0; i < n; i++) ids[size_t(i)] = i;
  CK(cudaMemcpy(b->row_stream, ids.data(), sizeof(int) * size_t(n), cudaMemcpyHostToDevice));
  WRows& r = b->rows;
  r.rows = n;
  r.st = st;
  r.nh = m->n_head;
  r.text_ctx = m->n_text_ctx;
  r.audio_ctx = m->n_audio_ctx;
  r.vocab = m->n_vocab;
  r.row_stream = b->row_stream;
  r.row_pos = b->row_pos;
  r.row_tok = b->row_tok;
  rc = ws1_setup(b.get());
  if (rc) return rc;
  *out = b.release();
  return GRX_OK;
}

void grx_whisper_batch_free(grx_whisper_batch* b) { delete b; }

}  // extern "C"

namespace {

// A new window for every stream: cross K/V from d_enc [n][ctx][state]
// (encoder.go:120-140), empty caches and fresh sampling states.
int set_audio(grx_whisper_batch* b, const float* d_enc) {
  const grx_whisper* m = b->m;
  const int n = b->n, st = m->n_state, ctx = m->n_audio_ctx;
  const float tsc = float(1 / std::sqrt(double(st / m->n_head)));
  for (size_t l = 0; l < m->layers.size(); l++) {
    const WLayerDev& L = m->layers[l];
    WmmArgs a;
    a.a = d_enc;
    a.lda = st;
    a.a_zs = size_t(ctx) * st;
    a.m = ctx;
    a.w = L.xk;
    a.mode = WM_CROSSK;
    a.c = b->ck + l * layer_stride_cross(m, n);
    a.nh = m->n_head;
    a.tsc = tsc;
    launch_wmm(a, n, b->st);
    a.w = L.xv;
    a.bias = L.xvb;
    a.mode = WM_CROSSV;
    a.c = b->cvt + l * layer_stride_cross(m, n);
    launch_wmm(a, n, b->st);
    b->launches += 2;
  }
  CK(cudaMemsetAsync(b->row_pos, 0, sizeof(int) * size_t(n), b->st));
  b->pos = 0;
  std::vector<WSample> s0(size_t(n), WSample{0, -1, -1, 0, 3000});  // seq{seekDelta: winFrames}
  CK(cudaMemcpyAsync(b->state, s0.data(), sizeof(WSample) * size_t(n), cudaMemcpyHostToDevice, b->st));
  CK(cudaMemsetAsync(b->step, 0, sizeof(int), b->st));
  launch_wtick(n, b->row_pos, b->dst_row, m->n_text_ctx, 0, nullptr, b->st);
  CK(cudaGetLastError());
  CK(cudaStreamSynchronize(b->st));
  return GRX_OK;
}

int ensure_run_out(grx_whisper_batch* b, int steps) {
  if (steps <= b->run_cap) return GRX_OK;
  // a new output buffer means new graphs (the pointer is captured)
  int rc = 0;
  b->run_out = b->ar.alloc<int>(size_t(steps) * b->n * 4, &rc);
  if (rc) return rc;
  b->run_cap = steps;
  if (b->g_step) {
    cudaGraphExecDestroy(b->g_step);
    b->g_step = nullptr;
  }
  return GRX_OK;
}

// One product of the prompt rows ([token][stream] order, np tokens per
// stream): whisper/gemm.go's matmul takes the packed kernel for each
// stream's first np/6·6 rows when np ≥ 6 and gemv for the rest.
void prompt_product(grx_whisper_batch* b, int np, const WMat& w, const float* a, int lda, const float* bias, int epi,
                    float* c, int ldc) {
  const int n = b->n, mfull = np >= 6 ? np / 6 * 6 : 0;
  if (mfull > 0) {
    WmmArgs p;
    p.a = a;
    p.lda = n * lda;  // consecutive tokens of one stream are n rows apart
    p.a_zs = size_t(lda);
    p.m = mfull;
    p.w = w;
    p.bias = bias;
    p.mode = epi == FE_RESID ? WM_RESID : epi == FE_GELU ? WM_GELU : epi == FE_ROWPOS ? WM_ROWPOS : WM_STORE;
    p.c = c;
    p.ldc = epi == FE_ROWPOS ? ldc : n * ldc;
    p.c_zs = size_t(ldc);
    p.dst_row = b->p_dst;
    p.rs_i = n;
    launch_wmm(p, n, b->st);
    b->launches++;
  }
  if (mfull < np) {
    const size_t r0 = size_t(mfull) * n;
    flin_w(w, a + r0 * lda, lda, (np - mfull) * n, bias, epi, epi == FE_ROWPOS ? c : c + r0 * ldc, ldc,
           epi == FE_ROWPOS ? b->p_dst + r0 : nullptr, b->st);
    b->launches++;
  }
}

// decode (decoder.go:33-140) of np prompt tokens per stream: all rows at
// once, causal self-attention per row; the no-speech probability from the
// logits of row sot_at, the next sample's logits from the last row.
int prefill(grx_whisper_batch* b, const int* prompt, int np, int sot_at) {
  const grx_whisper* m = b->m;
  const int n = b->n, st = m->n_state, R = np * n;
  int rc = 0;
  if (R > b->p_cap) {
    b->px = b->ar.alloc<float>(size_t(R) * st, &rc);
    b->pcur = b->ar.alloc<float>(size_t(R) * st, &rc);
    b->pq = b->ar.alloc<float>(size_t(R) * st, &rc);
    b->patt = b->ar.alloc<float>(size_t(R) * st, &rc);
    b->pff = b->ar.alloc<float>(size_t(R) * 4 * st, &rc);
    b->p_stream = b->ar.alloc<int>(R, &rc);
    b->p_pos = b->ar.alloc<int>(R, &rc);
    b->p_tok = b->ar.alloc<int>(R, &rc);
    b->p_dst = b->ar.alloc<int>(R, &rc);
    if (rc) return rc;
    b->p_cap = R;
  }
  std::vector<int> hs((size_t)R), hp((size_t)R), ht((size_t)R), hd((size_t)R);
  for (int i = 0; i < np; i++)
    for (int s = 0; s < n; s++) {
      const size_t r = size_t(i) * n + s;
      hs[r] = s;
      hp[r] = b->pos + i;
      ht[r] = prompt[size_t(s) * np + i];
      hd[r] = s * m->n_text_ctx + b->pos + i;
    }
  CK(cudaMemcpyAsync(b->p_stream, hs.data(), sizeof(int) * R, cudaMemcpyHostToDevice, b->st));
  CK(cudaMemcpyAsync(b->p_pos, hp.data(), sizeof(int) * R, cudaMemcpyHostToDevice, b->st));
  CK(cudaMemcpyAsync(b->p_tok, ht.data(), sizeof(int) * R, cudaMemcpyHostToDevice, b->st));
  CK(cudaMemcpyAsync(b->p_dst, hd.data(), sizeof(int) * R, cudaMemcpyHostToDevice, b->st));
  WRows pr = b->rows;
  pr.rows = R;
  pr.row_stream = b->p_stream;
  pr.row_pos = b->p_pos;
  pr.row_tok = b->p_tok;
  cudaStream_t s = b->st;
  launch_wembed(pr, m->tok_emb, m->dec_pos, b->px, s);
  for (size_t l = 0; l < m->layers.size(); l++) {
    const WLayerDev& L = m->layers[l];
    float* skl = b->sk + l * layer_stride_self(m, n);
    float* svl = b->sv + l * layer_stride_self(m, n);
    launch_wln(b->px, b->pcur, L.attn_ln_w, L.attn_ln_b, R, st, s);
    prompt_product(b, np, L.q, b->pcur, st, L.qb, FE_BIAS, b->pq, st);
    prompt_product(b, np, L.k, b->pcur, st, nullptr, FE_ROWPOS, skl, st);
    prompt_product(b, np, L.v, b->pcur, st, L.vb, FE_ROWPOS, svl, st);
    launch_wself(pr, b->pq, skl, svl, b->patt, s);
    prompt_product(b, np, L.o, b->patt, st, L.ob, FE_RESID, b->px, st);
    launch_wln(b->px, b->pcur, L.x_ln_w, L.x_ln_b, R, st, s);
    prompt_product(b, np, L.xq, b->pcur, st, L.xqb, FE_BIAS, b->pq, st);
    launch_wcross(pr, b->pq, b->ck + l * layer_stride_cross(m, n), b->cvt + l * layer_stride_cross(m, n), b->patt,
                  b->scratch, size_t(n) * m->n_vocab, s);
    prompt_product(b, np, L.xo, b->patt, st, L.xob, FE_RESID, b->px, st);
    launch_wln(b->px, b->pcur, L.mlp_ln_w, L.mlp_ln_b, R, st, s);
    prompt_product(b, np, L.fc1, b->pcur, st, L.fc1b, FE_GELU, b->pff, 4 * st);
    prompt_product(b, np, L.fc2, b->pff, 4 * st, L.fc2b, FE_RESID, b->px, st);
    b->launches += 6;
  }
  // the no-speech probability from row sot_at, then the logits of the last row
  launch_wln(b->px + size_t(sot_at) * n * st, b->pcur, m->ln_w, m->ln_b, n, st, s);
  flin_w(m->tok_emb, b->pcur, st, n, nullptr, FE_BIAS, b->logits, m->n_vocab, nullptr, s);
  launch_wnospeech(b->logits, m->n_vocab, m->voc.nosp, b->scratch, b->no_speech, n, s);
  launch_wln(b->px + size_t(np - 1) * n * st, b->pcur, m->ln_w, m->ln_b, n, st, s);
  flin_w(m->tok_emb, b->pcur, st, n, nullptr, FE_BIAS, b->logits, m->n_vocab, nullptr, s);
  b->launches += 6;
  // the token loop's rows continue after the prompt
  b->pos += np;
  std::vector<int> pos((size_t)n, b->pos);
  CK(cudaMemcpyAsync(b->row_pos, pos.data(), sizeof(int) * size_t(n), cudaMemcpyHostToDevice, s));
  launch_wtick(n, b->row_pos, b->dst_row, m->n_text_ctx, 0, nullptr, s);
  CK(cudaGetLastError());
  CK(cudaStreamSynchronize(s));  // the host arrays above are local
  return GRX_OK;
}

// One product of the encoder over `groups` streams of m rows each (all
// rows ≥ 6: whisper/gemm.go's packed kernel throughout).
void enc_product(grx_whisper_batch* b, const float* a, int lda, int m, const WMat& w, const float* bias, int mode,
                 float* c, int ldc, int groups, const float* aux = nullptr) {
  WmmArgs p;
  p.a = a;
  p.lda = lda;
  p.a_zs = size_t(m) * lda;
  p.m = m;
  p.w = w;
  p.bias = bias;
  p.mode = mode;
  p.c = c;
  p.ldc = ldc;
  p.c_zs = size_t(m) * ldc;
  p.aux = aux;
  launch_wmm(p, groups, b->st);
  b->launches++;
}

// encode (encoder.go:10-118) of every stream's window d_mel [n][n_mels][3000]
// into b->enc [n][ctx][state].
int encode(grx_whisper_batch* b, const float* d_mel) {
  const grx_whisper* m = b->m;
  const int n = b->n, st = m->n_state, ctx = m->n_audio_ctx, nmel = m->n_mels, W = 3000;
  const int nh = m->n_audio_head, hd = st / nh;
  int rc = 0;
  if (!b->e_x) {
    // attention's scores take nh·ctx² floats per stream: at most ~2 GB at once
    b->enc_chunk = int(std::max<size_t>(1, std::min<size_t>(n, (size_t(2) << 30) / (size_t(nh) * ctx * ctx * 4))));
    const size_t N = size_t(n);
    b->e_x1 = b->ar.alloc<float>(N * W * nmel * 3, &rc);
    b->e_h1 = b->ar.alloc<float>(N * W * st, &rc);
    b->e_x2 = b->ar.alloc<float>(N * ctx * st * 3, &rc);
    b->e_x = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_cur = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_q = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_k = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_v = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_att = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_ff = b->ar.alloc<float>(N * ctx * 4 * st, &rc);
    b->e_qh = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_kh = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_vt = b->ar.alloc<float>(N * ctx * st, &rc);
    b->e_sc = b->ar.alloc<float>(size_t(b->enc_chunk) * nh * ctx * ctx, &rc);
    if (rc) {
      b->e_x = nullptr;
      return rc;
    }
  }
  cudaStream_t s = b->st;
  // conv1 + GELU, conv2 + GELU + positions
  launch_wenc_conv1(d_mel, b->e_x1, nmel, n, s);
  enc_product(b, b->e_x1, nmel * 3, W, m->conv1, m->conv1b, WM_GELU, b->e_h1, st, n);
  launch_wenc_conv2(b->e_h1, b->e_x2, st, ctx, n, s);
  enc_product(b, b->e_x2, st * 3, ctx, m->conv2, m->conv2b, WM_GELU_ADD, b->e_x, st, n, m->enc_pos);
  b->launches += 2;
  const float sc = float(1 / std::sqrt(double(hd)));
  for (const WEncDev& L : m->enc) {
    launch_wln(b->e_x, b->e_cur, L.attn_ln_w, L.attn_ln_b, n * ctx, st, s);
    enc_product(b, b->e_cur, st, ctx, L.q, L.qb, WM_STORE, b->e_q, st, n);
    enc_product(b, b->e_cur, st, ctx, L.k, nullptr, WM_STORE, b->e_k, st, n);
    enc_product(b, b->e_cur, st, ctx, L.v, L.vb, WM_STORE, b->e_v, st, n);
    launch_wenc_heads(b->e_q, b->e_k, b->e_v, b->e_qh, b->e_kh, b->e_vt, ctx, st, nh, sc, n, s);
    b->launches += 2;
    for (int c0 = 0; c0 < n; c0 += b->enc_chunk) {
      const int cn = std::min(b->enc_chunk, n - c0), z0 = c0 * nh;
      // scores = qh·khᵀ per (stream, head), then the rows' softmax
      WmmArgs p;
      p.a = b->e_qh + size_t(z0) * ctx * hd;
      p.lda = hd;
      p.a_zs = size_t(ctx) * hd;
      p.m = ctx;
      p.w.f = b->e_kh + size_t(z0) * ctx * hd;
      p.w.rows = ctx;
      p.w.cols = hd;
      p.w_zs = size_t(ctx) * hd;
      p.c = b->e_sc;
      p.ldc = ctx;
      p.c_zs = size_t(ctx) * ctx;
      launch_wmm(p, cn * nh, s);
      launch_wenc_softmax(b->e_sc, ctx, long(cn) * nh * ctx, s);
      // oh = scores·vtᵀ, into the heads' columns of att
      for (int i = 0; i < cn; i++) {
        WmmArgs o;
        o.a = b->e_sc + size_t(i) * nh * ctx * ctx;
        o.lda = ctx;
        o.a_zs = size_t(ctx) * ctx;
        o.m = ctx;
        o.w.f = b->e_vt + size_t(c0 + i) * nh * hd * ctx;
        o.w.rows = hd;
        o.w.cols = ctx;
        o.w_zs = size_t(hd) * ctx;
        o.c = b->e_att + size_t(c0 + i) * ctx * st;
        o.ldc = st;
        o.c_zs = size_t(hd);
        launch_wmm(o, nh, s);
        b->launches++;
      }
      b->launches += 2;
    }
    enc_product(b, b->e_att, st, ctx, L.o, L.ob, WM_RESID, b->e_x, st, n);
    launch_wln(b->e_x, b->e_cur, L.mlp_ln_w, L.mlp_ln_b, n * ctx, st, s);
    enc_product(b, b->e_cur, st, ctx, L.fc1, L.fc1b, WM_GELU, b->e_ff, 4 * st, n);
    enc_product(b, b->e_ff, 4 * st, ctx, L.fc2, L.fc2b, WM_RESID, b->e_x, st, n);
    b->launches += 2;
  }
  launch_wln(b->e_x, b->enc, m->enc_ln_w, m->enc_ln_b, n * ctx, st, s);
  b->launches++;
  CK(cudaGetLastError());
  return GRX_OK;
}

}  // namespace

extern "C" {

int grx_whisper_encode(grx_whisper_batch* b, const float* mel) {
  if (!b || !mel) return fail(GRX_EINVAL, "grx_whisper_encode: null argument");
  const grx_whisper* m = b->m;
  if (!m->has_enc) return fail(GRX_EINVAL, "grx_whisper_encode: the model file has no encoder");
  CK(cudaSetDevice(b->ar.dev));
  const size_t nm = size_t(b->n) * m->n_mels * 3000;
  int rc = 0;
  if (!b->e_mel) b->e_mel = b->ar.alloc<float>(nm, &rc);
  if (rc) return rc;
  CK(cudaMemcpyAsync(b->e_mel, mel, sizeof(float) * nm, cudaMemcpyHostToDevice, b->st));
  rc = encode(b, b->e_mel);
  if (rc) return rc;
  return set_audio(b, b->enc);
}

int grx_whisper_encode_device(grx_whisper_batch* b, const float* d_mel) {
  if (!b || !d_mel) return fail(GRX_EINVAL, "grx_whisper_encode_device: null argument");
  if (!b->m->has_enc) return fail(GRX_EINVAL, "grx_whisper_encode_device: the model file has no encoder");
  CK(cudaSetDevice(b->ar.dev));
  int rc = encode(b, d_mel);
  if (rc) return rc;
  return set_audio(b, b->enc);
}

int grx_whisper_encoder_out(grx_whisper_batch* b, float* out) {
  if (!b || !out) return fail(GRX_EINVAL, "grx_whisper_encoder_out: null argument");
  CK(cudaSetDevice(b->ar.dev));
  CK(cudaMemcpyAsync(out, b->enc, sizeof(float) * layer_stride_cross(b->m, b->n), cudaMemcpyDeviceToHost, b->st));
  CK(cudaStreamSynchronize(b->st));
  return GRX_OK;
}

int grx_whisper_set_audio(grx_whisper_batch* b, const float* enc) {
  if (!b || !enc) return fail(GRX_EINVAL, "grx_whisper_set_audio: null argument");
  CK(cudaSetDevice(b->ar.dev));
  CK(cudaMemcpyAsync(b->enc, enc, sizeof(float) * layer_stride_cross(b->m, b->n), cudaMemcpyHostToDevice, b->st));
  return set_audio(b, b->enc);
}

int grx_whisper_set_audio_device(grx_whisper_batch* b, const float* d_enc) {
  if (!b || !d_enc) return fail(GRX_EINVAL, "grx_whisper_set_audio_device: null argument");
  CK(cudaSetDevice(b->ar.dev));
  return set_audio(b, d_enc);
}

int grx_whisper_prompt(grx_whisper_batch* b, const int* prompt, int np, int sot_at, float* no_speech) {
  if (!b || !prompt || np <= 0 || sot_at < 0 || sot_at >= np) return fail(GRX_EINVAL, "grx_whisper_prompt: bad argument");
  const grx_whisper* m = b->m;
  if (b->pos + np > m->n_text_ctx) return fail(GRX_ERANGE, "whisper: prompt too long");
  for (int i = 0; i < b->n * np; i++)
    if (prompt[i] < 0 || prompt[i] >= m->n_vocab) return fail(GRX_EINVAL, "grx_whisper_prompt: token out of range");
  CK(cudaSetDevice(b->ar.dev));
  int rc = prefill(b, prompt, np, sot_at);
  if (rc) return rc;
  if (no_speech) CK(cudaMemcpy(no_speech, b->no_speech, sizeof(float) * size_t(b->n), cudaMemcpyDeviceToHost));
  CK(cudaGetLastError());
  return GRX_OK;
}

// `steps` rounds of sample then decode of the sampled token, with the
// outputs left in the batch's run buffer.
static int run(grx_whisper_batch* b, int steps) {
  if (steps <= 0) return fail(GRX_EINVAL, "grx_whisper_run: steps must be positive");
  // every step decodes its token at the next position (decoder.go:41-43)
  if (b->pos == 0) return fail(GRX_EINVAL, "grx_whisper_run: no prompt decoded since the window was set");
  if (b->pos + steps > b->m->n_text_ctx)
    return fail(GRX_ERANGE, "grx_whisper_run: " + std::to_string(b->pos + steps) + " positions exceed the text context of " +
                                std::to_string(b->m->n_text_ctx));
  int rc = ensure_run_out(b, steps);
  if (rc) return rc;
  if (b->ws1) {  // the whole run in one launch
    if (b->ws1_out != b->run_out) {
      CK(cudaStreamSynchronize(b->st));
      CK(cudaMemcpy(&b->ws1_args->out, &b->run_out, sizeof(int*), cudaMemcpyHostToDevice));
      b->ws1_out = b->run_out;
    }
    CK(cudaMemsetAsync(b->ws1_bar, 0, sizeof(unsigned), b->st));
    CK(cudaMemsetAsync(b->step, 0, sizeof(int), b->st));
    CK(launch_wstep1(b->ws1_args, b->ws1_grid, b->ws1_smem, b->pos, steps, b->st));
    b->launches += 1;
    b->pos += steps;
    return GRX_OK;
  }
  if (!b->g_step) {
    rc = capture(b, true, &b->g_step);
    if (rc) return rc;
  }
  CK(cudaMemsetAsync(b->step, 0, sizeof(int), b->st));
  for (int i = 0; i < steps; i++) {
    CK(cudaGraphLaunch(b->g_step, b->st));
    b->launches += b->per_decode;
  }
  b->pos += steps;
  CK(cudaGetLastError());
  return GRX_OK;
}

int grx_whisper_run(grx_whisper_batch* b, int steps, int* tokens) {
  if (!b || !tokens) return fail(GRX_EINVAL, "grx_whisper_run: null argument");
  CK(cudaSetDevice(b->ar.dev));
  int rc = run(b, steps);
  if (rc) return rc;
  CK(cudaMemcpyAsync(tokens, b->run_out, sizeof(int) * 4 * size_t(steps) * b->n, cudaMemcpyDeviceToHost, b->st));
  CK(cudaStreamSynchronize(b->st));
  return ws1_check(b);
}

int grx_whisper_run_device(grx_whisper_batch* b, int steps, int* d_tokens) {
  if (!b || !d_tokens) return fail(GRX_EINVAL, "grx_whisper_run_device: null argument");
  CK(cudaSetDevice(b->ar.dev));
  int rc = run(b, steps);
  if (rc) return rc;
  CK(cudaMemcpyAsync(d_tokens, b->run_out, sizeof(int) * 4 * size_t(steps) * b->n, cudaMemcpyDeviceToDevice, b->st));
  return GRX_OK;
}

int grx_whisper_sync(grx_whisper_batch* b) {
  if (!b) return fail(GRX_EINVAL, "null batch");
  CK(cudaSetDevice(b->ar.dev));
  CK(cudaStreamSynchronize(b->st));
  CK(cudaGetLastError());
  return ws1_check(b);
}

int grx_whisper_persistent(const grx_whisper_batch* b) { return b && b->ws1 ? 1 : 0; }

int grx_whisper_watchdog_test(grx_whisper_batch* b) {
  if (!b) return fail(GRX_EINVAL, "null batch");
  if (!b->ws1) return fail(GRX_EINVAL, "grx_whisper_watchdog_test: the batch does not run the persistent kernel");
  if (b->pos == 0 || b->pos + 1 > b->m->n_text_ctx) return fail(GRX_EINVAL, "grx_whisper_watchdog_test: decode a prompt first");
  CK(cudaSetDevice(b->ar.dev));
  int rc = ensure_run_out(b, 1);
  if (rc) return rc;
  // one step whose first grid barrier nothing completes
  const int one = 1, zero = 0;
  CK(cudaStreamSynchronize(b->st));
  if (b->ws1_out != b->run_out) {
    CK(cudaMemcpy(&b->ws1_args->out, &b->run_out, sizeof(int*), cudaMemcpyHostToDevice));
    b->ws1_out = b->run_out;
  }
  CK(cudaMemcpy(&b->ws1_args->stall, &one, sizeof one, cudaMemcpyHostToDevice));
  CK(cudaMemset(b->ws1_bar, 0, sizeof(unsigned)));
  const cudaError_t e = launch_wstep1(b->ws1_args, b->ws1_grid, b->ws1_smem, b->pos, 1, b->st);
  const cudaError_t e2 = cudaStreamSynchronize(b->st);
  CK(cudaMemcpy(&b->ws1_args->stall, &zero, sizeof zero, cudaMemcpyHostToDevice));
  CK(e);
  CK(e2);
  return ws1_check(b);
}

// The stream's cross K ([heads][ctx][hd], scaled) and Vᵀ ([heads][hd][ctx]) of a layer.
int grx_whisper_cross(grx_whisper_batch* b, int i, int layer, float* k, float* vt) {
  if (!b || i < 0 || i >= b->n || layer < 0 || layer >= b->m->n_text_layer) return fail(GRX_EINVAL, "grx_whisper_cross: bad argument");
  CK(cudaSetDevice(b->ar.dev));
  const size_t one = size_t(b->m->n_audio_ctx) * b->m->n_state;
  const size_t o = size_t(layer) * layer_stride_cross(b->m, b->n) + size_t(i) * one;
  if (k) CK(cudaMemcpy(k, b->ck + o, one * 4, cudaMemcpyDeviceToHost));
  if (vt) CK(cudaMemcpy(vt, b->cvt + o, one * 4, cudaMemcpyDeviceToHost));
  return GRX_OK;
}

// The logits left by the last decode, [n][vocab] (the rules of the next
// sample not yet applied).
int grx_whisper_logits(grx_whisper_batch* b, float* out) {
  if (!b || !out) return fail(GRX_EINVAL, "grx_whisper_logits: null argument");
  CK(cudaSetDevice(b->ar.dev));
  CK(cudaStreamSynchronize(b->st));
  CK(cudaMemcpy(out, b->logits, sizeof(float) * size_t(b->n) * b->m->n_vocab, cudaMemcpyDeviceToHost));
  return GRX_OK;
}

void* grx_whisper_batch_cuda_stream(const grx_whisper_batch* b) { return b ? (void*)b->st : nullptr; }

int64_t grx_whisper_batch_launches(const grx_whisper_batch* b) { return b ? b->launches : -1; }

}  // extern "C"
