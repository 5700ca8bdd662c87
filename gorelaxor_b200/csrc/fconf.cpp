// The FastConformer encoder on the device (grx_fconf_*): the encoder half of
// conformer.FromGGUF (conformer/model.go:160-189, 350-410) and Model.encode
// (encoder.go:123-489) for the offline case — "regular" attention over all
// frames of the utterance, non-causal subsampling — one utterance per call.
// The loader does what the reference's does to the weights: the
// subsampling and depthwise taps transposed to [taps][channels], batch norm
// folded into a scale and bias, every matrix on the int8 path (the
// reference packs them and drops their rows), the conv module's float16
// 1×1 convolutions rounded by ToQ8 when the rest of the file is Q8_0.
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

struct FFW {
  float *nw = nullptr, *nb = nullptr, *b1 = nullptr, *b2 = nullptr;
  DQ8 w1, w2;
};

struct FBlock {
  FFW ff1, ff2;
  float *na_w, *na_b, *nc_w, *nc_b, *no_w, *no_b;
  DQ8 q, k, v, out, pos, pw1, pw2;
  float *qb = nullptr, *kb = nullptr, *vb = nullptr, *outb = nullptr, *pu = nullptr, *pv = nullptr;
  float *pw1b = nullptr, *pw2b = nullptr, *dw = nullptr, *dwb = nullptr, *cnw = nullptr, *cnb = nullptr;
};

int sub_out(int n) { return (n - 1) / 2 + 1; }

// Weight.ToQ8 (kern.go:139-170): each 32-value block scaled by its largest
// magnitude over 127 (float32 division), values rounded half away from zero,
// the scale stored as f16. Returns 34-byte blocks.
std::vector<uint8_t> to_q8_blocks(const std::vector<float>& v, int rows, int cols) {
  const int nb = cols / 32;
  std::vector<uint8_t> out(size_t(rows) * nb * 34);
  for (int j = 0; j < rows; j++)
    for (int b = 0; b < nb; b++) {
      const float* xs = &v[size_t(j) * cols + size_t(b) * 32];
      uint8_t* blk = &out[(size_t(j) * nb + b) * 34];
      float amax = 0.f;
      for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(xs[i]));
      const float d = amax / 127.f;
      const float id = d != 0.f ? 1.f / d : 0.f;
      const uint16_t h = f32_to_f16(d);
      blk[0] = uint8_t(h & 0xff);
      blk[1] = uint8_t(h >> 8);
      for (int i = 0; i < 32; i++) {
        const float p = xs[i] * id;
        blk[2 + i] = uint8_t(int8_t(std::round(double(p))));
      }
    }
  return out;
}

}  // namespace

struct grx_fconf {
  Arena ar;
  int dev = 0;
  int d = 0, heads = 0, layers = 0, dff = 0, kernel = 0, sub_c = 0, n_mels = 0, pad_l = 0;
  bool xscaling = false, ln_conv = false;
  float *w0 = nullptr, *b0 = nullptr, *w2 = nullptr, *b2 = nullptr, *w5 = nullptr, *b5 = nullptr;
  float *b3 = nullptr, *b6 = nullptr, *outb = nullptr;
  DQ8 w3, w6, out;
  std::vector<FBlock> blocks;
  cudaStream_t st = nullptr;
  // per-call work buffers, grown to the longest utterance seen
  Arena wk;
  long wk_frames = 0;
  float *mel = nullptr, *in = nullptr, *a = nullptr, *b = nullptr, *flat = nullptr, *x = nullptr, *ln = nullptr,
        *ff = nullptr, *tmp = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qu = nullptr, *qv = nullptr,
        *glu = nullptr, *conv = nullptr, *g = nullptr, *dwo = nullptr, *pos = nullptr, *pp = nullptr;
  int8_t* aq = nullptr;
  float2* as = nullptr;
  int64_t launches = 0;
  ~grx_fconf() {
    cudaSetDevice(ar.dev);
    if (st) cudaStreamDestroy(st);
  }
};

namespace {

// y = x·Wᵀ (+ bias), or y += (resid), on the int8 path for M rows.
void q8_product(grx_fconf* m, const float* x, int M, const DQ8& w, const float* bias, float* y, bool resid) {
  const int K = w.cols, N = w.rows;
  launch_quant(x, M, K, m->aq, m->as, m->st);
  EpiArgs e;
  e.epi = resid ? EPI_RESID : EPI_STORE;
  e.bias = bias;
  e.ldy = N;
  m->launches++;
  if (M <= 8 || K % 64 == 0) {
    e.y = y;
    launch_q8_product(m->aq, m->as, M, w, e, m->st);
    m->launches++;
    return;
  }
  for (int r = 0; r < M; r += 8) {
    e.y = y + size_t(r) * N;
    launch_q8_product(m->aq + size_t(r) * K, m->as + size_t(r) * (K / 32), std::min(8, M - r), w, e, m->st);
    m->launches++;
  }
}

int ensure_work(grx_fconf* m, int frames) {
  if (frames <= m->wk_frames) return GRX_OK;
  cudaStreamSynchronize(m->st);  // the old buffers may still be in use
  for (void* q : m->wk.ptrs) cudaFree(q);
  m->wk.ptrs.clear();
  m->wk.bytes = 0;
  int rc = 0;
  const int nm = m->n_mels, c = m->sub_c, D = m->d;
  const int T1 = sub_out(frames), F1 = sub_out(nm), T = sub_out(sub_out(T1)), F3 = sub_out(sub_out(F1));
  const size_t big = size_t(T1) * F1 * c;  // the largest subsampling activation
  Arena& a = m->wk;
  m->mel = a.alloc<float>(size_t(nm) * frames, &rc);
  m->in = a.alloc<float>(size_t(nm) * frames, &rc);
  m->a = a.alloc<float>(big, &rc);
  m->b = a.alloc<float>(big, &rc);
  m->flat = a.alloc<float>(size_t(T) * c * F3, &rc);
  const size_t td = size_t(T) * D;
  m->x = a.alloc<float>(td, &rc);
  m->ln = a.alloc<float>(td, &rc);
  m->ff = a.alloc<float>(size_t(T) * m->dff, &rc);
  m->tmp = a.alloc<float>(td, &rc);
  m->q = a.alloc<float>(td, &rc);
  m->k = a.alloc<float>(td, &rc);
  m->v = a.alloc<float>(td, &rc);
  m->qu = a.alloc<float>(td, &rc);
  m->qv = a.alloc<float>(td, &rc);
  m->glu = a.alloc<float>(td, &rc);
  m->conv = a.alloc<float>(2 * td, &rc);
  m->g = a.alloc<float>(td, &rc);
  m->dwo = a.alloc<float>(td, &rc);
  m->pos = a.alloc<float>(size_t(2 * T - 1) * D, &rc);
  m->pp = a.alloc<float>(size_t(2 * T - 1) * D, &rc);
  size_t qk = std::max({big, size_t(T) * c * F3, size_t(T) * m->dff, size_t(2 * T - 1) * D, 2 * td});
  m->aq = a.alloc<int8_t>(qk, &rc);
  m->as = a.alloc<float2>(qk / 32 + 1, &rc);
  if (rc) {
    m->wk_frames = 0;
    return rc;
  }
  m->wk_frames = frames;
  return GRX_OK;
}

// relPosEmb (encoder.go:171-194): rows for positions n − 1 down to −(n − 1).
std::vector<float> rel_pos_emb(int n, int d) {
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

void feed_forward(grx_fconf* m, const FFW& w, int T) {
  const int D = m->d;
  launch_wln(m->x, m->ln, w.nw, w.nb, T, D, m->st);
  q8_product(m, m->ln, T, w.w1, w.b1, m->ff, false);
  launch_fc_silu(m->ff, long(T) * m->dff, m->st);
  q8_product(m, m->ff, T, w.w2, w.b2, m->tmp, false);
  launch_fc_axpy_half(m->x, m->tmp, long(T) * D, m->st);
  m->launches += 3;
}

// Model.encode (encoder.go:436-489) of d_mel [n_mels][frames] into m->x
// ([T][d]); returns the valid rows L through *L.
int encode(grx_fconf* m, const float* d_mel, int frames, int valid, int* Lo) {
  const int nm = m->n_mels, c = m->sub_c, D = m->d;
  cudaStream_t st = m->st;
  // subsample (encoder.go:123-168)
  launch_fc_mel_in(d_mel, m->in, frames, nm, valid, st);
  int T = frames, F = nm, L = valid;
  int T1 = sub_out(T), F1 = sub_out(F);
  L = sub_out(L);
  launch_fc_conv0(m->in, T, F, m->w0, m->b0, c, m->a, T1, F1, L, st);
  T = T1, F = F1, T1 = sub_out(T), F1 = sub_out(F);
  L = sub_out(L);
  launch_fc_dwconv2(m->a, T, F, c, m->w2, m->b2, m->b, T1, F1, L, st);
  T = T1, F = F1;
  q8_product(m, m->b, T * F, m->w3, m->b3, m->a, false);
  launch_fc_mask_relu(m->a, long(T) * F * c, long(F) * c, L, st);
  T1 = sub_out(T), F1 = sub_out(F);
  L = sub_out(L);
  launch_fc_dwconv2(m->a, T, F, c, m->w5, m->b5, m->b, T1, F1, L, st);
  T = T1, F = F1;
  q8_product(m, m->b, T * F, m->w6, m->b6, m->a, false);
  launch_fc_mask_relu(m->a, long(T) * F * c, long(F) * c, L, st);
  launch_fc_flatten(m->a, m->flat, T, F, c, st);
  q8_product(m, m->flat, T, m->out, m->outb, m->x, false);
  m->launches += 7;
  L = std::max(0, std::min(L, T));
  if (m->xscaling) {
    launch_fc_scale(m->x, long(T) * D, float(std::sqrt(double(D))), st);
    m->launches++;
  }
  // the position table, projected per block
  {
    const std::vector<float> pos = rel_pos_emb(T, D);
    CK(cudaMemcpyAsync(m->pos, pos.data(), sizeof(float) * pos.size(), cudaMemcpyHostToDevice, st));
    CK(cudaStreamSynchronize(st));  // pos is a local
  }
  const float scale = float(1 / std::sqrt(double(D / m->heads)));
  for (const FBlock& b : m->blocks) {
    q8_product(m, m->pos, 2 * T - 1, b.pos, nullptr, m->pp, false);
    feed_forward(m, b.ff1, T);
    launch_wln(m->x, m->ln, b.na_w, b.na_b, T, D, st);
    q8_product(m, m->ln, T, b.q, b.qb, m->q, false);
    q8_product(m, m->ln, T, b.k, b.kb, m->k, false);
    q8_product(m, m->ln, T, b.v, b.vb, m->v, false);
    launch_fc_qpos(m->q, b.pu, b.pv, m->qu, m->qv, long(T) * D, D, st);
    launch_fc_attn(m->qu, m->qv, m->k, m->v, m->pp, m->glu, T, D, m->heads, L, scale, st);
    q8_product(m, m->glu, T, b.out, b.outb, m->x, true);
    launch_wln(m->x, m->ln, b.nc_w, b.nc_b, T, D, st);
    q8_product(m, m->ln, T, b.pw1, b.pw1b, m->conv, false);
    launch_fc_glu(m->conv, m->g, T, D, L, st);
    launch_fc_dwconv(m->g, b.dw, b.dwb, b.cnw, b.cnb, m->dwo, T, D, m->kernel, m->pad_l, !m->ln_conv, st);
    if (m->ln_conv) {
      launch_wln(m->dwo, m->dwo, b.cnw, b.cnb, T, D, st);
      launch_fc_silu(m->dwo, long(T) * D, st);
      m->launches += 2;
    }
    q8_product(m, m->dwo, T, b.pw2, b.pw2b, m->x, true);
    feed_forward(m, b.ff2, T);
    launch_wln(m->x, m->x, b.no_w, b.no_b, T, D, st);
    m->launches += 7;
  }
  CK(cudaGetLastError());
  *Lo = L;
  return GRX_OK;
}

}  // namespace

extern "C" {

int grx_fconf_load(const void* bytes, size_t len, int device, grx_fconf** out) {
  if (!bytes || !out) return fail(GRX_EINVAL, "grx_fconf_load: null argument");
  int rc = device_init(device);
  if (rc) return rc;
  GGUF f;
  if (!f.parse(bytes, len)) return fail(GRX_EFORMAT, f.err);
  if (f.get_string("general.architecture", "") != "parakeet")
    return fail(GRX_EFORMAT, "conformer: the file isn't a FastConformer transducer");
  auto m = std::make_unique<grx_fconf>();
  m->ar.dev = m->dev = device;
  m->wk.dev = device;
  // readEncoder, model.go:162-189
  const std::string p = "stt.parakeet.encoder.";
  m->d = int(f.get_int(p + "d_model", 0));
  m->heads = int(f.get_int(p + "n_heads", 0));
  m->layers = int(f.get_int(p + "n_layers", 0));
  m->dff = int(f.get_int(p + "d_ff", 0));
  m->kernel = int(f.get_int(p + "conv_kernel", 0));
  m->sub_c = int(f.get_int(p + "subsampling_channels", 0));
  const int sub = int(f.get_int(p + "subsampling_factor", 8));
  m->xscaling = f.get_int(p + "xscaling", 0) != 0;
  const std::string style = f.get_string(p + "att_context_style", "regular");
  const int att_l = int(f.get_int(p + "att_context_left", -1)), att_r = int(f.get_int(p + "att_context_right", -1));
  const int conv_l = int(f.get_int(p + "conv_context_left", -1)), conv_r = int(f.get_int(p + "conv_context_right", -1));
  std::string norm = f.get_string(p + "conv_norm_type", "batch_norm");
  if (norm.empty()) norm = "batch_norm";
  const bool causal_sub = f.get_int(p + "causal_downsampling", style == "chunked_limited" ? 1 : 0) != 0;
  m->n_mels = int(f.get_int("stt.frontend.num_mels", 80));
  if (m->d <= 0 || m->heads <= 0 || m->d % m->heads != 0 || m->layers <= 0 || m->kernel <= 0)
    return fail(GRX_EFORMAT, "conformer: the model file is missing its encoder settings");
  if (sub != 8) return fail(GRX_EFORMAT, "conformer: subsampling " + std::to_string(sub) + " is not supported (only 8)");
  if (style != "regular" || (att_l >= 0 && att_r >= 0) || causal_sub)
    return fail(GRX_EINVAL, "conformer: this build runs the offline encoder (regular attention over all frames, "
                            "non-causal subsampling)");
  const int hd = m->d / m->heads;
  if (hd > 128 || hd % 4 || m->d % 64 || m->dff % 64 || m->sub_c % 64 || m->n_mels < 1 || m->n_mels > 512 ||
      m->kernel > 64 || m->d > 8192)
    return fail(GRX_EINVAL, "conformer: encoder dimensions outside what the kernels take");
  m->ln_conv = norm == "layer_norm";
  m->pad_l = conv_l >= 0 && conv_r >= 0 ? conv_l : (m->kernel - 1) / 2;
  std::string err;
  auto vec = [&](const std::string& name, int64_t n, bool optional) -> std::vector<float> {
    std::vector<float> v;
    if (!err.empty()) return v;
    if (!f.has(name)) {
      if (!optional) err = "conformer: the model has no " + name;
      return v;
    }
    if (!f.float32(name, v) || int64_t(v.size()) != n) err = "conformer: " + name + " has the wrong size";
    return v;
  };
  auto up = [&](const std::vector<float>& v) -> float* {
    return v.empty() ? nullptr : m->ar.upload(v.data(), v.size(), &rc);
  };
  auto taps = [&](const std::string& name, int ch, int nt) -> float* {  // transposeTaps
    const std::vector<float> v = vec(name, int64_t(ch) * nt, false);
    if (v.empty()) return nullptr;
    std::vector<float> t(v.size());
    for (int i = 0; i < ch; i++)
      for (int j = 0; j < nt; j++) t[size_t(j) * ch + i] = v[size_t(i) * nt + j];
    return up(t);
  };
  bool float_model = false;
  auto mat = [&](const std::string& name, int64_t rows, int64_t cols, bool to_q8) -> DQ8 {
    if (!err.empty()) return DQ8{};
    int64_t r = 0, c = 0;
    if (!f.matrix_shape(name, &r, &c)) {
      err = "conformer: the model has no " + name;
      return DQ8{};
    }
    if (r != rows || c != cols) {
      err = "conformer: " + name + " is " + std::to_string(r) + "x" + std::to_string(c) + ", want " +
            std::to_string(rows) + "x" + std::to_string(cols);
      return DQ8{};
    }
    const GTensor& t = f.tensors.at(name);
    if (t.type == G_Q8_0) return upload_q8(m->ar, t.data, int(rows), int(cols), &rc);
    if (to_q8 && cols % 32 == 0) {  // ToQ8 at load (model.go:391-396)
      std::vector<float> v;
      f.float32(name, v);
      const std::vector<uint8_t> q = to_q8_blocks(v, int(rows), int(cols));
      return upload_q8(m->ar, q.data(), int(rows), int(cols), &rc);
    }
    float_model = true;
    return DQ8{};
  };
  const int c = m->sub_c, D = m->d;
  int F = m->n_mels;
  for (int i = 0; i < 3; i++) F = sub_out(F);
  const std::string pe = "enc.pre_encode.";
  m->w0 = taps(pe + "conv.0.weight", c, 9);
  m->b0 = up(vec(pe + "conv.0.bias", c, false));
  m->w2 = taps(pe + "conv.2.weight", c, 9);
  m->b2 = up(vec(pe + "conv.2.bias", c, false));
  m->w3 = mat(pe + "conv.3.weight", c, c, false);
  m->b3 = up(vec(pe + "conv.3.bias", c, false));
  m->w5 = taps(pe + "conv.5.weight", c, 9);
  m->b5 = up(vec(pe + "conv.5.bias", c, false));
  m->w6 = mat(pe + "conv.6.weight", c, c, false);
  m->b6 = up(vec(pe + "conv.6.bias", c, false));
  m->out = mat(pe + "out.weight", D, int64_t(c) * F, false);
  m->outb = up(vec(pe + "out.bias", D, false));
  for (int i = 0; i < m->layers && err.empty(); i++) {
    const std::string bp = "enc.blocks." + std::to_string(i) + ".";
    FBlock b;
    auto ff = [&](const std::string& n) {
      FFW w;
      w.nw = up(vec(bp + "norm_" + n + ".weight", D, false));
      w.nb = up(vec(bp + "norm_" + n + ".bias", D, false));
      w.w1 = mat(bp + n + ".linear1.weight", m->dff, D, false);
      w.b1 = up(vec(bp + n + ".linear1.bias", m->dff, true));
      w.w2 = mat(bp + n + ".linear2.weight", D, m->dff, false);
      w.b2 = up(vec(bp + n + ".linear2.bias", D, true));
      return w;
    };
    b.ff1 = ff("ff1");
    b.ff2 = ff("ff2");
    b.na_w = up(vec(bp + "norm_attn.weight", D, false));
    b.na_b = up(vec(bp + "norm_attn.bias", D, false));
    b.q = mat(bp + "attn.linear_q.weight", D, D, false);
    b.qb = up(vec(bp + "attn.linear_q.bias", D, true));
    b.k = mat(bp + "attn.linear_k.weight", D, D, false);
    b.kb = up(vec(bp + "attn.linear_k.bias", D, true));
    b.v = mat(bp + "attn.linear_v.weight", D, D, false);
    b.vb = up(vec(bp + "attn.linear_v.bias", D, true));
    b.out = mat(bp + "attn.linear_out.weight", D, D, false);
    b.outb = up(vec(bp + "attn.linear_out.bias", D, true));
    b.pos = mat(bp + "attn.linear_pos.weight", D, D, false);
    b.pu = up(vec(bp + "attn.pos_bias_u", D, false));
    b.pv = up(vec(bp + "attn.pos_bias_v", D, false));
    b.nc_w = up(vec(bp + "norm_conv.weight", D, false));
    b.nc_b = up(vec(bp + "norm_conv.bias", D, false));
    b.pw1 = mat(bp + "conv.pointwise1.weight", 2 * D, D, true);
    b.pw1b = up(vec(bp + "conv.pointwise1.bias", 2 * D, true));
    b.pw2 = mat(bp + "conv.pointwise2.weight", D, D, true);
    b.pw2b = up(vec(bp + "conv.pointwise2.bias", D, true));
    b.dw = taps(bp + "conv.depthwise.weight", D, m->kernel);
    b.dwb = up(vec(bp + "conv.depthwise.bias", D, true));
    b.no_w = up(vec(bp + "norm_out.weight", D, false));
    b.no_b = up(vec(bp + "norm_out.bias", D, false));
    const std::vector<float> gw = vec(bp + "conv.bn.weight", D, false), gb = vec(bp + "conv.bn.bias", D, false);
    if (m->ln_conv) {
      b.cnw = up(gw);
      b.cnb = up(gb);
    } else {
      const std::vector<float> mean = vec(bp + "conv.bn.running_mean", D, false);
      const std::vector<float> vr = vec(bp + "conv.bn.running_var", D, false);
      if (err.empty()) {
        std::vector<float> sw((size_t(D))), sb((size_t(D)));
        for (int j = 0; j < D; j++) {  // model.go:401-406
          const float s = float(double(gw[size_t(j)]) / std::sqrt(double(vr[size_t(j)]) + 1e-5));
          sw[size_t(j)] = s;
          const float ms = mean[size_t(j)] * s;
          sb[size_t(j)] = gb[size_t(j)] - ms;
        }
        b.cnw = up(sw);
        b.cnb = up(sb);
      }
    }
    m->blocks.push_back(b);
  }
  if (!err.empty()) return fail(GRX_EFORMAT, err);
  if (float_model)
    return fail(GRX_EINVAL, "conformer: this build runs encoders whose matrices are Q8_0 (the int8 path)");
  if (rc) return rc;
  CK(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking));
  *out = m.release();
  return GRX_OK;
}

void grx_fconf_free(grx_fconf* m) { delete m; }

int grx_fconf_dims(const grx_fconf* m, int* d_model, int* heads, int* layers, int* n_mels, int* sub_channels) {
  if (!m) return fail(GRX_EINVAL, "null model");
  if (d_model) *d_model = m->d;
  if (heads) *heads = m->heads;
  if (layers) *layers = m->layers;
  if (n_mels) *n_mels = m->n_mels;
  if (sub_channels) *sub_channels = m->sub_c;
  return GRX_OK;
}

int grx_fconf_out_rows(int frames) { return frames < 1 ? 0 : sub_out(sub_out(sub_out(frames))); }

static int fconf_check(grx_fconf* m, int frames, int valid) {
  if (frames < 1 || frames > (1 << 20) || valid < 0) return fail(GRX_EINVAL, "grx_fconf_encode: bad frame counts");
  return ensure_work(m, frames);
}

int grx_fconf_encode(grx_fconf* m, const float* mel, int frames, int valid, float* out, int* rows) {
  if (!m || !mel || !out) return fail(GRX_EINVAL, "grx_fconf_encode: null argument");
  CK(cudaSetDevice(m->dev));
  int rc = fconf_check(m, frames, valid);
  if (rc) return rc;
  CK(cudaMemcpyAsync(m->mel, mel, sizeof(float) * size_t(m->n_mels) * frames, cudaMemcpyHostToDevice, m->st));
  int L = 0;
  rc = encode(m, m->mel, frames, valid, &L);
  if (rc) return rc;
  CK(cudaMemcpyAsync(out, m->x, sizeof(float) * size_t(L) * m->d, cudaMemcpyDeviceToHost, m->st));
  CK(cudaStreamSynchronize(m->st));
  CK(cudaGetLastError());
  if (rows) *rows = L;
  return GRX_OK;
}

int grx_fconf_encode_device(grx_fconf* m, const float* d_mel, int frames, int valid, float* d_out, int* rows) {
  if (!m || !d_mel || !d_out) return fail(GRX_EINVAL, "grx_fconf_encode_device: null argument");
  CK(cudaSetDevice(m->dev));
  int rc = fconf_check(m, frames, valid);
  if (rc) return rc;
  int L = 0;
  rc = encode(m, d_mel, frames, valid, &L);
  if (rc) return rc;
  CK(cudaMemcpyAsync(d_out, m->x, sizeof(float) * size_t(L) * m->d, cudaMemcpyDeviceToDevice, m->st));
  if (rows) *rows = L;
  return GRX_OK;
}

int grx_fconf_sync(grx_fconf* m) {
  if (!m) return fail(GRX_EINVAL, "null model");
  CK(cudaSetDevice(m->dev));
  CK(cudaStreamSynchronize(m->st));
  CK(cudaGetLastError());
  return GRX_OK;
}

void* grx_fconf_cuda_stream(const grx_fconf* m) { return m ? (void*)m->st : nullptr; }

int64_t grx_fconf_launches(const grx_fconf* m) { return m ? m->launches : 0; }

}  // extern "C"
