// Host-side declarations of the token-loop kernels' launchers.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace grx {

// A Q8_0 weight on the device: int8 values [rows][cols] and the blocks'
// f16 scales [rows][cols/32], split from the 34-byte GGUF blocks so that
// both are 16-byte aligned for vector and async loads.
struct DQ8 {
  const int8_t* q = nullptr;
  const uint16_t* d = nullptr;
  // For the tensor-core product: per block dw and nm = −1.5·2^23·dw as
  // float32 (both exact; dw is a half), as quads per block and column pair
  // {dw[n], dw[n+1], nm[n], nm[n+1]} for n = 2p, [cols/32][(rows+1)/2] (the
  // second of an odd last row is 0).
  const float4* dwnm = nullptr;
  int rows = 0, cols = 0;
};

// What a Q8_0 product does with its outputs.
enum Epi {
  EPI_STORE = 0,    // y[m][n] = c (+ bias)
  EPI_RESID = 1,    // x[m][n] += c  (kern.Add after the product, nn.go:173-174, 178-179)
  EPI_ROPE_KV = 2,  // rotate q and k, append k and v to the cache (nn.go:153-171)
  EPI_GELU_Q8 = 3,  // GELU, then round each 32-block to Q8_0 for the next product (nn.go:176-178)
};

// Where the qkv product's outputs go (EPI_ROPE_KV).
struct KVArgs {
  float* q = nullptr;        // [M][d] rotated queries
  float* kv = nullptr;       // cache base: [M][L][2][H][cap][hd]
  const int* pos = nullptr;  // [M] position being written
  const float* rope = nullptr;  // [cap][hd/2][2] cos, sin
  int layer = 0, layers = 0, heads = 0, cap = 0, d = 0;
  // Rows of several positions per stream (text prefill): the cache slot of
  // row m is row_stream[m] (NULL: row m is stream m).
  const int* row_stream = nullptr;
  // A ring of this many positions (0: position p at row p); RoPE still
  // takes the position itself.
  int ring = 0;
};

struct EpiArgs {
  int epi = EPI_STORE;
  float* y = nullptr;  // STORE / RESID target, row stride ldy
  int ldy = 0;
  const float* bias = nullptr;
  int8_t* q8 = nullptr;  // GELU_Q8 outputs: values [M][N], scales [M][N/32]
  float2* q8s = nullptr;
  const float* ls = nullptr;  // RESID: y += ls[col]·c (addScaled, unfused) when set
  KVArgs kv;
};

// Per-frame inputs and outputs of a run, in device memory so that one
// captured frame graph serves every frame: the frame's slice of each array
// is base + frame·stride, and the last kernel of a frame moves `frame` on.
struct FrameIO {
  const float* noise;  // [frames][rows][ldim]
  float* latent;       // [frames][rows][ldim] (may be NULL)
  float* scaled;       // [frames][rows][ldim] (may be NULL)
  float* eos;          // [frames][rows] (may be NULL)
  int frame;
  // Optional instrumentation: per frame and layer, the attention kernel's
  // first CTA start and last CTA end (%globaltimer, ns) [frames][layers][2];
  // slots must start at {UINT64_MAX, 0}.
  unsigned long long* attn_ts;
  int rows;  // rows per frame in the arrays above (every stream of the job)
  int row0;  // this stream set's first row
  int part, parts;  // attn_ts is [frames][layers][parts][2]
};

// LayerNorm modes.
enum LnOut { LN_Q8 = 0, LN_F32 = 1, LN_MOD = 2 };

struct LnArgs {
  const float* x = nullptr;
  const float* w = nullptr;  // may be NULL (no affine)
  const float* b = nullptr;
  double eps = 1e-5;
  int mode = LN_Q8;
  int8_t* q8 = nullptr;
  float2* q8s = nullptr;
  float* y = nullptr;
  const float* mod = nullptr;  // LN_MOD: shift at mod[m*ldmod + shift], scale at +scale
  int ldmod = 0, shift = 0, scale = 0;
  // LN_F32 only, when eosw is set: the end-of-speech logit of each output
  // row, dotF32Go(y, eosw) + eosb (lm.go:193-194), to eos[m] and the frame's
  // io->eos slot; then pos[m] += 1 (the frame is done with the position).
  const float* eosw = nullptr;
  float eosb = 0.f;
  float* eos = nullptr;
  const FrameIO* io = nullptr;
  int* pos = nullptr;
};

void launch_ln(const LnArgs& a, int M, int D, cudaStream_t st);

// The widest Q8_0 row (values) the up-to-8-row product takes: its rows of
// activations sit in shared memory.
constexpr int kQ8GemvMaxK = 16384;

// Activation blocks rounded to Q8_0 travel as int8 values [M][K] and block
// scales [M][K/32], each scale stored twice as a float2 (s, s): the
// tensor-core product consumes it as one packed operand.
//
// C[M][N] = A·Wᵀ with the int8 path's arithmetic (q8int.go:148-223).
void launch_q8_product(const int8_t* a, const float2* as, int M, const DQ8& w, const EpiArgs& e, cudaStream_t st);

// Nonzero once a tensor-core product gave up on a wait (its outputs are then
// not written); read after the stream is synchronised.
int q8_tc_fault();

// The activations rounded to Q8_0 blocks (quantU8, q8int.go:88-105).
void launch_quant(const float* x, int M, int K, int8_t* q, float2* s, cudaStream_t st);

struct AttnArgs {
  const float* q = nullptr;   // [M][d]
  const float* kv = nullptr;  // cache, as KVArgs
  const int* pos = nullptr;   // [M]: keys 0..pos are attended
  float* out = nullptr;       // [M][d] (may be NULL)
  int8_t* q8 = nullptr;       // [M][d] output rounded to Q8_0 for attn_out
  float2* q8s = nullptr;      // [M][d/32]
  int layer = 0, layers = 0, heads = 0, cap = 0, d = 0;
  const FrameIO* io = nullptr;  // for io->attn_ts (may be NULL)
};

void launch_attn(const AttnArgs& a, int M, cudaStream_t st);

// transformer.attend for T queries per stream (text prefill, nn.go:200-243
// with T > 1): call-stream i owns rows row0[i] .. row0[i] + T[i] − 1 of q
// and the output, at positions pos0[i] ..; its keys are the cache slot
// slot[i]'s rows 0 .. pos0[i] + T[i] − 1 (already appended).
struct AttnRowsArgs {
  const float* q = nullptr;  // [R][d] rotated queries
  const float* kv = nullptr;
  const int *row0 = nullptr, *T = nullptr, *pos0 = nullptr, *slot = nullptr;
  float* out = nullptr;  // [R][d] (may be NULL)
  int8_t* q8 = nullptr;  // [R][d] output rounded to Q8_0
  float2* q8s = nullptr;
  int layer = 0, layers = 0, heads = 0, cap = 0, d = 0;
  // A context window (0: none): keys from max(0, pos0 − context + 1), query
  // p sees [max(that, p − context + 1), p]; and the cache as a ring of
  // `ring` positions (0: none).
  int context = 0, ring = 0;
  // Set by launch_attn_rows: score slots before the staged value rows (0: values read from the cache).
  int vstage = 0;
};

void launch_attn_rows(const AttnRowsArgs& a, int nstreams, int tmax, cudaStream_t st);
void attn_kernels_init();

// ---- Mimi's decoder (k_mimi.cu); rows [stream][time][channel], n streams ----
void launch_mimi_up(const float* z, const float* up, const float* part_in, float* x, float* part_out, int n, int S,
                    int C, cudaStream_t st);
// The ELU of each stream's len values (len % 4 == 0), in place when in == out.
void launch_mimi_elu(const float* in, float* out, int n, int len, cudaStream_t st);
// stage [n][P + T][C] = [carry_in; x or ELU(x)]; carry_out = its last P rows.
void launch_mimi_stage(const float* x, const float* carry_in, float* carry_out, float* stage, int n, int T, int C,
                       int P, bool elu, cudaStream_t st);
// gemvRows of a float32 weight of K < 16 columns for rows [off, T) of every
// stream (x rows at (s·sstride + t)·ldx; y [n][T][N], stored or added).
void launch_mimi_gemv_small(const float* x, int ldx, int sstride, int T, int off, const float* w, int N, int K,
                            const float* bias, float* y, bool resid, int n, cudaStream_t st);
// The row tables of a call of T rows per stream: rowslot[r] = r / T,
// crow0[i] = i·T, cT[i] = T, cslot[i] = i.
void launch_mimi_rowtab(int T, int n, int* rowslot, int* crow0, int* cT, int* cslot, cudaStream_t st);
// carry [n][P][C] = P copies of each stream's row 0 of x [n][T][C].
void launch_mimi_replicate(const float* x, int T, int C, float* carry, int P, int n, cudaStream_t st);
void launch_mimi_im2col(const float* x, const float* prev_in, float* prev_out, float* col, int n, int T, int cin, int k,
                        int stride, int dil, int P, cudaStream_t st);
// Q8_0 rounding of rows t < T of K values at x + (s·sstride + t)·ldx, ELU
// first when elu_len (> 0: the per-stream array length, x dense), into
// dense q [n·T][K], qs [n·T][K/32].
void launch_mimi_quant(const float* x, int ldx, int sstride, int n, int T, int K, int elu_len, int8_t* q, float2* qs,
                       cudaStream_t st);
// The packed-order float32 product over convolution windows (rows t < mf
// of each stream, y dense [n·T][N], stored or added to); row t's window is
// the K = k·cin values from window row t on: staged rows x + (s·sstride +
// t)·cin, or (virt) [carry_in (P); x or ELU(x)] read in place from dense x
// [n][T][cin], the next carry_out written on the way. mimi_fconv_fits says
// whether a shape fits.
struct FconvArgs {
  const float* x = nullptr;
  int sstride = 0, cin = 0, K = 0, T = 0, mf = 0;
  const float* w = nullptr;
  const float* bias = nullptr;
  int N = 0;
  float* y = nullptr;
  int resid = 0;
  int virt = 0, P = 0, elu = 0;
  const float* carry_in = nullptr;
  float* carry_out = nullptr;
  int ngp = 0;  // set by the launcher
};
bool mimi_fconv_fits(int cin, int K, int N);
void launch_mimi_fconv(const FconvArgs& a, int n, cudaStream_t st);
void launch_mimi_convtr(const float* z, const float* bias, const float* part_in, float* y, float* part_out, int n, int T,
                        int co, int k, int S, cudaStream_t st);
// rowpos[r] = pos[r / S] + r % S for the R rows of a call; pos[i] += S after it.
void launch_mimi_rows(const int* pos, int S, int R, int* rowpos, cudaStream_t st);
void launch_mimi_advance(int* pos, int S, int n, cudaStream_t st);
// The fade-in of each not yet started stream's frame (pcm [n][frame]); marks it started.
void launch_mimi_fade(float* pcm, int* started, int n, int frame, int fade, cudaStream_t st);
void mimi_kernels_init();

// x[r] = embedding row ids[r] (float32 rows of width d).
void launch_embed_rows(float* x, const float* embed, const int* ids, int rows, int d, cudaStream_t st);

// Float activations times a Q8_0 (rows kept), F32 or F16 matrix with the
// reference's float-path order (dot4q8avx / dot4f32avx / dot4f16avx,
// gemm.go:195-259; whisper/gemm.go:212-256).
enum FEpi {
  FE_BIAS = 0,    // y = dot + bias
  FE_COND = 1,    // y = silu(dot + bias + tc)        (lm.go:110-115 and :131-132 with one step)
  FE_SILU = 2,    // y = silu(dot + bias)             (lm.go:144-145)
  FE_GATE = 3,    // h += gate · (dot + bias)         (lm.go:146-149)
  FE_LATENT = 4,  // cur = noise + (dot + bias)/steps; latent, scaled  (lm.go:118-121; speak.go:165-168)
  FE_RESID = 5,   // y += dot + bias                  (whisper/decoder.go:89,121,129: matmul then addTo)
  FE_GELU = 6,    // y = geluAVX(dot + bias)          (whisper/decoder.go:127)
  FE_ROWPOS = 7,  // y[dst_row[m]·ldy + n] = dot + bias  (a cache row per input row)
  FE_QKV = 8,     // whisper's q, k, v stacked: q to y, k and v to their cache rows (decoder.go:62-68)
};

struct FArgs {
  int epi = FE_BIAS;
  const float* x = nullptr;  // [M][K], row stride ldx
  int ldx = 0;
  const int8_t* wq = nullptr;  // Q8_0 weight (values, scales), or
  const uint16_t* wd = nullptr;
  const float* wf = nullptr;  // F32 weight [N][K], or
  const uint16_t* wh = nullptr;  // F16 weight [N][K]
  // With wq: widen each value as the Whisper loader does, f16(q·d)
  // (whisper/model.go:486-490), and take the F16 product order.
  bool q8_as_f16 = false;
  const int* dst_row = nullptr;  // FE_ROWPOS: the destination row of each input row
  int N = 0, K = 0;
  const float* bias = nullptr;
  float* y = nullptr;  // [M][N], row stride ldy
  int ldy = 0;
  const float* aux = nullptr;  // tc [N] (COND); gate [M][ldaux] (GATE); noise (LATENT)
  int ldaux = 0;
  const float* mean = nullptr;  // LATENT: emb_mean, emb_std
  const float* stdv = nullptr;
  float* out2 = nullptr;  // LATENT: latent copy, scaled
  float* out3 = nullptr;
  float steps = 1.f;
  int M = 0;  // rows (streams); set by launch_flin
  // When set: x (FE_BIAS with x_noise) or aux (FE_LATENT with aux_noise)
  // is this frame's noise, and FE_LATENT also writes the frame's latent and
  // scaled rows to io.
  const FrameIO* io = nullptr;
  bool x_noise = false, aux_noise = false, io_out = false;
  // Row groups (FE_BIAS and FE_RESID only): logical row m is row
  // (m / rg_len)·rg_stride + rg_off + m % rg_len of x and row
  // (m / rg_len)·ry_stride + ry_off + m % rg_len of y (rg_len 0: row m).
  int rg_len = 0, rg_stride = 0, rg_off = 0, ry_stride = 0, ry_off = 0;
  // FE_QKV: the weight is three matrices of `seg` rows stacked (q, k, v).
  // Column c of the first goes to y[m·ldy + c] (+ qkv_bias[0][c]); of the
  // second and third to qkv_y[0] and qkv_y[1] at row dst_row[m] (stride
  // ldy), + qkv_bias[1] / [2] where given. `bias` stays null.
  int seg = 0;
  const float* qkv_bias[3] = {nullptr, nullptr, nullptr};
  float* qkv_y[2] = {nullptr, nullptr};
};

void launch_flin(const FArgs& a, int M, cudaStream_t st);

// io->frame += 1 (the end of a frame).
void launch_tick(FrameIO* io, cudaStream_t st);

// Per-device kernel attributes (dynamic shared memory limits).
void flow_kernels_init();
void flin_kernels_init();
// The largest K launch_flin takes with F32 and with Q8_0 weights.
int flin_max_k();
int flin_max_k_q8();

// The flow head's time conditioning (pockettts/lm.go:62-104) from the two
// embedders' MLP outputs: each row normalized (float64 mean, variance
// with n−1, + 1e-5) times alpha, then the two averaged.
void launch_time_norm(const float* y0, const float* y1, const float* a0, const float* a1, int N, int steps,
                      float* tc, cudaStream_t st);

// Elementwise: y = silu(y0 + tc) for decode steps beyond the first.
void launch_cond_step(const float* y0, const float* tc, float* sy, int M, int N, cudaStream_t st);


// ---- one stream's FlowLM frames in one persistent kernel (k_frame1.cu) ----
constexpr int F1_THREADS = 512, F1_SLOTS = 5, F1_MAX_LAYERS = 12, F1_MAX_DEPTH = 4;

struct F1Layer {
  const float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr;
  DQ8 qkv, out, ff1, ff2;
};
struct F1Res {
  const float *nw = nullptr, *nb = nullptr, *b1 = nullptr, *b2 = nullptr, *adab = nullptr;
  DQ8 fc1, fc2, ada;
};

// Everything the kernel reads and writes, in device memory (one copy per
// stream set); see engine.cpp for what each field is.
struct Frame1Args {
  int d = 0, heads = 0, ff = 0, L = 0, ldim = 0, fd = 0, depth = 0, cap = 0;
  F1Layer layers[F1_MAX_LAYERS];
  F1Res res[F1_MAX_DEPTH];
  const float *win = nullptr, *outw = nullptr, *outb = nullptr, *eosw = nullptr;
  float eosb = 0.f;
  const float *mean = nullptr, *stdv = nullptr;
  DQ8 cond, fada;
  const float *condb = nullptr, *fin = nullptr, *finb = nullptr, *fadab = nullptr, *fout = nullptr, *foutb = nullptr;
  const float* tc = nullptr;  // [fd]: the one decode step's time condition
  float* kv = nullptr;        // the stream's cache [L][2][H][cap][64]
  int* pos = nullptr;
  const float* rope = nullptr;
  float *x = nullptr, *q = nullptr, *att = nullptr, *lm_out = nullptr, *eos = nullptr, *lat = nullptr;
  int8_t* ffq = nullptr;
  float* ffs = nullptr;
  float *sy = nullptr, *h = nullptr, *mod = nullptr, *mod2 = nullptr, *mm = nullptr;
  FrameIO* io = nullptr;
  unsigned* bar = nullptr;  // grid barrier arrivals, zeroed before each launch
  int* err = nullptr;       // set when a bounded wait ran out
};

// Whether the model and set fit the kernel on a grid of G CTAs; its shared
// memory and weight slot size.
bool frame1_suits(const Frame1Args& A, size_t* smem, uint32_t* slot_bytes, int G);
int frame1_max_active(size_t smem);
// Queues `frames` frames (a cooperative launch of G CTAs); stall: the
// watchdog check, a run whose first grid barrier never completes.
cudaError_t launch_frame1(const Frame1Args* d_args, size_t smem, uint32_t slot_bytes, int G, int frames, int stall,
                          cudaStream_t st);

// ---- the FastConformer encoder (k_fconf.cu), one utterance, rows [time][channels] ----
void launch_fc_mel_in(const float* mel, float* in, int frames, int nm, int valid, cudaStream_t st);
void launch_fc_conv0(const float* in, int T, int F, const float* w, const float* b, int c, float* out, int T1, int F1,
                     int L, cudaStream_t st);
void launch_fc_dwconv2(const float* in, int T, int F, int c, const float* w, const float* b, float* out, int T1, int F1,
                       int L, cudaStream_t st);
void launch_fc_mask_relu(float* x, long n, long width, int L, cudaStream_t st);
void launch_fc_flatten(const float* y, float* flat, int T, int F, int c, cudaStream_t st);
void launch_fc_scale(float* x, long n, float s, cudaStream_t st);
void launch_fc_silu(float* x, long n, cudaStream_t st);
void launch_fc_axpy_half(float* x, const float* y, long n, cudaStream_t st);
void launch_fc_qpos(const float* q, const float* pu, const float* pv, float* qu, float* qv, long n, int D,
                    cudaStream_t st);
void launch_fc_glu(const float* a, float* g, int T, int D, int L, cudaStream_t st);
void launch_fc_dwconv(const float* g, const float* w, const float* dwb, const float* cnw, const float* cnb, float* out,
                      int T, int D, int K, int padL, bool bn_silu, cudaStream_t st);
void launch_fc_attn(const float* qu, const float* qv, const float* k, const float* v, const float* pp, float* out,
                    int T, int D, int H, int L, float scale, cudaStream_t st);
void fconf_kernels_init();

// ---- the greedy TDT / RNN-T decode loop (k_tdt.cu) ----
constexpr int TDT_MAX_LAYERS = 8, TDT_MAX_DURATIONS = 8;

// Device state of a batch of n decoder streams. Arrays indexed by stream s;
// the LSTM state is [2 halves][layers][n][H] (half cur[s] is the stream's
// DecoderState, the other one the prediction step's output).
struct TdtArgs {
  int n = 0, H = 0, layers = 0, V = 0, J = 0, nout = 0, ndur = 0, blank = 0, max_symbols = 0, tdt = 1, act = 0;
  int max_t = 0, cap = 0;
  int durations[TDT_MAX_DURATIONS] = {};
  const float* embed = nullptr;  // [V][H]
  DQ8 lstm_wx[TDT_MAX_LAYERS], lstm_wh[TDT_MAX_LAYERS];
  const float* lstm_b[TDT_MAX_LAYERS] = {};
  DQ8 jpred, jout;
  const float *jpred_b = nullptr, *jout_b = nullptr;
  const float* enc_proj = nullptr;  // [n][max_t][J]
  float* pred_proj = nullptr;       // [n][J]
  float* logits = nullptr;          // [n][nout]
  float *h = nullptr, *c = nullptr;
  int *cur = nullptr, *last = nullptr, *step = nullptr, *nsym = nullptr, *iter = nullptr, *ntok = nullptr;
  const int *T = nullptr, *frame_offset = nullptr;
  int* tokens = nullptr;  // [n][cap][4]: id, frame, duration, p (float bits)
  int *active = nullptr, *dirty = nullptr;  // [2][n] stream lists by iteration parity
  int* counts = nullptr;                    // [2][2]: active, dirty counts by parity
};

void tdt_kernels_init();
size_t tdt_lin_smem(int K, bool lstm);
void launch_tdt_begin(const TdtArgs& a, cudaStream_t st);
// One loop iteration for every stream on the parity's lists.
void launch_tdt_iteration(const TdtArgs& a, int parity, cudaStream_t st);


// ---- the Whisper text decoder's token loop (k_whisper.cu) ----
// A decoder weight matrix: Q8_0 values widened through f16(q·d) as the
// reference loads them, or float16.
struct WMat {
  const int8_t* q = nullptr;
  const uint16_t* d = nullptr;  // Q8_0 scales [rows][cols/32]
  const uint16_t* h = nullptr;  // or float16 values [rows][cols]
  const float* f = nullptr;     // or float32 values [rows][cols]
  int rows = 0, cols = 0;
};

// The rows of one call: row r is token row_tok[r] at position row_pos[r] of
// stream row_stream[r].
struct WRows {
  int rows = 0, st = 0, nh = 0, text_ctx = 0, audio_ctx = 0, vocab = 0;
  const int *row_stream = nullptr, *row_pos = nullptr, *row_tok = nullptr;
};

// Sampling state of a stream (transcribe.go:56-64): sampled so far, the last
// two tokens, timestamps seen, the window's seek delta.
struct WSample {
  int nt, last, penult, has_ts, seek_delta;
};

// The vocabulary's special tokens and the suppressed ones (vocab.go).
struct WVocabDev {
  int n = 0, n_lang = 0, eot = 0, sot = 0, translate = 0, transcribe = 0, solm = 0, prev = 0, nosp = 0, not_ = 0, beg = 0,
      space = -1, n_suppress = 0;
  const int* suppress = nullptr;
  int audio_ctx = 1500;
  // Rows k_wproc recomputed in the reference's sequential order because a
  // parallel decision fell within its margin (device counter).
  unsigned long long* exact_rows = nullptr;
};

// ---- the token loop of one Whisper stream in one cooperative launch
constexpr int WS1_MAX_LAYERS = 12;
constexpr int WS1_MAX_GRID = 160;  // CTAs of the persistent Whisper kernel at most
struct WS1Layer {
  WMat q, k, v, o, xq, xo, fc1, fc2;
  const float *qb, *vb, *ob, *xqb, *xob, *fc1b, *fc2b;
  const float *ln1w, *ln1b, *ln2w, *ln2b, *ln3w, *ln3b;
  float *sk, *sv;           // the stream's self K / V caches [text_ctx][st]
  const float *ck, *cvt;    // its cross K [nh][ctx][64] (scaled) and Vᵀ [nh][64][ctx]
};
struct WStep1Args {
  int st = 0, nh = 0, ctx = 0, text_ctx = 0, ff = 0, L = 0, vocab = 0;
  WS1Layer layers[WS1_MAX_LAYERS];
  WMat emb;
  const float *dec_pos = nullptr, *lnw = nullptr, *lnb = nullptr;
  WVocabDev voc;
  WSample* state = nullptr;
  int *out = nullptr, *row_tok = nullptr, *row_pos = nullptr, *dst_row = nullptr, *step = nullptr;
  float *logits = nullptr, *scratch = nullptr, *x = nullptr, *q = nullptr, *att = nullptr, *ffb = nullptr;
  float *sg = nullptr, *mg = nullptr, *part = nullptr;
  void* partv = nullptr;     // (value, index) partials [2][grid]
  unsigned* bar = nullptr;   // grid barrier arrivals (zeroed before a launch)
  int* err = nullptr;        // 1: a wait ran out
  int stall = 0;             // test hook: the first barrier never completes
  // shared-memory plan: two weight buffers of wb bytes, logits rows staged
  // lrows at a time, so_nd / xo_nd outputs of a head per CTA in the self-
  // and cross-attention values, xv_floats floats of staged V columns,
  // xk_floats of staged cross K rows
  int wb = 0, lrows = 0, so_nd = 0, xo_nd = 0, xv_floats = 0, xk_floats = 0;
};

// Bytes of R rows of K columns staged in shared memory by the persistent
// Whisper kernel: float16 rows of 2K + 16 bytes, or Q8_0 rows of K + 16
// int8 values and then the rows' float16 scales, rounded up to 16.
__host__ __device__ inline int ws_slice_bytes(bool f16, int R, int K) {
  return f16 ? R * (2 * K + 16) : (R * (K + 16) + R * (K / 16) + 15) / 16 * 16;
}
// Shared memory a CTA of the kernel needs; whether the device runs it (one
// 512-thread CTA per SM, cooperative launch); the launch (steps rounds of
// sample-then-decode from position pos0).
// h[i] = f16(q[i]·d[i/32]) for a Q8_0 matrix (the products' widening).
void launch_wwiden(const WMat& w, uint16_t* h, cudaStream_t st);
size_t wstep1_smem(const WStep1Args& a);
int wstep1_max_active(size_t smem);
cudaError_t launch_wstep1(const WStep1Args* d_args, int grid, size_t smem, int pos0, int steps, cudaStream_t st);

void launch_wembed(const WRows& r, const WMat& tok_emb, const float* dec_pos, float* x, cudaStream_t st);
void launch_wln(const float* x, float* y, const float* w, const float* b, int rows, int n, cudaStream_t st);
// Self-attention of every row over its stream's cache rows 0..pos.
void launch_wself(const WRows& r, const float* q, const float* sk, const float* sv, float* att, cudaStream_t st);
// Cross-attention over the stream's pre-scaled keys [nh][ctx][hd] and
// transposed values [nh][hd][ctx].
// Cross-attention of every row; `scratch` (scratch_floats floats) holds the
// scores when the heads are spread over several CTAs.
void launch_wcross(const WRows& r, const float* q, const float* ck, const float* cvt, float* att, float* scratch,
                   size_t scratch_floats, cudaStream_t st);
// The packed-order product (whisper/gemm.go:124-209, rows < m/6·6) for
// `groups` independent matrices (grid z): C = A·Wᵀ + bias, row i of group z
// at a + z·a_zs + i·lda. Epilogues (mode): WM_STORE / WM_RESID (+=) /
// WM_GELU (geluAVX) at c + z·c_zs + i·ldc; WM_ROWPOS at c + dst_row[i·rs_i +
// z]·ldc; WM_CROSSK keys ·tsc into [z][nh][m][hd] and WM_CROSSV values into
// [z][nh][hd][m] (the cross K/V prep, A = encoder output of stream z).
// WM_GELU_ADD: geluAVX, then + aux at the same place (the encoder's
// positional embedding after conv2). A float32 weight may differ per group:
// w.f + z·w_zs.
enum WmmMode { WM_STORE = 0, WM_CROSSK = 1, WM_CROSSV = 2, WM_RESID = 3, WM_GELU = 4, WM_ROWPOS = 5, WM_GELU_ADD = 6 };
struct WmmArgs {
  const float* a = nullptr;
  int lda = 0;
  size_t a_zs = 0;
  int m = 0;
  WMat w;
  const float* bias = nullptr;
  int mode = WM_STORE;
  float* c = nullptr;
  int ldc = 0;
  size_t c_zs = 0;
  int nh = 1;
  float tsc = 1.f;
  const int* dst_row = nullptr;
  int rs_i = 0;
  size_t w_zs = 0;
  const float* aux = nullptr;
};
void launch_wmm(const WmmArgs& a, int groups, cudaStream_t st);
// The audio encoder's steps between products (encode, encoder.go:10-118),
// n streams: conv1's window rows from a log-mel [n][nmel][3000] into x1
// [n][3000][nmel·3]; conv2's (stride 2) from h1 [n][3000][state] into x2
// [n][ctx][state·3]; q/k/v [n][ctx][state] split per (stream, head) into qh
// (·sc) and kh [n·nh][ctx][hd] and vt [n·nh][hd][ctx]; the softmax of rows of
// len values.
void launch_wenc_conv1(const float* mel, float* x1, int nmel, int n, cudaStream_t st);
void launch_wenc_conv2(const float* h1, float* x2, int state, int ctx, int n, cudaStream_t st);
void launch_wenc_heads(const float* q, const float* k, const float* v, float* qh, float* kh, float* vt, int ctx,
                       int state, int nh, float sc, int n, cudaStream_t st);
void launch_wenc_softmax(float* x, int len, long rows, cudaStream_t st);
// Once per device, outside any graph capture: which cluster sizes the
// process/sample kernel can use, and the shared memory limits of the
// cross-attention kernels.
void wdecode_init();
// process + sample at temperature 0 for every row (transcribe.go:370-494):
// logits [rows][vocab] are masked in place (scratch [rows][vocab]); writes
// out[*step][rows][4] (id, tid, p, plog), the next token and the stream's
// sampling state.
void launch_wproc(const WRows& r, float* logits, float* scratch, const WVocabDev& v, WSample* state, int* out,
                  const int* step, int* next_tok, cudaStream_t st);
// row_pos += advance; dst_row = r·text_ctx + row_pos; *step += 1 when step is given.
void launch_wtick(int rows, int* row_pos, int* dst_row, int text_ctx, int advance, int* step, cudaStream_t st);
void whisper_kernels_init();
// softmax(logits row)[nosp] (the no-speech probability, transcribe.go:176-180);
// scratch [rows][vocab].
void launch_wnospeech(const float* logits, int vocab, int nosp, float* scratch, float* out, int rows, cudaStream_t st);

}  // namespace grx
