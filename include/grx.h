/*
 * grx.h — the C ABI of the B200 token-loop library (libgrx.so).
 *
 * It replaces, for gorelaxor's autoregressive token loops, the Go calls
 * listed beside each entry point (paths are inside the gorelaxor source
 * tree). Plain pointers and sizes only; every call returns 0 or a negative
 * GRX_E* code and never aborts; grx_last_error() gives the calling thread's
 * message. Host buffers are the caller's; device memory is the library's.
 * One handle lives on one device. Model handles may be shared by threads;
 * a stream set is driven by one thread at a time (like the reference's
 * tstate, pockettts/nn.go:120).
 */
#ifndef GRX_H
#define GRX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GRX_OK 0
#define GRX_EINVAL -1     /* bad argument or shape (the reference panics or returns an error) */
#define GRX_EFORMAT -2    /* a model or voice file that does not parse or fit (internal/gguf) */
#define GRX_ENOMEM -3     /* device allocation failed */
#define GRX_ECUDA -4      /* a CUDA call failed */
#define GRX_ERANGE -5     /* a stream ran past the positions its state was made for, or a size above a fixed limit */
#define GRX_ENODEV -6     /* no such device */
#define GRX_ETIMEDOUT -7  /* a bounded wait inside a kernel ran out (its watchdog); the state it was working on is undefined until reset */

/* The calling thread's last error message (empty if none); returns the
 * message length. */
int grx_last_error(char* buf, size_t len);
/* Number of CUDA devices the library sees. */
int grx_device_count(void);

/* ------------------------------------------------------------- GGUF ----
 * internal/gguf: the subset the token loops read (v2/v3; F32, F16, BF16,
 * Q8_0 tensors), with the reference's hostile-input checks
 * (internal/gguf/gguf.go:292-354). */
typedef struct grx_gguf grx_gguf;
/* gguf.Parse, internal/gguf/gguf.go:262-274 (copies the bytes). */
int grx_gguf_open(const void* bytes, size_t len, grx_gguf** out);
void grx_gguf_close(grx_gguf* f);
/* File.Int / File.Float / File.String, gguf.go:416-460; def when absent. */
int64_t grx_gguf_int(const grx_gguf* f, const char* key, int64_t def);
double grx_gguf_float(const grx_gguf* f, const char* key, double def);
int grx_gguf_string(const grx_gguf* f, const char* key, char* buf, size_t len);
/* The tensor's type (0 F32, 1 F16, 8 Q8_0, 30 BF16) and GGUF dims
 * (dims[0] fastest); returns the number of dims, or GRX_EINVAL if absent. */
int grx_gguf_tensor(const grx_gguf* f, const char* name, int* type, int64_t dims[4]);
/* File.Float32, gguf.go:498-523: the tensor widened to float32. */
int grx_gguf_float32(const grx_gguf* f, const char* name, float* dst, size_t n);

/* ------------------------------------------------ operator (kern) ------
 * kern.Weight and kern.Linear (internal/kern/kern.go:41-201) on the GPU. */
typedef struct grx_weight grx_weight;
/* kern.NewQ8, kern.go:76-84: rows×cols as 34-byte Q8_0 blocks. */
int grx_weight_q8(int device, const void* blocks, int rows, int cols, grx_weight** out);
/* kern.NewF32, kern.go:53-58. */
int grx_weight_f32(int device, const float* v, int rows, int cols, grx_weight** out);
/* kern.Weight.Pack + DropRows, kern.go:89-103: after this every product
 * with the weight takes the int8 path, a single row too. */
int grx_weight_drop_rows(grx_weight* w);
void grx_weight_free(grx_weight* w);
/* kern.Linear, kern.go:199 (MatMul dispatch :185-196): dst[m][rows] =
 * x[m][cols]·Wᵀ + bias (bias may be NULL). A Q8_0 weight with dropped rows,
 * or any m ≥ 2, takes the int8 path (activations rounded to Q8_0 blocks,
 * q8int.go:148-223); otherwise the float path (gemm.go:195-259). Host
 * buffers; synchronous. Limits of this build: the float path takes at most
 * 16 rows and K ≤ 65536; the int8 path with more
 * than 8 rows needs K % 64 == 0 (an even number of blocks: the activation
 * scales are copied two blocks at a time), with up to 8 rows N % 32 == 0. */
int grx_linear(const grx_weight* w, const float* x, int m, const float* bias, float* dst);

/* grx_linear_q8_static: the int8 path of grx_linear for callers that must
 * not allocate GPU memory. No counterpart in the reference: its Go kernels
 * run on the CPU and take scratch from the Go heap.
 *
 * Who needs it: a host that owns every byte of device memory itself — a
 * serving process whose pool allocator has reserved the GPU's memory up
 * front, or a real-time audio loop, where cudaMalloc/cudaFree would fail
 * or stall the device mid-stream. grx_linear cannot serve them: it uploads
 * its inputs and allocates the rounded activations on every call.
 *
 * Same product and dispatch rule as grx_linear's int8 path, bit for bit: w
 * is a Q8_0 weight with dropped rows, or m >= 2 (otherwise GRX_EINVAL: the
 * reference takes the float path there, which needs no scratch). d_x
 * [m][cols], d_bias [rows] (may be NULL) and d_dst [m][rows] are DEVICE
 * pointers on the weight's device, owned by the caller; work is queued on
 * `stream` (a cudaStream_t, NULL for the default stream) and not waited
 * for; the caller's current device is the same after the call as before
 * it. The call allocates nothing: the activations rounded to Q8_0 go to one
 * fixed array in the library's device memory, GRX_STATIC_MAX_ELEMS int8
 * values plus their block scales (1.25 MiB), which every GPU that loads the
 * library holds until the process exits. m*cols above GRX_STATIC_MAX_ELEMS
 * is rejected with GRX_ERANGE before anything is queued.
 *
 * The first call on a device looks up that array's device address (with
 * the device current) and keeps it; make that first call before any stream
 * capture on the device. All calls share the one array, and each leaves its
 * rounded activations there: calls that may overlap on the GPU (two
 * streams, or two threads without ordering) race on it and must be ordered
 * by the caller. Nothing needs clearing between calls: each call writes all
 * of the array that it then reads. The same shape limits as grx_linear's
 * int8 path apply (m > 8: cols % 64 == 0; m <= 8: rows % 32 == 0). */
#define GRX_STATIC_MAX_ELEMS (1 << 20)
int grx_linear_q8_static(const grx_weight* w, const float* d_x, int m, const float* d_bias, float* d_dst,
                         void* stream);

/* ------------------------------------------- Pocket TTS FlowLM ---------
 * pockettts.Model (pockettts/model.go:14) restricted to the flow LM and
 * its flow head; Mimi and the text path stay with the caller. */
typedef struct grx_flowlm grx_flowlm;
typedef struct grx_voice grx_voice;
typedef struct grx_streams grx_streams;

/* pockettts.Load, model.go:202-322 (the flow LM's tensors and settings),
 * with the upload to `device`. */
int grx_flowlm_load(const void* gguf, size_t len, int device, grx_flowlm** out);
void grx_flowlm_free(grx_flowlm* m);
/* Model dims: d, heads, ff, layers, latent dim, flow dim, flow depth,
 * decode steps (any pointer may be NULL). */
int grx_flowlm_dims(const grx_flowlm* m, int* d, int* heads, int* ff, int* layers, int* ldim, int* fdim, int* depth,
                    int* steps);
/* Model.LoadVoice, voice.go:26-63 (kept on the host until streams use it). */
int grx_voice_load(grx_flowlm* m, const void* gguf, size_t len, grx_voice** out);
/* A voice from raw caches: kv is [layers][2][positions][d] float32. */
int grx_voice_raw(grx_flowlm* m, int positions, const float* kv, grx_voice** out);
void grx_voice_free(grx_voice* v);
/* The flow-LM half of Model.CloneVoice (pockettts/voice.go:94-106 and
 * cloneCond :113-127 after Mimi's encoder): latents are the clip's Mimi
 * latents [n][ldim] (1 ≤ n ≤ 4095); cond = kern.Linear(latents,
 * lm.speaker_proj), then [lm.bos_voice; cond] runs through the transformer
 * from an empty state and its caches become the voice (n + 1 positions).
 * Needs a model file with lm.speaker_proj (float32) and lm.bos_voice. */
int grx_voice_from_latents(grx_flowlm* m, const float* latents, int n, grx_voice** out);
/* A voice's positions and (kv may be NULL) its caches [layers][2][positions][d]
 * — the tstate a Voice holds (voice.go:14-17). */
int grx_voice_kv(const grx_voice* v, int* positions, float* kv);

/* n streams, stream i starting from voices[i] (speakChunk's
 * v.st.clone(...), speak.go:117), each with room for max_frames frames. */
int grx_streams_create(grx_flowlm* m, int n, const grx_voice* const* voices, int max_frames, grx_streams** out);
void grx_streams_free(grx_streams* s);
/* Puts every stream back at its voice prompt and the next frame at bos. */
int grx_streams_reset(grx_streams* s);
/* flowLM.text (pockettts/lm.go:172-181), what speakChunk runs before its
 * frames (speak.go:119): stream i's text tokens ids[offsets[i] ..
 * offsets[i+1]) go through the transformer after the positions it holds,
 * with attend's arithmetic for several queries (nn.go:200-243), and stay in
 * its caches; the next frame still starts at bos. offsets has n + 1
 * non-decreasing entries from 0 (a stream may have no tokens). The tokens
 * count against the room the set was made with (max_frames). out (host,
 * may be NULL) gets [n][d]: out_norm of each stream's last token row, which
 * the reference returns (streams without tokens keep their row). Needs a
 * model with lm.embed; ids must be rows of it. Synchronous. */
int grx_streams_text(grx_streams* s, const int* ids, const int* offsets, float* out);
/* One frame for every stream: flowLM.step then flowHead.sample
 * (pockettts/lm.go:185-195, 108-124; speak.go:146-174), the raw latent fed
 * back on the device. noise is [n][ldim]. Outputs (host, any may be NULL):
 * lm_out [n][d], eos [n], latent [n][ldim], scaled [n][ldim] (the latent
 * times emb_std plus emb_mean, what speak.go:165-173 sends to Mimi). */
int grx_streams_step(grx_streams* s, const float* noise, float* lm_out, float* eos, float* latent, float* scaled);
/* `frames` frames with the same meaning, device-resident in and out:
 * d_noise [frames][n][ldim], d_latent [frames][n][ldim], d_eos
 * [frames][n] (device pointers on the stream set's device; d_eos may be
 * NULL). Asynchronous on the library's stream; grx_streams_sync waits. */
int grx_streams_run_device(grx_streams* s, int frames, const float* d_noise, float* d_latent, float* d_eos);
int grx_streams_sync(grx_streams* s);
/* grx_streams_run_device with instrumentation: d_attn_ts (device,
 * [frames][layers][parts][2] uint64, each pair preset to {UINT64_MAX, 0})
 * gets each attention kernel's first-CTA start and last-CTA end in
 * %globaltimer ns. */
int grx_streams_run_device_timed(grx_streams* s, int frames, const float* d_noise, float* d_latent, float* d_eos,
                                 unsigned long long* d_attn_ts);
/* The cudaStream_t the stream set's work runs on (for events); work is
 * queued behind what this stream holds and finishes before what is queued
 * on it later. */
void* grx_streams_cuda_stream(const grx_streams* s);
/* A set of 128 or more streams runs as parts of at least 64 streams, each
 * on its own CUDA stream, so one part's memory-bound attention can overlap
 * another's products: two parts at most unless the environment variable
 * GRX_STREAM_PARTS (1 to 8, read when the set is created) allows more.
 * Returns the number of parts. */
int grx_streams_parts(const grx_streams* s);
/* Positions held by stream i (voice prompt plus frames so far). */
int grx_streams_pos(const grx_streams* s, int i);
/* Device kernel launches issued by this stream set since creation. */
int64_t grx_streams_launches(const grx_streams* s);
/* 1 when the set runs its frames in the persistent one-stream kernel: a set
 * of one stream whose model has one decode step (a flow head of depth 1 to
 * 4) runs every frame of a step or a device-resident run as one cooperative
 * launch, one block per SM, with grid barriers between the frame's
 * dependent steps (GRX_FRAME1=0, read when the set is created, keeps the
 * per-kernel path). Same results bit for bit. Its waits are bounded (about
 * a second each); one that runs out makes grx_streams_step /
 * grx_streams_sync return GRX_ETIMEDOUT. 0 otherwise. */
int grx_streams_persistent(const grx_streams* s);
/* Checks the persistent kernel's watchdog: runs it once with a grid barrier
 * that nothing completes and returns what its bounded waits report —
 * GRX_ETIMEDOUT, after about a second, when they work. The set's positions
 * are unchanged; reset it before the next frame. GRX_EINVAL for a set that
 * does not run the persistent kernel. */
int grx_streams_watchdog_test(grx_streams* s);

/* ------------------------------------------- Pocket TTS Mimi decoder ----
 * mimiDecoder (pockettts/mimi.go:24-150): the latent projection, the
 * depthwise upsampling, the windowed transformer with layer scales and the
 * SEANet decoder, streaming, for n independent streams that each turn one
 * latent into one frame of samples per call. */
typedef struct grx_mimi grx_mimi;
typedef struct grx_mimi_streams grx_mimi_streams;
/* The decoder half of pockettts.Load (model.go:102-178, 220-227, 280-307):
 * the pockettts.mimi.* and pockettts.seanet.* settings and the mimi.quant,
 * mimi.up, mimi.dec_tf.* and mimi.dec.* tensors of a Pocket TTS file, with
 * the same shape checks. Q8_0 matrices take the int8 path (the reference
 * packs them and drops their rows), float32 ones MatMul's float path. This
 * build takes 64-value heads, Q8_0 transformer matrices, Q8_0 matrices
 * with rows % 32 == 0 and cols <= 16384 and float32 ones with cols % 4 == 0
 * or cols < 16; other files give GRX_EINVAL or GRX_EFORMAT. A file with
 * Mimi's encoder (mimi.enc.*, mimi.enc_tf.*, mimi.down: model.go:181-200,
 * 308-313) also loads it, for grx_mimi_encoder_create. */
int grx_mimi_load(const void* gguf, size_t len, int device, grx_mimi** out);
void grx_mimi_free(grx_mimi* m);
/* d, heads, transformer layers, context, upsampling stride, latent dim,
 * samples per frame, sample rate (any pointer may be NULL). */
int grx_mimi_dims(const grx_mimi* m, int* d, int* heads, int* layers, int* context, int* upsample, int* ldim,
                  int* frame, int* sample_rate);
/* n streams (1 ≤ n ≤ 65535), each a fresh decState (mimi.go:108-124) with
 * room for max_frames frames. */
int grx_mimi_streams_create(grx_mimi* m, int n, int max_frames, grx_mimi_streams** out);
void grx_mimi_streams_free(grx_mimi_streams* s);
/* Every stream back to a fresh decState; the next frame fades in again. */
int grx_mimi_streams_reset(grx_mimi_streams* s);
/* mimiDecoder.decode of one latent per stream (latents [n][ldim], host, the
 * flow LM's scaled latents), then speakChunk's fade-in on each stream's
 * first frame (speak.go:185-190): pcm (host, may be NULL) gets [n][frame]
 * samples. Synchronous. */
int grx_mimi_decode(grx_mimi_streams* s, const float* latents, float* pcm);
/* `frames` calls of grx_mimi_decode, device-resident: d_latents
 * [frames][n][ldim] in, d_pcm [frames][n][frame] out (device pointers on
 * the set's device). Asynchronous on the library's stream; grx_mimi_sync
 * waits. A set's first decode call (either form) captures the call's
 * kernels into CUDA graphs on the set's stream, which later calls replay;
 * an encoder set does the same per piece shape. */
int grx_mimi_decode_device(grx_mimi_streams* s, int frames, const float* d_latents, float* d_pcm);
int grx_mimi_sync(grx_mimi_streams* s);
/* The cudaStream_t the set's kernels run on. */
void* grx_mimi_cuda_stream(const grx_mimi_streams* s);
/* Device kernel launches issued by this set since creation. */
int64_t grx_mimi_launches(const grx_mimi_streams* s);
/* Frames decoded since creation or the last reset. */
int grx_mimi_frames(const grx_mimi_streams* s);

/* ------------------------------------------- Pocket TTS Mimi encoder ----
 * mimiEncoder.encode (pockettts/mimi.go:152-179) as cloneCond runs it
 * (voice.go:113-124): the SEANet encoder, the windowed transformer and the
 * downsampling convolution to the latent rate, streaming over pieces of
 * twelve frames. The clip is 24 kHz audio after CloneVoice's resampling and
 * end_on_pause (voice.go:85-93, host work). */
/* A set of n clips of up to max_samples samples each; needs a model file
 * with the encoder (GRX_EINVAL otherwise). grx_mimi_streams_free frees it. */
int grx_mimi_encoder_create(grx_mimi* m, int n, int max_samples, grx_mimi_streams** out);
/* Every clip (d_pcm [n][samples], device) padded with zeros to whole frames
 * and encoded twelve frames at a time with one state per clip, from a fresh
 * state: d_latents [n][frames][ldim], frames = ceil(samples / frame).
 * Asynchronous on the set's stream; grx_mimi_sync waits. */
int grx_mimi_encode_device(grx_mimi_streams* s, int samples, const float* d_pcm, float* d_latents);
/* The same from and to host memory (pcm [n][samples], latents
 * [n][frames][ldim]). Synchronous. */
int grx_mimi_encode(grx_mimi_streams* s, int samples, const float* pcm, float* latents);
/* cloneCond's encoding of one clip: latents [frames][ldim] (room for
 * ceil(samples / frame) rows), *frames (may be NULL) the row count. */
int grx_mimi_clone_latents(grx_mimi* m, const float* pcm, int samples, float* latents, int* frames);
/* Model.CloneVoice after resampling and end_on_pause (voice.go:94-106):
 * the Mimi encoding of the clip (grx_mimi_clone_latents), then the flow-LM
 * half (grx_voice_from_latents). */
int grx_voice_clone(grx_flowlm* lm, grx_mimi* mimi, const float* pcm, int samples, grx_voice** out);

/* ----------------------------------------- FastConformer encoder --------
 * conformer.Model.encode (conformer/encoder.go:123-489): the 8x
 * depthwise-striding subsampling and the Conformer blocks (macaron
 * feed-forwards, relative-position attention, the convolution module), for
 * the offline case — "regular" attention over every frame of the utterance,
 * non-causal subsampling — one utterance per call. */
typedef struct grx_fconf grx_fconf;
/* The encoder half of conformer.FromGGUF (model.go:160-189, 350-410) from a
 * parakeet GGUF: the stt.parakeet.encoder.* settings, stt.frontend.num_mels
 * and the enc.* tensors, with the same names and shape checks; taps
 * transposed, batch norm folded, float16 1x1 convolutions rounded by ToQ8.
 * This build takes files whose matrices are Q8_0 (the int8 path) and the
 * offline attention; others give GRX_EINVAL. */
int grx_fconf_load(const void* gguf, size_t len, int device, grx_fconf** out);
void grx_fconf_free(grx_fconf* m);
int grx_fconf_dims(const grx_fconf* m, int* d_model, int* heads, int* layers, int* n_mels, int* sub_channels);
/* Rows the subsampling makes from `frames` (three stride-2 steps). */
int grx_fconf_out_rows(int frames);
/* Encode of log-mel features mel [n_mels][frames] (host), the first valid
 * frames real: out (host, room for grx_fconf_out_rows(frames) rows of
 * d_model) gets the valid rows, *rows their count. Synchronous; calls on
 * one handle must not overlap. */
int grx_fconf_encode(grx_fconf* m, const float* mel, int frames, int valid, float* out, int* rows);
/* The same with device buffers, asynchronous on the handle's stream
 * (grx_fconf_sync waits). */
int grx_fconf_encode_device(grx_fconf* m, const float* d_mel, int frames, int valid, float* d_out, int* rows);
int grx_fconf_sync(grx_fconf* m);
void* grx_fconf_cuda_stream(const grx_fconf* m);
int64_t grx_fconf_launches(const grx_fconf* m);

/* ------------------------------------------- TDT decoder (conformer) ------
 * conformer.Model.Decode (conformer/rnnt.go:111-173), the greedy RNN-T /
 * TDT loop over encoder output, for a batch of independent streams. */
typedef struct grx_tdt grx_tdt;
typedef struct grx_tdt_batch grx_tdt_batch;
/* conformer.Token (rnnt.go:10-15). */
typedef struct grx_tdt_token {
  int id;       /* token id */
  int frame;    /* encoder frame where it was emitted, plus the frame offset */
  int duration; /* frames it covers (TDT); 1 for RNN-T */
  float p;      /* softmax probability of the token */
} grx_tdt_token;
/* The decoder part of conformer.FromGGUF (model.go:190-236, 306-314): a
 * parakeet GGUF's decoder settings and its pred.* and joint.* tensors (Q8_0
 * matrices, as the converter writes them) on `device`. The encoder is not
 * loaded (its output is Decode's input). */
int grx_tdt_load(const void* bytes, size_t len, int device, grx_tdt** out);
void grx_tdt_free(grx_tdt* m);
/* Any pointer may be NULL. is_tdt: 1 TDT, 0 RNN-T. */
int grx_tdt_dims(const grx_tdt* m, int* hidden, int* layers, int* vocab, int* joint, int* d_enc, int* n_durations,
                 int* blank, int* is_tdt);
/* n DecoderStates (rnnt.go:19-33), each at its start, and room for max_t
 * encoder frames and cap tokens per stream and call. */
int grx_tdt_batch_create(grx_tdt* m, int n, int max_t, int cap, grx_tdt_batch** out);
void grx_tdt_batch_free(grx_tdt_batch* b);
/* NewDecoderState (rnnt.go:27) for every stream. */
int grx_tdt_batch_reset(grx_tdt_batch* b);
/* Stream i's DecoderState: h and c [layers][hidden], the last token. */
int grx_tdt_state_get(grx_tdt_batch* b, int i, float* h, float* c, int* last);
int grx_tdt_state_set(grx_tdt_batch* b, int i, const float* h, const float* c, int last);
/* Model.Decode for every stream i: enc [n][max_t][d_enc] (host), T[i] frames
 * (0..max_t), frame_offset (may be NULL: 0). Continues from each stream's
 * state and leaves it after the stream's last iteration, as Decode's st.
 * tokens [n][cap] (host) gets each stream's tokens in order and counts[n]
 * their number, which may exceed cap (only the first cap are kept). */
int grx_tdt_decode(grx_tdt_batch* b, const float* enc, const int* T, const int* frame_offset, grx_tdt_token* tokens,
                   int* counts);
/* The same with device-resident buffers: d_enc [n][max_t][d_enc], d_tokens
 * [n][cap], d_counts [n] on the batch's device (T and frame_offset on the
 * host). Returns when every stream has finished its loop. */
int grx_tdt_decode_device(grx_tdt_batch* b, const float* d_enc, const int* T, const int* frame_offset,
                          grx_tdt_token* d_tokens, int* d_counts);
/* The cudaStream_t the batch's work runs on. */
void* grx_tdt_batch_cuda_stream(const grx_tdt_batch* b);
/* Kernel launches and loop iterations (batch rounds) issued so far. */
int64_t grx_tdt_batch_launches(const grx_tdt_batch* b);
int64_t grx_tdt_batch_iterations(const grx_tdt_batch* b);
/* Loop iterations of the last decode summed over its streams (each is one
 * joint evaluation of one stream, the reference's unit of work in
 * rnnt.go:138-171); waits for the batch's stream. */
int64_t grx_tdt_batch_stream_iterations(grx_tdt_batch* b);

/* ------------------------------------------- Whisper text decoder ---------
 * The token loop of whisper.Model (whisper/decoder.go:33-140,
 * transcribe.go:150-269 and 370-520) for a batch of independent streams. */
typedef struct grx_whisper grx_whisper;
typedef struct grx_whisper_batch grx_whisper_batch;
/* whisper.Load's decoder part (model.go:94-223, 320-448): a whisper.cpp
 * ggml file; the encoder's tensors are read and left (the decoder is given
 * the encoder's output). Matrices keep Q8_0 in HBM, widened as f16(q·d) on
 * the fly exactly as the reference widens them at load; other types are
 * widened to float16 at load as the reference does. Heads of 64 values. */
int grx_whisper_load(const void* bytes, size_t len, int device, grx_whisper** out);
void grx_whisper_free(grx_whisper* m);
int grx_whisper_dims(const grx_whisper* m, int* n_vocab, int* n_audio_ctx, int* n_state, int* n_head,
                     int* n_text_layer, int* n_text_ctx);
/* The vocabulary's special tokens (vocab.go:19-43). */
int grx_whisper_tokens(const grx_whisper* m, int* eot, int* sot, int* prev, int* nosp, int* beg, int* n_lang);
/* vocab.suppressed() (vocab.go:103-118) into out (up to cap); returns the count. */
int grx_whisper_suppressed(const grx_whisper* m, int* out, int cap);
/* How many sampled rows, over every batch of this model since it was
 * loaded, were decided in the reference's sequential order: process/sample
 * sums the vocabulary as trees and recomputes a row in sequence when a
 * decision it feeds (the timestamp rule, the winner against an earlier
 * index) falls within the margin those sums' roundings could move. */
int64_t grx_whisper_exact_rows(const grx_whisper* m);
/* n streams, each a decoding sequence (its self-attention cache, this
 * window's cross K/V, its sampling state). */
int grx_whisper_batch_create(grx_whisper* m, int n, grx_whisper_batch** out);
void grx_whisper_batch_free(grx_whisper_batch* b);
/* A window for every stream: enc [n][n_audio_ctx][n_state] (host, or device
 * for _device) → each layer's cross keys (·1/√64) and values
 * (encoder.go:120-140, the packed product order of gemm.go:124-209); the
 * caches and sampling states start over. */
int grx_whisper_set_audio(grx_whisper_batch* b, const float* enc);
int grx_whisper_set_audio_device(grx_whisper_batch* b, const float* d_enc);
/* Model.encode (whisper/encoder.go:10-118) of every stream's window, then
 * what grx_whisper_set_audio does with its output: mel is [n][n_mels][3000]
 * (the log-mel as logMel lays it out, channel-major). conv1 and conv2 with
 * GELU, the positions, the encoder blocks and the final LayerNorm, every
 * product in whisper/gemm.go's packed order. Needs a model file with the
 * encoder's tensors. Synchronous. */
int grx_whisper_encode(grx_whisper_batch* b, const float* mel);
/* The same from device memory (d_mel on the batch's device). */
int grx_whisper_encode_device(grx_whisper_batch* b, const float* d_mel);
/* The last window's encoder output [n][1500][n_state] (from
 * grx_whisper_encode, or what grx_whisper_set_audio was given). */
int grx_whisper_encoder_out(grx_whisper_batch* b, float* out);
/* The prompt decode (transcribe.go:166-181): prompt [n][np] tokens, all
 * rows at once as decoder.go does (the packed product for each stream's
 * first np/6·6 rows when np ≥ 6); no_speech [n] (may be NULL) gets
 * softmax(logits at sot_at)[nosp]. */
int grx_whisper_prompt(grx_whisper_batch* b, const int* prompt, int np, int sot_at, float* no_speech);
/* `steps` rounds of the greedy loop at temperature 0 (transcribe.go:196-269:
 * process, sample, decode of the sampled token), for every stream, without
 * the window's stop rules. tokens [steps][n][4]: id, tid, p and plog (float
 * bits), host or device (_device, asynchronous; grx_whisper_sync waits). */
int grx_whisper_run(grx_whisper_batch* b, int steps, int* tokens);
int grx_whisper_run_device(grx_whisper_batch* b, int steps, int* d_tokens);
int grx_whisper_sync(grx_whisper_batch* b);
/* 1 when the batch runs its token loop in the persistent one-stream kernel:
 * a batch of one stream whose model has 64-value heads, Q8_0 or float16
 * matrices with whole groups of 16 columns and at most 12 layers runs every
 * step of grx_whisper_run(_device) as one cooperative launch, one block per
 * SM, with grid barriers between a step's dependent parts (GRX_WSTEP1=0,
 * read when the batch is created, keeps the per-kernel path). Same tokens
 * bit for bit. Its waits are bounded (about a second each); one that runs
 * out makes grx_whisper_run / grx_whisper_sync return GRX_ETIMEDOUT. 0
 * otherwise. */
int grx_whisper_persistent(const grx_whisper_batch* b);
/* Checks the persistent kernel's watchdog: runs one step with a grid barrier
 * that nothing completes and returns what its bounded waits report —
 * GRX_ETIMEDOUT, after about a second, when they work. The batch's decoding
 * state is undefined afterwards; set the window and decode a prompt again.
 * GRX_EINVAL for a batch that does not run the persistent kernel or has no
 * prompt decoded. */
int grx_whisper_watchdog_test(grx_whisper_batch* b);
/* Stream i's cross K [heads][ctx][64] and Vᵀ [heads][64][ctx] of a layer. */
int grx_whisper_cross(grx_whisper_batch* b, int i, int layer, float* k, float* vt);
/* The logits of the last decode, [n][n_vocab]. */
int grx_whisper_logits(grx_whisper_batch* b, float* out);
void* grx_whisper_batch_cuda_stream(const grx_whisper_batch* b);
int64_t grx_whisper_batch_launches(const grx_whisper_batch* b);

#ifdef __cplusplus
}
#endif
#endif /* GRX_H */
