"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU oracle (liboracle.so,
built from this folder by its Makefile). Imported by tests/, by
__graft_entry__.smoke() as the checker, and by bench.py's CPU-baseline
leg; never by the product (gorelaxor_b200/)."""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        P, I, F, D = C.c_void_p, C.c_int, C.c_float, C.c_double
        sig = {
            "orc_f16_to_f32": (F, [C.c_uint16]),
            "orc_f32_to_f16": (C.c_uint16, [F]),
            "orc_expf_go": (F, [F]),
            "orc_exp_avx": (F, [F]),
            "orc_gelu_go": (F, [F]),
            "orc_gelu_avx": (F, [F]),
            "orc_silu_go": (F, [F]),
            "orc_silu_avx": (F, [F]),
            "orc_expsub": (F, [P, I, F]),
            "orc_gelu_vec": (None, [P, I]),
            "orc_silu_vec": (None, [P, I]),
            "orc_quant_act": (None, [P, P, P, I]),
            "orc_to_q8": (None, [P, P, I, I]),
            "orc_linear": (None, [P, P, I, I, P, I, I, I, P]),
            "orc_layer_norm_pt": (None, [P, P, I, I, P, P, D]),
            "orc_rope_table": (None, [P, I, D, I]),
            "orc_attend_one": (None, [P, P, P, P, I, I, I]),
            "orc_flowlm_new": (P, [I, I, I, I, I, I, I, D]),
            "orc_flowlm_free": (None, [P]),
            "orc_flowlm_tensor": (None, [P, C.c_char_p, I, I, I, P]),
            "orc_flowlm_ready": (I, [P, I]),
            "orc_error": (C.c_char_p, [P]),
            "orc_flowlm_time_conds": (None, [P, P]),
            "orc_stream_new": (P, [P, I, P]),
            "orc_stream_free": (None, [P]),
            "orc_stream_pos": (I, [P]),
            "orc_flowlm_text": (I, [P, P, P, I, P]),
            "orc_flowlm_voice_latents": (I, [P, P, I, P]),
            "orc_mimi_new": (P, [I, I, I, I, D, I, P, I, I, I, I, I, I, I, I, I, I]),
            "orc_mimi_free": (None, [P]),
            "orc_mimi_tensor": (None, [P, C.c_char_p, I, I, I, P]),
            "orc_mimi_error": (C.c_char_p, [P]),
            "orc_mimi_ready": (I, [P]),
            "orc_mimi_state": (P, [P]),
            "orc_mimi_state_free": (None, [P]),
            "orc_mimi_decode": (None, [P, P, P, P]),
            "orc_mimi_frame": (I, [P]),
            "orc_elu": (None, [P, C.c_long]),
            "orc_flowlm_frame": (F, [P, P, P, P, P, P, P, P]),
            "orc_flowlm_run": (None, [P, I, P, I, P, P, P, P, I]),
            "orc_tdt_new": (P, [I, I, I, I, I, I, I, I, P, I]),
            "orc_tdt_free": (None, [P]),
            "orc_tdt_error": (C.c_char_p, [P]),
            "orc_tdt_tensor": (None, [P, C.c_char_p, I, I, I, P]),
            "orc_tdt_ready": (I, [P]),
            "orc_tdt_decode": (I, [P, P, I, I, P, P, P, P, I, P, P]),
            "orc_tdt_run": (None, [P, I, P, I, I, P, I, P, P, I]),
            "orc_q8_to_f16": (None, [P, C.c_long, P]),
            "orc_whisper_new": (P, [I, I, I, I, I]),
            "orc_whisper_free": (None, [P]),
            "orc_whisper_error": (C.c_char_p, [P]),
            "orc_whisper_tensor": (None, [P, C.c_char_p, I, I, I, P]),
            "orc_whisper_vocab": (None, [P, P, P, I]),
            "orc_whisper_suppress": (I, [P, P, I]),
            "orc_whisper_ready": (I, [P]),
            "orc_whisper_encoder": (None, [P, I, I, I]),
            "orc_mimi_conv_run": (None, [P, P, I, I, I, I, I, P, P, I, P]),
            "orc_mimi_clone_latents": (I, [P, P, I, P]),
            "orc_mimi_convtr_run": (None, [P, P, I, I, I, I, P, P, I, P]),
            "orc_attend_window": (None, [P, P, I, P, P, I, I, I, I]),
            "orc_fconf_new": (P, [I, I, I, I, I, I, I, I, I]),
            "orc_fconf_free": (None, [P]),
            "orc_fconf_error": (C.c_char_p, [P]),
            "orc_fconf_tensor": (None, [P, C.c_char_p, I, I, I, P]),
            "orc_fconf_ready": (I, [P]),
            "orc_fconf_encode": (I, [P, P, I, I, P, I]),
            "orc_whisper_encode": (None, [P, P, P]),
            "orc_whisper_encode_blocks": (None, [P, P, P, I]),
            "orc_wseq_new": (P, [P]),
            "orc_wseq_free": (None, [P]),
            "orc_whisper_cross_kv": (None, [P, P, P]),
            "orc_wseq_cross": (None, [P, I, P, P]),
            "orc_whisper_decode": (I, [P, P, P, I, P, I, P]),
            "orc_whisper_matmul": (None, [P, P, I, I, I, I, P, P]),
            "orc_whisper_process_sample": (None, [P, P, P, P]),
            "orc_whisper_greedy": (I, [P, P, P, I, I, I, P, P]),
            "orc_whisper_run": (None, [P, I, P, P, I, I, I, P, I]),
        }
        sig["orc_set_fast"] = (I, [I])
        sig["orc_set_pool"] = (None, [I])
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        _lib = L
    return _lib


class fast_mode:
    """The oracle's fast mode (fast.h: the same values from SIMD kernels in
    the reference's lane order) for the calls inside a with-block; `kind` is
    2 on AVX-512 VNNI, 1 on AVX2, 0 where neither exists (exact mode then).
    With `threads`, a single call's products and heads split over that many
    threads (calls made from this Python thread)."""

    def __init__(self, threads: int = 0):
        self.threads = threads

    def __enter__(self):
        self.kind = lib().orc_set_fast(1)
        if self.threads > 1:
            lib().orc_set_pool(self.threads)
        return self

    def __exit__(self, *exc):
        if self.threads > 1:
            lib().orc_set_pool(0)
        lib().orc_set_fast(0)
        return False


def p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ------------------------------------------------------------ kernels --


def quant_act(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    nb = x.size // 32
    q = np.empty(x.size, np.int8)
    s = np.empty(nb, np.float32)
    lib().orc_quant_act(p(q), p(s), p(x), nb)
    return q, s


def to_q8(v: np.ndarray) -> np.ndarray:
    """Weight.ToQ8 (kern.go:139-170) of a [rows][cols] float32 matrix."""
    v = np.ascontiguousarray(v, np.float32)
    rows, cols = v.shape
    out = np.empty(rows * cols // 32 * 34, np.uint8)
    lib().orc_to_q8(p(out), p(v), rows, cols)
    return out


def f16_to_f32(h: int) -> float:
    return lib().orc_f16_to_f32(h)


def f32_to_f16(f: float) -> int:
    return lib().orc_f32_to_f16(f)


def linear(x: np.ndarray, kind: str, w: np.ndarray, rows: int, cols: int, bias=None, dropped=False):
    """kern.Linear with the reference's dispatch; kind 'f32' | 'f16' | 'q8_0'."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    out = np.empty((x.shape[0], rows), np.float32)
    t = {"f32": 0, "f16": 1, "q8_0": 2}[kind]
    w = np.ascontiguousarray(w)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().orc_linear(p(out), p(x), x.shape[0], t, p(w), rows, cols, int(dropped), p(b))
    return out


def layer_norm_pt(x, w, b, eps):
    x = np.ascontiguousarray(x, np.float32)
    rows, n = x.reshape(-1, x.shape[-1]).shape
    out = np.empty_like(x)
    lib().orc_layer_norm_pt(p(out), p(x), rows, n, p(w), p(b), eps)
    return out


def attend_one(q, kc, vc, heads):
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(kc, np.float32)
    vc = np.ascontiguousarray(vc, np.float32)
    nk, d = kc.shape
    out = np.empty(d, np.float32)
    lib().orc_attend_one(p(out), p(q), p(kc), p(vc), nk, d, heads)
    return out


# -------------------------------------------------------------- FlowLM --


class FlowLM:
    """The oracle's FlowLM, from the synthetic generator's tensor dict."""

    def __init__(self, cfg, tensors: dict):
        from gorelaxor_b200.synth import Q8

        self.cfg = cfg
        self._keep = []
        L = lib()
        self.h = L.orc_flowlm_new(cfg.d, cfg.heads, cfg.ff, cfg.layers, cfg.ldim, cfg.flow_dim, cfg.flow_depth,
                                  cfg.max_period)
        for name, arr in tensors.items():
            if isinstance(arr, Q8):
                buf = np.ascontiguousarray(arr.blocks)
                L.orc_flowlm_tensor(self.h, name.encode(), 2, arr.rows, arr.cols, p(buf))
            else:
                buf = np.ascontiguousarray(arr, np.float32)
                rows, cols = (buf.shape if buf.ndim == 2 else (1, buf.size))
                L.orc_flowlm_tensor(self.h, name.encode(), 0, rows, cols, p(buf))
            self._keep.append(buf)
        if L.orc_flowlm_ready(self.h, cfg.decode_steps) != 0:
            raise RuntimeError(L.orc_error(self.h).decode())

    def time_conds(self):
        out = np.empty((self.cfg.decode_steps, self.cfg.flow_dim), np.float32)
        lib().orc_flowlm_time_conds(self.h, p(out))
        return out

    def stream(self, kv: np.ndarray):
        """kv: [layers][2][positions][d]."""
        kv = np.ascontiguousarray(kv, np.float32)
        return Stream(lib().orc_stream_new(self.h, kv.shape[2], p(kv)))

    def text(self, st: "Stream", ids):
        """flowLM.text (lm.go:172-181): the token ids through the
        transformer on st; returns the output at the last token."""
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(self.cfg.d, np.float32)
        if lib().orc_flowlm_text(self.h, st.h, p(ids), len(ids), p(out)) != 0:
            raise ValueError("orc_flowlm_text: no lm.embed or a token id out of range")
        return out

    def voice_from_latents(self, lat):
        """The voice caches [layers][2][n + 1][d] a clip's Mimi latents
        [n][ldim] make (voice.go:94-106 after the encoder)."""
        lat = np.ascontiguousarray(lat, np.float32)
        n = lat.shape[0]
        kv = np.empty((self.cfg.layers, 2, n + 1, self.cfg.d), np.float32)
        if lib().orc_flowlm_voice_latents(self.h, p(lat), n, p(kv)) != 0:
            raise ValueError("orc_flowlm_voice_latents: no float32 lm.speaker_proj / lm.bos_voice")
        return kv

    def frame(self, st: "Stream", latent, noise, trace=False):
        c = self.cfg
        lm_out = np.empty(c.d, np.float32)
        lat = np.empty(c.ldim, np.float32)
        sc = np.empty(c.ldim, np.float32)
        tr = np.empty((c.layers + 1, c.d), np.float32) if trace else None
        lat_in = None if latent is None else np.ascontiguousarray(latent, np.float32)
        nz = np.ascontiguousarray(noise, np.float32)
        eos = lib().orc_flowlm_frame(self.h, st.h, p(lat_in), p(nz), p(lm_out), p(lat), p(sc), p(tr))
        return dict(lm_out=lm_out, eos=np.float32(eos), latent=lat, scaled=sc, trace=tr)

    def run(self, streams: list, noise: np.ndarray, threads: int = 1, want_lm_out=False):
        """noise [frames][n][ldim] → latents [frames][n][ldim], eos [frames][n]."""
        frames, n, ld = noise.shape
        arr = (C.c_void_p * n)(*[s.h for s in streams])
        lat = np.empty((frames, n, ld), np.float32)
        eos = np.empty((frames, n), np.float32)
        lo = np.empty((frames, n, self.cfg.d), np.float32) if want_lm_out else None
        nz = np.ascontiguousarray(noise, np.float32)
        lib().orc_flowlm_run(self.h, n, arr, frames, p(nz), p(lat), p(eos), p(lo), threads)
        return lat, eos, lo

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_flowlm_free(self.h)
            self.h = None


class Stream:
    def __init__(self, h):
        self.h = h

    @property
    def pos(self):
        return lib().orc_stream_pos(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_stream_free(self.h)
            self.h = None


ACTS = {"relu": 0, "sigmoid": 1, "tanh": 2}


class TDT:
    """The oracle's greedy TDT / RNN-T decoder (conformer/rnnt.go), from the
    synthetic generator's tensor dict."""

    def __init__(self, cfg, tensors: dict):
        from gorelaxor_b200.synth import Q8

        self.cfg = cfg
        self._keep = []
        L = lib()
        dur = np.ascontiguousarray(cfg.durations, np.int32)
        self._keep.append(dur)
        self.h = L.orc_tdt_new(cfg.H, cfg.layers, cfg.V, cfg.J, cfg.blank, cfg.max_symbols,
                               int(cfg.head == "tdt"), ACTS[cfg.act], p(dur), len(dur))
        for name, arr in tensors.items():
            if isinstance(arr, Q8):
                buf = np.ascontiguousarray(arr.blocks)
                L.orc_tdt_tensor(self.h, name.encode(), 2, arr.rows, arr.cols, p(buf))
            else:
                buf = np.ascontiguousarray(arr, np.float32)
                rows, cols = (buf.shape if buf.ndim == 2 else (1, buf.size))
                L.orc_tdt_tensor(self.h, name.encode(), 0, rows, cols, p(buf))
            self._keep.append(buf)
        if L.orc_tdt_ready(self.h) != 0:
            raise RuntimeError(L.orc_tdt_error(self.h).decode())

    def state(self):
        """A fresh DecoderState: (h [layers][H], c [layers][H], last)."""
        z = np.zeros((self.cfg.layers, self.cfg.H), np.float32)
        return [z.copy(), z.copy(), -1]

    def decode(self, enc: np.ndarray, state=None, frame_offset: int = 0, cap: int | None = None):
        """Model.Decode (rnnt.go:111): tokens as an int array [n][4] (id,
        frame, duration, p as float32 bits), the state updated in place;
        also returns (iterations, prediction steps)."""
        enc = np.ascontiguousarray(enc, np.float32)
        T = enc.shape[0]
        st = state if state is not None else self.state()
        cap = cap or 16 * T + 1024
        toks = np.zeros((cap, 4), np.int32)
        last = C.c_int(st[2])
        it, npred = C.c_long(0), C.c_long(0)
        n = lib().orc_tdt_decode(self.h, p(enc), T, frame_offset, p(st[0]), p(st[1]), C.byref(last), p(toks), cap,
                                 C.byref(it), C.byref(npred))
        st[2] = last.value
        return toks[:min(n, cap)], it.value, npred.value

    def run(self, enc: np.ndarray, cap: int, threads: int):
        """n fresh decodes of enc [n][T][D] on host threads: (tokens [n][cap][4],
        counts [n], total iterations)."""
        enc = np.ascontiguousarray(enc, np.float32)
        n, T, D = enc.shape
        toks = np.zeros((n, cap, 4), np.int32)
        counts = np.zeros(n, np.int32)
        it = C.c_long(0)
        lib().orc_tdt_run(self.h, n, p(enc), T, D, p(toks), cap, p(counts), C.byref(it), threads)
        return toks, counts, it.value

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.orc_tdt_free(self.h)
            self.h = None


def q8_to_f16(q8) -> np.ndarray:
    """Q8_0 blocks widened as the Whisper loader does (model.go:486-490):
    float16 bits [rows][cols]."""
    out = np.empty((q8.rows, q8.cols), np.uint16)
    lib().orc_q8_to_f16(p(np.ascontiguousarray(q8.blocks)), q8.rows * q8.cols, p(out))
    return out


class Whisper:
    """The oracle's Whisper text decoder (whisper/decoder.go, transcribe.go)
    from the synthetic generator's tensors and words."""

    def __init__(self, cfg, tensors: dict, words: list[bytes]):
        from gorelaxor_b200.synth import Q8

        self.cfg = cfg
        self._keep = []
        L = lib()
        self.h = L.orc_whisper_new(cfg.n_vocab, cfg.n_text_ctx, cfg.n_state, cfg.n_head, cfg.n_text_layer)
        for name, arr in tensors.items():
            if isinstance(arr, Q8):
                buf = q8_to_f16(arr)
                L.orc_whisper_tensor(self.h, name.encode(), 1, arr.rows, arr.cols, p(buf))
            elif arr.dtype == np.float16:  # a float16 matrix (the convolutions)
                buf = np.ascontiguousarray(arr).view(np.uint16)
                L.orc_whisper_tensor(self.h, name.encode(), 1, arr.shape[0], arr.shape[1], p(buf))
            else:
                buf = np.ascontiguousarray(arr, np.float32)
                rows, cols = (buf.shape if buf.ndim == 2 else (1, buf.size))
                L.orc_whisper_tensor(self.h, name.encode(), 0, rows, cols, p(buf))
            self._keep.append(buf)
        blob = np.frombuffer(b"".join(words), np.uint8) if words else np.zeros(1, np.uint8)
        lens = np.array([len(w) for w in words], np.int32)
        self._keep += [blob, lens]
        L.orc_whisper_vocab(self.h, p(blob), p(lens), len(words))
        self.has_encoder = "encoder.conv1.weight" in tensors
        if self.has_encoder:
            L.orc_whisper_encoder(self.h, cfg.n_mels, cfg.n_head, cfg.n_audio_layer)
        if L.orc_whisper_ready(self.h) != 0:
            raise RuntimeError(L.orc_whisper_error(self.h).decode())

    def encode(self, mel: np.ndarray, blocks: int | None = None) -> np.ndarray:
        """encode (encoder.go:10-118): mel [n_mels][3000] → [1500][state];
        with `blocks`, the front end and that many blocks only (timing)."""
        out = np.empty((self.cfg.n_audio_ctx, self.cfg.n_state), np.float32)
        m = p(np.ascontiguousarray(mel, np.float32))
        if blocks is None:
            lib().orc_whisper_encode(self.h, m, p(out))
        else:
            lib().orc_whisper_encode_blocks(self.h, m, p(out), blocks)
        return out

    def suppress(self) -> list[int]:
        out = np.zeros(256, np.int32)
        n = lib().orc_whisper_suppress(self.h, p(out), 256)
        return out[:n].tolist()

    def seq(self, enc: np.ndarray | None = None):
        s = WSeq(lib().orc_wseq_new(self.h))
        if enc is not None:
            lib().orc_whisper_cross_kv(self.h, s.h, p(np.ascontiguousarray(enc, np.float32)))
        return s

    def cross(self, s, layer: int):
        c = self.cfg
        hd = c.n_state // c.n_head
        k = np.empty((c.n_head, c.n_audio_ctx, hd), np.float32)
        v = np.empty((c.n_head, hd, c.n_audio_ctx), np.float32)
        lib().orc_wseq_cross(s.h, layer, p(k), p(v))
        return k, v

    def decode(self, s, tokens, want):
        t = np.ascontiguousarray(tokens, np.int32)
        w = np.ascontiguousarray(want, np.int32)
        out = np.empty((len(w), self.cfg.n_vocab), np.float32)
        if lib().orc_whisper_decode(self.h, s.h, p(t), len(t), p(w), len(w), p(out)) != 0:
            return None
        return out

    def process_sample(self, state, lg):
        """state = (nt, last, penult, has_ts, seek_delta); lg is modified in
        place. Returns (id, tid, p, plog)."""
        st = np.ascontiguousarray(state, np.int32)
        out = np.zeros(4, np.int32)
        lib().orc_whisper_process_sample(self.h, p(st), p(lg), p(out))
        return int(out[0]), int(out[1]), float(out[2:3].view(np.float32)[0]), float(out[3:4].view(np.float32)[0])

    def greedy(self, s, prompt, sot_at: int, steps: int):
        """Tokens [n][4] (id, tid, p bits, plog bits) and the no-speech probability."""
        pr = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros((steps, 4), np.int32)
        ns = C.c_float(0)
        n = lib().orc_whisper_greedy(self.h, s.h, p(pr), len(pr), sot_at, steps, p(toks), C.byref(ns))
        return toks[:n], ns.value

    def run(self, enc: np.ndarray, prompt, sot_at: int, steps: int, threads: int) -> np.ndarray:
        """n streams (enc [n][ctx][state]) decoded on host threads: token ids [n][steps]."""
        enc = np.ascontiguousarray(enc, np.float32)
        pr = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros((enc.shape[0], steps), np.int32)
        lib().orc_whisper_run(self.h, enc.shape[0], p(enc), p(pr), len(pr), sot_at, steps, p(out), threads)
        return out

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.orc_whisper_free(self.h)
            self.h = None


class WSeq:
    def __init__(self, h):
        self.h = h

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.orc_wseq_free(self.h)
            self.h = None



# --------------------------------------------------------------- Mimi --


class Mimi:
    """The oracle's Mimi decoder (oracle/mimi.h), from a MimiConfig and the
    generator's tensor dict."""

    def __init__(self, mc, tensors: dict, ldim: int):
        from gorelaxor_b200.synth import Q8

        L = lib()
        self._keep = []
        r = np.ascontiguousarray(mc.ratios, np.int32)
        self._keep.append(r)
        self.h = L.orc_mimi_new(mc.d, mc.heads, mc.ff, mc.context, mc.max_period, mc.upsample, p(r), len(r), mc.nf,
                                mc.k, mc.resk, mc.lastk, mc.dil, mc.comp, mc.nres, ldim, mc.sample_rate)
        for name, arr in tensors.items():
            if not name.startswith("mimi."):
                continue
            if isinstance(arr, Q8):
                buf = np.ascontiguousarray(arr.blocks)
                L.orc_mimi_tensor(self.h, name.encode(), 2, arr.rows, arr.cols, p(buf))
            else:
                buf = np.ascontiguousarray(arr, np.float32)
                rows, cols = (buf.shape if buf.ndim == 2 else (1, buf.size))
                L.orc_mimi_tensor(self.h, name.encode(), 0, rows, cols, p(buf))
            self._keep.append(buf)
        if L.orc_mimi_ready(self.h) != 0:
            raise RuntimeError(L.orc_mimi_error(self.h).decode())
        self.frame = L.orc_mimi_frame(self.h)
        self.ldim = ldim

    def state(self):
        return MimiState(lib().orc_mimi_state(self.h))

    def clone_latents(self, x: np.ndarray) -> np.ndarray:
        """cloneCond's Mimi encoding (voice.go:113-124) of 24 kHz samples x:
        latents [frames][ldim]."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(((x.size + self.frame - 1) // self.frame, self.ldim), np.float32)
        n = lib().orc_mimi_clone_latents(self.h, p(x), x.size, p(out))
        if n < 0:
            raise RuntimeError("the Mimi tensors have no encoder")
        return out[:n]

    def decode(self, st: "MimiState", latent) -> np.ndarray:
        """One latent (already scaled) → one frame of samples, with
        speakChunk's fade-in on the state's first frame."""
        lat = np.ascontiguousarray(latent, np.float32)
        pcm = np.empty(self.frame, np.float32)
        lib().orc_mimi_decode(self.h, st.h, p(lat), p(pcm))
        return pcm

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_mimi_free(self.h)
            self.h = None


class MimiState:
    def __init__(self, h):
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_mimi_state_free(self.h)
            self.h = None


# ------------------------------------------------------- FastConformer --


class FConf:
    """The oracle's FastConformer encoder (oracle/conformer.h) from an
    FConfConfig and the generator's tensor dict."""

    def __init__(self, fc, tensors: dict):
        from gorelaxor_b200.synth import Q8

        L = lib()
        self.fc = fc
        self._keep = []
        self.h = L.orc_fconf_new(fc.d, fc.heads, fc.layers, fc.dff, fc.kernel, fc.sub_c, fc.n_mels,
                                 int(fc.xscaling), int(fc.conv_norm == "layer_norm"))
        for name, arr in tensors.items():
            if isinstance(arr, Q8):
                buf = np.ascontiguousarray(arr.blocks)
                L.orc_fconf_tensor(self.h, name.encode(), 2, arr.rows, arr.cols, p(buf))
            elif arr.dtype == np.float16:
                buf = np.ascontiguousarray(arr).view(np.uint16)
                L.orc_fconf_tensor(self.h, name.encode(), 1, arr.shape[0], arr.shape[-1], p(buf))
            else:
                buf = np.ascontiguousarray(arr, np.float32)
                L.orc_fconf_tensor(self.h, name.encode(), 0, 1, buf.size, p(buf))
            self._keep.append(buf)
        if L.orc_fconf_ready(self.h) != 0:
            raise RuntimeError(L.orc_fconf_error(self.h).decode())

    def encode(self, mel: np.ndarray, valid: int | None = None, blocks: int = -1) -> np.ndarray:
        """Model.encode (encoder.go:436-489): mel [n_mels][frames] → [L][d]."""
        mel = np.ascontiguousarray(mel, np.float32)
        frames = mel.shape[1]
        t = frames
        for _ in range(3):
            t = (t - 1) // 2 + 1
        out = np.empty((t, self.fc.d), np.float32)
        n = lib().orc_fconf_encode(self.h, p(mel), frames, frames if valid is None else valid, p(out), blocks)
        return out[:n]

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            lib().orc_fconf_free(self.h)
            self.h = None

