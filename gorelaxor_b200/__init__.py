"""B200 token-loop library: Python host mirror of include/grx.h.

The compute path is libgrx.so (CUDA kernels for sm_100a behind a C ABI);
this module only binds it with ctypes and mirrors the reference's Go API
for the token loop:

* ``Weight`` / ``linear`` — kern.Weight and kern.Linear
  (internal/kern/kern.go:41-201);
* ``FlowLM`` — pockettts.Model's flow LM (pockettts/model.go:202-322),
  ``FlowLM.load_voice`` — Model.LoadVoice (pockettts/voice.go:26-63);
* ``Streams`` — speakChunk's per-frame loop (pockettts/speak.go:146-175)
  for a batch of independent streams;
* ``GGUF`` — the internal/gguf reader.

There is no CPU fallback: importing works without a GPU, but every call
that computes needs libgrx.so and a CUDA device and raises otherwise.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libgrx.so"

GRX_ERRORS = {-1: "EINVAL", -2: "EFORMAT", -3: "ENOMEM", -4: "ECUDA", -5: "ERANGE", -6: "ENODEV", -7: "ETIMEDOUT"}

_lib = None


class GrxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"grx {GRX_ERRORS.get(code, code)}: {msg}")
        self.code = code


def _sig(lib):
    P, I, L, S, D, F = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_double, C.POINTER(C.c_float)
    PP = C.POINTER(C.c_void_p)
    sigs = {
        "grx_last_error": (I, [C.c_char_p, S]),
        "grx_device_count": (I, []),
        "grx_gguf_open": (I, [P, S, PP]),
        "grx_gguf_close": (None, [P]),
        "grx_gguf_int": (L, [P, C.c_char_p, L]),
        "grx_gguf_float": (D, [P, C.c_char_p, D]),
        "grx_gguf_string": (I, [P, C.c_char_p, C.c_char_p, S]),
        "grx_gguf_tensor": (I, [P, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int64)]),
        "grx_gguf_float32": (I, [P, C.c_char_p, P, S]),
        "grx_weight_q8": (I, [I, P, I, I, PP]),
        "grx_weight_f32": (I, [I, P, I, I, PP]),
        "grx_weight_drop_rows": (I, [P]),
        "grx_weight_free": (None, [P]),
        "grx_linear": (I, [P, P, I, P, P]),
        "grx_linear_q8_static": (I, [P, P, I, P, P, P]),
        "grx_flowlm_load": (I, [P, S, I, PP]),
        "grx_flowlm_free": (None, [P]),
        "grx_flowlm_dims": (I, [P] + [C.POINTER(C.c_int)] * 8),
        "grx_voice_load": (I, [P, P, S, PP]),
        "grx_voice_raw": (I, [P, I, P, PP]),
        "grx_voice_free": (None, [P]),
        "grx_voice_from_latents": (I, [P, P, I, PP]),
        "grx_voice_kv": (I, [P, P, P]),
        "grx_streams_create": (I, [P, I, P, I, PP]),
        "grx_streams_free": (None, [P]),
        "grx_streams_reset": (I, [P]),
        "grx_streams_text": (I, [P, P, P, P]),
        "grx_streams_step": (I, [P, P, P, P, P, P]),
        "grx_streams_run_device": (I, [P, I, P, P, P]),
        "grx_streams_sync": (I, [P]),
        "grx_streams_run_device_timed": (I, [P, I, P, P, P, P]),
        "grx_streams_pos": (I, [P, I]),
        "grx_streams_launches": (L, [P]),
        "grx_streams_cuda_stream": (P, [P]),
        "grx_streams_parts": (I, [P]),
        "grx_streams_persistent": (I, [P]),
        "grx_streams_watchdog_test": (I, [P]),
        "grx_mimi_load": (I, [P, S, I, PP]),
        "grx_mimi_free": (None, [P]),
        "grx_mimi_dims": (I, [P] + [C.POINTER(C.c_int)] * 8),
        "grx_mimi_streams_create": (I, [P, I, I, PP]),
        "grx_mimi_streams_free": (None, [P]),
        "grx_mimi_streams_reset": (I, [P]),
        "grx_mimi_decode": (I, [P, P, P]),
        "grx_mimi_decode_device": (I, [P, I, P, P]),
        "grx_mimi_sync": (I, [P]),
        "grx_mimi_cuda_stream": (P, [P]),
        "grx_mimi_launches": (L, [P]),
        "grx_mimi_frames": (I, [P]),
        "grx_mimi_encoder_create": (I, [P, I, I, PP]),
        "grx_mimi_encode_device": (I, [P, I, P, P]),
        "grx_mimi_encode": (I, [P, I, P, P]),
        "grx_mimi_clone_latents": (I, [P, P, I, P, C.POINTER(C.c_int)]),
        "grx_voice_clone": (I, [P, P, P, I, PP]),
        "grx_fconf_load": (I, [P, S, I, PP]),
        "grx_fconf_free": (None, [P]),
        "grx_fconf_dims": (I, [P] + [C.POINTER(C.c_int)] * 5),
        "grx_fconf_out_rows": (I, [I]),
        "grx_fconf_encode": (I, [P, P, I, I, P, C.POINTER(C.c_int)]),
        "grx_fconf_encode_device": (I, [P, P, I, I, P, C.POINTER(C.c_int)]),
        "grx_fconf_sync": (I, [P]),
        "grx_fconf_cuda_stream": (P, [P]),
        "grx_fconf_launches": (L, [P]),
        "grx_tdt_load": (I, [P, S, I, PP]),
        "grx_tdt_free": (None, [P]),
        "grx_tdt_dims": (I, [P] + [C.POINTER(C.c_int)] * 8),
        "grx_tdt_batch_create": (I, [P, I, I, I, PP]),
        "grx_tdt_batch_free": (None, [P]),
        "grx_tdt_batch_reset": (I, [P]),
        "grx_tdt_state_get": (I, [P, I, P, P, C.POINTER(C.c_int)]),
        "grx_tdt_state_set": (I, [P, I, P, P, I]),
        "grx_tdt_decode": (I, [P, P, P, P, P, P]),
        "grx_tdt_decode_device": (I, [P, P, P, P, P, P]),
        "grx_tdt_batch_cuda_stream": (P, [P]),
        "grx_tdt_batch_launches": (L, [P]),
        "grx_tdt_batch_iterations": (L, [P]),
        "grx_tdt_batch_stream_iterations": (L, [P]),
        "grx_whisper_load": (I, [P, S, I, PP]),
        "grx_whisper_free": (None, [P]),
        "grx_whisper_dims": (I, [P] + [C.POINTER(C.c_int)] * 6),
        "grx_whisper_tokens": (I, [P] + [C.POINTER(C.c_int)] * 6),
        "grx_whisper_suppressed": (I, [P, P, I]),
        "grx_whisper_exact_rows": (L, [P]),
        "grx_whisper_batch_create": (I, [P, I, PP]),
        "grx_whisper_batch_free": (None, [P]),
        "grx_whisper_set_audio": (I, [P, P]),
        "grx_whisper_set_audio_device": (I, [P, P]),
        "grx_whisper_encode": (I, [P, P]),
        "grx_whisper_encode_device": (I, [P, P]),
        "grx_whisper_encoder_out": (I, [P, P]),
        "grx_whisper_prompt": (I, [P, P, I, I, P]),
        "grx_whisper_run": (I, [P, I, P]),
        "grx_whisper_run_device": (I, [P, I, P]),
        "grx_whisper_sync": (I, [P]),
        "grx_whisper_persistent": (I, [P]),
        "grx_whisper_watchdog_test": (I, [P]),
        "grx_whisper_cross": (I, [P, I, I, P, P]),
        "grx_whisper_logits": (I, [P, P]),
        "grx_whisper_batch_cuda_stream": (P, [P]),
        "grx_whisper_batch_launches": (L, [P]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


# Free functions bound when the library loads: destructors that run while
# the interpreter shuts down must not look up module globals.
_FREE: dict = {}


def lib():
    """libgrx.so, loaded once. Raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m gorelaxor_b200.build`")
        _lib = _sig(C.CDLL(str(LIB_PATH)))
        for n in ("grx_gguf_close", "grx_weight_free", "grx_flowlm_free", "grx_voice_free", "grx_streams_free",
                  "grx_mimi_free", "grx_mimi_streams_free", "grx_fconf_free", "grx_tdt_free", "grx_tdt_batch_free", "grx_whisper_free",
                  "grx_whisper_batch_free"):
            _FREE[n] = getattr(_lib, n)
    return _lib


def last_error() -> str:
    """The calling thread's last error message (grx_last_error)."""
    buf = C.create_string_buffer(4096)
    lib().grx_last_error(buf, 4096)
    return buf.value.decode(errors="replace")


def _check(rc: int):
    if rc < 0:
        raise GrxError(rc, last_error())
    return rc


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def device_count() -> int:
    return lib().grx_device_count()


class GGUF:
    """internal/gguf's File: settings and tensors of a GGUF file."""

    def __init__(self, data: bytes):
        h = C.c_void_p()
        self._buf = data
        _check(lib().grx_gguf_open(data, len(data), C.byref(h)))
        self._h = h

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_gguf_close"](h)

    def int(self, key: str, default: int = -1) -> int:
        return lib().grx_gguf_int(self._h, key.encode(), default)

    def float(self, key: str, default: float = float("nan")) -> float:
        return lib().grx_gguf_float(self._h, key.encode(), default)

    def string(self, key: str) -> str:
        n = _check(lib().grx_gguf_string(self._h, key.encode(), None, 0))
        buf = C.create_string_buffer(n + 1)
        lib().grx_gguf_string(self._h, key.encode(), buf, n + 1)
        return buf.value.decode()

    def tensor(self, name: str):
        t = C.c_int()
        dims = (C.c_int64 * 4)()
        nd = _check(lib().grx_gguf_tensor(self._h, name.encode(), C.byref(t), dims))
        return t.value, [dims[i] for i in range(nd)]

    def float32(self, name: str) -> np.ndarray:
        _, dims = self.tensor(name)
        n = int(np.prod(dims))
        out = np.empty(n, dtype=np.float32)
        _check(lib().grx_gguf_float32(self._h, name.encode(), _ptr(out), n))
        return out.reshape(list(reversed(dims)))


class Weight:
    """kern.Weight on a device (kern.go:41-103)."""

    def __init__(self, h, rows, cols, kind):
        self._h, self.rows, self.cols, self.kind = h, rows, cols, kind

    @classmethod
    def q8(cls, blocks: np.ndarray, rows: int, cols: int, device: int = 0) -> "Weight":
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        h = C.c_void_p()
        _check(lib().grx_weight_q8(device, _ptr(b), rows, cols, C.byref(h)))
        return cls(h, rows, cols, "q8_0")

    @classmethod
    def f32(cls, v: np.ndarray, device: int = 0) -> "Weight":
        a = np.ascontiguousarray(v, dtype=np.float32)
        h = C.c_void_p()
        _check(lib().grx_weight_f32(device, _ptr(a), a.shape[0], a.shape[1], C.byref(h)))
        return cls(h, a.shape[0], a.shape[1], "f32")

    def drop_rows(self) -> "Weight":
        _check(lib().grx_weight_drop_rows(self._h))
        return self

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_weight_free"](h)


def linear(w: Weight, x: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """kern.Linear (kern.go:199): x [m][cols] → [m][rows]."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, w.cols)
    out = np.empty((x.shape[0], w.rows), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    _check(lib().grx_linear(w._h, _ptr(x), x.shape[0], _ptr(b), _ptr(out)))
    return out


STATIC_MAX_ELEMS = 1 << 20  # GRX_STATIC_MAX_ELEMS: the largest m × cols of linear_q8_static


def linear_q8_static(w: Weight, d_x: int, m: int, d_bias: int | None, d_dst: int, stream: int = 0) -> None:
    """grx_linear_q8_static: the int8 path of `linear` on caller-owned device
    buffers (addresses), queued on `stream`, allocating nothing — for hosts
    whose device memory is all owned by their own allocator. The rounded
    activations go to one fixed array shared by every call on the device:
    calls that may overlap on the GPU must be ordered by the caller."""
    _check(lib().grx_linear_q8_static(w._h, d_x, m, d_bias, d_dst, stream or None))


class FlowLM:
    """pockettts.Model's flow LM and flow head on one device."""

    def __init__(self, gguf: bytes, device: int = 0):
        h = C.c_void_p()
        _check(lib().grx_flowlm_load(gguf, len(gguf), device, C.byref(h)))
        self._h = h
        self.device = device
        v = [C.c_int() for _ in range(8)]
        _check(lib().grx_flowlm_dims(h, *[C.byref(x) for x in v]))
        self.d, self.heads, self.ff, self.layers, self.ldim, self.fdim, self.depth, self.steps = [x.value for x in v]

    def load_voice(self, gguf: bytes) -> "Voice":
        h = C.c_void_p()
        _check(lib().grx_voice_load(self._h, gguf, len(gguf), C.byref(h)))
        return Voice(h)

    def voice(self, kv: np.ndarray) -> "Voice":
        """A voice from caches [layers][2][positions][d]."""
        a = np.ascontiguousarray(kv, dtype=np.float32)
        h = C.c_void_p()
        _check(lib().grx_voice_raw(self._h, a.shape[2], _ptr(a), C.byref(h)))
        return Voice(h)

    def voice_clone(self, mimi: "Mimi", pcm: np.ndarray) -> "Voice":
        """Model.CloneVoice after resampling and end_on_pause (voice.go:
        94-106): Mimi's encoding of the 24 kHz clip, then the flow LM."""
        x = np.ascontiguousarray(pcm, dtype=np.float32).ravel()
        h = C.c_void_p()
        _check(lib().grx_voice_clone(self._h, mimi._h, _ptr(x), x.size, C.byref(h)))
        v = Voice(h)
        v._model = self
        return v

    def voice_from_latents(self, latents: np.ndarray) -> "Voice":
        """The voice a clip's Mimi latents [n][ldim] make (the flow-LM half
        of CloneVoice, voice.go:94-106)."""
        a = np.ascontiguousarray(latents, dtype=np.float32)
        h = C.c_void_p()
        _check(lib().grx_voice_from_latents(self._h, _ptr(a), a.shape[0], C.byref(h)))
        v = Voice(h)
        v._model = self
        return v

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_flowlm_free"](h)


class Voice:
    def __init__(self, h):
        self._h = h

    def kv(self, layers: int, d: int) -> np.ndarray:
        """The caches [layers][2][positions][d]."""
        n = C.c_int()
        _check(lib().grx_voice_kv(self._h, C.byref(n), None))
        out = np.empty((layers, 2, n.value, d), np.float32)
        _check(lib().grx_voice_kv(self._h, None, _ptr(out)))
        return out

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_voice_free"](h)


class Streams:
    """n independent FlowLM streams, each starting from its voice."""

    def __init__(self, model: FlowLM, voices: list[Voice], max_frames: int):
        self.model, self.n = model, len(voices)
        self._voices = voices
        arr = (C.c_void_p * self.n)(*[v._h.value for v in voices])
        h = C.c_void_p()
        _check(lib().grx_streams_create(model._h, self.n, arr, max_frames, C.byref(h)))
        self._h = h

    def reset(self):
        _check(lib().grx_streams_reset(self._h))

    def text(self, ids: list) -> np.ndarray:
        """flowLM.text for every stream (lm.go:172-181): ids[i] is stream i's
        list of token ids (may be empty). Returns [n][d], out_norm at each
        stream's last token (zeros for streams without tokens)."""
        if len(ids) != self.n:
            raise ValueError(f"text: {len(ids)} token lists for {self.n} streams")
        off = np.zeros(self.n + 1, np.int32)
        off[1:] = np.cumsum([len(t) for t in ids])
        flat = np.ascontiguousarray(np.concatenate([np.asarray(t, np.int32) for t in ids]) if off[-1] else
                                    np.zeros(1, np.int32), np.int32)
        out = np.zeros((self.n, self.model.d), np.float32)
        _check(lib().grx_streams_text(self._h, _ptr(flat), _ptr(off), _ptr(out)))
        return out

    def step(self, noise: np.ndarray, want_lm_out: bool = False):
        """One frame for every stream: returns (latent, eos, scaled, lm_out)."""
        m = self.model
        nz = np.ascontiguousarray(noise, dtype=np.float32).reshape(self.n, m.ldim)
        lat = np.empty((self.n, m.ldim), np.float32)
        sc = np.empty((self.n, m.ldim), np.float32)
        eos = np.empty(self.n, np.float32)
        lo = np.empty((self.n, m.d), np.float32) if want_lm_out else None
        _check(lib().grx_streams_step(self._h, _ptr(nz), _ptr(lo), _ptr(eos), _ptr(lat), _ptr(sc)))
        return lat, eos, sc, lo

    def run_device(self, frames: int, d_noise: int, d_latent: int, d_eos: int | None):
        """frames frames with device pointers (ints): noise [frames][n][ldim] in,
        latent [frames][n][ldim] and eos [frames][n] out. Asynchronous."""
        _check(lib().grx_streams_run_device(self._h, frames, C.c_void_p(d_noise), C.c_void_p(d_latent),
                                            C.c_void_p(d_eos) if d_eos else None))

    def run_device_timed(self, frames: int, d_noise: int, d_latent: int, d_eos: int | None, d_ts: int):
        """run_device that also records each attention kernel's span into the
        device array d_ts [frames][layers][parts][2] (uint64 ns, preset to
        {UINT64_MAX, 0})."""
        _check(lib().grx_streams_run_device_timed(self._h, frames, C.c_void_p(d_noise), C.c_void_p(d_latent),
                                                  C.c_void_p(d_eos) if d_eos else None, C.c_void_p(d_ts)))

    def sync(self):
        _check(lib().grx_streams_sync(self._h))

    def pos(self, i: int) -> int:
        return _check(lib().grx_streams_pos(self._h, i))

    def cuda_stream(self) -> int:
        """The cudaStream_t (as an int) the stream set's kernels run on."""
        return lib().grx_streams_cuda_stream(self._h) or 0

    def launches(self) -> int:
        return lib().grx_streams_launches(self._h)

    def parts(self) -> int:
        """1, or 2 when the set runs as two concurrent parts."""
        return _check(lib().grx_streams_parts(self._h))

    def persistent(self) -> bool:
        """Whether the set runs its frames in the persistent one-stream kernel."""
        return bool(_check(lib().grx_streams_persistent(self._h)))

    def watchdog_test(self) -> int:
        """Runs the persistent kernel with a grid barrier nothing completes;
        returns the status code its bounded waits give (GRX_ETIMEDOUT, -7)."""
        return lib().grx_streams_watchdog_test(self._h)

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_streams_free"](h)


# ------------------------------------------------------- Mimi decoder


class Mimi:
    """Pocket TTS's Mimi decoder (pockettts/mimi.go:24-150) on one device,
    from a Pocket TTS file."""

    def __init__(self, gguf: bytes, device: int = 0):
        h = C.c_void_p()
        _check(lib().grx_mimi_load(gguf, len(gguf), device, C.byref(h)))
        self._h = h
        self.device = device
        v = [C.c_int() for _ in range(8)]
        _check(lib().grx_mimi_dims(h, *[C.byref(x) for x in v]))
        (self.d, self.heads, self.layers, self.context, self.upsample, self.ldim, self.frame,
         self.sample_rate) = [x.value for x in v]

    def clone_latents(self, pcm: np.ndarray) -> np.ndarray:
        """cloneCond's Mimi encoding of one 24 kHz clip (voice.go:113-124):
        latents [frames][ldim], frames = ceil(len / frame)."""
        x = np.ascontiguousarray(pcm, dtype=np.float32).ravel()
        frames = -(-x.size // self.frame)
        out = np.empty((frames, self.ldim), np.float32)
        _check(lib().grx_mimi_clone_latents(self._h, _ptr(x), x.size, _ptr(out), None))
        return out

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_mimi_free"](h)


class MimiEncoder:
    """n clips through Mimi's encoder together (mimi.go:152-179), each from
    a fresh state, as cloneCond encodes one (voice.go:113-124)."""

    def __init__(self, model: Mimi, n: int, max_samples: int):
        self.model, self.n, self.max_samples = model, n, max_samples
        h = C.c_void_p()
        _check(lib().grx_mimi_encoder_create(model._h, n, max_samples, C.byref(h)))
        self._h = h

    def encode(self, pcm: np.ndarray) -> np.ndarray:
        """pcm [n][samples] → latents [n][frames][ldim]."""
        m = self.model
        x = np.ascontiguousarray(pcm, dtype=np.float32).reshape(self.n, -1)
        frames = -(-x.shape[1] // m.frame)
        out = np.empty((self.n, frames, m.ldim), np.float32)
        _check(lib().grx_mimi_encode(self._h, x.shape[1], _ptr(x), _ptr(out)))
        return out

    def encode_device(self, samples: int, d_pcm: int, d_latents: int):
        """Device pointers (ints): pcm [n][samples] in, latents
        [n][frames][ldim] out. Asynchronous."""
        _check(lib().grx_mimi_encode_device(self._h, samples, C.c_void_p(d_pcm), C.c_void_p(d_latents)))

    def sync(self):
        _check(lib().grx_mimi_sync(self._h))

    def cuda_stream(self) -> int:
        return lib().grx_mimi_cuda_stream(self._h) or 0

    def launches(self) -> int:
        return lib().grx_mimi_launches(self._h)

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_mimi_streams_free"](h)


class MimiStreams:
    """n independent decoder states (decState, mimi.go:108-124); each call
    turns one latent per stream into one frame per stream."""

    def __init__(self, model: Mimi, n: int, max_frames: int):
        self.model, self.n = model, n
        h = C.c_void_p()
        _check(lib().grx_mimi_streams_create(model._h, n, max_frames, C.byref(h)))
        self._h = h

    def reset(self):
        _check(lib().grx_mimi_streams_reset(self._h))

    def decode(self, latents: np.ndarray) -> np.ndarray:
        """latents [n][ldim] → samples [n][frame] (the first frame of each
        stream faded in, speak.go:185-190)."""
        m = self.model
        lat = np.ascontiguousarray(latents, dtype=np.float32).reshape(self.n, m.ldim)
        out = np.empty((self.n, m.frame), np.float32)
        _check(lib().grx_mimi_decode(self._h, _ptr(lat), _ptr(out)))
        return out

    def decode_device(self, frames: int, d_latents: int, d_pcm: int):
        """frames calls with device pointers (ints): latents [frames][n][ldim]
        in, samples [frames][n][frame] out. Asynchronous."""
        _check(lib().grx_mimi_decode_device(self._h, frames, C.c_void_p(d_latents), C.c_void_p(d_pcm)))

    def sync(self):
        _check(lib().grx_mimi_sync(self._h))

    def frames(self) -> int:
        return _check(lib().grx_mimi_frames(self._h))

    def cuda_stream(self) -> int:
        return lib().grx_mimi_cuda_stream(self._h) or 0

    def launches(self) -> int:
        return lib().grx_mimi_launches(self._h)

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_mimi_streams_free"](h)


# -------------------------------------------------- FastConformer encoder


class FConf:
    """conformer.Model's FastConformer encoder (encoder.go:123-489) on one
    device, from a parakeet GGUF; offline attention over all frames."""

    def __init__(self, gguf: bytes, device: int = 0):
        h = C.c_void_p()
        _check(lib().grx_fconf_load(gguf, len(gguf), device, C.byref(h)))
        self._h = h
        self.device = device
        v = [C.c_int() for _ in range(5)]
        _check(lib().grx_fconf_dims(h, *[C.byref(x) for x in v]))
        self.d, self.heads, self.layers, self.n_mels, self.sub_c = [x.value for x in v]

    def encode(self, mel: np.ndarray, valid: int | None = None) -> np.ndarray:
        """mel [n_mels][frames] (the first `valid` real) → [L][d]."""
        a = np.ascontiguousarray(mel, np.float32)
        frames = a.shape[1]
        out = np.empty((lib().grx_fconf_out_rows(frames), self.d), np.float32)
        rows = C.c_int()
        _check(lib().grx_fconf_encode(self._h, _ptr(a), frames, frames if valid is None else valid, _ptr(out),
                                      C.byref(rows)))
        return out[:rows.value]

    def encode_device(self, d_mel: int, frames: int, valid: int, d_out: int) -> int:
        """Device pointers (ints); asynchronous. Returns the valid rows."""
        rows = C.c_int()
        _check(lib().grx_fconf_encode_device(self._h, C.c_void_p(d_mel), frames, valid, C.c_void_p(d_out),
                                             C.byref(rows)))
        return rows.value

    def sync(self):
        _check(lib().grx_fconf_sync(self._h))

    def cuda_stream(self) -> int:
        return lib().grx_fconf_cuda_stream(self._h) or 0

    def launches(self) -> int:
        return lib().grx_fconf_launches(self._h)

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_fconf_free"](h)


# ------------------------------------------------------------ TDT decoder

TOKEN = np.dtype([("id", "<i4"), ("frame", "<i4"), ("duration", "<i4"), ("p", "<f4")])  # grx_tdt_token


class TDT:
    """The decoder of a conformer.Model (RNN-T or TDT head) on one device:
    conformer.FromGGUF's pred.* and joint.* part (model.go:306-314)."""

    def __init__(self, gguf: bytes, device: int = 0):
        h = C.c_void_p()
        _check(lib().grx_tdt_load(gguf, len(gguf), device, C.byref(h)))
        self._h = h
        self.device = device
        v = [C.c_int() for _ in range(8)]
        _check(lib().grx_tdt_dims(h, *[C.byref(x) for x in v]))
        (self.hidden, self.layers, self.vocab, self.joint, self.d_enc, self.n_durations, self.blank,
         is_tdt) = [x.value for x in v]
        self.is_tdt = bool(is_tdt)

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_tdt_free"](h)


class TDTBatch:
    """n DecoderStates decoded together: Model.Decode for each stream."""

    def __init__(self, model: TDT, n: int, max_t: int, cap: int):
        self.model, self.n, self.max_t, self.cap = model, n, max_t, cap
        h = C.c_void_p()
        _check(lib().grx_tdt_batch_create(model._h, n, max_t, cap, C.byref(h)))
        self._h = h

    def reset(self):
        _check(lib().grx_tdt_batch_reset(self._h))

    def state(self, i: int):
        """Stream i's DecoderState: (h [layers][hidden], c, last)."""
        m = self.model
        hh = np.empty((m.layers, m.hidden), np.float32)
        cc = np.empty_like(hh)
        last = C.c_int()
        _check(lib().grx_tdt_state_get(self._h, i, _ptr(hh), _ptr(cc), C.byref(last)))
        return hh, cc, last.value

    def set_state(self, i: int, h: np.ndarray, c: np.ndarray, last: int):
        h = np.ascontiguousarray(h, np.float32)
        c = np.ascontiguousarray(c, np.float32)
        _check(lib().grx_tdt_state_set(self._h, i, _ptr(h), _ptr(c), last))

    def decode(self, enc: np.ndarray, T, frame_offset=None):
        """enc [n][max_t][d_enc]; T [n]. Returns each stream's tokens (TOKEN
        records) and the full counts (which may exceed cap)."""
        e = np.ascontiguousarray(enc, np.float32).reshape(self.n, self.max_t, self.model.d_enc)
        t = np.ascontiguousarray(T, np.int32).reshape(self.n)
        off = None if frame_offset is None else np.ascontiguousarray(frame_offset, np.int32).reshape(self.n)
        toks = np.zeros((self.n, self.cap), TOKEN)
        counts = np.zeros(self.n, np.int32)
        _check(lib().grx_tdt_decode(self._h, _ptr(e), _ptr(t), _ptr(off), toks.ctypes.data, _ptr(counts)))
        return [toks[i, :min(int(counts[i]), self.cap)] for i in range(self.n)], counts

    def decode_device(self, d_enc: int, T, d_tokens: int, d_counts: int, frame_offset=None):
        t = np.ascontiguousarray(T, np.int32).reshape(self.n)
        off = None if frame_offset is None else np.ascontiguousarray(frame_offset, np.int32).reshape(self.n)
        _check(lib().grx_tdt_decode_device(self._h, C.c_void_p(d_enc), _ptr(t), _ptr(off), C.c_void_p(d_tokens),
                                           C.c_void_p(d_counts)))

    def cuda_stream(self) -> int:
        return lib().grx_tdt_batch_cuda_stream(self._h) or 0

    def launches(self) -> int:
        return lib().grx_tdt_batch_launches(self._h)

    def stream_iterations(self) -> int:
        """The last decode's loop iterations summed over its streams."""
        return int(_check(lib().grx_tdt_batch_stream_iterations(self._h)))

    def iterations(self) -> int:
        return lib().grx_tdt_batch_iterations(self._h)

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_tdt_batch_free"](h)


# ---------------------------------------------------------------- Whisper


class Whisper:
    """whisper.Model's text decoder on one device, from a whisper.cpp ggml file."""

    def __init__(self, data: bytes, device: int = 0):
        h = C.c_void_p()
        _check(lib().grx_whisper_load(data, len(data), device, C.byref(h)))
        self._h = h
        self.device = device
        v = [C.c_int() for _ in range(6)]
        _check(lib().grx_whisper_dims(h, *[C.byref(x) for x in v]))
        self.n_vocab, self.n_audio_ctx, self.n_state, self.n_head, self.n_text_layer, self.n_text_ctx = [x.value for x in v]
        t = [C.c_int() for _ in range(6)]
        _check(lib().grx_whisper_tokens(h, *[C.byref(x) for x in t]))
        self.eot, self.sot, self.prev, self.nosp, self.beg, self.n_lang = [x.value for x in t]

    def suppressed(self) -> list[int]:
        out = np.zeros(512, np.int32)
        n = _check(lib().grx_whisper_suppressed(self._h, _ptr(out), 512))
        return out[:n].tolist()

    def exact_rows(self) -> int:
        """Rows process/sample decided in the reference's sequential order
        (a parallel decision fell within its margin), since the model loaded."""
        return int(lib().grx_whisper_exact_rows(self._h))

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_whisper_free"](h)


class WhisperBatch:
    """n decoding sequences of a Whisper model."""

    def __init__(self, model: Whisper, n: int):
        self.model, self.n = model, n
        h = C.c_void_p()
        _check(lib().grx_whisper_batch_create(model._h, n, C.byref(h)))
        self._h = h

    def set_audio(self, enc: np.ndarray):
        e = np.ascontiguousarray(enc, np.float32)
        _check(lib().grx_whisper_set_audio(self._h, _ptr(e)))

    def set_audio_device(self, d_enc: int):
        _check(lib().grx_whisper_set_audio_device(self._h, C.c_void_p(d_enc)))

    def encode(self, mel: np.ndarray):
        """Model.encode (encoder.go:10-118) of each stream's window, mel
        [n][n_mels][3000], then the window's cross K/V (as set_audio)."""
        a = np.ascontiguousarray(mel, np.float32)
        _check(lib().grx_whisper_encode(self._h, _ptr(a)))

    def encode_device(self, d_mel: int):
        _check(lib().grx_whisper_encode_device(self._h, C.c_void_p(d_mel)))

    def encoder_out(self) -> np.ndarray:
        """The window's encoder output [n][1500][n_state]."""
        m = self.model
        out = np.empty((self.n, m.n_audio_ctx, m.n_state), np.float32)
        _check(lib().grx_whisper_encoder_out(self._h, _ptr(out)))
        return out

    def prompt(self, prompt, sot_at: int) -> np.ndarray:
        """prompt [n][np] (or one prompt for all); returns no_speech [n]."""
        pr = np.ascontiguousarray(np.broadcast_to(np.asarray(prompt, np.int32), (self.n, np.shape(prompt)[-1])))
        ns = np.zeros(self.n, np.float32)
        _check(lib().grx_whisper_prompt(self._h, _ptr(pr), pr.shape[1], sot_at, _ptr(ns)))
        return ns

    def run(self, steps: int) -> np.ndarray:
        """Tokens [steps][n][4] int32 (id, tid, p bits, plog bits)."""
        out = np.zeros((steps, self.n, 4), np.int32)
        _check(lib().grx_whisper_run(self._h, steps, _ptr(out)))
        return out

    def run_device(self, steps: int, d_tokens: int):
        _check(lib().grx_whisper_run_device(self._h, steps, C.c_void_p(d_tokens)))

    def sync(self):
        _check(lib().grx_whisper_sync(self._h))

    def persistent(self) -> bool:
        """Whether the batch runs its token loop in the persistent kernel."""
        return bool(_check(lib().grx_whisper_persistent(self._h)))

    def watchdog_test(self) -> int:
        """Runs one step with a grid barrier nothing completes; returns the
        status its bounded waits report (GRX_ETIMEDOUT when they work)."""
        return lib().grx_whisper_watchdog_test(self._h)

    def cross(self, i: int, layer: int):
        m = self.model
        k = np.empty((m.n_head, m.n_audio_ctx, m.n_state // m.n_head), np.float32)
        vt = np.empty((m.n_head, m.n_state // m.n_head, m.n_audio_ctx), np.float32)
        _check(lib().grx_whisper_cross(self._h, i, layer, _ptr(k), _ptr(vt)))
        return k, vt

    def logits(self) -> np.ndarray:
        out = np.empty((self.n, self.model.n_vocab), np.float32)
        _check(lib().grx_whisper_logits(self._h, _ptr(out)))
        return out

    def cuda_stream(self) -> int:
        return lib().grx_whisper_batch_cuda_stream(self._h) or 0

    def launches(self) -> int:
        return lib().grx_whisper_batch_launches(self._h)

    def __del__(self, _free=_FREE):
        h, self._h = getattr(self, "_h", None), None
        if h:
            _free["grx_whisper_batch_free"](h)

