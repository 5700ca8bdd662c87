"""Synthetic model and voice files for the token-loop workloads.

No weights ship with the reference (its model files are gitignored), so every
workload runs on seeded synthetic files written in the reference's own
formats:

* Pocket TTS FlowLM: a GGUF v3 file with the tensor names and settings that
  ``pockettts.Load`` reads (pockettts/model.go:202-278), and a voice GGUF with
  the keys ``LoadVoice`` reads (pockettts/voice.go:26-63).
* Parakeet TDT decoder: a GGUF v3 file with the decoder tensors
  ``conformer.fromGGUF`` reads (conformer/model.go:305-313).
* Whisper: a whisper.cpp ggml ``.bin`` file (whisper/model.go:117-226).

Which tensors are Q8_0 follows the converter's placement rule: matrices of at
least 64 by 64 whose rows are whole blocks (tools/convert_pocket_tts.py:150-156,
the same rule in tools/convert_nemo.py:289-339). Q8_0 blocks are drawn
directly from the benchmark's distributions (f16 scale = f16(|N(0, 0.002)|),
int8 uniform on [-127, 127]); everything else is float32.

The GGUF layout (header, key/value section, tensor table, 32-byte aligned
data) is the one internal/gguf/gguf.go:292-354 reads; tests/test_golden.py
checks a file written by the reference's own converter against this
library's reader.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
ALIGN = 32
QK = 32
Q8_BYTES = 34


# --------------------------------------------------------------------- GGUF


def _s(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


@dataclass
class Q8:
    """A Q8_0 matrix [rows][cols] held as raw 34-byte blocks."""

    rows: int
    cols: int
    blocks: np.ndarray  # uint8 [rows * cols/32 * 34]

    @property
    def shape(self):
        return (self.rows, self.cols)


def _le(v: int, width: int, signed: bool = False) -> bytes:
    return int(v).to_bytes(width, "little", signed=signed)


class GGUFWriter:
    """A GGUF v3 file built in memory, in the layout internal/gguf/gguf.go:
    292-354 parses: "GGUF", version 3, the tensor and key/value counts (u64);
    each key/value as a string key, a u32 type code and the value; the
    tensor table (name, dimension count, dims fastest-first as u64, the ggml
    type, the offset into the data section); zero padding to a 32-byte
    boundary, then each tensor's bytes, each starting on a 32-byte boundary
    of the data section (general.alignment's default)."""

    def __init__(self, arch: str):
        self._meta = bytearray()  # the encoded key/value pairs
        self._count = 0
        self._tensors: list[tuple[str, int, list[int], bytes]] = []
        self.str("general.architecture", arch)

    def _begin(self, key: str, code: int) -> bytearray:
        self._meta += _s(key) + _le(code, 4)
        self._count += 1
        return self._meta

    def u32(self, key, v):
        self._begin(key, T_U32).extend(_le(v, 4))

    def i32(self, key, v):
        self._begin(key, T_I32).extend(_le(v, 4, signed=True))

    def f32(self, key, v):
        self._begin(key, T_F32).extend(np.float32(v).tobytes())

    def bool(self, key, v):
        self._begin(key, T_BOOL).append(1 if v else 0)

    def str(self, key, v):
        self._begin(key, T_STR).extend(_s(str(v)))

    def i32s(self, key, v):
        vals = np.asarray([int(x) for x in v], dtype="<i4")
        self._begin(key, T_ARR).extend(_le(T_I32, 4) + _le(len(vals), 8) + vals.tobytes())

    def tensor(self, name: str, arr) -> None:
        """A Q8 matrix keeps its blocks; float16 and float32 arrays their
        values (dims listed fastest first, as ggml does)."""
        if isinstance(arr, Q8):
            self._tensors.append((name, GGML_Q8_0, [arr.cols, arr.rows], arr.blocks.tobytes()))
            return
        kind, dt = (GGML_F16, "<f2") if np.asarray(arr).dtype == np.float16 else (GGML_F32, "<f4")
        a = np.ascontiguousarray(arr, dtype=dt)
        self._tensors.append((name, kind, [int(d) for d in a.shape[::-1]] or [1], a.tobytes()))

    def to_bytes(self) -> bytes:
        def pad(n):
            return bytes((-n) % ALIGN)

        out = bytearray(b"GGUF" + _le(3, 4) + _le(len(self._tensors), 8) + _le(self._count, 8))
        out += self._meta
        at = 0  # where each tensor's bytes start in the data section
        for name, kind, dims, data in self._tensors:
            out += _s(name) + _le(len(dims), 4) + b"".join(_le(d, 8) for d in dims) + _le(kind, 4) + _le(at, 8)
            at += len(data) + len(pad(len(data)))
        out += pad(len(out))
        for _, _, _, data in self._tensors:
            out += data + pad(len(data))
        return bytes(out)


# ------------------------------------------------------- value distributions


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to IEEE half, ties to even (numpy's astype does RNE)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def rand_q8(rng: np.random.Generator, rows: int, cols: int, scale_sd: float = 0.002) -> Q8:
    """Q8_0 blocks with f16 scale f16(|N(0, scale_sd)|) and int8 uniform on
    [-127, 127]: the benchmark configs' weight distribution."""
    assert cols % QK == 0
    nblk = rows * cols // QK
    d = f32_to_f16_bits(np.abs(rng.normal(0.0, scale_sd, nblk)).astype(np.float32))
    q = rng.integers(-127, 128, size=(nblk, QK), dtype=np.int16).astype(np.int8)
    blk = np.empty((nblk, Q8_BYTES), dtype=np.uint8)
    blk[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
    blk[:, 2:] = q.view(np.uint8)
    return Q8(rows, cols, blk.reshape(-1))


def q8_dequant(w: Q8) -> np.ndarray:
    """Q8_0 blocks widened to float32: f16 scale times int8 (exact)."""
    b = w.blocks.reshape(-1, Q8_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(w.rows, w.cols)


def _n(rng, shape, sd):
    return rng.normal(0.0, sd, shape).astype(np.float32)


# ------------------------------------------------------------ Pocket TTS


@dataclass
class FlowLMConfig:
    d: int = 1024
    heads: int = 16
    ff: int = 4096
    layers: int = 6
    ldim: int = 32
    flow_dim: int = 512
    flow_depth: int = 1
    decode_steps: int = 1
    text_vocab: int = 4000  # text tokens; lm.embed has one row more (model.go:246)
    temperature: float = 0.3
    max_period: float = 10000.0
    sha: str = "synthetic-flowlm-seed0"


def flowlm_tensors(cfg: FlowLMConfig, seed: int = 0) -> dict:
    """Every tensor of a synthetic FlowLM, in the converter's names."""
    rng = np.random.default_rng(seed)
    d, ff, ld, fd = cfg.d, cfg.ff, cfg.ldim, cfg.flow_dim
    t: dict = {}
    for i in range(cfg.layers):
        p = f"lm.blk.{i}."
        t[p + "norm1.weight"] = 1.0 + _n(rng, d, 0.1)
        t[p + "norm1.bias"] = _n(rng, d, 0.1)
        t[p + "norm2.weight"] = 1.0 + _n(rng, d, 0.1)
        t[p + "norm2.bias"] = _n(rng, d, 0.1)
        t[p + "attn_qkv.weight"] = rand_q8(rng, 3 * d, d)
        t[p + "attn_out.weight"] = rand_q8(rng, d, d)
        t[p + "ff1.weight"] = rand_q8(rng, ff, d)
        t[p + "ff2.weight"] = rand_q8(rng, d, ff)
    t["lm.input.weight"] = _n(rng, (d, ld), 1.0 / np.sqrt(ld))
    t["lm.bos"] = _n(rng, ld, 1.0)
    t["lm.bos_voice"] = _n(rng, d, 1.0)
    t["lm.out_norm.weight"] = 1.0 + _n(rng, d, 0.1)
    t["lm.out_norm.bias"] = _n(rng, d, 0.1)
    t["lm.eos.weight"] = _n(rng, (1, d), 1.0 / np.sqrt(d))
    t["lm.eos.bias"] = np.array([-2.0], dtype=np.float32)
    t["lm.emb_mean"] = _n(rng, ld, 0.1)
    t["lm.emb_std"] = (0.5 + np.abs(_n(rng, ld, 1.0))).astype(np.float32)
    t["flow.cond.weight"] = rand_q8(rng, fd, d)
    t["flow.cond.bias"] = _n(rng, fd, 0.02)
    t["flow.input.weight"] = _n(rng, (fd, ld), 1.0 / np.sqrt(ld))
    t["flow.input.bias"] = _n(rng, fd, 0.02)
    half = 128
    for k in range(2):
        p = f"flow.time.{k}."
        t[p + "freqs"] = np.exp(-np.log(10000.0) * np.arange(half) / half).astype(np.float32)
        t[p + "fc1.weight"] = rand_q8(rng, fd, 2 * half)
        t[p + "fc1.bias"] = _n(rng, fd, 0.02)
        t[p + "fc2.weight"] = rand_q8(rng, fd, fd)
        t[p + "fc2.bias"] = _n(rng, fd, 0.02)
        t[p + "norm.alpha"] = 1.0 + _n(rng, fd, 0.1)
    for i in range(cfg.flow_depth):
        p = f"flow.res.{i}."
        t[p + "norm.weight"] = 1.0 + _n(rng, fd, 0.1)
        t[p + "norm.bias"] = _n(rng, fd, 0.1)
        t[p + "fc1.weight"] = rand_q8(rng, fd, fd)
        t[p + "fc1.bias"] = _n(rng, fd, 0.02)
        t[p + "fc2.weight"] = rand_q8(rng, fd, fd)
        t[p + "fc2.bias"] = _n(rng, fd, 0.02)
        t[p + "ada.weight"] = rand_q8(rng, 3 * fd, fd)
        t[p + "ada.bias"] = _n(rng, 3 * fd, 0.02)
    t["flow.final.ada.weight"] = rand_q8(rng, 2 * fd, fd)
    t["flow.final.ada.bias"] = _n(rng, 2 * fd, 0.02)
    t["flow.final.out.weight"] = _n(rng, (ld, fd), 1.0 / np.sqrt(fd))
    t["flow.final.out.bias"] = _n(rng, ld, 0.02)
    # the text embedding, drawn from its own generator so that the tensors
    # above do not depend on it
    t["lm.embed"] = rand_q8(np.random.default_rng(seed + 7919), cfg.text_vocab + 1, d)
    # voice cloning's projection of Mimi latents (float32: too narrow for
    # the converter's Q8_0 rule, convert_pocket_tts.py:150-156)
    t["lm.speaker_proj"] = _n(np.random.default_rng(seed + 104729), (d, ld), 1.0 / np.sqrt(ld))
    return t


@dataclass
class MimiConfig:
    """Mimi's decoder as a Pocket TTS file configures it (model.go:280-300);
    the defaults are a small one that still takes every product path: Q8_0
    for the first convolution, the first transposed one and the transformer
    (the converter's rule: both dimensions at least 64, columns whole
    blocks, convert_pocket_tts.py:150-156), float32 for the narrow last
    stages, and rows past 16 so that those take the packed kernel."""

    d: int = 128
    heads: int = 2
    ff: int = 256
    layers: int = 2
    context: int = 8
    max_period: float = 10000.0
    upsample: int = 4
    ratios: tuple = (5, 2)
    nf: int = 16
    k: int = 7
    resk: int = 3
    lastk: int = 3
    dil: int = 2
    comp: int = 2
    nres: int = 1
    frame_rate: float = 12.5

    @property
    def frame(self) -> int:
        return int(np.prod(self.ratios)) * self.upsample

    @property
    def sample_rate(self) -> int:
        return int(round(self.frame * self.frame_rate))


def _mat(rng, rows, cols):
    """A matrix the way the converter stores it: Q8_0 when both dimensions
    are at least 64 and the columns whole blocks, else float32; values of
    standard deviation 1/√cols."""
    sd = 1.0 / np.sqrt(cols)
    if rows >= 64 and cols >= 64 and cols % QK == 0:
        return rand_q8(rng, rows, cols, scale_sd=sd / 73.0)
    return _n(rng, (rows, cols), sd)


def mimi_tensors(mc: MimiConfig, ldim: int, seed: int = 0, encoder: bool = False) -> dict:
    """Mimi decoder tensors in the converter's names (model.go:102-200); with
    encoder, also the encoder's (SEANet encoder, mimi.enc_tf, mimi.down,
    model.go:181-200, 308-313)."""
    rng = np.random.default_rng(seed + 31337)
    d = mc.d
    t: dict = {"mimi.quant": _n(rng, (d, ldim), 1.0 / np.sqrt(ldim)),
               "mimi.up": _n(rng, d * 2 * mc.upsample, 0.5)}
    for i in range(mc.layers):
        p = f"mimi.dec_tf.{i}."
        t[p + "norm1.weight"] = 1.0 + _n(rng, d, 0.1)
        t[p + "norm1.bias"] = _n(rng, d, 0.1)
        t[p + "norm2.weight"] = 1.0 + _n(rng, d, 0.1)
        t[p + "norm2.bias"] = _n(rng, d, 0.1)
        t[p + "attn_qkv.weight"] = _mat(rng, 3 * d, d)
        t[p + "attn_out.weight"] = _mat(rng, d, d)
        t[p + "ff1.weight"] = _mat(rng, mc.ff, d)
        t[p + "ff2.weight"] = _mat(rng, d, mc.ff)
        t[p + "ls1"] = np.abs(_n(rng, d, 0.2))
        t[p + "ls2"] = np.abs(_n(rng, d, 0.2))

    def conv(name, cin, cout, k):
        t[name + ".weight"] = _mat(rng, cout, k * cin)
        t[name + ".bias"] = _n(rng, cout, 0.05)

    mult = 1 << len(mc.ratios)
    conv("mimi.dec.0", d, mult * mc.nf, mc.k)
    idx = 1
    for r in mc.ratios:
        idx += 1
        cin, cout = mult * mc.nf, mult * mc.nf // 2
        t[f"mimi.dec.{idx}.weight"] = _mat(rng, 2 * r * cout, cin)
        t[f"mimi.dec.{idx}.bias"] = _n(rng, cout, 0.05)
        idx += 1
        for _ in range(mc.nres):
            conv(f"mimi.dec.{idx}.1", cout, cout // mc.comp, mc.resk)
            conv(f"mimi.dec.{idx}.3", cout // mc.comp, cout, 1)
            idx += 1
        mult //= 2
    idx += 1
    conv(f"mimi.dec.{idx}", mc.nf, 1, mc.lastk)
    if encoder:
        rng2 = np.random.default_rng(seed + 65537)
        for i in range(mc.layers):
            p = f"mimi.enc_tf.{i}."
            t[p + "norm1.weight"] = 1.0 + _n(rng2, d, 0.1)
            t[p + "norm1.bias"] = _n(rng2, d, 0.1)
            t[p + "norm2.weight"] = 1.0 + _n(rng2, d, 0.1)
            t[p + "norm2.bias"] = _n(rng2, d, 0.1)
            t[p + "attn_qkv.weight"] = _mat(rng2, 3 * d, d)
            t[p + "attn_out.weight"] = _mat(rng2, d, d)
            t[p + "ff1.weight"] = _mat(rng2, mc.ff, d)
            t[p + "ff2.weight"] = _mat(rng2, d, mc.ff)
            t[p + "ls1"] = np.abs(_n(rng2, d, 0.2))
            t[p + "ls2"] = np.abs(_n(rng2, d, 0.2))

        def econv(name, cin, cout, k):
            t[name + ".weight"] = _mat(rng2, cout, k * cin)
            t[name + ".bias"] = _n(rng2, cout, 0.05)

        econv("mimi.enc.0", 1, mc.nf, mc.k)
        idx, mult = 1, 1
        for r in reversed(mc.ratios):
            dim = mult * mc.nf
            for _ in range(mc.nres):
                econv(f"mimi.enc.{idx}.1", dim, dim // mc.comp, mc.resk)
                econv(f"mimi.enc.{idx}.3", dim // mc.comp, dim, 1)
                idx += 1
            idx += 1
            econv(f"mimi.enc.{idx}", dim, 2 * dim, 2 * r)
            idx += 1
            mult *= 2
        idx += 1
        econv(f"mimi.enc.{idx}", mult * mc.nf, d, mc.lastk)
        t["mimi.down"] = _mat(rng2, ldim, 2 * mc.upsample * d)
    return t


def mimi_keys(g: "GGUFWriter", mc: MimiConfig) -> None:
    g.u32("pockettts.sample_rate", mc.sample_rate)
    g.f32("pockettts.frame_rate", mc.frame_rate)
    g.u32("pockettts.mimi.d_model", mc.d)
    g.u32("pockettts.mimi.heads", mc.heads)
    g.u32("pockettts.mimi.ff", mc.ff)
    g.u32("pockettts.mimi.context", mc.context)
    g.f32("pockettts.mimi.max_period", mc.max_period)
    g.u32("pockettts.mimi.upsample", mc.upsample)
    g.i32s("pockettts.seanet.ratios", list(mc.ratios))
    g.u32("pockettts.seanet.n_filters", mc.nf)
    g.u32("pockettts.seanet.dimension", mc.d)
    g.u32("pockettts.seanet.kernel_size", mc.k)
    g.u32("pockettts.seanet.residual_kernel_size", mc.resk)
    g.u32("pockettts.seanet.last_kernel_size", mc.lastk)
    g.u32("pockettts.seanet.dilation_base", mc.dil)
    g.u32("pockettts.seanet.compress", mc.comp)
    g.u32("pockettts.seanet.n_residual_layers", mc.nres)


def flowlm_gguf(cfg: FlowLMConfig, tensors: dict, mimi: "MimiConfig | None" = None) -> bytes:
    """A Pocket TTS file with the FlowLM's tensors (and, given mimi, the
    decoder's tensors in `tensors` and its keys)."""
    g = GGUFWriter("pockettts")
    if mimi is not None:
        mimi_keys(g, mimi)
    g.str("general.name", "Pocket TTS synthetic")
    g.str("general.source.sha256", cfg.sha)
    g.u32("pockettts.latent_dim", cfg.ldim)
    g.u32("pockettts.lm.d_model", cfg.d)
    g.u32("pockettts.lm.heads", cfg.heads)
    g.f32("pockettts.lm.max_period", cfg.max_period)
    g.u32("pockettts.lm.layers", cfg.layers)
    g.u32("pockettts.lm.ff", cfg.ff)
    g.u32("pockettts.flow.dim", cfg.flow_dim)
    g.u32("pockettts.flow.depth", cfg.flow_depth)
    g.f32("pockettts.temperature", cfg.temperature)
    g.u32("pockettts.decode_steps", cfg.decode_steps)
    g.f32("pockettts.eos_threshold", -4.0)
    g.u32("pockettts.min_frames_before_eos", 6)
    for name, arr in tensors.items():
        g.tensor(name, arr)
    return g.to_bytes()


def voice_tensors(cfg: FlowLMConfig, positions: int = 64, seed: int = 1) -> dict:
    """A voice prefill: per layer, keys and values [positions][d] of N(0,1)."""
    rng = np.random.default_rng(seed)
    t = {}
    for i in range(cfg.layers):
        t[f"voice.{i}.k"] = _n(rng, (positions, cfg.d), 1.0)
        t[f"voice.{i}.v"] = _n(rng, (positions, cfg.d), 1.0)
    return t


def voice_gguf(cfg: FlowLMConfig, tensors: dict) -> bytes:
    positions = next(iter(tensors.values())).shape[0]
    g = GGUFWriter("pockettts-voice")
    g.str("general.name", "synthetic voice")
    g.str("pockettts.voice.model.sha256", cfg.sha)
    g.u32("pockettts.voice.layers", cfg.layers)
    g.u32("pockettts.voice.positions", positions)
    for name, arr in tensors.items():
        g.tensor(name, arr)
    return g.to_bytes()


def noise_frames(seed: int, frames: int, ldim: int, temperature: float) -> np.ndarray:
    """Per-frame flow-head noise N(0,1)·√temperature (speak.go:148-154 draws
    it from Go's PCG; the reference tests inject it, ref_test.go:168-172, and
    so does this harness)."""
    rng = np.random.default_rng(10_000 + seed)
    std = np.float32(np.sqrt(np.float64(np.float32(temperature))))
    return (rng.normal(0.0, 1.0, (frames, ldim)).astype(np.float32) * std).astype(np.float32)


# ---------------------------------------------------------- Parakeet TDT


@dataclass
class TDTConfig:
    """The decoder of a Parakeet-TDT-shaped transducer (conformer/model.go
    HParams): 2-layer LSTM prediction net, relu joint, 1025 tokens (blank
    last) plus 5 durations."""

    H: int = 640  # predictor.hidden
    layers: int = 2  # predictor.n_layers
    V: int = 1025  # predictor.vocab, tokens plus blank
    J: int = 640  # joint.hidden
    D: int = 640  # encoder output width
    durations: tuple = (0, 1, 2, 3, 4)
    max_symbols: int = 10
    act: str = "relu"
    head: str = "tdt"
    # The blank logit is lifted by blank_lift × √(2 ln V) token-logit
    # deviations (about the expected maximum of the others) so that, as in a
    # trained model, many iterations emit nothing; random weights alone would
    # emit a token nearly every time.
    blank_lift: float = 0.8

    @property
    def blank(self) -> int:
        return self.V - 1


def tdt_tensors(cfg: TDTConfig, seed: int = 0) -> dict:
    """The decoder tensors in the converter's names (convert_nemo.py:686-695):
    matrices as Q8_0, the embedding and biases F32."""
    rng = np.random.default_rng(seed)
    H, J, D = cfg.H, cfg.J, cfg.D
    t: dict = {"pred.embed.weight": _n(rng, (cfg.V, H), 1.0)}
    for i in range(cfg.layers):
        p = f"pred.lstm.{i}."
        t[p + "Wx"] = rand_q8(rng, 4 * H, H)
        t[p + "Wh"] = rand_q8(rng, 4 * H, H)
        t[p + "bias"] = _n(rng, 4 * H, 0.1)
    t["joint.enc.weight"] = rand_q8(rng, J, D)
    t["joint.enc.bias"] = _n(rng, J, 0.1)
    t["joint.pred.weight"] = rand_q8(rng, J, H)
    t["joint.pred.bias"] = _n(rng, J, 0.1)
    nout = cfg.V + (len(cfg.durations) if cfg.head == "tdt" else 0)
    t["joint.out.weight"] = rand_q8(rng, nout, J)
    # Centre each output on the relu hidden's mean, σ/√(2π) for the hidden's
    # spread σ (encoder part N(0,1) inputs, prediction part |h| ≈ 0.55), so
    # that no token wins on its row sum alone; then lift the blank: most
    # iterations emit nothing, as with a trained model.
    we = q8_dequant(t["joint.enc.weight"]).astype(np.float64)
    wp = q8_dequant(t["joint.pred.weight"]).astype(np.float64)
    sigma = np.sqrt((we ** 2).sum(axis=1).mean() + 0.3 * (wp ** 2).sum(axis=1).mean())
    rowsum = q8_dequant(t["joint.out.weight"]).astype(np.float64).sum(axis=1)
    b = (_n(rng, nout, 0.1) - sigma / np.sqrt(2 * np.pi) * rowsum).astype(np.float32)
    wo = q8_dequant(t["joint.out.weight"]).astype(np.float64)
    sd_logit = np.sqrt((wo ** 2).sum(axis=1).mean() * sigma ** 2 / 2)
    b[cfg.blank] += np.float32(cfg.blank_lift * np.sqrt(2 * np.log(cfg.V)) * sd_logit)
    t["joint.out.bias"] = b
    return t


def tdt_gguf(cfg: TDTConfig, tensors: dict) -> bytes:
    """A parakeet GGUF with the decoder settings conformer/model.go:190-236
    reads (the encoder's tensors are out of scope and not written)."""
    g = GGUFWriter("parakeet")
    p = "stt.parakeet."
    g.str("general.name", "Parakeet TDT synthetic decoder")
    g.str(p + "head_kind", cfg.head)
    g.u32(p + "predictor.hidden", cfg.H)
    g.u32(p + "predictor.n_layers", cfg.layers)
    g.u32(p + "predictor.vocab", cfg.V)
    g.u32(p + "joint.hidden", cfg.J)
    g.str(p + "joint.activation", cfg.act)
    g.u32(p + "encoder.d_model", cfg.D)
    if cfg.head == "tdt":
        g.i32s(p + "tdt.durations", cfg.durations)
        g.u32(p + "tdt.max_symbols", cfg.max_symbols)
    g.u32("tokenizer.ggml.blank_token_id", cfg.blank)
    for name, arr in tensors.items():
        g.tensor(name, arr)
    return g.to_bytes()


@dataclass
class FConfConfig:
    """A FastConformer encoder (conformer/model.go:160-189, 350-410); the
    defaults are a small one of Parakeet's shape rules (8× depthwise-striding
    subsampling, relative-position attention over all frames, centred
    depthwise convolution, batch norm). Parakeet TDT 0.6B is d 1024, 8 heads,
    24 layers, d_ff 4096, 256 subsampling channels, 128 mels."""

    d: int = 128
    heads: int = 2
    layers: int = 2
    dff: int = 512
    kernel: int = 9
    sub_c: int = 64
    n_mels: int = 32
    xscaling: bool = True
    conv_norm: str = "batch_norm"

    @property
    def sub_f(self) -> int:
        f = self.n_mels
        for _ in range(3):
            f = (f - 1) // 2 + 1
        return f


def fconf_tensors(fc: FConfConfig, seed: int = 0) -> dict:
    """The encoder's tensors in the converter's names (model.go:350-410):
    the blocks' linear layers and the subsampling's pointwise convolutions
    Q8_0, the 1×1 convolutions of the conv module float16 (as the converter
    keeps them), taps, norms, biases and batch-norm statistics float32.
    Weights of standard deviation about 1/√fan-in."""
    rng = np.random.default_rng(seed + 777)
    d, c, K = fc.d, fc.sub_c, fc.kernel

    def q8(rows, cols):
        return rand_q8(rng, rows, cols, scale_sd=1 / np.sqrt(cols) / 73.0)

    pe = "enc.pre_encode."
    t: dict = {pe + "conv.0.weight": _n(rng, (c, 1, 3, 3), 1 / 3.0), pe + "conv.0.bias": _n(rng, c, 0.1),
               pe + "conv.2.weight": _n(rng, (c, 1, 3, 3), 1 / 3.0), pe + "conv.2.bias": _n(rng, c, 0.1),
               pe + "conv.3.weight": q8(c, c), pe + "conv.3.bias": _n(rng, c, 0.1),
               pe + "conv.5.weight": _n(rng, (c, 1, 3, 3), 1 / 3.0), pe + "conv.5.bias": _n(rng, c, 0.1),
               pe + "conv.6.weight": q8(c, c), pe + "conv.6.bias": _n(rng, c, 0.1),
               pe + "out.weight": q8(d, c * fc.sub_f), pe + "out.bias": _n(rng, d, 0.1)}
    for i in range(fc.layers):
        p = f"enc.blocks.{i}."
        for n in ("norm_ff1", "norm_attn", "norm_conv", "norm_ff2", "norm_out"):
            t[p + n + ".weight"] = 1.0 + _n(rng, d, 0.1)
            t[p + n + ".bias"] = _n(rng, d, 0.1)
        for ff in ("ff1", "ff2"):
            t[f"{p}{ff}.linear1.weight"] = q8(fc.dff, d)
            t[f"{p}{ff}.linear1.bias"] = _n(rng, fc.dff, 0.1)
            t[f"{p}{ff}.linear2.weight"] = q8(d, fc.dff)
            t[f"{p}{ff}.linear2.bias"] = _n(rng, d, 0.1)
        for w in ("q", "k", "v", "out"):
            t[f"{p}attn.linear_{w}.weight"] = q8(d, d)
            t[f"{p}attn.linear_{w}.bias"] = _n(rng, d, 0.1)
        t[p + "attn.linear_pos.weight"] = q8(d, d)
        t[p + "attn.pos_bias_u"] = _n(rng, (fc.heads, d // fc.heads), 0.1)
        t[p + "attn.pos_bias_v"] = _n(rng, (fc.heads, d // fc.heads), 0.1)
        t[p + "conv.pointwise1.weight"] = (rng.normal(0, 1 / np.sqrt(d), (2 * d, d))).astype(np.float16)
        t[p + "conv.pointwise1.bias"] = _n(rng, 2 * d, 0.1)
        t[p + "conv.depthwise.weight"] = _n(rng, (d, 1, K), 1 / np.sqrt(K))
        t[p + "conv.depthwise.bias"] = _n(rng, d, 0.1)
        t[p + "conv.bn.weight"] = 1.0 + _n(rng, d, 0.1)
        t[p + "conv.bn.bias"] = _n(rng, d, 0.1)
        t[p + "conv.bn.running_mean"] = _n(rng, d, 0.1)
        t[p + "conv.bn.running_var"] = (1.0 + np.abs(_n(rng, d, 0.3))).astype(np.float32)
        t[p + "conv.pointwise2.weight"] = (rng.normal(0, 1 / np.sqrt(d), (d, d))).astype(np.float16)
        t[p + "conv.pointwise2.bias"] = _n(rng, d, 0.1)
    return t


def fconf_gguf(fc: FConfConfig, tensors: dict, style: str = "regular") -> bytes:
    """A parakeet GGUF with the encoder's settings (model.go:160-189) and
    tensors (style: the attention's att_context_style)."""
    g = GGUFWriter("parakeet")
    p = "stt.parakeet.encoder."
    g.str("general.name", "Parakeet FastConformer synthetic encoder")
    g.u32(p + "d_model", fc.d)
    g.u32(p + "n_heads", fc.heads)
    g.u32(p + "n_layers", fc.layers)
    g.u32(p + "d_ff", fc.dff)
    g.u32(p + "conv_kernel", fc.kernel)
    g.u32(p + "subsampling_channels", fc.sub_c)
    g.u32(p + "subsampling_factor", 8)
    g.bool(p + "xscaling", fc.xscaling)
    g.str(p + "att_context_style", style)
    g.str(p + "conv_norm_type", fc.conv_norm)
    g.u32("stt.frontend.num_mels", fc.n_mels)
    for name, arr in tensors.items():
        g.tensor(name, arr)
    return g.to_bytes()


def fconf_mel(seed: int, n_mels: int, frames: int) -> np.ndarray:
    """Log-mel features [mels][frames] as NeMo's per-feature normalisation
    leaves them (about N(0, 1))."""
    return np.random.default_rng(50_000 + seed).normal(0.0, 1.0, (n_mels, frames)).astype(np.float32)


def encoder_frames(seed: int, T: int, D: int) -> np.ndarray:
    """Encoder output [T][D] of N(0,1) values for stream `seed`."""
    return np.random.default_rng(20_000 + seed).normal(0.0, 1.0, (T, D)).astype(np.float32)


# --------------------------------------------------------------- Whisper


@dataclass
class WhisperConfig:
    """A whisper.cpp ggml model's hparams (whisper/model.go:16-21, 117-135);
    the defaults are base.en's."""

    n_vocab: int = 51864
    n_audio_ctx: int = 1500
    n_state: int = 512
    n_head: int = 8
    n_audio_layer: int = 6
    n_text_ctx: int = 448
    n_text_layer: int = 6
    n_mels: int = 80
    ftype: int = 8  # matrices as Q8_0
    n_words: int = 50256  # vocabulary entries written to the file (text tokens)


GGML_MAGIC = 0x67676D6C

# Words placed in the synthetic vocabulary at fixed ids so that the
# reference's suppression rules (vocab.go:96-118) and the initial " " rule
# (transcribe.go:383-385) have tokens to act on.
WHISPER_MARKED = {220: " ", 12: "(", 13: " (", 60: "♪", 61: " ♪", 1000: " -", 1001: " '", 1002: "<<", 5000: "[["}


def whisper_words(cfg: WhisperConfig) -> list[bytes]:
    words = [f"w{i}".encode() for i in range(cfg.n_words)]
    for i, w in WHISPER_MARKED.items():
        if i < cfg.n_words:
            words[i] = w.encode()
    return words


def whisper_q8_bytes(cfg: "WhisperConfig") -> int:
    """Q8_0 bytes a decode step reads once per token row: the token
    embedding (the logits product), and per layer the self-attention's q, k,
    v, o, the cross-attention's q and o (its k and v act on the encoder
    output once per window) and the two MLP matrices."""
    st = cfg.n_state
    return (cfg.n_vocab * st + cfg.n_text_layer * (6 * st * st + 8 * st * st)) * Q8_BYTES // QK


def whisper_tensors(cfg: WhisperConfig, seed: int = 0) -> dict:
    """The text decoder's tensors in whisper.cpp's names (model.go:464-484):
    matrices as Q8_0 (ftype 8), vectors and positions float32. The encoder's
    tensors are not made (the decoder consumes its output)."""
    rng = np.random.default_rng(seed)
    st = cfg.n_state
    t: dict = {"decoder.positional_embedding": _n(rng, (cfg.n_text_ctx, st), 0.1),
               "decoder.token_embedding.weight": rand_q8(rng, cfg.n_vocab, st),
               "decoder.ln.weight": 1.0 + _n(rng, st, 0.1), "decoder.ln.bias": _n(rng, st, 0.1)}
    for i in range(cfg.n_text_layer):
        p = f"decoder.blocks.{i}."
        for ln in ("attn_ln", "cross_attn_ln", "mlp_ln"):
            t[p + ln + ".weight"] = 1.0 + _n(rng, st, 0.1)
            t[p + ln + ".bias"] = _n(rng, st, 0.1)
        for a in ("attn", "cross_attn"):
            for w in ("query", "key", "value", "out"):
                t[f"{p}{a}.{w}.weight"] = rand_q8(rng, st, st)
                if w != "key":
                    t[f"{p}{a}.{w}.bias"] = _n(rng, st, 0.1)
        t[p + "mlp.0.weight"] = rand_q8(rng, 4 * st, st)
        t[p + "mlp.0.bias"] = _n(rng, 4 * st, 0.1)
        t[p + "mlp.2.weight"] = rand_q8(rng, st, 4 * st)
        t[p + "mlp.2.bias"] = _n(rng, st, 0.1)
    return t


def whisper_encoder_tensors(cfg: WhisperConfig, seed: int = 0) -> dict:
    """The audio encoder's tensors in whisper.cpp's names (model.go:352-372):
    the convolutions float16 (as whisper.cpp's quantized files keep them;
    [state][in·3], a row's values (channel, tap) → channel·3 + tap), the
    blocks' matrices Q8_0, vectors and positions float32. Weights of
    standard deviation about 1/√cols keep activations O(1) through the
    layers."""
    rng = np.random.default_rng(seed + 4242)
    st = cfg.n_state

    def f16(rows, cols):
        return (rng.normal(0, 1 / np.sqrt(cols), (rows, cols))).astype(np.float16)

    def q8(rows, cols):
        return rand_q8(rng, rows, cols, scale_sd=1 / np.sqrt(cols) / 73.0)

    t: dict = {"encoder.positional_embedding": _n(rng, (cfg.n_audio_ctx, st), 0.1),
               "encoder.conv1.weight": f16(st, cfg.n_mels * 3), "encoder.conv1.bias": _n(rng, st, 0.1),
               "encoder.conv2.weight": f16(st, st * 3), "encoder.conv2.bias": _n(rng, st, 0.1),
               "encoder.ln_post.weight": 1.0 + _n(rng, st, 0.1), "encoder.ln_post.bias": _n(rng, st, 0.1)}
    for i in range(cfg.n_audio_layer):
        p = f"encoder.blocks.{i}."
        for ln in ("attn_ln", "mlp_ln"):
            t[p + ln + ".weight"] = 1.0 + _n(rng, st, 0.1)
            t[p + ln + ".bias"] = _n(rng, st, 0.1)
        for w in ("query", "key", "value", "out"):
            t[f"{p}attn.{w}.weight"] = q8(st, st)
            if w != "key":
                t[f"{p}attn.{w}.bias"] = _n(rng, st, 0.1)
        t[p + "mlp.0.weight"] = q8(4 * st, st)
        t[p + "mlp.0.bias"] = _n(rng, 4 * st, 0.1)
        t[p + "mlp.2.weight"] = q8(st, 4 * st)
        t[p + "mlp.2.bias"] = _n(rng, st, 0.1)
    return t


def whisper_mel(seed: int, cfg: WhisperConfig) -> np.ndarray:
    """A window's log-mel [n_mels][3000] for stream `seed`: values in the
    range logMel gives (its floor max − 8 and the (v + 4)/4 scaling, mel.go:
    80-95), here N(0, 0.5) around −0.3."""
    return np.random.default_rng(40_000 + seed).normal(-0.3, 0.5, (cfg.n_mels, 3000)).astype(np.float32)


def whisper_ggml(cfg: WhisperConfig, tensors: dict, words: list[bytes] | None = None, seed: int = 0,
                 f16_bits: dict | None = None) -> bytes:
    """A whisper.cpp model file (model.go:115-223): magic, hparams, mel
    filters, vocabulary, then the tensors (dims fastest first). f16_bits
    maps names to float16 bit arrays written as F16 tensors instead."""
    rng = np.random.default_rng(seed + 77)
    words = whisper_words(cfg) if words is None else words
    out = [struct.pack("<I", GGML_MAGIC)]
    out.append(struct.pack("<11i", cfg.n_vocab, cfg.n_audio_ctx, cfg.n_state, cfg.n_head, cfg.n_audio_layer,
                           cfg.n_text_ctx, cfg.n_state, cfg.n_head, cfg.n_text_layer, cfg.n_mels, cfg.ftype))
    out.append(struct.pack("<ii", cfg.n_mels, 201))
    out.append(np.abs(rng.normal(0, 0.01, (cfg.n_mels, 201))).astype("<f4").tobytes())
    out.append(struct.pack("<i", len(words)))
    for w in words:
        out.append(struct.pack("<i", len(w)) + w)
    for name, arr in tensors.items():
        nb = name.encode()
        if f16_bits and name in f16_bits:
            h = np.ascontiguousarray(f16_bits[name], dtype="<u2")
            dims, typ, data = list(reversed(h.shape)), 1, h.tobytes()
        elif isinstance(arr, Q8):
            dims, typ, data = [arr.cols, arr.rows], 8, arr.blocks.tobytes()
        elif arr.dtype == np.float16:
            h = np.ascontiguousarray(arr, dtype="<f2")
            dims, typ, data = list(reversed(h.shape)), 1, h.tobytes()
        else:
            a = np.ascontiguousarray(arr, dtype="<f4")
            dims, typ, data = list(reversed(a.shape)), 0, a.tobytes()
        out.append(struct.pack("<iii", len(dims), len(nb), typ) + struct.pack(f"<{len(dims)}i", *dims) + nb + data)
    return b"".join(out)


def whisper_encoder_out(seed: int, cfg: WhisperConfig) -> np.ndarray:
    """Encoder output [n_audio_ctx][n_state] of N(0,1) values for stream `seed`."""
    return np.random.default_rng(30_000 + seed).normal(0.0, 1.0, (cfg.n_audio_ctx, cfg.n_state)).astype(np.float32)
