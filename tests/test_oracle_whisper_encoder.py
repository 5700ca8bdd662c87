"""The Whisper audio encoder oracle (oracle/whisper.h whisper_encode, which
restates whisper/encoder.go:10-118) against an independent float64 numpy
encoder written from the model: the same weights (float16 as the
reference's loader holds them), float64 arithmetic throughout."""

import dataclasses

import numpy as np

from gorelaxor_b200 import synth
from oracle import oracle as orc

SMALL_ENC = dataclasses.replace(synth.WhisperConfig(), n_state=64, n_head=1, n_audio_layer=2, n_text_layer=1,
                                n_mels=16, n_text_ctx=64)


def _np_encode(cfg, t, mel):
    D = lambda a: np.asarray(a, np.float64)

    def W(name):
        a = t[name]
        if isinstance(a, synth.Q8):  # the loader's widening: f16(q·d)
            return D(orc.q8_to_f16(a).view(np.float16))
        return D(a)

    def ln(x, w, b):
        m = x.mean(-1, keepdims=True)
        return (x - m) / np.sqrt(((x - m) ** 2).mean(-1, keepdims=True) + 1e-5) * D(t[w]) + D(t[b])

    gelu = lambda v: 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * v * (1 + 0.044715 * v * v)))
    st, W_ = cfg.n_state, 3000
    melp = np.pad(D(mel), ((0, 0), (1, 1)))
    x1 = np.stack([melp[:, k:k + W_] for k in range(3)], -1).transpose(1, 0, 2).reshape(W_, -1)  # [t][c·3+k]
    h1 = gelu(x1 @ W("encoder.conv1.weight").T + D(t["encoder.conv1.bias"]))
    h1p = np.pad(h1, ((1, 1), (0, 0)))
    x2 = np.stack([h1p[2 * np.arange(cfg.n_audio_ctx) + k] for k in range(3)], -1).reshape(cfg.n_audio_ctx, -1)
    x = gelu(x2 @ W("encoder.conv2.weight").T + D(t["encoder.conv2.bias"])) + D(t["encoder.positional_embedding"])
    nh, hd = cfg.n_head, st // cfg.n_head
    for i in range(cfg.n_audio_layer):
        p = f"encoder.blocks.{i}."
        cur = ln(x, p + "attn_ln.weight", p + "attn_ln.bias")
        q = cur @ W(p + "attn.query.weight").T + D(t[p + "attn.query.bias"])
        k = cur @ W(p + "attn.key.weight").T
        v = cur @ W(p + "attn.value.weight").T + D(t[p + "attn.value.bias"])
        att = np.empty_like(q)
        for h in range(nh):
            s = slice(h * hd, (h + 1) * hd)
            sc = (q[:, s] / np.sqrt(hd)) @ k[:, s].T
            e = np.exp(sc - sc.max(-1, keepdims=True))
            att[:, s] = (e / e.sum(-1, keepdims=True)) @ v[:, s]
        x = x + att @ W(p + "attn.out.weight").T + D(t[p + "attn.out.bias"])
        cur = ln(x, p + "mlp_ln.weight", p + "mlp_ln.bias")
        ff = gelu(cur @ W(p + "mlp.0.weight").T + D(t[p + "mlp.0.bias"]))
        x = x + ff @ W(p + "mlp.2.weight").T + D(t[p + "mlp.2.bias"])
    return ln(x, "encoder.ln_post.weight", "encoder.ln_post.bias")


def test_whisper_encode_against_numpy_model():
    """One window through the restated encoder (float32, the reference's
    orders) against the float64 model: within 1e-4 relative RMS."""
    cfg = SMALL_ENC
    t = synth.whisper_tensors(cfg, 0)
    t.update(synth.whisper_encoder_tensors(cfg, 0))
    om = orc.Whisper(cfg, t, synth.whisper_words(cfg))
    mel = synth.whisper_mel(1, cfg)
    got = om.encode(mel)
    want = _np_encode(cfg, t, mel)
    err = np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum())
    assert got.shape == (1500, cfg.n_state)
    assert err < 1e-4, err
