"""GPU parity for the Whisper audio encoder: grx_whisper_encode through the
C ABI against the oracle's encode (oracle/whisper.h, restating
whisper/encoder.go:10-118), bit for bit, on a small model of the
reference's shape rules (1500 positions, 3000 frames, 64-value heads); then
the window's cross K/V from that output, and a token loop from it."""

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import mismatch
from tests.test_oracle_whisper_encoder import SMALL_ENC

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _model(cfg, seed=0):
    t = synth.whisper_tensors(cfg, seed)
    t.update(synth.whisper_encoder_tensors(cfg, seed))
    words = synth.whisper_words(cfg)
    return t, words, synth.whisper_ggml(cfg, t, words)


def _check(got, want, what):
    ne, rel = mismatch(got, want)
    assert ne == 0, f"{what}: {ne} of {got.size} differ (max rel {rel:.2e})"
    assert rel <= TOL


@pytest.mark.parametrize("n", [1, 3])
def test_whisper_encode_bit_exact(have_gpu, n):
    """Each stream's window through the encoder: identical float32 to the
    oracle's, then the cross K/V of every decoder layer from it."""
    cfg = SMALL_ENC
    t, words, gg = _model(cfg, n)
    om = orc.Whisper(cfg, t, words)
    mel = np.stack([synth.whisper_mel(10 * n + i, cfg) for i in range(n)])
    gm = g.Whisper(gg)
    b = g.WhisperBatch(gm, n)
    b.encode(mel)
    got = b.encoder_out()
    for i in range(n):
        want = om.encode(mel[i])
        _check(got[i], want, f"encoder output, stream {i}")
        s = om.seq(want)
        for layer in range(cfg.n_text_layer):
            gk, gv = b.cross(i, layer)
            ok, ov = om.cross(s, layer)
            _check(gk, ok, f"cross K stream {i} layer {layer}")
            _check(gv, ov, f"cross V stream {i} layer {layer}")


def test_whisper_encode_then_tokens(have_gpu):
    """A window from audio to tokens on the device: encode, prompt, greedy
    steps; the tokens equal the oracle's loop on the oracle's encoder output."""
    cfg = SMALL_ENC
    t, words, gg = _model(cfg, 5)
    om = orc.Whisper(cfg, t, words)
    mel = synth.whisper_mel(77, cfg)[None]
    gm = g.Whisper(gg)
    b = g.WhisperBatch(gm, 1)
    b.encode(mel)
    prompt, sot_at = [gm.prev, 100, 200, gm.sot], 3
    b.prompt(prompt, sot_at)
    got = b.run(12)
    want, _ = om.greedy(om.seq(om.encode(mel[0])), prompt, sot_at, 12)
    assert np.array_equal(got[:, 0, 0], want[:, 0]), f"{got[:, 0, 0].tolist()} vs {want[:, 0].tolist()}"


def test_whisper_encode_needs_encoder(have_gpu):
    cfg = SMALL_ENC
    t = synth.whisper_tensors(cfg, 0)
    gm = g.Whisper(synth.whisper_ggml(cfg, t, synth.whisper_words(cfg)))
    b = g.WhisperBatch(gm, 1)
    with pytest.raises(g.GrxError, match="no encoder"):
        b.encode(np.zeros((1, cfg.n_mels, 3000), np.float32))
