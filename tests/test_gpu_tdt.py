"""GPU parity of the TDT / RNN-T decode loop (conformer/rnnt.go:111-173)
through the C ABI against the CPU oracle, on seeded synthetic decoders and
N(0,1) encoder output. Token ids, frames and durations must be identical;
the probabilities and the final LSTM states bit-identical (the tests allow
the 1e-3 relative tolerance the spec states for float outputs, and 1e-6 for
p, whose float64 sum the GPU reduces in another order)."""

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import bits_equal

pytestmark = pytest.mark.gpu
TOL, PTOL = 1e-3, 1e-6

SMALL_TDT = dict(H=128, V=65, J=96, D=128)


def _models(cfg, seed=0):
    t = synth.tdt_tensors(cfg, seed)
    return g.TDT(synth.tdt_gguf(cfg, t)), orc.TDT(cfg, t)


def _enc(cfg, n, max_t, seed0=1):
    return np.stack([synth.encoder_frames(seed0 + i, max_t, cfg.D) for i in range(n)])


def _check_stream(got, counts_i, want, cap):
    assert counts_i == len(want), (counts_i, len(want))
    want = want[:cap]
    assert len(got) == len(want)
    assert np.array_equal(got["id"], want[:, 0]), "token ids differ"
    assert np.array_equal(got["frame"], want[:, 1]), "frames differ"
    assert np.array_equal(got["duration"], want[:, 2]), "durations differ"
    wp = want[:, 3].copy().view(np.float32)
    if len(wp):
        assert np.max(np.abs(got["p"] - wp) / np.abs(wp)) <= PTOL


def _decode_both(gm, om, cfg, enc, T, offsets=None, cap=None, batch=None, ostates=None):
    n, max_t = enc.shape[0], enc.shape[1]
    cap = cap or 16 * max_t + 1024
    b = batch or g.TDTBatch(gm, n, max_t, cap)
    toks, counts = b.decode(enc, T, offsets)
    ostates = ostates or [om.state() for _ in range(n)]
    for i in range(n):
        want, _, _ = om.decode(enc[i, :T[i]], ostates[i], 0 if offsets is None else offsets[i])
        _check_stream(toks[i], int(counts[i]), want, cap)
        h, c, last = b.state(i)
        assert last == ostates[i][2]
        assert bits_equal(h, ostates[i][0]) and bits_equal(c, ostates[i][1]), f"stream {i}: LSTM state differs"
    return b, ostates, toks, counts


@pytest.mark.parametrize("head,act,lift", [("tdt", "relu", 0.8), ("rnnt", "relu", 0.8), ("tdt", "sigmoid", 0.3),
                                           ("rnnt", "tanh", 0.8)])
def test_tdt_small_batch_ragged(have_gpu, head, act, lift):
    """Five streams of 40, 1, 0, 23 and 40 frames (T = 1 takes the float
    path for the encoder projection, T = 0 returns nothing)."""
    cfg = synth.TDTConfig(**SMALL_TDT, head=head, act=act, blank_lift=lift)
    gm, om = _models(cfg)
    T = [40, 1, 0, 23, 40]
    enc = _enc(cfg, len(T), 40)
    _, _, toks, counts = _decode_both(gm, om, cfg, enc, T)
    assert counts[2] == 0
    assert counts.sum() > 0


def test_tdt_chunked_state_and_offsets(have_gpu):
    """Decode in two chunks, the state carried (DecoderState) and frames
    offset, as a streaming caller does; then reset."""
    cfg = synth.TDTConfig(**SMALL_TDT)
    gm, om = _models(cfg, seed=3)
    n, max_t = 3, 30
    b = g.TDTBatch(gm, n, max_t, 256)
    ost = [om.state() for _ in range(n)]
    e1, e2 = _enc(cfg, n, max_t, 10), _enc(cfg, n, max_t, 20)
    _decode_both(gm, om, cfg, e1, [30, 30, 17], None, 256, b, ost)
    _decode_both(gm, om, cfg, e2, [25, 30, 30], [30, 30, 17], 256, b, ost)
    b.reset()
    _decode_both(gm, om, cfg, e1, [30, 30, 30], None, 256, b, None)


def test_tdt_state_set_and_cap(have_gpu):
    """A state written through the C ABI is the one decoded from; tokens past
    cap are counted but not written."""
    cfg = synth.TDTConfig(**SMALL_TDT, blank_lift=0.4)
    gm, om = _models(cfg, seed=5)
    n, max_t, cap = 2, 40, 4
    b = g.TDTBatch(gm, n, max_t, cap)
    rng = np.random.default_rng(7)
    ost = []
    for i in range(n):
        h = np.tanh(rng.normal(0, 1, (cfg.layers, cfg.H))).astype(np.float32)
        c = rng.normal(0, 1, (cfg.layers, cfg.H)).astype(np.float32)
        b.set_state(i, h, c, 17 + i)
        ost.append([h.copy(), c.copy(), 17 + i])
    _, _, toks, counts = _decode_both(gm, om, cfg, _enc(cfg, n, max_t, 30), [40, 40], None, cap, b, ost)
    assert (counts > cap).any()


def test_tdt_c3_shape(have_gpu):
    """The Parakeet-TDT decoder shape (H 640, 2 layers, 1025 tokens + 5
    durations, joint 640) on four streams of 48 frames."""
    cfg = synth.TDTConfig()
    gm, om = _models(cfg)
    T = [48, 48, 31, 48]
    _decode_both(gm, om, cfg, _enc(cfg, 4, 48), T)


def test_tdt_loader_rejects_bad_files(have_gpu):
    """conformer.FromGGUF's checks on the decoder part (model.go:190-236)."""
    cfg = synth.TDTConfig(**SMALL_TDT)
    t = synth.tdt_tensors(cfg, 0)
    bad_arch = synth.tdt_gguf(cfg, t).replace(b"parakeet", b"parakeeX", 1)
    with pytest.raises(g.GrxError) as e:
        g.TDT(bad_arch)
    assert e.value.code == -2
    t2 = dict(t)
    del t2["joint.out.bias"]
    with pytest.raises(g.GrxError) as e:
        g.TDT(synth.tdt_gguf(cfg, t2))
    assert "joint.out.bias" in str(e.value)
    with pytest.raises(g.GrxError) as e:
        g.TDT(synth.tdt_gguf(synth.TDTConfig(**SMALL_TDT, durations=()), t))
    assert "durations" in str(e.value)
