"""GPU parity of the Whisper text decoder's token loop (whisper/decoder.go,
encoder.go:120-140, transcribe.go:370-520) through the C ABI against the CPU
oracle, on seeded synthetic ggml models and N(0,1) encoder output. Token ids
and timestamps must be identical; the cross K/V, the logits and the float
outputs (p, plog, no-speech probability) bit-identical or within the 1e-3
relative tolerance the spec states for float outputs (p and plog come from
sums over the vocabulary that the GPU reduces in another order)."""

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import bits_equal, mismatch

pytestmark = pytest.mark.gpu
TOL = 1e-3
SMALL_W = dict(n_state=128, n_head=2, n_text_layer=2, n_text_ctx=64)


def _models(cfg, seed=0, f16=False):
    t = synth.whisper_tensors(cfg, seed)
    words = synth.whisper_words(cfg)
    bits = {k: orc.q8_to_f16(v) for k, v in t.items() if isinstance(v, synth.Q8)} if f16 else None
    gm = g.Whisper(synth.whisper_ggml(cfg, t, words, f16_bits=bits))
    return gm, orc.Whisper(cfg, t, words)


def _enc(cfg, n, seed0=1):
    return np.stack([synth.whisper_encoder_out(seed0 + i, cfg) for i in range(n)])


def _prompt(gm):
    return [gm.prev, 100, 200, gm.sot], 3


def _check_tokens(got, want):
    """got [steps][4] int32 from the GPU, want [steps][4] from the oracle.
    p within TOL relative; plog, a log-probability, within TOL absolute
    (both come from float32 sums over the 51864 logits that the reference
    takes in sequence and the GPU as a tree; the two roundings differ by
    ~1e-4 relative in the sum)."""
    assert len(got) == len(want)
    assert np.array_equal(got[:, 0], want[:, 0]), f"ids differ: {got[:, 0].tolist()} vs {want[:, 0].tolist()}"
    assert np.array_equal(got[:, 1], want[:, 1]), "timestamps differ"
    p, wp = got[:, 2].copy().view(np.float32), want[:, 2].copy().view(np.float32)
    assert np.all(np.abs(p - wp) <= TOL * np.abs(wp))
    lp, wlp = got[:, 3].copy().view(np.float32), want[:, 3].copy().view(np.float32)
    fin = np.isfinite(wlp)
    assert np.array_equal(np.isfinite(lp), fin)
    assert np.all(np.abs(lp[fin] - wlp[fin]) <= TOL)


def test_whisper_vocab_and_suppress(have_gpu):
    cfg = synth.WhisperConfig(**SMALL_W)
    gm, om = _models(cfg)
    assert gm.suppressed() == om.suppress()
    assert (gm.eot, gm.sot, gm.prev, gm.nosp, gm.beg) == (50256, 50257, 50360, 50361, 50363)


@pytest.mark.parametrize("f16", [False, True])
def test_whisper_cross_kv_and_greedy(have_gpu, f16):
    """Cross K/V of two streams, the 4-token prompt and 24 greedy steps:
    tokens identical, logits and K/V bit-identical."""
    cfg = synth.WhisperConfig(**SMALL_W)
    gm, om = _models(cfg, f16=f16)
    n, steps = 2, 24
    enc = _enc(cfg, n)
    b = g.WhisperBatch(gm, n)
    b.set_audio(enc)
    prompt, sot_at = _prompt(gm)
    seqs = [om.seq(enc[i]) for i in range(n)]
    for i in range(n):
        for layer in range(cfg.n_text_layer):
            k, vt = b.cross(i, layer)
            wk, wv = om.cross(seqs[i], layer)
            assert bits_equal(k, wk) and bits_equal(vt, wv), f"stream {i} layer {layer}: cross K/V differ"
    ns = b.prompt(prompt, sot_at)
    lg = b.logits()
    for i in range(n):
        s = om.seq(enc[i])
        want = om.decode(s, prompt, [sot_at, len(prompt) - 1])
        ne, rel = mismatch(lg[i], want[1])
        assert ne == 0, f"prompt logits: {ne} differ (max rel {rel:.2e})"
    toks = b.run(steps)
    for i in range(n):
        want, wns = om.greedy(om.seq(enc[i]), prompt, sot_at, steps)
        _check_tokens(toks[:, i], want)
        assert abs(ns[i] - wns) <= TOL * abs(wns)


def test_whisper_mixed_qkv_types(have_gpu):
    """A file whose first layer stores attn.key as float16 and attn.query and
    attn.value as Q8_0: that layer keeps three product launches (its matrices
    are not stacked) while the second takes the stacked q/k/v launch. Greedy
    tokens as the oracle's over three streams (the per-kernel decode step)."""
    cfg = synth.WhisperConfig(**SMALL_W)
    t = synth.whisper_tensors(cfg, 5)
    words = synth.whisper_words(cfg)
    name = "decoder.blocks.0.attn.key.weight"
    gm = g.Whisper(synth.whisper_ggml(cfg, t, words, f16_bits={name: orc.q8_to_f16(t[name])}))
    om = orc.Whisper(cfg, t, words)
    n, steps = 3, 16
    enc = _enc(cfg, n, seed0=21)
    b = g.WhisperBatch(gm, n)
    assert not b.persistent()
    b.set_audio(enc)
    prompt, sot_at = _prompt(gm)
    b.prompt(prompt, sot_at)
    toks = b.run(steps)
    for i in range(n):
        want, _ = om.greedy(om.seq(enc[i]), prompt, sot_at, steps)
        _check_tokens(toks[:, i], want)


def test_whisper_base_shape(have_gpu):
    """The base.en decoder shape (state 512, 8 heads, 6 layers, vocab 51864,
    text context 448) on one stream: prompt and 6 greedy steps."""
    cfg = synth.WhisperConfig()
    gm, om = _models(cfg)
    enc = _enc(cfg, 1, seed0=7)
    b = g.WhisperBatch(gm, 1)
    b.set_audio(enc)
    prompt, sot_at = _prompt(gm)
    b.prompt(prompt, sot_at)
    toks = b.run(6)
    want, _ = om.greedy(om.seq(enc[0]), prompt, sot_at, 6)
    _check_tokens(toks[:, 0], want)


def test_whisper_loader_rejects_bad_files(have_gpu):
    """whisper.Load's checks (model.go:115-223, 320-402)."""
    cfg = synth.WhisperConfig(**SMALL_W)
    t = synth.whisper_tensors(cfg, 0)
    good = synth.whisper_ggml(cfg, t)
    with pytest.raises(g.GrxError) as e:
        g.Whisper(b"ggjt" + good[4:])
    assert e.value.code == -2
    with pytest.raises(g.GrxError):
        g.Whisper(synth.whisper_ggml(synth.WhisperConfig(**SMALL_W, n_audio_ctx=1499), t))
    t2 = dict(t)
    del t2["decoder.ln.bias"]
    with pytest.raises(g.GrxError) as e:
        g.Whisper(synth.whisper_ggml(cfg, t2))
    assert "decoder.ln.bias" in str(e.value)
    t3 = dict(t)
    t3["decoder.extra.weight"] = np.zeros(4, np.float32)
    with pytest.raises(g.GrxError) as e:
        g.Whisper(synth.whisper_ggml(cfg, t3))
    assert "doesn't know" in str(e.value)
    with pytest.raises(g.GrxError):
        g.Whisper(good[: len(good) - 7])


@pytest.mark.parametrize("np_", [6, 9])
def test_whisper_long_prompt_packed_rows(have_gpu, np_):
    """A prompt of 6 or more tokens takes the packed product for each
    stream's first np/6·6 rows (whisper/gemm.go:150-186) and gemv for the
    rest; logits, no-speech probability and the following tokens match."""
    cfg = synth.WhisperConfig(**SMALL_W)
    gm, om = _models(cfg, seed=2)
    n = 2
    enc = _enc(cfg, n, seed0=11)
    prompt = [gm.prev] + list(range(300, 300 + np_ - 2)) + [gm.sot]
    sot_at = np_ - 1
    b = g.WhisperBatch(gm, n)
    b.set_audio(enc)
    ns = b.prompt(prompt, sot_at)
    lg = b.logits()
    for i in range(n):
        want = om.decode(om.seq(enc[i]), prompt, [sot_at, np_ - 1])
        ne, rel = mismatch(lg[i], want[1])
        assert ne == 0, f"{ne} logits differ (max rel {rel:.2e})"
    toks = b.run(5)
    for i in range(n):
        want, wns = om.greedy(om.seq(enc[i]), prompt, sot_at, 5)
        _check_tokens(toks[:, i], want)
        assert abs(ns[i] - wns) <= TOL * abs(wns)



@pytest.mark.parametrize("n", [1, 20, 40, 80, 160])
def test_whisper_launch_shapes(have_gpu, n):
    """Every launch shape of the token step on the small model: cross-
    attention spread over key chunks and output slices (fewer than 296
    (row, head) pairs) or one CTA per pair (the 160-stream decode and every
    prompt pass from 80 streams up), process/sample on clusters of 8, 4 or 2
    CTAs per row or one CTA per row. Ids identical for every stream, and
    every output of the first and last stream."""
    cfg = synth.WhisperConfig(**SMALL_W)
    gm, om = _models(cfg, seed=7)
    steps = 6
    enc = _enc(cfg, n, seed0=31)
    b = g.WhisperBatch(gm, n)
    b.set_audio(enc)
    prompt, sot_at = _prompt(gm)
    b.prompt(prompt, sot_at)
    toks = b.run(steps)
    ids = om.run(enc, prompt, sot_at, steps, 8)
    for i in range(n):
        assert np.array_equal(toks[:, i, 0], ids[i]), f"stream {i}: ids differ"
    for i in {0, n - 1}:
        want, _ = om.greedy(om.seq(enc[i]), prompt, sot_at, steps)
        _check_tokens(toks[:, i], want)
