"""GPU parity of Mimi's encoder: grx_mimi_encoder_*, grx_mimi_clone_latents
and grx_voice_clone through the C ABI against the oracle's cloneCond
encoding (oracle/mimi.h mimi_clone_latents, which restates pockettts/
mimi.go:152-179 and voice.go:113-124: the clip padded to whole frames, then
twelve frames at a time through the SEANet encoder, the windowed transformer
and the downsampling convolution whose first call is padded by replicating
the first row). The bar is bit-identical float32 latents and voice caches;
the tolerance the spec allows (1e-3 relative) is stated for the record."""

import dataclasses

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import SMALL, mismatch

pytestmark = pytest.mark.gpu
TOL = 1e-3
LDIM = 32

_BASE = synth.MimiConfig()
CONFIGS = {
    # 40-sample frames: the one-channel first convolution (7 columns, float32)
    # on the packed kernel plus dotF32Go rows, float32 residual blocks and the
    # first strided convolution, Q8_0 second strided and last convolutions
    "base": _BASE,
    # 24 and 48 filters: Q8_0 convolutions with odd block counts (the int8
    # path in groups of up to 8 rows)
    "odd_blocks": dataclasses.replace(_BASE, nf=24),
    # two residual blocks per ratio, the second dilated (explicit im2col)
    "dilated": dataclasses.replace(_BASE, nres=2),
    # Mimi's own 2 transformer rows per latent and a 5-position window
    "upsample2": dataclasses.replace(_BASE, upsample=2, ratios=(5, 4), context=5),
}


def _models(mc, seed):
    t = synth.mimi_tensors(mc, LDIM, seed, encoder=True)
    gg = synth.flowlm_gguf(synth.FlowLMConfig(ldim=LDIM), t, mimi=mc)
    return g.Mimi(gg), orc.Mimi(mc, t, LDIM)


def _check(got, want, what):
    assert got.shape == want.shape, (got.shape, want.shape)
    ne, rel = mismatch(got, want)
    assert ne == 0, f"{what}: {ne} of {got.size} latent values differ (max rel {rel:.2e})"
    assert rel <= TOL


@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("frames", [0.25, 1, 12, 25, 30.85])
def test_mimi_clone_latents_bit_exact(have_gpu, name, frames):
    """One clip of a quarter frame up to 31 frames (several pieces, a short
    last one, a length that is not whole frames): latents bit-identical."""
    mc = CONFIGS[name]
    gm, om = _models(mc, seed=int(frames * 10))
    n = max(1, int(frames * mc.frame))
    x = np.random.default_rng(n).normal(0, 0.3, n).astype(np.float32)
    _check(gm.clone_latents(x), om.clone_latents(x), f"{name}, {n} samples")


def test_mimi_encoder_batch_and_reuse(have_gpu):
    """Three clips encoded together, each from its own fresh state, then the
    same set again on shorter clips: every clip's latents equal the oracle's
    for that clip alone."""
    mc = CONFIGS["base"]
    gm, om = _models(mc, seed=5)
    enc = g.MimiEncoder(gm, 3, 2000)
    rng = np.random.default_rng(9)
    for n in (1234, 500):
        x = rng.normal(0, 0.3, (3, n)).astype(np.float32)
        got = enc.encode(x)
        for i in range(3):
            _check(got[i], om.clone_latents(x[i]), f"clip {i} of {n} samples")


def test_voice_clone_end_to_end(have_gpu):
    """grx_voice_clone (CloneVoice after resampling and end_on_pause,
    voice.go:94-124): the voice's caches equal the oracle's flow-LM half run
    on the oracle's latents of the clip, and frames from it match too."""
    cfg = synth.FlowLMConfig(**SMALL)
    mc = CONFIGS["base"]
    t = dict(synth.flowlm_tensors(cfg, 3))
    t.update(synth.mimi_tensors(mc, cfg.ldim, 3, encoder=True))
    gg = synth.flowlm_gguf(cfg, t, mimi=mc)
    lm, mimi = g.FlowLM(gg), g.Mimi(gg)
    olm, omimi = orc.FlowLM(cfg, t), orc.Mimi(mc, t, cfg.ldim)
    x = np.random.default_rng(11).normal(0, 0.3, 777).astype(np.float32)
    v = lm.voice_clone(mimi, x)
    kv_o = olm.voice_from_latents(omimi.clone_latents(x))
    kv = v.kv(cfg.layers, cfg.d)
    ne, rel = mismatch(kv, kv_o)
    assert ne == 0, f"{ne} of {kv.size} cache values differ, max rel {rel:.2e}"
    st = g.Streams(lm, [v], 2)
    noise = synth.noise_frames(4, 2, cfg.ldim, cfg.temperature)[:, None, :]
    lat_o, eos_o, _ = olm.run([olm.stream(kv_o)], noise)
    for f in range(2):
        lat, eos, _, _ = st.step(noise[f])
        assert mismatch(lat, lat_o[f])[0] == 0 and mismatch(eos, eos_o[f])[0] == 0, f"frame {f}"


def test_mimi_encoder_errors(have_gpu):
    """A file without the encoder, a clip longer than the set was made for,
    an empty clip: errors, not faults."""
    mc = CONFIGS["base"]
    t = synth.mimi_tensors(mc, LDIM, 1)
    gm = g.Mimi(synth.flowlm_gguf(synth.FlowLMConfig(ldim=LDIM), t, mimi=mc))
    with pytest.raises(g.GrxError) as e:
        g.MimiEncoder(gm, 1, 100)
    assert "voice cloning" in str(e.value)
    gm2, _ = _models(mc, seed=1)
    enc = g.MimiEncoder(gm2, 2, 100)
    with pytest.raises(g.GrxError):
        enc.encode(np.zeros((2, 101), np.float32))
    with pytest.raises(g.GrxError):
        gm2.clone_latents(np.zeros(0, np.float32))
