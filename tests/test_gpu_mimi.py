"""GPU parity for Mimi's decoder: grx_mimi_* through the C ABI against the
oracle's mimiDecoder.decode (oracle/mimi.h, which restates
pockettts/mimi.go:24-150 and nn.go), frame after frame with the streaming
state carried, for several independent streams. The bar is bit-identical
float32 samples; the tolerance the spec allows (1e-3 relative) is stated
for the record and passed trivially."""

import dataclasses

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import mismatch

pytestmark = pytest.mark.gpu
TOL = 1e-3
LDIM = 32

_BASE = synth.MimiConfig()
CONFIGS = {
    # Q8_0 first conv, first transposed conv and transformer; float32 tail
    # stages with rows past 16 (the packed kernel plus gemvRows); 4 rows per
    # latent, so T >= 4 takes attend's product for the values
    "base": _BASE,
    # the first transposed conv's rows are 3 blocks long (odd): the int8
    # path in groups of up to 8 rows
    "odd_blocks": dataclasses.replace(_BASE, nf=24),
    # Mimi's own 2 rows per latent (attend's AddScaled for the values), a
    # 5-position window over a 6-row ring
    "upsample2": dataclasses.replace(_BASE, upsample=2, ratios=(5, 4), context=5),
    # two residual blocks per ratio, the second dilated (its window through
    # an explicit im2col)
    "dilated": dataclasses.replace(_BASE, nres=2),
    # a last stage of 48 rows per latent: every row of its float32 convs
    # takes the packed kernel (the window read in place, ELU fused)
    "whole_packed": dataclasses.replace(_BASE, upsample=2, ratios=(6, 4)),
}


def _model(mc, seed):
    t = synth.mimi_tensors(mc, LDIM, seed)
    return t, synth.flowlm_gguf(synth.FlowLMConfig(ldim=LDIM), t, mimi=mc)


def _check(got, want, what):
    ne, rel = mismatch(got, want)
    assert ne == 0, f"{what}: {ne} of {got.size} samples differ (max rel {rel:.2e})"
    assert rel <= TOL


@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("n", [1, 3, 9])
def test_mimi_decode_bit_exact(have_gpu, name, n):
    """n streams, 10 frames each (past the attention window and around the
    ring), each stream's latents its own: every frame equals the oracle's."""
    mc = CONFIGS[name]
    t, gg = _model(mc, n)
    om = orc.Mimi(mc, t, LDIM)
    states = [om.state() for _ in range(n)]
    gm = g.Mimi(gg)
    assert (gm.d, gm.upsample, gm.frame, gm.sample_rate, gm.ldim) == (mc.d, mc.upsample, mc.frame, mc.sample_rate,
                                                                       LDIM)
    gs = g.MimiStreams(gm, n, max_frames=10)
    rng = np.random.default_rng(100 + n)
    for f in range(10):
        lat = rng.normal(0, 1, (n, LDIM)).astype(np.float32)
        got = gs.decode(lat)
        assert got.shape == (n, mc.frame)
        for i in range(n):
            _check(got[i], om.decode(states[i], lat[i]), f"{name} frame {f} stream {i}")
    assert gs.frames() == 10


def test_mimi_reset_and_device_run(have_gpu):
    """decode_device gives the host calls' samples; after reset a set
    starts over (fresh state, the first frame faded in again)."""
    import torch

    mc = CONFIGS["base"]
    _, gg = _model(mc, 7)
    gm = g.Mimi(gg)
    n, frames = 5, 6
    rng = np.random.default_rng(5)
    lat = rng.normal(0, 1, (frames, n, LDIM)).astype(np.float32)
    a = g.MimiStreams(gm, n, max_frames=frames)
    host = np.stack([a.decode(lat[f]) for f in range(frames)])
    a.reset()
    again = np.stack([a.decode(lat[f]) for f in range(3)])
    _check(again, host[:3], "after reset")
    b = g.MimiStreams(gm, n, max_frames=frames)
    dl = torch.from_numpy(lat).cuda()
    dp = torch.empty((frames, n, mc.frame), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    b.decode_device(frames, dl.data_ptr(), dp.data_ptr())
    b.sync()
    _check(dp.cpu().numpy(), host, "device run")
    assert b.launches() > 0


def test_mimi_errors(have_gpu):
    mc = CONFIGS["base"]
    t, gg = _model(mc, 1)
    gm = g.Mimi(gg)
    s = g.MimiStreams(gm, 2, max_frames=2)
    z = np.zeros((2, LDIM), np.float32)
    s.decode(z)
    s.decode(z)
    with pytest.raises(g.GrxError, match="ERANGE"):
        s.decode(z)
    bad = dict(t)
    del bad["mimi.dec.0.bias"]
    with pytest.raises(g.GrxError, match="mimi.dec.0.bias"):
        g.Mimi(synth.flowlm_gguf(synth.FlowLMConfig(ldim=LDIM), bad, mimi=mc))
    with pytest.raises(g.GrxError, match="EINVAL"):
        g.MimiStreams(gm, 0, 4)
