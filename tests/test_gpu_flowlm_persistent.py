"""GPU parity of the persistent one-stream FlowLM kernel (k_frame1.cu): a set
of one stream runs every frame of a call as one cooperative launch with grid
barriers between the frame's steps. Its results must be the oracle's bits
(flowLM.step + flowHead.sample, pockettts/lm.go:108-195, speak.go:146-175)
and the per-kernel path's; its bounded waits must report a wait that runs
out as GRX_ETIMEDOUT without faulting or hanging the device."""

import os

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import SMALL, bits_equal, mismatch, voice_kv

pytestmark = pytest.mark.gpu
TOL = 1e-3  # the relative tolerance the spec allows; identical bits pass it

# d, ff and the flow dim multiples of 256 (the kernel's slice alignment), a
# flow head of two residual blocks.
MID = dict(d=256, heads=4, ff=512, layers=2, flow_dim=256, flow_depth=2)


def _models(cfg, seed=0):
    t = synth.flowlm_tensors(cfg, seed)
    return g.FlowLM(synth.flowlm_gguf(cfg, t)), orc.FlowLM(cfg, t)


def _device_run(st, noise):
    import torch

    frames = noise.shape[0]
    dn = torch.from_numpy(np.ascontiguousarray(noise)).cuda()
    dl = torch.empty_like(dn)
    de = torch.empty((frames, noise.shape[1]), device="cuda")
    st.run_device(frames, dn.data_ptr(), dl.data_ptr(), de.data_ptr())
    st.sync()
    return dl.cpu().numpy(), de.cpu().numpy()


def test_persistent_kernel_chosen_for_one_stream(have_gpu):
    cfg = synth.FlowLMConfig()
    gm, _ = _models(cfg)
    kv = voice_kv(cfg, 8, 1)
    assert g.Streams(gm, [gm.voice(kv)], 4).persistent()
    assert not g.Streams(gm, [gm.voice(kv), gm.voice(kv)], 4).persistent()
    small = synth.FlowLMConfig(**SMALL)  # d 128: not a multiple of 256
    gs, _ = _models(small)
    assert not g.Streams(gs, [gs.voice(voice_kv(small, 8, 1))], 4).persistent()


def test_persistent_depth2_steps_and_device_run(have_gpu):
    """A model with a two-block flow head, 40 frames through grx_streams_step
    (lm_out, eos, latent and scaled every frame), then the same frames again
    after a reset as one device-resident run."""
    cfg = synth.FlowLMConfig(**MID)
    gm, om = _models(cfg, seed=3)
    kv = voice_kv(cfg, 9, 2)
    frames = 40
    st = g.Streams(gm, [gm.voice(kv)], frames)
    assert st.persistent()
    os_ = om.stream(kv)
    noise = synth.noise_frames(2, frames, cfg.ldim, cfg.temperature)
    lat_o = None
    want_lat, want_eos = [], []
    for f in range(frames):
        lat, eos, sc, lo = st.step(noise[f][None], want_lm_out=True)
        r = om.frame(os_, lat_o, noise[f])
        lat_o = r["latent"]
        want_lat.append(r["latent"])
        want_eos.append(r["eos"])
        for name, a, b in (("lm_out", lo[0], r["lm_out"]), ("eos", eos[:1], [r["eos"]]),
                           ("latent", lat[0], r["latent"]), ("scaled", sc[0], r["scaled"])):
            ne, rel = mismatch(a, b)
            assert ne == 0, f"frame {f} {name}: {ne} differ, max rel {rel:.2e} (tolerance {TOL})"
    assert st.pos(0) == 9 + frames
    st.reset()
    dl, de = _device_run(st, noise[:, None, :])
    assert bits_equal(dl[:, 0], np.stack(want_lat)) and bits_equal(de[:, 0], np.asarray(want_eos, np.float32))


def test_persistent_matches_per_kernel_path(have_gpu, monkeypatch):
    """The Pocket-TTS-shaped model over 64 device-resident frames: the
    persistent kernel and the per-kernel graph path (GRX_FRAME1=0) give the
    same bits."""
    cfg = synth.FlowLMConfig()
    gm, _ = _models(cfg)
    kv = voice_kv(cfg, 64, 1)
    frames = 64
    noise = synth.noise_frames(1, frames, cfg.ldim, cfg.temperature)[:, None, :]
    a = g.Streams(gm, [gm.voice(kv)], frames)
    assert a.persistent()
    la, ea = _device_run(a, noise)
    monkeypatch.setenv("GRX_FRAME1", "0")
    b = g.Streams(gm, [gm.voice(kv)], frames)
    assert not b.persistent()
    lb, eb = _device_run(b, noise)
    assert bits_equal(la, lb) and bits_equal(ea, eb)


def test_persistent_text_then_frames(have_gpu):
    """flowLM.text on a one-stream set (the per-kernel prefill), then frames
    in the persistent kernel from the positions the text left."""
    cfg = synth.FlowLMConfig(**MID)
    gm, om = _models(cfg, seed=4)
    kv = voice_kv(cfg, 5, 3)
    ids = [[(7 * j + 3) % cfg.text_vocab for j in range(11)]]
    frames = 6
    st = g.Streams(gm, [gm.voice(kv)], 11 + frames)
    assert st.persistent()
    out = st.text(ids)
    os_ = om.stream(kv)
    assert bits_equal(out[0], om.text(os_, ids[0]))
    noise = synth.noise_frames(3, frames, cfg.ldim, cfg.temperature)[:, None, :]
    lat_o, eos_o, _ = om.run([os_], noise, threads=1)
    for f in range(frames):
        lat, eos, _, _ = st.step(noise[f])
        assert bits_equal(lat, lat_o[f]) and bits_equal(eos, eos_o[f]), f"frame {f}"


def test_persistent_watchdog_reports_and_recovers(have_gpu):
    """A run whose first grid barrier nothing completes: every block gives up
    after its one-second limit, the call returns GRX_ETIMEDOUT (-7), the
    positions are untouched, and after a reset the set decodes correctly on
    the same context."""
    cfg = synth.FlowLMConfig(**MID)
    gm, om = _models(cfg, seed=5)
    kv = voice_kv(cfg, 7, 4)
    st = g.Streams(gm, [gm.voice(kv)], 8)
    assert st.persistent()
    assert st.watchdog_test() == -7
    assert "one-second limit" in g.last_error()
    assert st.pos(0) == 7
    st.reset()
    noise = synth.noise_frames(4, 3, cfg.ldim, cfg.temperature)[:, None, :]
    lat_o, eos_o, _ = om.run([om.stream(kv)], noise, threads=1)
    dl, de = _device_run(st, noise)
    assert bits_equal(dl, lat_o) and bits_equal(de, eos_o)
