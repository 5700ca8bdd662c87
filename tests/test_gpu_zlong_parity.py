"""Full-length GPU parity at BASELINE.json's configurations: the CUDA path
through the C ABI against the oracle (its fast mode: the reference's SIMD
kernels restated in their lane order, bit-identical to the exact mode, which
tests/test_oracle_fast.py checks) over the whole runs the spec quotes:

  * C0: one FlowLM stream, 256 frames from a 64-position prefill
    (speak.go:146-175), every frame's latent and EOS logit;
  * C1: 256 streams (two concurrent parts) x 512 frames, device-resident;
    eight streams spread over both parts compared every frame, so attention
    is checked up to 576 keys;
  * C2: the Whisper base.en decoder, 224 greedy tokens from a 4-token prompt
    (transcribe.go:206-257) at one stream (ids, timestamps, p and plog) and
    at 32 streams (the ids of four of them);
  * C3: the Parakeet-TDT decoder, 128 streams x 750 encoder frames
    (rnnt.go:111-173): every token, frame and duration of every stream.

The file is named to run after the quick tests."""

import os

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import bits_equal, mismatch, voice_kv

pytestmark = pytest.mark.gpu
TOL = 1e-3  # the relative tolerance the spec allows for float outputs
THREADS = max(1, os.cpu_count() or 1)


def _device_run(st, noise):
    import torch

    frames, n = noise.shape[0], noise.shape[1]
    dn = torch.from_numpy(np.ascontiguousarray(noise)).cuda()
    dl = torch.empty_like(dn)
    de = torch.empty((frames, n), device="cuda")
    st.run_device(frames, dn.data_ptr(), dl.data_ptr(), de.data_ptr())
    st.sync()
    return dl.cpu().numpy(), de.cpu().numpy()


def _first_diff(a, b):
    d = np.nonzero(np.asarray(a, np.float32).view(np.uint32) != np.asarray(b, np.float32).view(np.uint32))
    return tuple(int(v[0]) for v in d) if len(d[0]) else None


def test_c0_one_stream_256_frames(have_gpu):
    cfg = synth.FlowLMConfig()
    t = synth.flowlm_tensors(cfg, 0)
    gm, om = g.FlowLM(synth.flowlm_gguf(cfg, t)), orc.FlowLM(cfg, t)
    kv = voice_kv(cfg, 64, 1)
    frames = 256
    st = g.Streams(gm, [gm.voice(kv)], frames)
    noise = synth.noise_frames(1, frames, cfg.ldim, cfg.temperature)[:, None, :].copy()
    dl, de = _device_run(st, noise)
    with orc.fast_mode():
        lat_o, eos_o, _ = om.run([om.stream(kv)], noise, threads=THREADS)
    ne, rel = mismatch(dl, lat_o)
    assert ne == 0, f"{ne} latent values differ (first at {_first_diff(dl, lat_o)}), max rel {rel:.2e}"
    assert bits_equal(de, eos_o), f"EOS logits differ, first at {_first_diff(de, eos_o)}"
    assert st.pos(0) == 64 + frames


def test_c1_256_streams_512_frames(have_gpu):
    cfg = synth.FlowLMConfig()
    t = synth.flowlm_tensors(cfg, 0)
    gm, om = g.FlowLM(synth.flowlm_gguf(cfg, t)), orc.FlowLM(cfg, t)
    n, frames = 256, 512
    st = g.Streams(gm, [gm.voice(voice_kv(cfg, 64, 1 + i)) for i in range(n)], frames)
    assert st.parts() == 2
    noise = np.stack([synth.noise_frames(1 + i, frames, cfg.ldim, cfg.temperature) for i in range(n)], axis=1)
    dl, de = _device_run(st, noise)
    pick = [0, 37, 90, 127, 128, 170, 211, 255]  # both parts, their edges
    with orc.fast_mode():
        lat_o, eos_o, _ = om.run([om.stream(voice_kv(cfg, 64, 1 + i)) for i in pick], noise[:, pick], threads=THREADS)
    for j, i in enumerate(pick):
        ne, rel = mismatch(dl[:, i], lat_o[:, j])
        assert ne == 0, f"stream {i}: {ne} latent values differ (first at {_first_diff(dl[:, i], lat_o[:, j])})"
        assert bits_equal(de[:, i], eos_o[:, j]), f"stream {i}: EOS logits differ"
    assert st.pos(0) == st.pos(n - 1) == 64 + frames


def _whisper_check(got, want):
    assert np.array_equal(got[:, 0], want[:, 0]), (
        f"ids differ from step {int(np.nonzero(got[:, 0] != want[:, 0])[0][0])}")
    assert np.array_equal(got[:, 1], want[:, 1]), "timestamps differ"
    p, wp = got[:, 2].copy().view(np.float32), want[:, 2].copy().view(np.float32)
    assert np.all(np.abs(p - wp) <= TOL * np.abs(wp))
    lp, wlp = got[:, 3].copy().view(np.float32), want[:, 3].copy().view(np.float32)
    fin = np.isfinite(wlp)
    assert np.array_equal(np.isfinite(lp), fin)
    assert np.all(np.abs(lp[fin] - wlp[fin]) <= TOL)


def test_c2_whisper_224_tokens(have_gpu):
    cfg = synth.WhisperConfig()
    t = synth.whisper_tensors(cfg, 0)
    words = synth.whisper_words(cfg)
    gm, om = g.Whisper(synth.whisper_ggml(cfg, t, words)), orc.Whisper(cfg, t, words)
    steps = 224
    prompt, sot_at = [gm.prev, 100, 200, gm.sot], 3
    # one stream: ids, timestamps, p and plog every step
    enc1 = np.stack([synth.whisper_encoder_out(7, cfg)])
    b1 = g.WhisperBatch(gm, 1)
    b1.set_audio(enc1)
    b1.prompt(prompt, sot_at)
    toks1 = b1.run(steps)
    with orc.fast_mode(THREADS):
        want, _ = om.greedy(om.seq(enc1[0]), prompt, sot_at, steps)
    _whisper_check(toks1[:, 0], want)
    # 32 streams: the ids of four of them
    n = 32
    enc = np.stack([synth.whisper_encoder_out(1 + i, cfg) for i in range(n)])
    b = g.WhisperBatch(gm, n)
    b.set_audio(enc)
    b.prompt(prompt, sot_at)
    toks = b.run(steps)
    pick = [0, 11, 22, 31]
    with orc.fast_mode():
        ids = om.run(enc[pick], prompt, sot_at, steps, min(THREADS, len(pick)))
    for j, i in enumerate(pick):
        assert np.array_equal(toks[:, i, 0], ids[j]), f"stream {i}: ids differ"
    print(f"\nk_wproc decided {gm.exact_rows()} of {(1 + n) * (steps + 1)} rows in the sequential order")


def test_c3_tdt_128_streams_750_frames(have_gpu):
    cfg = synth.TDTConfig()
    t = synth.tdt_tensors(cfg, 0)
    gm, om = g.TDT(synth.tdt_gguf(cfg, t)), orc.TDT(cfg, t)
    n, T = 128, 750
    enc = np.stack([synth.encoder_frames(1 + i, T, cfg.D) for i in range(n)])
    cap = 16 * T + 1024
    b = g.TDTBatch(gm, n, T, cap)
    toks, counts = b.decode(enc, [T] * n)
    with orc.fast_mode():
        wt, wc, _ = om.run(enc, cap, THREADS)
    assert np.array_equal(counts, wc), "token counts differ"
    for i in range(n):
        w = wt[i, :wc[i]]
        assert np.array_equal(toks[i]["id"], w[:, 0]), f"stream {i}: token ids differ"
        assert np.array_equal(toks[i]["frame"], w[:, 1]), f"stream {i}: frames differ"
        assert np.array_equal(toks[i]["duration"], w[:, 2]), f"stream {i}: durations differ"
        wp = w[:, 3].copy().view(np.float32)
        assert np.all(np.abs(toks[i]["p"] - wp) <= 1e-6 * np.abs(wp)), f"stream {i}: p beyond 1e-6"
    for i in (0, 127):  # the LSTM state each stream ends with
        st = om.state()
        with orc.fast_mode():
            om.decode(enc[i], st, 0)
        h, c, last = b.state(i)
        assert last == st[2] and bits_equal(h, st[0]) and bits_equal(c, st[1]), f"stream {i}: LSTM state"
