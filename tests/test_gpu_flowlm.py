"""GPU parity: the CUDA path through the C ABI against the CPU oracle (a
restatement of the reference's amd64 arithmetic), on the same seeded
synthetic inputs. The bar is bit-identical float32 outputs; each test also
states the 1e-3 relative tolerance the spec allows, which identical bits
pass trivially."""

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import SMALL, bits_equal, mismatch, voice_kv

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _q8(rng, n, k):
    return synth.rand_q8(rng, n, k)


@pytest.mark.parametrize("m,n,k", [(1, 3072, 1024), (1, 1024, 4096), (3, 64, 96), (8, 96, 128), (17, 64, 128),
                                   (64, 1024, 1024), (256, 4096, 1024), (130, 200, 256), (40, 96, 192),
                                   (130, 1000, 64), (100, 3072, 1024), (33, 4096, 1024), (200, 1024, 4096),
                                   (128, 1024, 192), (300, 512, 512)])
def test_q8_int8_path_bit_exact(have_gpu, m, n, k):
    """kern.Linear on a packed Q8_0 weight (int8 path, q8int.go:148-223):
    per-block int32 dots and the FMA chain give identical float32."""
    rng = np.random.default_rng(m * 7919 + n)
    w = _q8(rng, n, k)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32)
    if n % 32 and m <= 8:
        pytest.skip("the small-M kernel takes whole 32-row groups")
    gw = g.Weight.q8(w.blocks, n, k).drop_rows()
    for b in (None, bias):
        got = g.linear(gw, x, b)
        want = orc.linear(x, "q8_0", w.blocks, n, k, bias=b, dropped=True)
        ne, rel = mismatch(got, want)
        assert ne == 0, f"{ne} of {got.size} differ (max rel {rel:.2e})"


@pytest.mark.parametrize("n,k", [(512, 1024), (1536, 512), (1030, 640), (7, 64)])
def test_q8_float_path_bit_exact(have_gpu, n, k):
    """One row times a Q8_0 weight that keeps its rows: the float path
    (dot4q8avx per four rows, dotQ8Go for the rest, gemm.go:195-259)."""
    rng = np.random.default_rng(n + k)
    w = _q8(rng, n, k)
    x = rng.normal(0, 1, (1, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32)
    gw = g.Weight.q8(w.blocks, n, k)
    got = g.linear(gw, x, bias)
    want = orc.linear(x, "q8_0", w.blocks, n, k, bias=bias)
    ne, rel = mismatch(got, want)
    assert ne == 0, f"{ne} differ, max rel {rel:.2e}"
    assert rel <= TOL


@pytest.mark.parametrize("n,k,m", [(1024, 32, 1), (32, 512, 1), (512, 32, 13), (1, 1024, 1), (6, 48, 16),
                                   (100, 96, 3)])
def test_f32_float_path_bit_exact(have_gpu, n, k, m):
    """F32 weights take the float path for any number of rows (dot4f32avx
    per four rows, dotF32Go for the rest)."""
    rng = np.random.default_rng(n * k)
    w = rng.normal(0, 0.2, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    got = g.linear(g.Weight.f32(w), x)
    want = orc.linear(x, "f32", w, n, k)
    assert bits_equal(got, want)


def _models(cfg, seed=0):
    t = synth.flowlm_tensors(cfg, seed)
    return g.FlowLM(synth.flowlm_gguf(cfg, t)), orc.FlowLM(cfg, t)


@pytest.mark.parametrize("n,frames,prefill", [(1, 12, 8), (5, 10, 3), (16, 6, 9)])
def test_flowlm_small_frames_bit_exact(have_gpu, n, frames, prefill):
    """Whole frames (flowLM.step + flowHead.sample, speak.go:146-174) of a
    small model for several streams, the latent fed back each frame."""
    cfg = synth.FlowLMConfig(**SMALL)
    gm, om = _models(cfg)
    kvs = [voice_kv(cfg, prefill + (i % 3), 1 + i) for i in range(n)]
    st = g.Streams(gm, [gm.voice(kv) for kv in kvs], frames)
    os_ = [om.stream(kv) for kv in kvs]
    noise = np.stack([synth.noise_frames(1 + i, frames, cfg.ldim, cfg.temperature) for i in range(n)], axis=1)
    lat_o = [None] * n
    for f in range(frames):
        lat, eos, sc, lo = st.step(noise[f], want_lm_out=True)
        for i in range(n):
            r = om.frame(os_[i], lat_o[i], noise[f, i])
            lat_o[i] = r["latent"]
            for name, a, b in (("lm_out", lo[i], r["lm_out"]), ("eos", eos[i:i + 1], [r["eos"]]),
                               ("latent", lat[i], r["latent"]), ("scaled", sc[i], r["scaled"])):
                ne, rel = mismatch(a, b)
                assert ne == 0, f"frame {f} stream {i} {name}: {ne} differ, max rel {rel:.2e}"
    for i in range(n):
        assert st.pos(i) == os_[i].pos


def test_flowlm_c0_model_bit_exact(have_gpu):
    """The C0 model (6 layers, d 1024, 16 heads, FFN 4096, flow head
    1024→512→32) from a 64-position prefill, one stream, 24 frames."""
    cfg = synth.FlowLMConfig()
    gm, om = _models(cfg)
    kv = voice_kv(cfg, 64, 1)
    st = g.Streams(gm, [gm.voice(kv)], 24)
    os_ = om.stream(kv)
    noise = synth.noise_frames(1, 24, cfg.ldim, cfg.temperature)
    lat_o = None
    for f in range(24):
        lat, eos, sc, lo = st.step(noise[f][None], want_lm_out=True)
        r = om.frame(os_, lat_o, noise[f])
        lat_o = r["latent"]
        assert bits_equal(lo[0], r["lm_out"]), f"frame {f} lm_out {mismatch(lo[0], r['lm_out'])}"
        assert bits_equal(lat[0], r["latent"]), f"frame {f} latent {mismatch(lat[0], r['latent'])}"
        assert bits_equal(eos[:1], [r["eos"]])


def test_flowlm_batched_run_device_bit_exact(have_gpu):
    """C1's shape at 64 streams (the M=64 tensor-core path), device-resident
    run of 6 frames against the oracle's independent streams."""
    import torch

    cfg = synth.FlowLMConfig()
    gm, om = _models(cfg)
    n, frames = 64, 6
    kvs = [voice_kv(cfg, 64, 1 + i) for i in range(n)]
    st = g.Streams(gm, [gm.voice(kv) for kv in kvs], frames)
    noise = np.stack([synth.noise_frames(1 + i, frames, cfg.ldim, cfg.temperature) for i in range(n)], axis=1)
    dn = torch.from_numpy(noise).cuda()
    dl = torch.empty_like(dn)
    de = torch.empty((frames, n), device="cuda")
    st.run_device(frames, dn.data_ptr(), dl.data_ptr(), de.data_ptr())
    st.sync()
    lat_o, eos_o, _ = om.run([om.stream(kv) for kv in kvs], noise, threads=8)
    ne, rel = mismatch(dl.cpu().numpy(), lat_o)
    assert ne == 0, f"{ne} latents differ, max rel {rel:.2e}"
    assert bits_equal(de.cpu().numpy(), eos_o)


@pytest.mark.parametrize("n", [128, 131])
def test_flowlm_parts_run_device_and_step(have_gpu, n):
    """A set of 128 or more streams runs as two parts on their own CUDA
    streams (an odd count splits unevenly): device-resident frames and the
    per-frame host call both match the oracle bit for bit."""
    import torch

    cfg = synth.FlowLMConfig(**SMALL)
    gm, om = _models(cfg, seed=4)
    frames = 3
    kvs = [voice_kv(cfg, 8 + i % 5, 1 + i) for i in range(n)]  # ragged prefills
    noise = np.stack([synth.noise_frames(1 + i, frames, cfg.ldim, cfg.temperature) for i in range(n)], axis=1)
    lat_o, eos_o, _ = om.run([om.stream(kv) for kv in kvs], noise, threads=8)
    st = g.Streams(gm, [gm.voice(kv) for kv in kvs], frames)
    dn = torch.from_numpy(noise).cuda()
    dl = torch.empty_like(dn)
    de = torch.empty((frames, n), device="cuda")
    st.run_device(frames, dn.data_ptr(), dl.data_ptr(), de.data_ptr())
    st.sync()
    ne, rel = mismatch(dl.cpu().numpy(), lat_o)
    assert ne == 0, f"{ne} latents differ, max rel {rel:.2e}"
    assert bits_equal(de.cpu().numpy(), eos_o)
    assert [st.pos(i) for i in (0, n - 1)] == [8 + frames, 8 + (n - 1) % 5 + frames]
    st.reset()
    for f in range(frames):
        lat, eos, _, _ = st.step(noise[f])
        assert bits_equal(lat, lat_o[f]) and bits_equal(eos, eos_o[f]), f"frame {f}"


def _text_ids(cfg, lens, seed):
    return [[(11 * i + 5 * j + seed) % cfg.text_vocab for j in range(T)] for i, T in enumerate(lens)]


@pytest.mark.parametrize("lens", [[1, 3, 5, 16], [17, 30, 0, 4], [2, 40, 6, 23]])
def test_flowlm_text_prefill_bit_exact(have_gpu, lens):
    """flowLM.text (lm.go:172-181) for ragged token counts — attend's T < 4
    (values key by key), 4 ≤ T ≤ 16 (gemvRows products) and T > 16 (packed
    rows below T/6·6) — then frames from bos: the output at each stream's
    last token, the positions and every frame bit-identical to the oracle."""
    cfg = synth.FlowLMConfig(**SMALL)
    gm, om = _models(cfg, seed=5)
    n, frames = len(lens), 3
    kvs = [voice_kv(cfg, 6 + i, 1 + i) for i in range(n)]
    ids = _text_ids(cfg, lens, 3)
    st = g.Streams(gm, [gm.voice(kv) for kv in kvs], max(lens) + frames)
    out = st.text(ids)
    os_ = [om.stream(kv) for kv in kvs]
    for i in range(n):
        if ids[i]:
            ne, rel = mismatch(out[i], om.text(os_[i], ids[i]))
            assert ne == 0, f"stream {i} (T={lens[i]}): {ne} of the output differ, max rel {rel:.2e}"
        assert st.pos(i) == os_[i].pos == 6 + i + lens[i]
    noise = np.stack([synth.noise_frames(1 + i, frames, cfg.ldim, cfg.temperature) for i in range(n)], axis=1)
    lat_o, eos_o, _ = om.run(os_, noise, threads=4)
    for f in range(frames):
        lat, eos, _, _ = st.step(noise[f])
        assert bits_equal(lat, lat_o[f]) and bits_equal(eos, eos_o[f]), f"frame {f}"


def test_flowlm_text_prefill_parts(have_gpu):
    """A set of 130 streams (two parts on their own CUDA streams) prefilled
    with ragged texts of 0-20 tokens, then two device-resident frames."""
    import torch

    cfg = synth.FlowLMConfig(**SMALL)
    gm, om = _models(cfg, seed=6)
    n, frames = 130, 2
    rng = np.random.default_rng(7)
    lens = [int(v) for v in rng.integers(0, 21, n)]
    kvs = [voice_kv(cfg, 4 + i % 5, 1 + i) for i in range(n)]
    ids = _text_ids(cfg, lens, 9)
    st = g.Streams(gm, [gm.voice(kv) for kv in kvs], 20 + frames)
    assert st.parts() == 2
    out = st.text(ids)
    os_ = [om.stream(kv) for kv in kvs]
    for i in range(n):
        if ids[i]:
            assert bits_equal(out[i], om.text(os_[i], ids[i])), f"stream {i}"
    noise = np.stack([synth.noise_frames(1 + i, frames, cfg.ldim, cfg.temperature) for i in range(n)], axis=1)
    lat_o, eos_o, _ = om.run(os_, noise, threads=8)
    dn = torch.from_numpy(noise).cuda()
    dl = torch.empty_like(dn)
    de = torch.empty((frames, n), device="cuda")
    st.run_device(frames, dn.data_ptr(), dl.data_ptr(), de.data_ptr())
    st.sync()
    assert bits_equal(dl.cpu().numpy(), lat_o) and bits_equal(de.cpu().numpy(), eos_o)


def test_flowlm_text_errors(have_gpu):
    """Token ids outside lm.embed and texts longer than the set's room are
    refused before anything runs."""
    cfg = synth.FlowLMConfig(**SMALL)
    gm, _ = _models(cfg)
    st = g.Streams(gm, [gm.voice(voice_kv(cfg, 4, 1))], 5)
    with pytest.raises(g.GrxError):
        st.text([[cfg.text_vocab + 1]])
    with pytest.raises(g.GrxError):
        st.text([list(range(6))])
    assert st.pos(0) == 4


@pytest.mark.parametrize("n", [3, 16, 17, 40])
def test_flowlm_voice_from_latents_bit_exact(have_gpu, n):
    """The flow-LM half of CloneVoice (voice.go:94-106): the speaker
    projection (gemvRows up to 16 rows, packed rows beyond) and [bos_voice;
    cond] through the transformer from an empty state give caches
    bit-identical to the oracle's; frames from that voice match too."""
    cfg = synth.FlowLMConfig(**SMALL)
    gm, om = _models(cfg, seed=8)
    lat = np.random.default_rng(n).normal(0, 1, (n, cfg.ldim)).astype(np.float32)
    v = gm.voice_from_latents(lat)
    kv_o = om.voice_from_latents(lat)
    kv = v.kv(cfg.layers, cfg.d)
    ne, rel = mismatch(kv, kv_o)
    assert ne == 0, f"{ne} of {kv.size} cache values differ, max rel {rel:.2e}"
    frames = 2
    st = g.Streams(gm, [v], frames)
    os_ = om.stream(kv_o)
    noise = synth.noise_frames(3, frames, cfg.ldim, cfg.temperature)[:, None, :]
    lat_o, eos_o, _ = om.run([os_], noise)
    for f in range(frames):
        l_, e_, _, _ = st.step(noise[f])
        assert bits_equal(l_, lat_o[f]) and bits_equal(e_, eos_o[f]), f"frame {f}"
