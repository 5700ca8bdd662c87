"""The oracle's fast mode (oracle/fast.h, the timed CPU baseline) against its
exact mode: the reference's SIMD kernels restated in their lane order must
give the exact restatement's float32 bits, product by product, in one-query
attention, in the activations and over whole FlowLM and TDT runs. Both the
AVX-512 VNNI tile (q8tileEVEX, vnni_amd64.s:58-138) and the 256-bit form are
checked (the latter in a child process with ORC_FAST_AVX2=1). CPU only."""

import os
import subprocess
import sys

import numpy as np
import pytest

from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import SMALL, bits_equal, voice_kv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# (m, n, k, rows dropped): the int8 path (dropped, or m >= 2) and the float
# path (one row, rows kept), FlowLM / TDT / Whisper shapes and ragged ones.
Q8_SHAPES = [(1, 3072, 1024, True), (1, 1024, 4096, True), (6, 1024, 4096, True), (7, 100, 64, True),
             (13, 4096, 1024, False), (2, 37, 96, False), (1, 512, 1024, False), (1, 1030, 640, False),
             (1, 2560, 640, False), (1, 33, 32, False)]
F32_SHAPES = [(1, 1024, 32), (1, 32, 512), (3, 17, 48), (1, 5, 7)]


def _kind():
    with orc.fast_mode() as fm:
        return fm.kind


def _need_simd():
    if _kind() == 0:
        pytest.skip("this processor has neither AVX2 nor AVX-512 VNNI: the fast mode is the exact mode")


def _both(fn):
    a = fn()
    with orc.fast_mode():
        b = fn()
    return a, b


@pytest.mark.parametrize("m,n,k,dropped", Q8_SHAPES)
def test_fast_q8_products(m, n, k, dropped):
    _need_simd()
    rng = np.random.default_rng(m * 7919 + n + k)
    w = synth.rand_q8(rng, n, k)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    b = rng.normal(0, 0.1, n).astype(np.float32)
    e, f = _both(lambda: orc.linear(x, "q8_0", w.blocks, n, k, b, dropped))
    assert bits_equal(e, f)


@pytest.mark.parametrize("m,n,k", F32_SHAPES)
def test_fast_f32_products(m, n, k):
    _need_simd()
    rng = np.random.default_rng(n * 31 + k)
    w = rng.normal(0, 0.1, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    e, f = _both(lambda: orc.linear(x, "f32", w, n, k, None))
    assert bits_equal(e, f)


@pytest.mark.parametrize("nk", [1, 3, 4, 5, 8, 63, 64, 65, 320, 577])
def test_fast_attention(nk):
    """attend (nn.go:200-243): the groups of four keys and the tail, EXP8
    lane sums over nk & ~7 keys and expf for the rest."""
    _need_simd()
    rng = np.random.default_rng(nk)
    q = rng.normal(0, 1, 1024).astype(np.float32)
    kc = rng.normal(0, 1, (nk, 1024)).astype(np.float32)
    vc = rng.normal(0, 1, (nk, 1024)).astype(np.float32)
    e, f = _both(lambda: orc.attend_one(q, kc, vc, 16))
    assert bits_equal(e, f)


def test_fast_activations():
    _need_simd()
    x = np.random.default_rng(5).normal(0, 3, 4099).astype(np.float32)
    x[:8] = [0, -0.0, 9.5, -9.5, 40, -40, 1e-30, -87.5]
    L = orc.lib()
    for fn in (L.orc_gelu_vec, L.orc_silu_vec):
        def run():
            y = x.copy()
            fn(orc.p(y), len(y))
            return y
        e, f = _both(run)
        assert bits_equal(e, f)


def test_fast_flowlm_frames_small_model():
    """A small FlowLM over 6 frames from a 9-position prefill, two streams on
    two threads (one stream per thread) and one stream on four threads (its
    products and heads split over them)."""
    _need_simd()
    cfg = synth.FlowLMConfig(**SMALL)
    t = synth.flowlm_tensors(cfg, 0)
    om = orc.FlowLM(cfg, t)
    frames = 6
    for n, threads in ((2, 2), (1, 4)):
        kvs = [voice_kv(cfg, 9, 1 + i) for i in range(n)]
        noise = np.stack([synth.noise_frames(1 + i, frames, cfg.ldim, cfg.temperature) for i in range(n)], axis=1)

        def run():
            return om.run([om.stream(kv) for kv in kvs], noise, threads=threads, want_lm_out=True)

        (la, ea, oa), (lb, eb, ob) = _both(run)
        assert bits_equal(la, lb) and bits_equal(ea, eb) and bits_equal(oa, ob)


def test_fast_flowlm_full_model_frames():
    """The Pocket-TTS-shaped model over 3 frames from a
    64-position prefill, one stream whose products split over 4 threads."""
    _need_simd()
    cfg = synth.FlowLMConfig()
    t = synth.flowlm_tensors(cfg, 0)
    om = orc.FlowLM(cfg, t)
    kv = voice_kv(cfg, 64, 1)
    noise = synth.noise_frames(1, 3, cfg.ldim, cfg.temperature)[:, None, :].copy()
    (la, ea, oa), (lb, eb, ob) = _both(lambda: om.run([om.stream(kv)], noise, threads=4, want_lm_out=True))
    assert bits_equal(la, lb) and bits_equal(ea, eb) and bits_equal(oa, ob)


def test_fast_tdt_decode():
    """The TDT loop's float-path products (LSTM, joint) through the fast
    kernels: tokens, frames and durations identical."""
    _need_simd()
    cfg = synth.TDTConfig(H=64, J=64, V=33, D=64, layers=2)
    t = synth.tdt_tensors(cfg, 0)
    om = orc.TDT(cfg, t)
    enc = np.stack([synth.encoder_frames(1 + i, 20, cfg.D) for i in range(3)])
    e, f = _both(lambda: om.run(enc, 400, 2))
    for a, b in zip(e, f):
        assert np.array_equal(np.asarray(a), np.asarray(b))


def test_fast_256bit_path_matches_exact():
    """The 256-bit kernels (no AVX-512 VNNI) in a child process."""
    if _kind() == 0:
        pytest.skip("no AVX2")
    code = (
        "import numpy as np\n"
        "from gorelaxor_b200 import synth\n"
        "from oracle import oracle as orc\n"
        "from tests.helpers import bits_equal\n"
        "rng = np.random.default_rng(1)\n"
        "for m, n, k, dr in [(1, 3072, 1024, True), (6, 1024, 4096, True), (7, 100, 64, True), (13, 77, 96, False)]:\n"
        "    w = synth.rand_q8(rng, n, k)\n"
        "    x = rng.normal(0, 1, (m, k)).astype(np.float32)\n"
        "    e = orc.linear(x, 'q8_0', w.blocks, n, k, None, dr)\n"
        "    with orc.fast_mode() as fm:\n"
        "        assert fm.kind == 1, fm.kind\n"
        "        f = orc.linear(x, 'q8_0', w.blocks, n, k, None, dr)\n"
        "    assert bits_equal(e, f), (m, n, k)\n"
        "print('ok')\n"
    )
    env = dict(os.environ, ORC_FAST_AVX2="1", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("m,n,k,kind", [(6, 512, 512, 1), (7, 64, 300, 0), (13, 40, 96, 1), (1500, 64, 512, 1)])
def test_fast_whisper_packed_product(m, n, k, kind):
    """whisper/gemm.go:124-209 (bias, then += each 256-deep fused chain for
    rows below m/6·6, gemv for the rest), F16 (kind 1) and F32 weights."""
    _need_simd()
    rng = np.random.default_rng(m + n + k)
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    wf = rng.normal(0, 0.1, (n, k)).astype(np.float32)
    w = wf.astype(np.float16).view(np.uint16) if kind == 1 else wf
    w = np.ascontiguousarray(w)
    bias = rng.normal(0, 0.1, n).astype(np.float32)

    def run():
        c = np.empty((m, n), np.float32)
        orc.lib().orc_whisper_matmul(orc.p(c), orc.p(a), m, n, k, kind, orc.p(w), orc.p(bias))
        return c

    e, f = _both(run)
    assert bits_equal(e, f)


def test_fast_whisper_greedy_small():
    """A small Whisper decoder's cross K/V prep and 12 greedy steps, the
    fast mode with a pool of 4 threads against the exact mode."""
    _need_simd()
    cfg = synth.WhisperConfig(n_state=128, n_head=2, n_text_layer=2, n_text_ctx=64)
    t = synth.whisper_tensors(cfg, 0)
    om = orc.Whisper(cfg, t, synth.whisper_words(cfg))
    enc = synth.whisper_encoder_out(3, cfg)
    prompt = [50360, 100, 200, 50257]
    want, wns = om.greedy(om.seq(enc), prompt, 3, 12)
    with orc.fast_mode(4):
        got, ns = om.greedy(om.seq(enc), prompt, 3, 12)
    assert np.array_equal(got, want) and np.float32(ns).view(np.uint32) == np.float32(wns).view(np.uint32)
