"""The oracle's self-checks: gorelaxor's own kernel tests restated against the
C++ restatement (internal/kern/*_test.go, whisper/whisper_test.go,
pockettts/nn_test.go), with the same shapes, tolerances and known answers,
plus an independent float64 numpy model of one FlowLM frame. CPU only."""

import math

import numpy as np
import pytest

from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import SMALL, voice_kv


def test_quant_known_answers():
    """q8int_test.go:9-35: a zero block gives scale 0 and bytes 128 (value
    0 here, the signed form); an extreme of -40 gives byte 1 (value -127)."""
    r = np.random.default_rng(3)
    nb = 9
    x = np.concatenate([r.normal(0, 1, 32) * (1 + b) for b in range(nb)]).astype(np.float32)
    x[2 * 32:3 * 32] = 0
    x[5 * 32] = -40
    q, s = orc.quant_act(x)
    assert s[2] == 0 and np.all(q[64:96] == 0)
    assert q[5 * 32] == -127
    # RNE of v·(127/amax), amax·(1/127) with the float32 constant 0x3c010204
    for b in range(nb):
        blk = x[b * 32:(b + 1) * 32]
        amax = np.float32(np.max(np.abs(blk)))
        assert s[b] == np.float32(amax * np.float32(np.uint32(0x3c010204).view(np.float32)))
        if amax:
            want = np.clip(np.rint((blk * np.float32(np.float32(127) / amax)).astype(np.float64)), -128, 127)
            assert np.array_equal(q[b * 32:(b + 1) * 32], want.astype(np.int8))


def test_expf_against_exp():
    """whisper_test.go:99-105: expf within 1e-6 relative of exp over [-87, 88];
    the vector (EXP8) form too."""
    v = np.float32(-87.0)
    while v < 88:
        want = math.exp(float(v))
        assert abs(orc.lib().orc_expf_go(float(v)) - want) <= 1e-6 * want
        assert abs(orc.lib().orc_exp_avx(float(v)) - want) <= 1e-6 * want
        v = np.float32(v + np.float32(0.731))


def test_expsub_and_gelu_vector_vs_scalar():
    """whisper_test.go:70-97: expSub's AVX and Go forms agree to 1e-5 (sum
    1e-4); GELU's to 1e-5."""
    x = (np.arange(1003) % 97 * 0.37 - 20).astype(np.float32)
    y = x.copy()
    s1 = orc.lib().orc_expsub(orc.p(x), x.size, 3.0)
    s2 = sum(float(orc.lib().orc_expf_go(float(v - np.float32(3)))) for v in y)
    e2 = np.array([orc.lib().orc_expf_go(float(v - np.float32(3))) for v in y], np.float32)
    assert np.all(np.abs(x - e2) <= 1e-5 * e2 + 1e-30)
    assert abs(s1 - s2) <= 1e-4 * s2
    g = (np.arange(1003) % 211 * 0.05 - 5).astype(np.float32)
    for v in g:
        assert abs(orc.lib().orc_gelu_avx(float(v)) - orc.lib().orc_gelu_go(float(v))) <= 1e-5


def test_silu_vector_vs_scalar():
    """vec_test.go:9-46: SiLU's AVX and Go forms agree to 1e-6, ±120 included."""
    for v in list(np.linspace(-120, 120, 481, dtype=np.float32)):
        a, b = orc.lib().orc_silu_avx(float(v)), orc.lib().orc_silu_go(float(v))
        assert abs(a - b) <= 1e-6 * max(1.0, abs(b))


def test_f16_conversions():
    """f16.go: widening is exact for all halves (odd_test.go:79-113 pins the
    subnormal, negative-zero-ish 0x8001 scale); narrowing rounds to nearest
    even like numpy."""
    for h in [0x0000, 0x8000, 0x0001, 0x8001, 0x03ff, 0x0400, 0x3c00, 0x7bff, 0x7c00, 0xfc00]:
        assert orc.f16_to_f32(h) == float(np.uint16(h).view(np.float16))
    allh = np.arange(0, 1 << 16, 97, dtype=np.uint16)
    fin = allh[np.isfinite(allh.view(np.float16))]
    got = np.array([orc.f16_to_f32(int(h)) for h in fin], np.float32)
    assert np.array_equal(got, fin.view(np.float16).astype(np.float32))
    r = np.random.default_rng(11)
    vals = np.concatenate([r.normal(0, 1, 2000), r.normal(0, 1e-6, 500), r.normal(0, 3e4, 200)]).astype(np.float32)
    for v in vals:
        assert orc.f32_to_f16(float(v)) == int(np.float32(v).astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("m,n,k", [(2, 1, 32), (5, 15, 64), (6, 16, 96), (7, 17, 32), (13, 40, 128), (50, 33, 256),
                                   (100, 70, 64)])
def test_int8_matmul_against_fp64(m, n, k):
    """q8int_test.go:80-126: the int8 path within 0.02 RMS relative of the
    float64 product with the widened weight."""
    r = np.random.default_rng(5 + m)
    x = r.normal(0, 1, (m, k)).astype(np.float32)
    wv = (r.random((n, k)) * 2 - 1).astype(np.float32)
    w = orc.to_q8(wv)
    wf = synth.q8_dequant(synth.Q8(n, k, w)).astype(np.float64)
    bias = r.random(n).astype(np.float32)
    got = orc.linear(x, "q8_0", w, n, k, bias=bias, dropped=True)
    ref = x.astype(np.float64) @ wf.T + bias
    assert np.sqrt(((got - ref) ** 2).sum() / (ref ** 2).sum()) <= 0.02


@pytest.mark.parametrize("m,n,k", [(1, 70, 64), (3, 33, 96), (1, 40, 128)])
def test_float_path_types(m, n, k):
    """kern_test.go:30-73: F32 and Q8_0 (float path) products within 1e-3 of
    float64."""
    r = np.random.default_rng(1)
    x = (r.random((m, k)) * 2 - 1).astype(np.float32)
    wv = (r.random((n, k)) * 2 - 1).astype(np.float32)
    got = orc.linear(x, "f32", wv, n, k)
    assert np.abs(got - x.astype(np.float64) @ wv.T.astype(np.float64)).max() <= 1e-3
    w = orc.to_q8(wv)
    wf = synth.q8_dequant(synth.Q8(n, k, w)).astype(np.float64)
    # the test forces the float path (setInt(intNone), kern_test.go:32): one row at a time
    got = np.vstack([orc.linear(x[i:i + 1], "q8_0", w, n, k) for i in range(m)])
    assert np.abs(got - x.astype(np.float64) @ wf.T).max() <= 1e-3


def test_attention_against_fp64():
    """nn_test.go:108-153 (the known-answer test for attend): single-query
    attention equals float64 softmax attention to 1e-5."""
    r = np.random.default_rng(9)
    d, heads = 128, 2
    for nk in (1, 3, 4, 7, 8, 9, 33, 64):
        q = r.normal(0, 1, d).astype(np.float32)
        kc = r.normal(0, 1, (nk, d)).astype(np.float32)
        vc = r.normal(0, 1, (nk, d)).astype(np.float32)
        got = orc.attend_one(q, kc, vc, heads)
        hd = d // heads
        want = np.zeros(d)
        for h in range(heads):
            sl = slice(h * hd, (h + 1) * hd)
            s = kc[:, sl].astype(np.float64) @ q[sl].astype(np.float64) / math.sqrt(hd)
            e = np.exp(s - s.max())
            want[sl] = (e / e.sum()) @ vc[:, sl].astype(np.float64)
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())


def test_layer_norm_against_fp64():
    r = np.random.default_rng(2)
    x = (r.normal(0, 3, (4, 1024)) + 5).astype(np.float32)
    w = r.normal(1, 0.1, 1024).astype(np.float32)
    b = r.normal(0, 0.1, 1024).astype(np.float32)
    got = orc.layer_norm_pt(x, w, b, 1e-5)
    xd = x.astype(np.float64)
    ref = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-5) * w + b
    assert np.abs(got - ref).max() <= 1e-5


def _np_frame(cfg, t, kvs, latent, noise, tc, pos):
    """One FlowLM frame in float64 numpy with the int8 path's activation
    rounding, written from the model's definition (pockettts/lm.go, nn.go)."""
    D = lambda a: np.asarray(a, np.float64)
    W = lambda name: D(synth.q8_dequant(t[name])) if isinstance(t[name], synth.Q8) else D(t[name])

    def q8round(x):
        out = np.empty_like(x)
        for b in range(0, x.size, 32):
            blk = x[b:b + 32]
            amax = np.abs(blk).max()
            out[b:b + 32] = np.rint(blk * 127 / amax) * amax / 127 if amax else 0
        return out

    def ln(x, w, b, eps):
        y = (x - x.mean()) / np.sqrt(x.var() + eps)
        return y * w + b if w is not None else y

    def rope(v):
        hd = cfg.d // cfg.heads
        f = np.exp(-np.log(cfg.max_period) * 2 / hd * np.arange(hd // 2))
        a = f * pos
        v = v.reshape(cfg.heads, hd // 2, 2).copy()
        r, i = v[..., 0].copy(), v[..., 1].copy()
        v[..., 0], v[..., 1] = r * np.cos(a) - i * np.sin(a), r * np.sin(a) + i * np.cos(a)
        return v.reshape(-1)

    gelu = lambda v: 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * v * (1 + 0.044715 * v * v)))
    silu = lambda v: v / (1 + np.exp(-v))
    x = W("lm.input.weight") @ D(latent)
    for l in range(cfg.layers):
        p = f"lm.blk.{l}."
        h = ln(x, D(t[p + "norm1.weight"]), D(t[p + "norm1.bias"]), 1e-5)
        qkv = W(p + "attn_qkv.weight") @ q8round(h)
        q, k, v = rope(qkv[:cfg.d]), rope(qkv[cfg.d:2 * cfg.d]), qkv[2 * cfg.d:]
        K = np.vstack([D(kvs[l][0]), k])
        V = np.vstack([D(kvs[l][1]), v])
        kvs[l] = (K, V)
        hd = cfg.d // cfg.heads
        att = np.zeros(cfg.d)
        for hh in range(cfg.heads):
            sl = slice(hh * hd, (hh + 1) * hd)
            s = K[:, sl] @ q[sl] / np.sqrt(hd)
            e = np.exp(s - s.max())
            att[sl] = (e / e.sum()) @ V[:, sl]
        x = x + W(p + "attn_out.weight") @ q8round(att)
        h = ln(x, D(t[p + "norm2.weight"]), D(t[p + "norm2.bias"]), 1e-5)
        x = x + W(p + "ff2.weight") @ q8round(gelu(W(p + "ff1.weight") @ q8round(h)))
    out = ln(x, D(t["lm.out_norm.weight"]), D(t["lm.out_norm.bias"]), 1e-5)
    eos = float(W("lm.eos.weight") @ out + t["lm.eos.bias"][0])
    y = W("flow.cond.weight") @ out + D(t["flow.cond.bias"]) + D(tc)
    sy = silu(y)
    h = W("flow.input.weight") @ D(noise) + D(t["flow.input.bias"])
    fd = cfg.flow_dim
    for i in range(cfg.flow_depth):
        p = f"flow.res.{i}."
        mod = W(p + "ada.weight") @ sy + D(t[p + "ada.bias"])
        n = ln(h, D(t[p + "norm.weight"]), D(t[p + "norm.bias"]), 1e-6) * (1 + mod[fd:2 * fd]) + mod[:fd]
        m = silu(W(p + "fc1.weight") @ n + D(t[p + "fc1.bias"]))
        h = h + mod[2 * fd:] * (W(p + "fc2.weight") @ m + D(t[p + "fc2.bias"]))
    mod = W("flow.final.ada.weight") @ sy + D(t["flow.final.ada.bias"])
    n = ln(h, None, None, 1e-6) * (1 + mod[fd:]) + mod[:fd]
    v = W("flow.final.out.weight") @ n + D(t["flow.final.out.bias"])
    return out, eos, D(noise) + v


def test_flowlm_frame_against_numpy_model():
    """The restated step and flow head follow the model: three frames of a
    small model against an independent float64 numpy model (same int8
    activation rounding) within 2% RMS — the int8 path's own bound
    (q8int_test.go:120) — fed the oracle's latents (teacher forcing)."""
    cfg = synth.FlowLMConfig(**SMALL)
    t = synth.flowlm_tensors(cfg, 0)
    om = orc.FlowLM(cfg, t)
    kv = voice_kv(cfg, 6, 1)
    st = om.stream(kv)
    kvs = [(kv[l, 0].astype(np.float64), kv[l, 1].astype(np.float64)) for l in range(cfg.layers)]
    tc = om.time_conds()[0]
    noise = synth.noise_frames(1, 3, cfg.ldim, cfg.temperature)
    latent = None
    for f in range(3):
        lat_in = t["lm.bos"] if latent is None else latent
        r = om.frame(st, latent, noise[f])
        out, eos, lat = _np_frame(cfg, t, kvs, lat_in, noise[f], tc, 6 + f)
        rel = lambda a, b: np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum())
        assert rel(r["lm_out"], out) < 0.02
        assert rel(r["latent"], lat) < 0.02
        assert abs(r["eos"] - eos) < 0.02 * max(1, abs(eos))
        latent = r["latent"]


def _np_text(cfg, t, kvs, ids, pos0):
    """flowLM.text in float64 numpy: the token rows through the transformer
    with causal attention over the voice prefill and the earlier tokens, the
    int8 path's activation rounding per row; the output at the last token."""
    D = lambda a: np.asarray(a, np.float64)
    W = lambda name: D(synth.q8_dequant(t[name])) if isinstance(t[name], synth.Q8) else D(t[name])

    def q8round(x):
        out = np.empty_like(x)
        for b in range(0, x.size, 32):
            blk = x[b:b + 32]
            amax = np.abs(blk).max()
            out[b:b + 32] = np.rint(blk * 127 / amax) * amax / 127 if amax else 0
        return out

    def ln(x, w, b, eps):
        return (x - x.mean()) / np.sqrt(x.var() + eps) * w + b

    hd = cfg.d // cfg.heads

    def rope(v, pos):
        f = np.exp(-np.log(cfg.max_period) * 2 / hd * np.arange(hd // 2))
        a = f * pos
        v = v.reshape(cfg.heads, hd // 2, 2).copy()
        r, i = v[..., 0].copy(), v[..., 1].copy()
        v[..., 0], v[..., 1] = r * np.cos(a) - i * np.sin(a), r * np.sin(a) + i * np.cos(a)
        return v.reshape(-1)

    gelu = lambda v: 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * v * (1 + 0.044715 * v * v)))
    E = W("lm.embed")
    xs = [E[i].copy() for i in ids]
    T = len(ids)
    for l in range(cfg.layers):
        p = f"lm.blk.{l}."
        qs, K, V = [], D(kvs[l][0]), D(kvs[l][1])
        for r in range(T):
            qkv = W(p + "attn_qkv.weight") @ q8round(ln(xs[r], D(t[p + "norm1.weight"]), D(t[p + "norm1.bias"]), 1e-5))
            qs.append(rope(qkv[:cfg.d], pos0 + r))
            K = np.vstack([K, rope(qkv[cfg.d:2 * cfg.d], pos0 + r)])
            V = np.vstack([V, qkv[2 * cfg.d:]])
        for r in range(T):
            nk = pos0 + r + 1
            att = np.zeros(cfg.d)
            for hh in range(cfg.heads):
                sl = slice(hh * hd, (hh + 1) * hd)
                s = K[:nk, sl] @ qs[r][sl] / np.sqrt(hd)
                e = np.exp(s - s.max())
                att[sl] = (e / e.sum()) @ V[:nk, sl]
            xs[r] = xs[r] + W(p + "attn_out.weight") @ q8round(att)
            h = ln(xs[r], D(t[p + "norm2.weight"]), D(t[p + "norm2.bias"]), 1e-5)
            xs[r] = xs[r] + W(p + "ff2.weight") @ q8round(gelu(W(p + "ff1.weight") @ q8round(h)))
    return ln(xs[-1], D(t["lm.out_norm.weight"]), D(t["lm.out_norm.bias"]), 1e-5)


@pytest.mark.parametrize("T", [1, 3, 5, 17])
def test_flowlm_text_against_numpy_model(T):
    """flowLM.text restated (T rows through the transformer, attend's T > 1
    products) follows the model: the output at the last token against an
    independent float64 numpy model within 2% RMS."""
    cfg = synth.FlowLMConfig(**SMALL)
    t = synth.flowlm_tensors(cfg, 0)
    om = orc.FlowLM(cfg, t)
    kv = voice_kv(cfg, 6, 1)
    st = om.stream(kv)
    ids = [(7 * i + 3) % cfg.text_vocab for i in range(T)]
    got = om.text(st, ids)
    assert st.pos == 6 + T
    want = _np_text(cfg, t, [(kv[l, 0], kv[l, 1]) for l in range(cfg.layers)], ids, 6)
    assert np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()) < 0.02


@pytest.mark.parametrize("n", [3, 20])
def test_flowlm_voice_latents_against_numpy_model(n):
    """The flow-LM half of CloneVoice (voice.go:94-106): [bos_voice;
    latents·speaker_projᵀ] through the transformer from an empty state. The
    last layer's cached values against an independent float64 model within
    2% RMS."""
    cfg = synth.FlowLMConfig(**SMALL)
    t = synth.flowlm_tensors(cfg, 0)
    om = orc.FlowLM(cfg, t)
    lat = np.random.default_rng(n).normal(0, 1, (n, cfg.ldim)).astype(np.float32)
    kv = om.voice_from_latents(lat)
    D = lambda a: np.asarray(a, np.float64)
    W = lambda name: D(synth.q8_dequant(t[name])) if isinstance(t[name], synth.Q8) else D(t[name])

    def q8round(x):
        out = np.empty_like(x)
        for b in range(0, x.size, 32):
            blk = x[b:b + 32]
            amax = np.abs(blk).max()
            out[b:b + 32] = np.rint(blk * 127 / amax) * amax / 127 if amax else 0
        return out

    ln = lambda x, w, b: (x - x.mean()) / np.sqrt(x.var() + 1e-5) * w + b
    hd = cfg.d // cfg.heads

    def rope(v, pos):
        f = np.exp(-np.log(cfg.max_period) * 2 / hd * np.arange(hd // 2))
        v = v.reshape(cfg.heads, hd // 2, 2).copy()
        r, i = v[..., 0].copy(), v[..., 1].copy()
        v[..., 0], v[..., 1] = r * np.cos(f * pos) - i * np.sin(f * pos), r * np.sin(f * pos) + i * np.cos(f * pos)
        return v.reshape(-1)

    gelu = lambda v: 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * v * (1 + 0.044715 * v * v)))
    xs = [D(t["lm.bos_voice"])] + list(D(lat) @ W("lm.speaker_proj").T)
    for l in range(cfg.layers):
        p = f"lm.blk.{l}."
        qs, K, V = [], [], []
        for r, x in enumerate(xs):
            qkv = W(p + "attn_qkv.weight") @ q8round(ln(x, D(t[p + "norm1.weight"]), D(t[p + "norm1.bias"])))
            qs.append(rope(qkv[:cfg.d], r))
            K.append(rope(qkv[cfg.d:2 * cfg.d], r))
            V.append(qkv[2 * cfg.d:])
        K, V = np.array(K), np.array(V)
        if l == cfg.layers - 1:
            got = kv[l, 1].astype(np.float64)
            assert np.sqrt(((got - V) ** 2).sum() / (V ** 2).sum()) < 0.02
        for r in range(len(xs)):
            att = np.zeros(cfg.d)
            for hh in range(cfg.heads):
                sl = slice(hh * hd, (hh + 1) * hd)
                s = K[:r + 1, sl] @ qs[r][sl] / np.sqrt(hd)
                e = np.exp(s - s.max())
                att[sl] = (e / e.sum()) @ V[:r + 1, sl]
            xs[r] = xs[r] + W(p + "attn_out.weight") @ q8round(att)
            h = ln(xs[r], D(t[p + "norm2.weight"]), D(t[p + "norm2.bias"]))
            xs[r] = xs[r] + W(p + "ff2.weight") @ q8round(gelu(W(p + "ff1.weight") @ q8round(h)))
