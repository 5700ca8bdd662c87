"""The Mimi decoder oracle (oracle/mimi.h) on the CPU: its ELU against the
definition, and whole frames against an independent float64 numpy decoder
written from the model (pockettts/mimi.go, nn.go), with the int8 path's
activation rounding wherever a weight is Q8_0."""

import numpy as np
import pytest

from gorelaxor_b200 import synth
from oracle import oracle as orc

LDIM = 32


def test_elu_matches_definition():
    """elu (nn.go:52-64): EXP8 lanes per 512-value chunk, Go's expf for each
    chunk's tail; within float32 rounding of x > 0 ? x : eˣ − 1."""
    x = np.random.default_rng(0).normal(0, 3, 1300).astype(np.float32)
    y = x.copy()
    orc.lib().orc_elu(orc.p(y), y.size)
    want = np.where(x > 0, x.astype(np.float64), np.expm1(x.astype(np.float64)))
    assert np.abs(y - want).max() <= 4e-7 * np.maximum(1, np.abs(want)).max()


def _np_decoder(mc, t):
    """A float64 streaming decoder: returns decode(latent) → frame."""
    D = lambda a: np.asarray(a, np.float64)
    isq = lambda name: isinstance(t[name], synth.Q8)
    W = lambda name: D(synth.q8_dequant(t[name])) if isq(name) else D(t[name])

    def q8round(x):
        out = np.empty_like(x)
        for b in range(0, x.size, 32):
            blk = x[b:b + 32]
            amax = np.abs(blk).max()
            out[b:b + 32] = np.rint(blk * 127 / amax) * amax / 127 if amax else 0
        return out

    def lin(name, x, bias=None):
        """x [rows][k] → [rows][n] with the weight named; rows rounded to Q8_0
        blocks first when the weight is Q8_0."""
        w = W(name)
        if isq(name):
            x = np.stack([q8round(r) for r in x])
        y = x @ w.T
        return y + D(bias) if bias is not None else y

    d, hd = mc.d, mc.d // mc.heads
    f = np.exp(-np.log(mc.max_period) * 2 / hd * np.arange(hd // 2))

    def rope(v, pos):
        v = v.reshape(mc.heads, hd // 2, 2).copy()
        r, i = v[..., 0].copy(), v[..., 1].copy()
        v[..., 0], v[..., 1] = r * np.cos(f * pos) - i * np.sin(f * pos), r * np.sin(f * pos) + i * np.cos(f * pos)
        return v.reshape(-1)

    ln = lambda x, w, b: (x - x.mean(-1, keepdims=True)) / np.sqrt(x.var(-1, keepdims=True) + 1e-5) * D(w) + D(b)
    gelu = lambda v: 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * v * (1 + 0.044715 * v * v)))
    elu = lambda v: np.where(v > 0, v, np.expm1(np.minimum(v, 0)))
    S = mc.upsample
    st = {"pos": 0, "up": np.zeros((S, d)), "K": [np.zeros((0, d))] * mc.layers, "V": [np.zeros((0, d))] * mc.layers,
          "prev": {}, "started": False}

    def conv(name, x, cin, cout, k, dil=1):
        P = (k - 1) * dil
        if k == 1:
            return lin(name + ".weight", x, t[name + ".bias"])
        prev = st["prev"].get(name, np.zeros((P, cin)))
        buf = np.vstack([prev, x])
        T = x.shape[0]
        col = np.stack([np.concatenate([buf[tt + j * dil] for j in range(k)]) for tt in range(T)])
        st["prev"][name] = buf[T:]
        return lin(name + ".weight", col, t[name + ".bias"])

    def convtr(name, x, cout, k, s):
        T = x.shape[0]
        z = lin(name + ".weight", x).reshape(T, k, cout)
        L = (T - 1) * s + k
        full = np.tile(D(t[name + ".bias"]), (L, 1))
        for tt in range(T):
            full[tt * s:tt * s + k] += z[tt]
        PT = k - s
        part = st["prev"].get(name, np.zeros((PT, cout)))
        full[:PT] += part
        st["prev"][name] = full[L - PT:] - D(t[name + ".bias"])
        return full[:T * s]

    def decode(lat):
        z = W("mimi.quant") @ D(lat)
        up = D(t["mimi.up"]).reshape(d, 2 * S)
        full = (z[:, None] * up).T  # [2S][d]
        full[:S] += st["up"]
        st["up"] = full[S:].copy()
        x = full[:S].copy()
        pos0 = st["pos"]
        for l in range(mc.layers):
            p = f"mimi.dec_tf.{l}."
            qkv = lin(p + "attn_qkv.weight", ln(x, t[p + "norm1.weight"], t[p + "norm1.bias"]))
            q = np.stack([rope(qkv[r, :d], pos0 + r) for r in range(S)])
            k = np.stack([rope(qkv[r, d:2 * d], pos0 + r) for r in range(S)])
            st["K"][l] = np.vstack([st["K"][l], k])
            st["V"][l] = np.vstack([st["V"][l], qkv[:, 2 * d:]])
            att = np.zeros((S, d))
            for r in range(S):
                pp = pos0 + r
                lo = max(0, pp - mc.context + 1)
                for h in range(mc.heads):
                    sl = slice(h * hd, (h + 1) * hd)
                    sc = st["K"][l][lo:pp + 1, sl] @ q[r, sl] / np.sqrt(hd)
                    e = np.exp(sc - sc.max())
                    att[r, sl] = (e / e.sum()) @ st["V"][l][lo:pp + 1, sl]
            x = x + D(t[p + "ls1"]) * lin(p + "attn_out.weight", att)
            hh = ln(x, t[p + "norm2.weight"], t[p + "norm2.bias"])
            x = x + D(t[p + "ls2"]) * lin(p + "ff2.weight", gelu(lin(p + "ff1.weight", hh)))
        st["pos"] += S
        mult = 1 << len(mc.ratios)
        x = conv("mimi.dec.0", x, d, mult * mc.nf, mc.k)
        idx = 1
        for r in mc.ratios:
            idx += 1
            x = convtr(f"mimi.dec.{idx}", elu(x), mult * mc.nf // 2, 2 * r, r)
            idx += 1
            dim = mult * mc.nf // 2
            for j in range(mc.nres):
                v = elu(x)
                hres = conv(f"mimi.dec.{idx}.1", v, dim, dim // mc.comp, mc.resk, mc.dil ** j)
                x = x + conv(f"mimi.dec.{idx}.3", elu(hres), dim // mc.comp, dim, 1)
                idx += 1
            mult //= 2
        idx += 1
        y = conv(f"mimi.dec.{idx}", elu(x), mc.nf, 1, mc.lastk)[:, 0]
        if not st["started"]:
            fade = mc.sample_rate // 200
            y[:fade] *= np.arange(fade) / (fade - 1)
            st["started"] = True
        return y

    return decode


@pytest.mark.parametrize("seed", [0, 1])
def test_mimi_decode_against_numpy_model(seed):
    """Six frames of the restated decoder (its streaming state carried from
    frame to frame) against the float64 model within 2% RMS per frame."""
    mc = synth.MimiConfig()
    t = synth.mimi_tensors(mc, LDIM, seed)
    om = orc.Mimi(mc, t, LDIM)
    st = om.state()
    dec = _np_decoder(mc, t)
    rng = np.random.default_rng(seed + 5)
    for f in range(6):
        lat = rng.normal(0, 1, LDIM).astype(np.float32)
        got = om.decode(st, lat)
        want = dec(lat)
        assert got.shape == want.shape == (mc.frame,)
        err = np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum())
        assert err < 0.02, f"frame {f}: {err:.4f}"


# The reference's model-free checks of the streaming pieces
# (pockettts/nn_test.go:37-153), restated on the oracle: a causal conv run
# in pieces equals the whole input convolved after zero padding of
# (k−1)·dil+1−stride; a transposed conv in pieces equals the whole output;
# windowed attention fed in pieces equals softmax attention over each
# query's window. Inputs are N(0,1) (the properties hold for any).


def _near(got, want, tol=1e-5):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= tol * (1 + np.abs(want)))


@pytest.mark.parametrize("cin,cout,k,stride,dil", [(3, 5, 3, 1, 1), (4, 2, 8, 4, 1), (2, 3, 3, 1, 2), (6, 4, 1, 1, 1)])
def test_conv_streaming(cin, cout, k, stride, dil):
    rng = np.random.default_rng(1)
    w = rng.normal(0, 1, (cout, k * cin)).astype(np.float32)  # [co][j][ci]
    b = rng.normal(0, 1, cout).astype(np.float32)
    T = 12 * stride
    x = rng.normal(0, 1, (T, cin)).astype(np.float32)
    P = (k - 1) * dil + 1 - stride
    pad = np.vstack([np.zeros((P, cin)), x.astype(np.float64)])
    want = np.array([[b[co] + sum(w[co, j * cin:(j + 1) * cin].astype(np.float64) @ pad[to * stride + j * dil]
                                  for j in range(k)) for co in range(cout)] for to in range(T // stride)])
    prev = np.zeros(max(P, 1) * cin, np.float32)
    got, a = [], 0
    for n in (2, 1, 5, 4):  # pieces, in strides
        piece = np.ascontiguousarray(x[a * stride:(a + n) * stride])
        y = np.empty((n, cout), np.float32)
        orc.lib().orc_mimi_conv_run(orc.p(w), orc.p(b), cin, cout, k, stride, dil, orc.p(prev), orc.p(piece),
                                    n * stride, orc.p(y))
        got.append(y)
        a += n
    _near(np.vstack(got), want)


def test_convtr_streaming():
    rng = np.random.default_rng(3)
    cin, cout, k, S, T = 3, 2, 8, 4, 9
    w = rng.normal(0, 1, (k * cout, cin)).astype(np.float32)  # [j][co][ci]
    b = rng.normal(0, 1, cout).astype(np.float32)
    x = rng.normal(0, 1, (T, cin)).astype(np.float32)
    full = np.tile(b.astype(np.float64), ((T - 1) * S + k, 1))
    for ti in range(T):
        full[ti * S:ti * S + k] += (w.astype(np.float64) @ x[ti]).reshape(k, cout)
    part = np.zeros((k - S) * cout, np.float32)
    got, start = [], 0
    for n in (4, 1, 4):
        piece = np.ascontiguousarray(x[start:start + n])
        y = np.empty((n * S, cout), np.float32)
        orc.lib().orc_mimi_convtr_run(orc.p(w), orc.p(b), cin, cout, k, S, orc.p(part), orc.p(piece), n, orc.p(y))
        got.append(y)
        start += n
    _near(np.vstack(got), full[:T * S])


def test_attend_window():
    rng = np.random.default_rng(5)
    d, heads, ctx, T = 8, 2, 5, 13
    hd = d // heads
    qkv = rng.normal(0, 1, (T, 3 * d)).astype(np.float32)
    want = np.zeros((T, d))
    for p_ in range(T):
        lo = max(0, p_ - ctx + 1)
        for h in range(heads):
            s = slice(h * hd, (h + 1) * hd)
            sc = np.array([qkv[p_, s].astype(np.float64) @ qkv[j, d:2 * d][s] for j in range(lo, p_ + 1)])
            e = np.exp(sc / np.sqrt(hd))
            want[p_, s] = (e / e.sum()) @ qkv[lo:p_ + 1, 2 * d:][:, s]
    kc = np.ascontiguousarray(qkv[:, d:2 * d])
    vc = np.ascontiguousarray(qkv[:, 2 * d:])
    got, pos = [], 0
    for n in (1, 6, 1, 5):
        out = np.empty((n, d), np.float32)
        part = np.ascontiguousarray(qkv[pos:pos + n])
        orc.lib().orc_attend_window(orc.p(out), orc.p(part), n, orc.p(kc), orc.p(vc), pos, d, heads, ctx)
        got.append(out)
        pos += n
    _near(np.vstack(got), want)


def _np_clone_latents(mc, t, x, ldim):
    """A float64 Mimi encoder (SEANet encoder, windowed layer-scaled
    transformer, the downsampling conv with its first row replicated) over
    the whole clip at once — what the streaming encoder computes piece by
    piece — with the int8 path's activation rounding where a weight is Q8_0."""
    D = lambda a: np.asarray(a, np.float64)
    isq = lambda name: isinstance(t[name], synth.Q8)
    W = lambda name: D(synth.q8_dequant(t[name])) if isq(name) else D(t[name])

    def q8round(v):
        out = np.empty_like(v)
        for b in range(0, v.size, 32):
            blk = v[b:b + 32]
            amax = np.abs(blk).max()
            out[b:b + 32] = np.rint(blk * 127 / amax) * amax / 127 if amax else 0
        return out

    def lin(name, v, bias=None):
        if isq(name):
            v = np.stack([q8round(r) for r in v])
        y = v @ W(name).T
        return y + D(bias) if bias is not None else y

    elu = lambda v: np.where(v > 0, v, np.expm1(np.minimum(v, 0)))

    def conv(name, v, k, stride=1, dil=1, pad_rows=None, wname=None):
        P = (k - 1) * dil + 1 - stride
        pre = np.zeros((P, v.shape[1])) if pad_rows is None else pad_rows
        buf = np.vstack([pre, v])
        To = v.shape[0] // stride
        col = np.stack([np.concatenate([buf[tt * stride + j * dil] for j in range(k)]) for tt in range(To)])
        b = t.get(name + ".bias")
        return lin(wname or name + ".weight", col, b)

    frame = mc.frame
    x = np.concatenate([D(x), np.zeros((frame - len(x) % frame) % frame)])[:, None]
    x = conv("mimi.enc.0", x, mc.k)
    idx, mult = 1, 1
    for r in reversed(mc.ratios):
        for j in range(mc.nres):
            h = conv(f"mimi.enc.{idx}.1", elu(x), mc.resk, 1, mc.dil ** j)
            x = x + conv(f"mimi.enc.{idx}.3", elu(h), 1)
            idx += 1
        idx += 1
        x = conv(f"mimi.enc.{idx}", elu(x), 2 * r, r)
        idx += 1
        mult *= 2
    idx += 1
    x = conv(f"mimi.enc.{idx}", elu(x), mc.lastk)
    d, hd = mc.d, mc.d // mc.heads
    f = np.exp(-np.log(mc.max_period) * 2 / hd * np.arange(hd // 2))

    def rope(v, pos):
        v = v.reshape(mc.heads, hd // 2, 2).copy()
        r_, i_ = v[..., 0].copy(), v[..., 1].copy()
        v[..., 0], v[..., 1] = r_ * np.cos(f * pos) - i_ * np.sin(f * pos), r_ * np.sin(f * pos) + i_ * np.cos(f * pos)
        return v.reshape(-1)

    ln = lambda v, w, b: (v - v.mean(-1, keepdims=True)) / np.sqrt(v.var(-1, keepdims=True) + 1e-5) * D(w) + D(b)
    gelu = lambda v: 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * v * (1 + 0.044715 * v * v)))
    T = x.shape[0]
    for l in range(mc.layers):
        p = f"mimi.enc_tf.{l}."
        qkv = lin(p + "attn_qkv.weight", ln(x, t[p + "norm1.weight"], t[p + "norm1.bias"]))
        q = np.stack([rope(qkv[r, :d], r) for r in range(T)])
        k = np.stack([rope(qkv[r, d:2 * d], r) for r in range(T)])
        v = qkv[:, 2 * d:]
        att = np.zeros((T, d))
        for r in range(T):
            lo = max(0, r - mc.context + 1)
            for h in range(mc.heads):
                s = slice(h * hd, (h + 1) * hd)
                sc = k[lo:r + 1, s] @ q[r, s] / np.sqrt(hd)
                e = np.exp(sc - sc.max())
                att[r, s] = (e / e.sum()) @ v[lo:r + 1, s]
        x = x + D(t[p + "ls1"]) * lin(p + "attn_out.weight", att)
        hh = ln(x, t[p + "norm2.weight"], t[p + "norm2.bias"])
        x = x + D(t[p + "ls2"]) * lin(p + "ff2.weight", gelu(lin(p + "ff1.weight", hh)))
    up = mc.upsample
    return conv("mimi.down", x, 2 * up, up, 1, pad_rows=np.repeat(x[:1], up, axis=0), wname="mimi.down")


@pytest.mark.parametrize("n", [1000, 1234])
def test_mimi_clone_latents_against_numpy_model(n):
    """cloneCond's Mimi encoding (voice.go:113-124, mimi.go:164-179) of a
    clip padded to whole frames and encoded twelve frames at a time, against
    the float64 encoder over the whole clip: within 2% relative RMS."""
    mc = synth.MimiConfig()
    t = synth.mimi_tensors(mc, LDIM, 2, encoder=True)
    om = orc.Mimi(mc, t, LDIM)
    x = np.random.default_rng(n).normal(0, 0.3, n).astype(np.float32)
    got = om.clone_latents(x)
    want = _np_clone_latents(mc, t, x, LDIM)
    assert got.shape == want.shape == (-(-n // mc.frame), LDIM)
    err = np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum())
    assert err < 0.02, err
