"""The FastConformer encoder oracle (oracle/conformer.h, restating
conformer/encoder.go:41-489) against an independent float64 numpy encoder
written from the model, with the int8 path's activation rounding wherever
the reference multiplies by a Q8_0 weight (every linear layer: the loader
packs them and drops their rows, and rounds the float16 1×1 convolutions
to Q8_0)."""

import numpy as np
import pytest

from gorelaxor_b200 import synth
from oracle import oracle as orc


def _q8round(x):
    out = np.empty_like(x)
    flat, o = x.reshape(-1, 32), out.reshape(-1, 32)
    amax = np.abs(flat).max(1, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        o[:] = np.where(amax > 0, np.rint(flat * 127 / amax) * amax / 127, 0)
    return out


def _np_encode(fc, t, mel, valid):
    D = lambda a: np.asarray(a, np.float64)

    def W(name):
        a = t[name]
        if isinstance(a, synth.Q8):
            return D(synth.q8_dequant(a))
        v = D(a.astype(np.float32))  # float16 1×1 convolutions: ToQ8 at load
        blk = v.reshape(v.shape[0], -1, 32)
        dq = (np.abs(blk).max(2, keepdims=True) / 127).astype(np.float32).astype(np.float16).astype(np.float64)
        with np.errstate(invalid="ignore", divide="ignore"):
            q = np.where(dq > 0, np.round(blk / dq), 0)
        return (q * dq).reshape(v.shape)

    def lin(x, name, bias=None):
        y = _q8round(x) @ W(name).T
        return y + D(t[bias]) if bias else y

    def ln(x, p):
        m = x.mean(-1, keepdims=True)
        return (x - m) / np.sqrt(((x - m) ** 2).mean(-1, keepdims=True) + 1e-5) * D(t[p + ".weight"]) + D(t[p + ".bias"])

    silu = lambda v: v / (1 + np.exp(-v))
    sub = lambda n: (n - 1) // 2 + 1
    c, d, H = fc.sub_c, fc.d, fc.heads
    pe = "enc.pre_encode."
    frames = mel.shape[1]
    x = np.zeros((frames, fc.n_mels))
    x[:valid] = D(mel[:, :valid]).T
    L = valid

    def conv(x, w, b, depthwise):
        T, F = x.shape[:2]
        T1, F1 = sub(T), sub(F)
        xp = np.pad(x, ((1, 2), (1, 2)) + (((0, 0),) if depthwise else ()))
        w = D(t[w]).reshape(c, 9)
        out = np.tile(D(t[b]), (T1, F1, 1))
        for kt in range(3):
            for kf in range(3):
                tap = xp[kt:kt + 2 * T1:2, kf:kf + 2 * F1:2]
                out += (tap if depthwise else tap[..., None]) * w[:, kt * 3 + kf]
        return out

    def mask(x, L):
        x[L:] = 0
        return x

    x = conv(x, pe + "conv.0.weight", pe + "conv.0.bias", False)
    L = sub(L)
    x = np.maximum(mask(x, L), 0)
    x = mask(conv(x, pe + "conv.2.weight", pe + "conv.2.bias", True), sub(L))
    L = sub(L)
    T, F = x.shape[:2]
    x = np.maximum(mask(lin(x.reshape(-1, c), pe + "conv.3.weight", pe + "conv.3.bias").reshape(T, F, c), L), 0)
    x = mask(conv(x, pe + "conv.5.weight", pe + "conv.5.bias", True), sub(L))
    L = sub(L)
    T, F = x.shape[:2]
    x = np.maximum(mask(lin(x.reshape(-1, c), pe + "conv.6.weight", pe + "conv.6.bias").reshape(T, F, c), L), 0)
    x = lin(x.transpose(0, 2, 1).reshape(T, c * F), pe + "out.weight", pe + "out.bias")
    if fc.xscaling:
        x = x * np.sqrt(d)
    hd = d // H
    i = np.arange(2 * T - 1)
    pos = (T - 1 - i)[:, None] * np.exp(np.arange(0, d, 2) * -(np.log(10000) / d))[None]
    pe_tab = np.zeros((2 * T - 1, d))
    pe_tab[:, 0::2], pe_tab[:, 1::2] = np.sin(pos), np.cos(pos)
    for li in range(fc.layers):
        p = f"enc.blocks.{li}."

        def ff(x, n):
            h = silu(lin(ln(x, p + "norm_" + n), f"{p}{n}.linear1.weight", f"{p}{n}.linear1.bias"))
            return x + 0.5 * lin(h, f"{p}{n}.linear2.weight", f"{p}{n}.linear2.bias")

        x = ff(x, "ff1")
        h = ln(x, p + "norm_attn")
        q = lin(h, p + "attn.linear_q.weight", p + "attn.linear_q.bias")
        k = lin(h, p + "attn.linear_k.weight", p + "attn.linear_k.bias")
        v = lin(h, p + "attn.linear_v.weight", p + "attn.linear_v.bias")
        pp = lin(pe_tab, p + "attn.linear_pos.weight")
        att = np.zeros((T, d))
        for hh in range(H):
            s = slice(hh * hd, (hh + 1) * hd)
            qu = q[:, s] + D(t[p + "attn.pos_bias_u"]).reshape(-1)[s]
            qv = q[:, s] + D(t[p + "attn.pos_bias_v"]).reshape(-1)[s]
            ac = qu @ k[:, s].T
            bd_full = qv @ pp[:, s].T  # [T][2T−1], column j is relative position T−1−j
            bd = np.stack([bd_full[r, T - 1 - r:2 * T - 1 - r] for r in range(T)])
            sc = (ac + bd) / np.sqrt(hd)
            sc[:, L:] = -np.inf
            e = np.exp(sc - sc.max(1, keepdims=True))
            w = e / e.sum(1, keepdims=True)
            w[L:] = 0
            att[:, s] = w @ v[:, s]
        x = x + lin(att, p + "attn.linear_out.weight", p + "attn.linear_out.bias")
        h = lin(ln(x, p + "norm_conv"), p + "conv.pointwise1.weight", p + "conv.pointwise1.bias")
        g = h[:, :d] / (1 + np.exp(-h[:, d:]))
        g[L:] = 0
        K = fc.kernel
        gp = np.pad(g, (((K - 1) // 2, K // 2), (0, 0)))
        wdw = D(t[p + "conv.depthwise.weight"]).reshape(d, K)
        dw = D(t[p + "conv.depthwise.bias"]) + sum(gp[j:j + T] * wdw[:, j] for j in range(K))
        bw, bb = D(t[p + "conv.bn.weight"]), D(t[p + "conv.bn.bias"])
        mean, var = D(t[p + "conv.bn.running_mean"]), D(t[p + "conv.bn.running_var"])
        dw = (dw - mean) / np.sqrt(var + 1e-5) * bw + bb
        x = x + lin(silu(dw), p + "conv.pointwise2.weight", p + "conv.pointwise2.bias")
        x = ln(ff(x, "ff2"), p + "norm_out")
    return x[:L]


@pytest.mark.parametrize("frames,valid", [(200, 200), (203, 150)])
def test_fconf_encode_against_numpy_model(frames, valid):
    """One utterance (and one with padding frames) through the restated
    encoder against the float64 model: within 2% relative RMS (the int8
    path's rounding of activations bounds the agreement)."""
    fc = synth.FConfConfig()
    t = synth.fconf_tensors(fc, 0)
    oc = orc.FConf(fc, t)
    mel = synth.fconf_mel(1, fc.n_mels, frames)
    got = oc.encode(mel, valid)
    want = _np_encode(fc, t, mel, valid)
    assert got.shape == want.shape
    err = np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum())
    assert err < 0.02, err
