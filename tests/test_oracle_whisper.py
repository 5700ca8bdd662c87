"""The Whisper oracle (oracle/whisper.h) on the CPU: its products against
float64, its decode against an independent float64 numpy decoder, and
process/sample against the rules of transcribe.go:370-494 on crafted logits."""

import numpy as np
import pytest

from gorelaxor_b200 import synth
from oracle import oracle as orc

SMALL_W = dict(n_state=128, n_head=2, n_text_layer=2, n_text_ctx=64)


def _f16(bits):
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float64)


@pytest.mark.parametrize("m", [1, 5, 6, 13])
def test_matmul_orders_match_float64(m):
    """Fewer than 6 rows: gemv per row; 6 or more: the packed kernel with
    256-deep passes; rows past the last multiple of 6 by gemv again."""
    rng = np.random.default_rng(m)
    n, k = 40, 600
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = rng.normal(0, 0.05, (n, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32)
    c = np.empty((m, n), np.float32)
    L = orc.lib()
    L.orc_whisper_matmul(orc.p(c), orc.p(a), m, n, k, 0, orc.p(w), orc.p(bias))
    want = a.astype(np.float64) @ w.T.astype(np.float64) + bias
    assert np.max(np.abs(c - want)) <= 1e-5 * np.max(np.abs(want))


def _np_decode(cfg, t, enc, prompt):
    """float64 decoder (decoder.go) on the f16-widened weights; returns the
    logits of the prompt's last row."""
    W = {}
    for k, v in t.items():
        W[k] = _f16(orc.q8_to_f16(v)) if isinstance(v, synth.Q8) else v.astype(np.float64)
    st, nh = cfg.n_state, cfg.n_head
    hd = st // nh

    def ln(x, w, b):
        mu = x.mean(-1, keepdims=True)
        return (x - mu) / np.sqrt(((x - mu) ** 2).mean(-1, keepdims=True) + 1e-5) * w + b

    def gelu(v):
        return 0.5 * v * (1 + np.tanh(0.7978845608028654 * v * (1 + 0.044715 * v * v)))

    def sm(x):
        e = np.exp(x - x.max(-1, keepdims=True))
        return e / e.sum(-1, keepdims=True)

    enc = enc.astype(np.float64)
    nt = len(prompt)
    x = W["decoder.token_embedding.weight"][prompt] + W["decoder.positional_embedding"][:nt]
    mask = np.triu(np.full((nt, nt), -np.inf), 1)
    for i in range(cfg.n_text_layer):
        p = f"decoder.blocks.{i}."
        c = ln(x, W[p + "attn_ln.weight"], W[p + "attn_ln.bias"])
        q = c @ W[p + "attn.query.weight"].T + W[p + "attn.query.bias"]
        k = c @ W[p + "attn.key.weight"].T
        v = c @ W[p + "attn.value.weight"].T + W[p + "attn.value.bias"]
        o = np.concatenate([sm(q[:, h * hd:(h + 1) * hd] @ k[:, h * hd:(h + 1) * hd].T / np.sqrt(hd) + mask)
                            @ v[:, h * hd:(h + 1) * hd] for h in range(nh)], axis=1)
        x = x + o @ W[p + "attn.out.weight"].T + W[p + "attn.out.bias"]
        c = ln(x, W[p + "cross_attn_ln.weight"], W[p + "cross_attn_ln.bias"])
        q = c @ W[p + "cross_attn.query.weight"].T + W[p + "cross_attn.query.bias"]
        k = enc @ W[p + "cross_attn.key.weight"].T
        v = enc @ W[p + "cross_attn.value.weight"].T + W[p + "cross_attn.value.bias"]
        o = np.concatenate([sm(q[:, h * hd:(h + 1) * hd] @ k[:, h * hd:(h + 1) * hd].T / np.sqrt(hd))
                            @ v[:, h * hd:(h + 1) * hd] for h in range(nh)], axis=1)
        x = x + o @ W[p + "cross_attn.out.weight"].T + W[p + "cross_attn.out.bias"]
        c = ln(x, W[p + "mlp_ln.weight"], W[p + "mlp_ln.bias"])
        f = gelu(c @ W[p + "mlp.0.weight"].T + W[p + "mlp.0.bias"])
        x = x + f @ W[p + "mlp.2.weight"].T + W[p + "mlp.2.bias"]
    return ln(x[-1], W["decoder.ln.weight"], W["decoder.ln.bias"]) @ W["decoder.token_embedding.weight"].T


def test_decode_matches_float64_model():
    cfg = synth.WhisperConfig(**SMALL_W)
    t = synth.whisper_tensors(cfg, 0)
    om = orc.Whisper(cfg, t, synth.whisper_words(cfg))
    enc = synth.whisper_encoder_out(1, cfg)
    prompt = [50360, 100, 200, 50257]
    got = om.decode(om.seq(enc), prompt, [3])[0]
    want = _np_decode(cfg, t, enc, prompt)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err < 2e-3, err


def _om():
    cfg = synth.WhisperConfig(**SMALL_W)
    return orc.Whisper(cfg, synth.whisper_tensors(cfg, 0), synth.whisper_words(cfg))


def test_process_initial_rules():
    """Initially eot, " " and the timestamps past 1 s are out; the special
    and suppressed tokens always (transcribe.go:378-408)."""
    om = _om()
    V, beg = 51864, 50363
    lg = np.zeros(V, np.float32)
    lg[50256] = 50.0  # eot
    lg[220] = 40.0  # " "
    lg[12] = 30.0  # "(" (suppressed)
    lg[beg + 51] = 20.0  # timestamp past 1 s
    lg[777] = 10.0
    tid, ts, p, plog = om.process_sample((0, -1, -1, 0, 3000), lg)
    assert tid == 777
    assert lg[50256] == -np.inf and lg[220] == -np.inf and lg[12] == -np.inf and lg[beg + 51] == -np.inf
    assert lg[beg + 50] == 0.0 and np.isfinite(plog) and 0 < p <= 1


def test_process_timestamp_pairs():
    """After a timestamp preceded by text only text or eot may follow; after
    two timestamps only text (transcribe.go:396-407); timestamps before the
    last one's delta are out once one was seen."""
    om = _om()
    V, beg, eot = 51864, 50363, 50256
    lg = np.zeros(V, np.float32)
    lg[beg + 100] = 30.0
    lg[500] = 10.0
    lg[eot] = 5.0
    # last = timestamp, penult = text: text (< eot) is out
    out = lg.copy()
    tid, *_ = om.process_sample((2, beg + 10, 300, 1, 20), out)
    assert np.all(out[:eot] == -np.inf) and tid == beg + 100
    # last two timestamps: every timestamp is out
    out = lg.copy()
    tid, *_ = om.process_sample((2, beg + 10, beg + 5, 1, 20), out)
    assert np.all(out[beg:] == -np.inf) and tid == 500
    # has_ts with seek_delta 400: timestamps below beg + 200 are out
    out = lg.copy()
    om.process_sample((1, 300, -1, 1, 400), out)
    assert np.all(out[beg:beg + 200] == -np.inf) and out[beg + 200] == 0.0


def test_process_timestamp_mass_wins():
    """When the timestamps' total log-probability beats every text token,
    text is masked and a timestamp is sampled (transcribe.go:414-434)."""
    om = _om()
    V, beg = 51864, 50363
    lg = np.full(V, -10.0, np.float32)
    lg[beg:beg + 50] = 2.0  # 50 timestamps at 2.0 outweigh
    lg[600] = 4.0  # one text token at 4.0
    tid, ts, p, plog = om.process_sample((1, 300, -1, 0, 3000), lg)
    assert beg <= tid < beg + 50 and ts == tid
    assert np.all(lg[:beg] == -np.inf)
