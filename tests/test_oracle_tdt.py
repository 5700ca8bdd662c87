"""The TDT oracle (oracle/tdt.h) against an independent float64 numpy
statement of the same decoder (conformer/rnnt.go), CPU only: the loop's
control flow (frame skipping, max_symbols, the state swap) must give the same
tokens; the float32 arithmetic differs from float64 by far less than the
gaps between the argmax winners on these seeds."""

import numpy as np
import pytest

from gorelaxor_b200 import synth
from oracle import oracle as orc

SMALL_TDT = dict(H=128, V=65, J=96, D=128)


def _np_decode(cfg, t, enc):
    W = {k: (synth.q8_dequant(v) if isinstance(v, synth.Q8) else v).astype(np.float64) for k, v in t.items()}
    H, L, V = cfg.H, cfg.layers, cfg.V
    sig = lambda x: 1 / (1 + np.exp(-x))
    act = {"relu": lambda v: np.maximum(v, 0), "sigmoid": sig, "tanh": np.tanh}[cfg.act]
    cur = [np.zeros((L, H)), np.zeros((L, H)), -1]
    # Linear of T >= 2 rows takes the int8 path: the rows are first rounded
    # to Q8_0 blocks (q8int.go:88-105), amax/127 steps, to nearest.
    blk = enc.reshape(enc.shape[0], -1, 32).astype(np.float32)
    amax = np.abs(blk).max(axis=2, keepdims=True)
    q = np.clip(np.rint(blk * (np.float32(127) / np.where(amax > 0, amax, 1))), -127, 127)
    encq = (q.astype(np.float64) * (amax.astype(np.float64) / 127)).reshape(enc.shape)
    enc_proj = encq @ W["joint.enc.weight"].T + W["joint.enc.bias"]

    def predict(st):
        x = W["pred.embed.weight"][st[2]] if st[2] >= 0 and st[2] != cfg.blank else np.zeros(H)
        h, c = np.zeros((L, H)), np.zeros((L, H))
        for l in range(L):
            gt = W[f"pred.lstm.{l}.Wx"] @ x + W[f"pred.lstm.{l}.bias"] + W[f"pred.lstm.{l}.Wh"] @ st[0][l]
            i, f, gg, o = sig(gt[:H]), sig(gt[H:2 * H]), np.tanh(gt[2 * H:3 * H]), sig(gt[3 * H:])
            c[l] = f * st[1][l] + i * gg
            h[l] = o * np.tanh(c[l])
            x = h[l]
        return [h, c, st[2]], x

    out, step, nsym, T, dirty = [], 0, 0, enc.shape[0], True
    tdt = cfg.head == "tdt"
    for _ in range(16 * T + 1024):
        if step >= T:
            break
        if dirty:
            nxt, pred = predict(cur)
            dirty = False
        hidden = act(enc_proj[step] + W["joint.pred.weight"] @ pred + W["joint.pred.bias"])
        lg = W["joint.out.weight"] @ hidden + W["joint.out.bias"]
        tok = int(np.argmax(lg[:V]))
        dur = cfg.durations[int(np.argmax(lg[V:V + len(cfg.durations)]))] if tdt else 1
        if tok != cfg.blank:
            out.append((tok, step, dur))
            nxt[2] = tok
            cur = nxt
            dirty = True
        if not tdt:
            if tok == cfg.blank:
                step, nsym = step + 1, 0
            else:
                nsym += 1
                if nsym >= cfg.max_symbols:
                    step, nsym = step + 1, 0
            continue
        step += dur
        nsym += 1
        if dur != 0:
            nsym = 0
        elif nsym >= cfg.max_symbols:
            step, nsym = step + 1, 0
    return out


@pytest.mark.parametrize("head,seed", [("tdt", 1), ("tdt", 2), ("rnnt", 3)])
def test_tdt_oracle_matches_float64_model(head, seed):
    cfg = synth.TDTConfig(**SMALL_TDT, head=head)
    t = synth.tdt_tensors(cfg, seed)
    enc = synth.encoder_frames(seed, 30, cfg.D)
    toks, iters, preds = orc.TDT(cfg, t).decode(enc)
    want = _np_decode(cfg, t, enc)
    assert [tuple(x[:3]) for x in toks.tolist()] == want
    assert len(want) > 0 and iters > len(want)  # both blanks and tokens


def test_tdt_oracle_probability_and_max_symbols():
    """p = softmax of the winning token (rnnt.go:80-89) and no frame emits
    more than max_symbols tokens of duration 0 in a row."""
    cfg = synth.TDTConfig(**SMALL_TDT, blank_lift=0.2, max_symbols=3)
    t = synth.tdt_tensors(cfg, 4)
    toks, _, _ = orc.TDT(cfg, t).decode(synth.encoder_frames(4, 30, cfg.D))
    p = toks[:, 3].copy().view(np.float32)
    assert ((p > 0) & (p <= 1)).all()
    run, prev = 0, None
    for tok, frame, dur, _ in toks.tolist():
        run = run + 1 if frame == prev else 1
        prev = frame
        assert run <= cfg.max_symbols
