"""GPU parity of the persistent one-stream Whisper kernel (k_whisper.cu
k_wstep1): a batch of one stream runs grx_whisper_run's whole token loop —
process/sample (transcribe.go:370-494) and the decode of the sampled token
(decoder.go:33-140) — in one cooperative launch. Token ids and timestamps
identical to the oracle's greedy loop, p and plog within the 1e-3 tolerance
the spec states for float outputs (their vocabulary sums are reduced over
the grid in another order), and the logits after the run bit-identical to
the per-kernel path's (GRX_WSTEP1=0)."""

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from tests.helpers import mismatch
from tests.test_gpu_whisper import SMALL_W, _check_tokens, _enc, _models, _prompt

pytestmark = pytest.mark.gpu


def _batch(gm, enc, prompt, sot_at):
    b = g.WhisperBatch(gm, 1)
    b.set_audio(enc)
    b.prompt(prompt, sot_at)
    return b


def test_persistent_chosen_for_one_stream(have_gpu, monkeypatch):
    cfg = synth.WhisperConfig(**SMALL_W)
    gm, _ = _models(cfg)
    assert g.WhisperBatch(gm, 1).persistent()
    assert not g.WhisperBatch(gm, 2).persistent()
    monkeypatch.setenv("GRX_WSTEP1", "0")
    assert not g.WhisperBatch(gm, 1).persistent()


@pytest.mark.parametrize("f16", [False, True])
def test_persistent_greedy_matches_oracle(have_gpu, f16):
    """Prompt, then 40 greedy steps in runs of 1, 15 and 24 steps (the run's
    output buffer grows between them)."""
    cfg = synth.WhisperConfig(**SMALL_W)
    gm, om = _models(cfg, seed=3, f16=f16)
    enc = _enc(cfg, 1, seed0=5)
    prompt, sot_at = _prompt(gm)
    b = _batch(gm, enc, prompt, sot_at)
    assert b.persistent()
    toks = np.concatenate([b.run(k) for k in (1, 15, 24)])
    want, _ = om.greedy(om.seq(enc[0]), prompt, sot_at, 40)
    _check_tokens(toks[:, 0], want)
    assert b.launches() > 0


def test_persistent_matches_per_kernel_path(have_gpu, monkeypatch):
    """The base.en shape (state 512, 8 heads, 6 layers, vocab 51864): the
    persistent kernel and the per-kernel graph path give the same ids and
    timestamps and bit-identical logits after 12 steps, the persistent one
    in a launch per run."""
    cfg = synth.WhisperConfig()
    gm, om = _models(cfg, seed=4)
    enc = _enc(cfg, 1, seed0=9)
    prompt, sot_at = _prompt(gm)
    a = _batch(gm, enc, prompt, sot_at)
    assert a.persistent()
    l0 = a.launches()
    ta = a.run(12)
    assert a.launches() - l0 == 1
    monkeypatch.setenv("GRX_WSTEP1", "0")
    b = _batch(gm, enc, prompt, sot_at)
    assert not b.persistent()
    tb = b.run(12)
    assert np.array_equal(ta[:, 0, :2], tb[:, 0, :2])
    ne, rel = mismatch(a.logits()[0], b.logits()[0])
    assert ne == 0, f"{ne} logits differ (max rel {rel:.2e})"
    want, _ = om.greedy(om.seq(enc[0]), prompt, sot_at, 12)
    _check_tokens(ta[:, 0], want)


def test_persistent_device_run_and_sync(have_gpu):
    """run_device then sync: the tokens land in device memory as run gives
    them."""
    import torch

    cfg = synth.WhisperConfig(**SMALL_W)
    gm, om = _models(cfg, seed=6)
    enc = _enc(cfg, 1, seed0=13)
    prompt, sot_at = _prompt(gm)
    b = _batch(gm, enc, prompt, sot_at)
    d = torch.zeros((10, 1, 4), dtype=torch.int32, device="cuda")
    b.run_device(10, d.data_ptr())
    b.sync()
    want, _ = om.greedy(om.seq(enc[0]), prompt, sot_at, 10)
    _check_tokens(d.cpu().numpy()[:, 0], want)


def test_persistent_watchdog_reports_and_recovers(have_gpu):
    """A step whose first grid barrier nothing completes: every block gives
    up after its one-second limit and the call returns GRX_ETIMEDOUT (-7);
    after the window and prompt are set again the batch decodes correctly on
    the same context."""
    cfg = synth.WhisperConfig(**SMALL_W)
    gm, om = _models(cfg, seed=8)
    enc = _enc(cfg, 1, seed0=17)
    prompt, sot_at = _prompt(gm)
    b = _batch(gm, enc, prompt, sot_at)
    assert b.watchdog_test() == -7
    assert "one-second limit" in g.last_error()
    b.set_audio(enc)
    b.prompt(prompt, sot_at)
    toks = b.run(8)
    want, _ = om.greedy(om.seq(enc[0]), prompt, sot_at, 8)
    _check_tokens(toks[:, 0], want)


def test_persistent_watchdog_rejects_other_batches(have_gpu):
    """GRX_EINVAL (-1) for a batch without a prompt decoded and for one of
    two streams (the per-kernel path)."""
    cfg = synth.WhisperConfig(**SMALL_W)
    gm, _ = _models(cfg)
    assert g.WhisperBatch(gm, 1).watchdog_test() == -1
    assert g.WhisperBatch(gm, 2).watchdog_test() == -1
