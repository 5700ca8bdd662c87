"""GPU parity for the FastConformer encoder: grx_fconf_encode through the C
ABI against the oracle's Model.encode (oracle/conformer.h, restating
conformer/encoder.go:123-489), bit for bit, on a small encoder of Parakeet's
shape rules: utterances that fill whole query blocks and ragged ones, short
ones whose attention takes gemvRows only, and padded ones (valid < frames)."""

import numpy as np
import pytest

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from oracle import oracle as orc
from tests.helpers import mismatch

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.mark.parametrize("frames,valid", [(200, 200), (203, 150), (70, 70), (600, 600), (600, 411)])
def test_fconf_encode_bit_exact(have_gpu, frames, valid):
    fc = synth.FConfConfig()
    t = synth.fconf_tensors(fc, 0)
    gm = g.FConf(synth.fconf_gguf(fc, t))
    assert (gm.d, gm.heads, gm.layers, gm.n_mels) == (fc.d, fc.heads, fc.layers, fc.n_mels)
    mel = synth.fconf_mel(frames + valid, fc.n_mels, frames)
    got = gm.encode(mel, valid)
    want = orc.FConf(fc, t).encode(mel, valid)
    assert got.shape == want.shape
    ne, rel = mismatch(got, want)
    assert ne == 0, f"{ne} of {got.size} differ (max rel {rel:.2e})"
    assert rel <= TOL


def test_fconf_layer_norm_conv_and_device_run(have_gpu):
    """The conv module normalizing with layer norm; the device-resident call
    gives the host call's rows."""
    import torch

    fc = synth.FConfConfig(conv_norm="layer_norm", xscaling=False)
    t = synth.fconf_tensors(fc, 3)
    gm = g.FConf(synth.fconf_gguf(fc, t))
    mel = synth.fconf_mel(9, fc.n_mels, 160)
    got = gm.encode(mel)
    want = orc.FConf(fc, t).encode(mel)
    ne, rel = mismatch(got, want)
    assert ne == 0, f"{ne} of {got.size} differ (max rel {rel:.2e})"
    dm = torch.from_numpy(mel).cuda()
    dout = torch.empty((want.shape[0], fc.d), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    rows = gm.encode_device(dm.data_ptr(), mel.shape[1], mel.shape[1], dout.data_ptr())
    gm.sync()
    assert rows == want.shape[0]
    ne, _ = mismatch(dout.cpu().numpy(), want)
    assert ne == 0


def test_fconf_rejects_streaming_models(have_gpu):
    fc = synth.FConfConfig()
    t = synth.fconf_tensors(fc, 0)
    with pytest.raises(g.GrxError, match="EINVAL"):
        g.FConf(synth.fconf_gguf(fc, t, style="chunked_limited"))
