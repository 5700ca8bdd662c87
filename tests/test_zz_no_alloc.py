"""grx_linear_q8_static, the entry point for callers that cannot allocate
GPU memory (a pool allocator owns the device, or a real-time loop must not
stall it), against grx_linear, the allocating entry point, through the C
ABI. The bar of the other parity tests holds: identical float32 bits.

The calls run back to back and share the library's fixed scratch array,
so the second and third see what the earlier ones left there. The file is
named to be collected last; it also passes alone in a fresh process (the
first call on the device looks the array up)."""

import numpy as np
import pytest
import torch

import gorelaxor_b200 as g
from gorelaxor_b200 import synth
from tests.helpers import bits_equal, mismatch

pytestmark = pytest.mark.gpu
TOL = 1e-3  # the relative tolerance the parity tests state; identical bits pass it


def _case(seed, m, n, k, bias, dropped):
    rng = np.random.default_rng(seed)
    w = synth.rand_q8(rng, n, k)
    gw = g.Weight.q8(w.blocks, n, k)
    if dropped:
        gw.drop_rows()
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    b = rng.normal(0, 0.1, n).astype(np.float32) if bias else None
    return gw, x, b


def _static(gw, x, b, side_stream=False):
    m = x.shape[0]
    dx = torch.from_numpy(x).to("cuda:0")
    db = torch.from_numpy(b).to("cuda:0") if b is not None else None
    dy = torch.full((m, gw.rows), float("nan"), device="cuda:0")
    s = torch.cuda.Stream(0) if side_stream else torch.cuda.current_stream(0)
    s.wait_stream(torch.cuda.current_stream(0))  # the inputs are written on the current stream
    before = torch.cuda.current_device()
    g.linear_q8_static(gw, dx.data_ptr(), m, db.data_ptr() if db is not None else None, dy.data_ptr(), s.cuda_stream)
    assert torch.cuda.current_device() == before, "the call changed the caller's current device"
    torch.cuda.synchronize(0)
    return dy.cpu().numpy()


def test_static_scratch_matches_linear_on_consecutive_calls(have_gpu):
    # a large call (the batched int8 product of more than 8 rows, with bias),
    # then a smaller one (the product of up to 8 rows, rows dropped, no bias)
    # over the first one's leftovers, then the first again over the second's,
    # this time on a stream of its own instead of the default one.
    cases = [_case(1, 256, 1024, 4096, True, False),  # m*cols = 2^20, the whole array
             _case(2, 5, 256, 512, False, True)]
    for i, (gw, x, b) in enumerate(cases + cases[:1]):
        want = g.linear(gw, x, b)
        got = _static(gw, x, b, side_stream=i == 2)
        ne, rel = mismatch(got, want)
        assert bits_equal(got, want), f"{ne} of {got.size} differ (max rel {rel:.2e}, tolerance {TOL})"


def test_static_scratch_rejects_oversize_and_float_path(have_gpu):
    gw, x, _ = _case(3, 2, 64, 1024, False, False)
    dy = torch.empty((2048, 64), device="cuda:0")
    dx = torch.zeros((2048, 1024), device="cuda:0")
    with pytest.raises(g.GrxError) as e:  # 2048 x 1024 values: twice the array
        g.linear_q8_static(gw, dx.data_ptr(), 2048, None, dy.data_ptr())
    assert e.value.code == -5 and "scratch" in str(e.value)
    with pytest.raises(g.GrxError) as e:  # one row, rows kept: the reference's float path
        g.linear_q8_static(gw, dx.data_ptr(), 1, None, dy.data_ptr())
    assert e.value.code == -1
