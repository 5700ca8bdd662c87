"""Golden fixtures made by the reference's own converter (see
golden/make_golden.py) against the oracle and the library's GGUF reader,
and the reader's hostile-input checks (internal/gguf/hostile_test.go).
CPU only: the GGUF entry points touch no device."""

import json
import struct
from pathlib import Path

import numpy as np
import pytest

import gorelaxor_b200 as g
from oracle import oracle as orc

GOLD = Path(__file__).resolve().parent / "golden"


def test_to_q8_matches_converter_bytes():
    """q8int_test.go:129-150: ToQ8 rounds exactly as the converter does."""
    z = np.load(GOLD / "q8_converter.npz")
    got = orc.to_q8(z["x"])
    assert got.tobytes() == z["q8"].tobytes()


def test_gguf_reader_reads_converter_file():
    """gguf_test.go:51-113 known answers, on a file the converter wrote."""
    data = (GOLD / "gguf_converter.gguf").read_bytes()
    want = json.loads((GOLD / "gguf_converter.json").read_text())
    vals = np.load(GOLD / "gguf_values.npz")
    f = g.GGUF(data)
    assert f.string("general.architecture") == want["general.architecture"]
    assert f.string("general.name") == want["general.name"]
    assert f.int("pockettts.lm.d_model") == want["pockettts.lm.d_model"]
    assert f.int("pockettts.frames_after_eos") == want["pockettts.frames_after_eos"]
    assert f.float("pockettts.temperature") == pytest.approx(want["pockettts.temperature"], abs=0)
    assert f.int("pockettts.text.capitalize_first_letter") == 1
    assert f.int("missing.key", 42) == 42
    for name, t in want["tensors"].items():
        assert f.tensor(name) == (t["type"], t["dims"])
    a = f.float32("a")
    assert a.reshape(-1)[4] == 4.5  # gguf_test.go:99
    assert np.array_equal(a, vals["a"])
    assert np.array_equal(f.float32("w"), vals["w"].astype(np.float32))
    assert np.array_equal(f.float32("v"), vals["v"])


def _gguf(kvs=b"", nkv=0, tensors=(), version=3, pad=True):
    """A minimal GGUF (gguf_test.go:18-49): header, settings, tensor table,
    32-byte aligned data."""
    s = lambda x: struct.pack("<Q", len(x)) + x
    b = b"GGUF" + struct.pack("<IQQ", version, len(tensors), nkv) + kvs
    off, datas = 0, []
    for name, dims, typ, data in tensors:
        b += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        b += struct.pack("<IQ", typ, off)
        datas.append(data)
        off += len(data)
        off += (-off) % 32
    if pad:
        b += b"\0" * ((-len(b)) % 32)
    for d in datas:
        b += d + b"\0" * ((-len(d)) % 32)
    return b


def test_gguf_known_answers_q8_and_conv_dims():
    """gguf_test.go:51-113: a 1x1 convolution kernel [1,4,8] is 8 rows of
    4; Q8_0 with scale 0.25 and values i-16 reads back -4 .. 3.75."""
    f16 = b"".join(struct.pack("<e", float(i)) for i in range(32))
    q8 = struct.pack("<e", 0.25) + bytes((i - 16) & 0xff for i in range(32))
    f = g.GGUF(_gguf(tensors=[(b"pw", [1, 4, 8], 1, f16), (b"q", [32, 1], 8, q8)]))
    q = f.float32("q").reshape(-1)
    assert q[0] == -4 and q[31] == 3.75
    assert f.tensor("pw") == (1, [1, 4, 8])


@pytest.mark.parametrize("mutate", ["cut", "magic", "version", "counts", "dims", "overflow", "offset", "align",
                                    "array", "strlen", "q8rows", "type", "overlap"])
def test_gguf_hostile_inputs(mutate):
    """hostile_test.go: lying headers, wraps and overflows fail with an
    error, never a crash or a huge allocation."""
    good = _gguf(tensors=[(b"a", [4, 2], 0, b"\0" * 32)])
    s = lambda x: struct.pack("<Q", len(x)) + x
    bad = {
        "cut": good[:-20],
        "magic": b"GGUX" + good[4:],
        "version": good[:4] + struct.pack("<I", 7) + good[8:],
        "counts": good[:8] + struct.pack("<Q", 1 << 40) + good[16:],
        "dims": _gguf(tensors=[(b"a", [0, 2], 0, b"")]),
        "overflow": _gguf(tensors=[(b"a", [1 << 40, 1 << 40], 0, b"\0" * 32)]),
        "offset": _gguf(tensors=[(b"a", [64, 64], 0, b"\0" * 32)]),
        "align": _gguf(kvs=s(b"general.alignment") + struct.pack("<II", 4, 3), nkv=1),
        "array": _gguf(kvs=s(b"x") + struct.pack("<IIQ", 9, 4, 1 << 40), nkv=1),
        "strlen": _gguf(kvs=s(b"x") + struct.pack("<IQ", 8, 1 << 50), nkv=1),
        "q8rows": _gguf(tensors=[(b"q", [33, 1], 8, b"\0" * 34)]),
        "type": _gguf(tensors=[(b"q", [32, 1], 99, b"\0" * 34)]),
        "overlap": _gguf(tensors=[(b"a", [8], 0, b"\0" * 32), (b"b", [8], 0, b"\0" * 32)])[:-32],
    }[mutate]
    with pytest.raises(g.GrxError) as e:
        g.GGUF(bad)
    assert e.value.code == -2
