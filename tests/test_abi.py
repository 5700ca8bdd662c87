"""The C ABI: libgrx.so loads without a GPU and exports every entry point
include/grx.h declares; calls that need a device fail with an error code,
not a crash. The oracle library builds. CPU only."""

import ctypes
import re
from pathlib import Path

import pytest

import gorelaxor_b200 as g
from oracle import oracle as orc

ROOT = Path(__file__).resolve().parents[1]


def declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(grx_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(g.LIB_PATH))
    names = declared()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_mirror_binds_every_symbol():
    lib = g.lib()
    for n in declared():
        assert getattr(lib, n).restype is not None or n.endswith(("_free", "_close")), n


def test_device_calls_fail_cleanly_without_device():
    if g.device_count() > 0:
        pytest.skip("a device is present")
    with pytest.raises(g.GrxError) as e:
        g.FlowLM(b"GGUF" + b"\0" * 64)
    assert e.value.code in (-2, -6)
    with pytest.raises(g.GrxError):
        g.Weight.f32(__import__("numpy").ones((2, 2), "float32"))


def test_oracle_library_builds():
    orc.build()
    assert orc.LIB.exists()
    assert orc.lib().orc_expf_go(0.0) == 1.0


def test_next_rows_fail_cleanly_without_device():
    """The Mimi decoder, Whisper encoder and FastConformer handles refuse to
    load without a device (an error code, no crash); the subsampling's row
    count is plain host arithmetic (three stride-2 steps, encoder.go:32-39)."""
    lib = g.lib()
    for n, want in ((1, 1), (2, 1), (8, 1), (9, 2), (70, 9), (200, 25), (203, 26), (3000, 375)):
        assert lib.grx_fconf_out_rows(n) == want
    assert lib.grx_fconf_out_rows(0) == 0
    if g.device_count() > 0:
        pytest.skip("a device is present")
    for cls in (g.Mimi, g.FConf):
        with pytest.raises(g.GrxError) as e:
            cls(b"GGUF" + b"\0" * 64)
        assert e.value.code in (-2, -6)
