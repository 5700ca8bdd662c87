"""Makes the golden fixtures in this folder from the reference's own Python.

gorelaxor's converter tools/convert_nemo.py is plain numpy; its Q8_0
quantizer (q8_0, :154-167) and its GGUF writer (class GGUF, :71-147) are
what produce every model file the Go engines read. This script imports that
file from a gorelaxor checkout and records:

* q8_converter.npz — float32 inputs and the converter's Q8_0 bytes for
  them (edge cases included: a zero block, exact .5 ties, ±extremes, tiny
  and huge magnitudes). Pins the oracle's ToQ8 restatement
  (internal/kern/kern.go:139-170), which q8int_test.go:129 requires to
  match the converter byte for byte, and with it the f16 rounding.
* gguf_converter.gguf + gguf_converter.json — a small GGUF written by the
  converter's GGUF class (settings of several types, an F32 matrix, a
  Q8_0 matrix of at least 64×64 as the converter's placement rule makes
  them, a vector) and the values it must read back as. Pins the library's
  GGUF reader against the writer of the files it has to load.

Run it where a gorelaxor checkout exists (the path is an argument); the
fixtures it writes are committed, so the tests never need the checkout.

    python tests/golden/make_golden.py <gorelaxor checkout>
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_converter(root: Path):
    spec = importlib.util.spec_from_file_location("convert_nemo", root / "tools" / "convert_nemo.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def q8_inputs() -> np.ndarray:
    rng = np.random.default_rng(20261201)
    blocks = [
        rng.normal(0, 1, 32),
        np.zeros(32),                                   # a block of zeros: scale 0, values 0
        np.linspace(-127, 127, 32),                     # exact integers at the scale 1
        np.array([0.5, -0.5, 1.5, -1.5, 2.5, -2.5] * 5 + [127, -127]),  # ties (round half away)
        rng.normal(0, 1e-6, 32),                        # tiny values (subnormal f16 scale)
        rng.normal(0, 3e4, 32),                         # large values
        np.concatenate([[-40.0], rng.uniform(-1, 1, 31)]),  # the extreme is negative
        rng.uniform(-1, 1, 32) * 1000,
    ]
    blocks += [rng.normal(0, s, 32) for s in (0.02, 0.5, 7.0, 250.0) for _ in range(4)]
    return np.concatenate(blocks).astype(np.float32).reshape(-1, 64)


def main(root: Path) -> None:
    cn = load_converter(root)
    x = q8_inputs()
    q = np.frombuffer(cn.q8_0(x), dtype=np.uint8)
    np.savez_compressed(HERE / "q8_converter.npz", x=x, q8=q)

    rng = np.random.default_rng(7)
    g = cn.GGUF("pockettts")
    g.str("general.name", "golden")
    g.u32("pockettts.lm.d_model", 64)
    g.i32("pockettts.frames_after_eos", -1)
    g.f32("pockettts.temperature", 0.3)
    g.bool("pockettts.text.capitalize_first_letter", True)
    g.i32s("pockettts.seanet.ratios", [8, 6, 5, 4])
    g.strs("tokenizer.ggml.tokens", ["a", "▁b", "c"])
    a = (np.arange(6, dtype=np.float32) + 0.5).reshape(2, 3)   # gguf_test.go:69-72
    w = rng.normal(0, 1, (64, 96)).astype(np.float32)
    v = rng.normal(0, 1, 96).astype(np.float32)
    g.tensor("a", a, cn.GGML_F32)
    g.tensor("w", w, cn.GGML_Q8_0)
    g.tensor("v", v, cn.GGML_F32)
    path = HERE / "gguf_converter.gguf"
    g.write(path)
    wq = np.frombuffer(cn.q8_0(w), dtype=np.uint8).reshape(-1, 34)
    d = wq[:, :2].copy().view(np.float16).astype(np.float32)
    qs = wq[:, 2:].view(np.int8).astype(np.float32)
    w_back = (qs * d).reshape(64, 96)
    expect = {
        "general.architecture": "pockettts",
        "general.name": "golden",
        "pockettts.lm.d_model": 64,
        "pockettts.frames_after_eos": -1,
        "pockettts.temperature": float(np.float32(0.3)),
        "pockettts.text.capitalize_first_letter": 1,
        "tensors": {"a": {"type": 0, "dims": [3, 2]}, "w": {"type": 8, "dims": [96, 64]},
                    "v": {"type": 0, "dims": [96]}},
    }
    (HERE / "gguf_converter.json").write_text(json.dumps(expect, indent=1) + "\n")
    np.savez_compressed(HERE / "gguf_values.npz", a=a, w=w_back, v=v)
    print("wrote", sorted(p.name for p in HERE.glob("*_converter*")))


if __name__ == "__main__":
    main(Path(sys.argv[1]))
