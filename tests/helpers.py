"""Shared helpers for the parity tests: synthetic models, both sides."""

from __future__ import annotations

import numpy as np

from gorelaxor_b200 import synth

SMALL = dict(d=128, heads=2, ff=256, layers=2, flow_dim=128)


def voice_kv(cfg, positions, seed):
    v = synth.voice_tensors(cfg, positions, seed)
    return np.stack([np.stack([v[f"voice.{l}.k"], v[f"voice.{l}.v"]]) for l in range(cfg.layers)])


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


def mismatch(a, b):
    a = np.asarray(a, np.float32).ravel()
    b = np.asarray(b, np.float32).ravel()
    ne = np.count_nonzero(a.view(np.uint32) != b.view(np.uint32))
    rel = np.max(np.abs(a.astype(np.float64) - b) / (np.abs(b.astype(np.float64)) + 1e-6)) if a.size else 0.0
    return ne, rel
