"""Parity tolerance of the attention path (the target stated for the port).

fp16 outputs with fp32 accumulation must match the reference restatement to
max-abs error <= 2e-3 and max-rel error <= 1e-2, where the relative error of
an element is |got - ref| / max(|ref|, 1e-3) (the floor keeps the measure
meaningful for outputs near zero, which long softmax averages produce).
kv_append and the generator are bit-exact.
"""
from __future__ import annotations

import numpy as np

ATOL = 2e-3
RTOL = 1e-2
REL_FLOOR = 1e-3


def errors(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(got - ref)
    rel = d / np.maximum(np.abs(ref), REL_FLOOR)
    return float(d.max(initial=0.0)), float(rel.max(initial=0.0))


def assert_attn_close(got, ref, what=""):
    got = np.asarray(got, dtype=np.float64)
    assert got.shape == np.shape(ref), (got.shape, np.shape(ref))
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    mab, mrel = errors(got, ref)
    assert mab <= ATOL and mrel <= RTOL, f"{what}: max-abs {mab:.3e} (<= {ATOL}), max-rel {mrel:.3e} (<= {RTOL})"
    return mab, mrel


def f16(bits: np.ndarray) -> np.ndarray:
    """fp16 bit patterns -> float64 values."""
    return np.ascontiguousarray(bits).view(np.float16).astype(np.float64)
