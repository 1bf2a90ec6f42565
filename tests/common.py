"""Shared test helpers."""
from __future__ import annotations

import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def compare(got, want):
    """The reference harness's pass criterion, Opure_TestHarness.cpp:70-101.

    Returns (passed, max_abs, rms): NaN on either side fails; otherwise passes when
    rms <= 1e-5 * max|want| (floored at 1e-6) or rms <= 1e-7.
    """
    g = np.asarray(got, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    n = min(g.size, w.size)
    g, w = g[:n], w[:n]
    if np.isnan(g).any() or np.isnan(w).any():
        return False, float("inf"), float("nan")
    d = np.abs(g - w)
    max_abs = float(d.max()) if n else 0.0
    rms = float(np.sqrt((d * d).sum() / n)) if n else 0.0
    scale = max(1e-6, float(np.abs(w).max()) if n else 0.0)
    return (rms <= 1e-5 * scale) or (rms <= 1e-7), max_abs, rms


def rel_err(got, want, floor=1e-6):
    """max |got - want| / max(max|want|, floor): the per-kernel 1e-3 relative gate."""
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    return float(np.abs(g - w).max() / max(float(np.abs(w).max()), floor))


def kats():
    return np.load(os.path.join(GOLDEN, "harness_kats.npz"))
