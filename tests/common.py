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


# Greedy token decisions whose top-2 logit gap in the oracle is below this are ties under
# the logits tolerance (BASELINE: logits max_abs <= 2e-2): fp32 GEMVs, fp16 KV rounding
# and tensor-core summation orders legitimately move logits by ~1e-5..1e-4, so a GPU may
# pick the runner-up there. Every other decision must be bit-exact.
TIE_MARGIN = 1e-3


def greedy_tokens_agree(got, want, margins, second, tie=TIE_MARGIN):
    """Compares a GPU greedy sequence with the oracle's. Returns (n_compared, note): equal
    tokens throughout, or equal up to a first difference where the oracle's top-2 margin
    is below `tie` and the GPU took the oracle's runner-up (both continuations are valid
    greedy decodes; the sequences are compared up to that decision only). Anything else
    raises AssertionError naming the step and margin."""
    got, want = np.asarray(got), np.asarray(want)
    n = min(got.size, want.size)
    diff = np.nonzero(got[:n] != want[:n])[0]
    if diff.size == 0 and got.size == want.size:
        return n, "equal"
    i = int(diff[0]) if diff.size else n
    if i < n and margins[i] < tie and int(got[i]) == int(second[i]):
        return i, f"tie at step {i} (oracle margin {margins[i]:.2e}, GPU took the runner-up {int(got[i])})"
    raise AssertionError(f"token mismatch at step {i}: gpu {got[i] if i < got.size else None} oracle "
                         f"{want[i] if i < want.size else None} (oracle margin {margins[min(i, n - 1)]:.3e}, "
                         f"runner-up {second[min(i, n - 1)]})")
