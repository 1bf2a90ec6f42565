"""Filtered sampling (temperature, top-k, top-p, repetition penalty) and the on-device
logit statistics vs the CPU restatements in the oracle.

Gates: sampled token ids bit-exact against oracle.sample_filtered on the same seeded
logits and uniforms (masses are integers, so the decisions do not depend on summation
order); the argmax key written for the next self-driving step decodes to the same id;
logit statistics within 1e-6 relative of oracle.logit_stats, and within the reference
harness's own criterion (norm 1e-2 relative, entropy 1e-3 absolute,
src/app/Opure_TestHarness.cpp:687-692).
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from voxelengine import cuda as cu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = cu.Ctx(0)
    yield c
    c.close()


def run_sample(ctx, lg, u, temperature, top_k, top_p, rep=1.0, hist=None, hist_len=None):
    R, V = lg.shape
    d_l, d_u = ctx.to_device(lg), ctx.to_device(u.astype(np.float32))
    d_o, d_k = ctx.buffer(R * 4), ctx.buffer(R * 8)
    a = cu.SampleArgs()
    a.logits, a.vocab, a.rows, a.stride = d_l.ptr, V, R, V
    a.temperature, a.top_k, a.top_p, a.rep_penalty = temperature, top_k, top_p, rep
    keep = []
    if hist is not None:
        d_h, d_hl = ctx.to_device(hist.astype(np.int32)), ctx.to_device(hist_len.astype(np.int32))
        keep += [d_h, d_hl]
        a.hist, a.max_len, a.seq, a.hist_len = d_h.ptr, hist.shape[1], None, d_hl.ptr
    a.u, a.out, a.keys = d_u.ptr, d_o.ptr, d_k.ptr
    ctx.sample_filtered(a)
    out = d_o.download(np.int32, R)
    keys = d_k.download(np.uint64, R)
    assert [0xFFFFFFFF - int(k & 0xFFFFFFFF) for k in keys] == list(out)
    return out


CASES = [
    # temperature, top_k, top_p, rep
    (0.0, 0, 1.0, 1.0),      # greedy
    (1.0, 1, 1.0, 1.0),      # top_k 1 = greedy
    (1.0, 0, 1.0, 1.0),      # plain softmax draw
    (0.7, 50, 1.0, 1.0),
    (1.0, 0, 0.9, 1.0),      # nucleus over the whole vocabulary
    (0.8, 50, 0.95, 1.0),    # the reference chat defaults (Opure_Chat.cpp:69)
    (1.3, 1000, 0.5, 1.0),
    (1.0, 40, 0.9, 1.3),     # with a repetition penalty
]


@pytest.mark.parametrize("V", [49152, 1000, 17])
@pytest.mark.parametrize("case", CASES)
def test_sample_filtered_matches_oracle(ctx, V, case):
    T, k, p, rep = case
    rng = np.random.default_rng(V * 31 + int(T * 10) + k)
    R = 12
    lg = (rng.standard_normal((R, V)) * 3).astype(np.float32)
    u = rng.random(R).astype(np.float32)
    u[0], u[1] = 0.0, np.nextafter(np.float32(1.0), np.float32(0.0))  # both ends of the CDF
    hist = hist_len = None
    if rep != 1.0:
        hist = rng.integers(0, V, (R, 64)).astype(np.int32)
        hist_len = rng.integers(0, 65, R).astype(np.int32)
    got = run_sample(ctx, lg, u, T, k, p, rep, hist, hist_len)
    want = [oracle.sample_filtered(lg[r], float(u[r]), T, k, p, rep,
                                   None if hist is None else hist[r, :hist_len[r]]) for r in range(R)]
    assert list(got) == want


def test_sample_filtered_ties_nans_and_infinities(ctx):
    V, R = 4096, 8
    rng = np.random.default_rng(3)
    lg = np.round(rng.standard_normal((R, V)) * 2).astype(np.float32)  # many exact ties
    lg[0, :] = np.nan
    lg[1, ::3] = np.nan
    lg[2, :] = -np.inf
    lg[2, 100] = 1.0
    lg[3, 7] = np.inf
    u = rng.random(R).astype(np.float32)
    for T, k, p in [(0.0, 0, 1.0), (1.0, 5, 1.0), (1.0, 0, 0.6), (2.0, 100, 0.9)]:
        got = run_sample(ctx, lg, u, T, k, p)
        want = [oracle.sample_filtered(lg[r], float(u[r]), T, k, p) for r in range(R)]
        assert list(got) == want, (T, k, p)


def test_sample_filtered_distribution(ctx):
    """Over a uniform grid of u the draws reproduce the filtered softmax."""
    V, R = 64, 4096
    rng = np.random.default_rng(9)
    row = (rng.standard_normal(V) * 1.5).astype(np.float32)
    lg = np.tile(row, (R, 1))
    u = ((np.arange(R) + 0.5) / R).astype(np.float32)
    T, k = 0.9, 10
    got = run_sample(ctx, lg, u, T, k, 1.0)
    top = np.argsort(-row, kind="stable")[:k]
    w = np.exp((row[top].astype(np.float64) - row[top].max()) / T)
    want = w / w.sum()
    freq = np.array([(got == t).sum() for t in top]) / R
    assert set(got) <= set(top)
    assert np.abs(freq - want).max() < 2.0 / R + 1e-3


def test_sample_filtered_refuses_bad_arguments(ctx):
    a = cu.SampleArgs()
    with pytest.raises(cu.OpureError):
        ctx.sample_filtered(a)


@pytest.mark.parametrize("scale", [0.5, 3.0, 30.0])
def test_logit_stats_matches_oracle(ctx, scale):
    rng = np.random.default_rng(int(scale * 10))
    R, V = 6, 49152
    lg = (rng.standard_normal((R, V)) * scale).astype(np.float32)
    lg[5, 11] = np.nan  # skipped for the max, as the argmax
    d_l, d_o = ctx.to_device(lg), ctx.buffer(R * 16)
    ctx.call("opure_logit_stats", C.c_void_p(d_l.ptr), V, R - 1, V, C.c_void_p(d_o.ptr))
    got = d_o.download(np.float32, (R - 1) * 4).reshape(R - 1, 4)
    for r in range(R - 1):
        want = oracle.logit_stats(lg[r])
        np.testing.assert_allclose(got[r], want, rtol=1e-6, atol=1e-6)
        # The reference harness's own pass criterion.
        assert abs(got[r, 1] - want[1]) <= 1e-2 * max(1.0, want[1])
        assert abs(got[r, 2] - want[2]) <= 1e-3 and 0.0 <= got[r, 2] <= np.log(V)
