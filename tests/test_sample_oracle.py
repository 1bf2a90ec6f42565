"""CPU checks of the oracle's filtered sampler and logit statistics (the checkers of
tests/test_gpu_sample.py): the sampling rules against direct numpy statements of them,
and the statistics against the reference's RefreshLogitStats arithmetic
(src/engine/Opure_VoxelEngine.cpp:832-876) written out in numpy."""
import numpy as np
import pytest

import oracle


def kept_set(row, T, k, p, hist=None, rep=1.0):
    lp = row.astype(np.float32).copy()
    if hist is not None and rep != 1.0:
        for t in set(int(x) for x in hist):
            lp[t] = lp[t] / np.float32(rep) if lp[t] > 0 else lp[t] * np.float32(rep)
    order = sorted(range(lp.size), key=lambda i: (-lp[i], i))
    if 1 < k < lp.size:
        order = order[:k]
    z = np.array([lp[i] for i in order], np.float64) * (1.0 / np.float64(T))
    mass = np.rint(np.exp(z - z[0]) * 2.0**40).astype(np.uint64)
    if p < 1.0:
        target = max(1, int(np.ceil(np.float64(np.float32(p)) * float(mass.sum()))))
        if target < int(mass.sum()):
            cum = np.cumsum(mass)
            order = order[: int(np.argmax(cum >= target)) + 1]
    return lp, order


def test_greedy_is_lowest_index_argmax():
    row = np.array([1, 3, 3, -2, 3], np.float32)
    assert oracle.sample_filtered(row, 0.5, 0.0) == 1
    assert oracle.sample_filtered(row, 0.5, 1.0, 1) == 1


@pytest.mark.parametrize("T,k,p", [(1.0, 5, 1.0), (0.7, 0, 0.8), (1.5, 20, 0.6), (1.0, 0, 0.05)])
def test_draws_stay_in_the_kept_set_and_cover_it(T, k, p):
    rng = np.random.default_rng(int(T * 100) + k)
    row = (rng.standard_normal(200) * 2).astype(np.float32)
    _, order = kept_set(row, T, k, p)
    got = {oracle.sample_filtered(row, float(u), T, k, p) for u in np.linspace(0, 1, 2001, endpoint=False)}
    assert got <= set(order)
    # Every kept token with at least 1/1000 of the kept mass is drawn on the grid.
    lp = row[order].astype(np.float64) / T
    w = np.exp(lp - lp.max())
    w /= w.sum()
    assert {order[i] for i in range(len(order)) if w[i] > 2e-3} <= got


def test_draw_is_the_index_order_inverse_cdf():
    row = np.array([0.0, 1.0, 2.0, 0.5], np.float32)
    lp, order = kept_set(row, 1.0, 0, 1.0)
    mass = np.rint(np.exp(row.astype(np.float64) - 2.0) * 2.0**40).astype(np.uint64)
    cum = np.cumsum(mass)
    for u in (0.0, 0.1, 0.3, 0.6, 0.9, 0.999):
        thr = int(np.floor(np.float64(np.float32(u)) * float(cum[-1])))
        assert oracle.sample_filtered(row, u, 1.0) == int(np.argmax(cum > thr))


def test_repetition_penalty():
    row = np.array([2.0, 1.9, -1.0, -1.1], np.float32)
    # Token 0 in the history: 2.0 / 1.5 < 1.9, so the greedy pick moves to token 1.
    assert oracle.sample_filtered(row, 0.5, 0.0, 0, 1.0, 1.5, np.array([0], np.int32)) == 1
    # A negative logit is multiplied: -1.0 * 1.5 < -1.1.
    lp, _ = kept_set(row, 1.0, 0, 1.0, hist=[2], rep=1.5)
    assert lp[2] == np.float32(-1.5)


def test_top_p_keeps_the_shortest_prefix():
    row = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float64)).astype(np.float32)
    for p, n_kept in [(0.4, 1), (0.5, 1), (0.75, 2), (0.9, 3), (0.99, 4)]:
        _, order = kept_set(row, 1.0, 0, p)
        assert len(order) == n_kept, (p, order)
        got = {oracle.sample_filtered(row, float(u), 1.0, 0, p) for u in np.linspace(0, 1, 101, endpoint=False)}
        assert got == set(order)


def test_infinite_and_nan_logits():
    row = np.zeros(10, np.float32)
    row[3] = np.inf
    assert oracle.sample_filtered(row, 0.7, 1.0) == 3
    row = np.full(10, np.nan, np.float32)
    assert oracle.sample_filtered(row, 0.7, 1.0) == 0
    row[4] = -1.0
    assert oracle.sample_filtered(row, 0.7, 1.0) == 4


@pytest.mark.parametrize("scale", [0.1, 2.0, 40.0])
def test_logit_stats_follow_the_reference_arithmetic(scale):
    rng = np.random.default_rng(int(scale * 7))
    g = (rng.standard_normal(49152) * scale).astype(np.float32)
    got = oracle.logit_stats(g)
    mx = g.max()
    ref_norm = np.sqrt((g.astype(np.float64) ** 2).sum())
    e = np.exp((g - mx).astype(np.float64))  # fp32 shift, then double (the reference's cast order)
    pr = e / e.sum()
    ref_ent = -(pr[pr > 0] * np.log(pr[pr > 0])).sum()
    assert got[0] == mx
    np.testing.assert_allclose(got[1], ref_norm, rtol=1e-6)
    np.testing.assert_allclose(got[2], ref_ent, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got[3], mx + np.log(e.sum()), rtol=1e-6)
