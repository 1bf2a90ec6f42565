"""Sampled generation through the engine (temperature / top-k / top-p / repetition
penalty, per-token logit statistics) vs the oracle.

Per generated token: the engine's own logits (returned for verification) drive
oracle.sample_filtered with the sequence's uniform stream (Rng(seed ^ s * 0x9E3779B97F4A7C15),
one draw per token) and the history so far; the sampled id must be bit-exact. The logits
themselves are checked against the oracle's scalar forward fed the same tokens (teacher
forcing) within max_abs 2e-2, and the statistics against oracle.logit_stats.
"""
import os

import numpy as np
import pytest

import oracle
from oracle.spec import GOLDEN, MASK, Rng
from voxelengine import engine as ve

pytestmark = pytest.mark.gpu
oracle.set_threads(os.cpu_count() or 1)

SMALL = dict(vocab=4096, hidden=576, inter=1536, layers=3, heads=9, kv_heads=3, max_pos=512)


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    return ve.synth_model(str(tmp_path_factory.mktemp("sample") / "m"), seed=41, **SMALL)


@pytest.mark.parametrize("T,k,p,rep", [(1.0, 0, 1.0, 1.0), (0.8, 50, 0.95, 1.0), (1.2, 0, 0.7, 1.3),
                                       (0.0, 0, 1.0, 1.2)])
def test_sample_generate_matches_oracle(model, T, k, p, rep):
    n, plen, budget, seed = 3, 6, 12, 77
    prompts = [ve.prompt(100 + s, SMALL["vocab"], plen) for s in range(n)]
    with ve.Engine(model, max_batch=n, max_len=plen + budget + 4) as eng:
        toks, stats, logits = eng.sample_generate(prompts, budget, temperature=T, top_k=k, top_p=p,
                                                  rep_penalty=rep, seed=seed, stats=True, logits=True)
    om = oracle.Model(model)
    for s in range(n):
        rng = Rng(seed ^ ((s * GOLDEN) & MASK))
        hist = list(int(t) for t in prompts[s])
        st = om.state(plen + budget + 2)
        ref = None
        for i, t in enumerate(hist):
            ref, _ = st.forward(t, logits=(i == plen - 1))
        for j in range(budget):
            u = rng.uniform()
            lg = logits[s, j]
            want = oracle.sample_filtered(lg, u, T, k, p, rep, np.asarray(hist, np.int32))
            assert toks[s, j] == want, (s, j)
            assert np.abs(lg - ref).max() <= 2e-2, (s, j)
            np.testing.assert_allclose(stats[s, j], oracle.logit_stats(lg), rtol=1e-5, atol=1e-6)
            hist.append(int(toks[s, j]))
            ref, _ = st.forward(int(toks[s, j]), logits=True)


def test_greedy_sampling_is_generate(model):
    """temperature 0 without penalty reproduces the engine's greedy generation."""
    prompts = [ve.prompt(7 + s, SMALL["vocab"], 5) for s in range(2)]
    with ve.Engine(model, max_batch=2, max_len=32) as eng:
        got = eng.sample_generate(prompts, 10, temperature=0.0)
        want, _ = eng.generate(prompts, 10)
    assert np.array_equal(got, want)
