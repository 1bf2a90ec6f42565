"""Speculative decoding on the GPU (draft + target engines on one stream) vs the CPU
restatement of the same loop (oracle/spec.py).

the draft is the target with every weight perturbed by seeded
N(0, 0.004) noise; k = 4 and 8; acceptance (a) greedy token match, (b) rejection sampling
at temperature 1 with seeded uniforms. Gates: generated tokens and per-round accept
counts bit-exact against the oracle; greedy speculative output equals the target's own
greedy generation.
"""
import os

import numpy as np
import pytest

import oracle
from oracle import spec as spec_oracle
from voxelengine import engine as ve

pytestmark = pytest.mark.gpu
oracle.set_threads(os.cpu_count() or 1)

SMALL = dict(vocab=4096, hidden=576, inter=1536, layers=3, heads=9, kv_heads=3, max_pos=512)


@pytest.fixture(scope="module")
def pair(tmp_path_factory):
    root = tmp_path_factory.mktemp("spec")
    tgt = ve.synth_model(str(root / "target"), seed=21, **SMALL)
    drf = ve.synth_model(str(root / "draft"), seed=21, noise_seed=5, noise_std=0.004, **SMALL)
    return tgt, drf


def engines(pair, n, k, max_len=96):
    t = ve.Engine(pair[0], max_batch=n * (k + 1), max_len=max_len)
    d = ve.Engine(pair[1], max_batch=n, max_len=max_len, share=t)
    return t, d


def close(t, d):
    d.close()
    t.close()


@pytest.mark.parametrize("n,k", [(1, 4), (2, 8), (3, 4)])
def test_spec_greedy_matches_oracle_and_target(pair, n, k):
    prompts = [ve.prompt(1 + s, SMALL["vocab"], 8) for s in range(n)]
    budget = 20
    t, d = engines(pair, n, k)
    try:
        got, st, log = t.spec_generate(d, prompts, budget, k=k, mode=ve.SPEC_GREEDY, log_rounds=64)
        plain, _ = t.generate(prompts, budget)
    finally:
        close(t, d)
    want, want_log = spec_oracle.spec_generate(oracle.Model(pair[0]), oracle.Model(pair[1]), prompts,
                                               budget, k, rejection=False)
    assert np.array_equal(got, want), (got, want)
    # Greedy speculation never changes the target's output.
    assert np.array_equal(got, plain)
    for s in range(n):
        gpu_log = [int(a) for a in log[:, s] if a >= 0]
        assert gpu_log == want_log[s], (s, gpu_log, want_log[s])
    assert st.rounds == log.shape[0] and st.accepted <= st.drafted
    assert st.accepted == sum(sum(x) for x in want_log)
    assert st.draft_ms > 0 and st.verify_ms > 0


@pytest.mark.parametrize("n,k,seed", [(1, 4, 11), (2, 8, 12)])
def test_spec_rejection_matches_oracle(pair, n, k, seed):
    prompts = [ve.prompt(40 + s, SMALL["vocab"], 8) for s in range(n)]
    budget = 20
    t, d = engines(pair, n, k)
    try:
        got, st, log = t.spec_generate(d, prompts, budget, k=k, mode=ve.SPEC_REJECTION, seed=seed,
                                       log_rounds=64)
    finally:
        close(t, d)
    want, want_log = spec_oracle.spec_generate(oracle.Model(pair[0]), oracle.Model(pair[1]), prompts,
                                               budget, k, rejection=True, seed=seed)
    for s in range(n):
        gpu_log = [int(a) for a in log[:, s] if a >= 0]
        assert gpu_log == want_log[s], (s, gpu_log, want_log[s])
    assert np.array_equal(got, want), (got, want)
    assert 0 < st.accepted <= st.drafted


def test_spec_refuses_bad_pairings(pair):
    t = ve.Engine(pair[0], max_batch=5, max_len=96)
    other = ve.Engine(pair[1], max_batch=1, max_len=96)      # own ctx: not a valid draft
    shared = ve.Engine(pair[1], max_batch=1, max_len=96, share=t)
    try:
        p = [ve.prompt(1, SMALL["vocab"], 8)]
        with pytest.raises(ve.cuda.OpureError):
            t.spec_generate(other, p, 8, k=4)
        with pytest.raises(ve.cuda.OpureError):
            t.spec_generate(shared, p, 8, k=8)               # target max_batch < n (k + 1)
        with pytest.raises(ve.cuda.OpureError):
            t.spec_generate(shared, p, 200, k=4)             # exceeds max_len
        out, st, _ = t.spec_generate(shared, p, 8, k=4)      # still usable afterwards
        assert out.shape == (1, 8)
    finally:
        shared.close()
        other.close()
        t.close()


# ---- BASELINE config 3 on its own pair: the config-0 model and its N(0, 0.004) draft -----
@pytest.fixture(scope="module")
def cfg3_oracles(smollm_dirs):
    return oracle.Model(smollm_dirs[0]), oracle.Model(smollm_dirs[1])


@pytest.mark.parametrize("k", [4, 8])
@pytest.mark.parametrize("mode", [ve.SPEC_GREEDY, ve.SPEC_REJECTION])
def test_config3_b16_matches_oracle(smollm_dirs, cfg3_oracles, k, mode):
    # B = 16 sequences (prompt seeds 1..16, 32 tokens), 32 generated tokens each: the
    # verify pass is B (k + 1) = 80 / 144 vectors on the tcgen05 GEMV. Accept counts per
    # round and tokens bit-exact against the oracle's loop (sequences on host threads).
    B, budget, seed = 16, 32, 3
    prompts = [ve.prompt(1 + b, 49152, 32) for b in range(B)]
    t = ve.Engine(smollm_dirs[0], max_batch=B * (k + 1), max_len=32 + budget + k + 8)
    d = ve.Engine(smollm_dirs[1], max_batch=B, max_len=32 + budget + k + 8, share=t)
    try:
        got, st, log = t.spec_generate(d, prompts, budget, k=k, mode=mode, seed=seed, log_rounds=64)
        acceptance = t.metrics().speculative_acceptance
    finally:
        close(t, d)
    want, want_log = spec_oracle.spec_generate(*cfg3_oracles, prompts, budget, k,
                                               rejection=(mode == ve.SPEC_REJECTION), seed=seed,
                                               threads=os.cpu_count() or 1)
    for s in range(B):
        gpu_log = [int(a) for a in log[:, s] if a >= 0]
        assert gpu_log == want_log[s], (s, gpu_log, want_log[s])
    assert np.array_equal(got, want)
    # The partial acceptance the noisy draft is meant to give, reported by the target's
    # SnapshotMetrics (the reference fixes it at -1).
    assert 0 < st.accepted < st.drafted
    assert acceptance == pytest.approx(st.accepted / st.drafted, rel=1e-6)
