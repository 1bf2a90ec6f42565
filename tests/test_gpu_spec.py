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
from common import greedy_tokens_agree
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
DRAW_DRIFT = 64     # token ids: an inverse-CDF draw moved by cumulative-sum rounding
RATIO_MARGIN = 0.02  # |u q(d) / p(d) - 1| below this: an accept decision within logit noise


def rejection_rounds_agree(got, gpu_log, want, recs, budget, gpu_drafts=None):
    """Rejection sampling at temperature 1 on a random-init model draws from nearly uniform
    distributions over 49152 ids (each id ~2e-5 of the mass): logits that differ by fp32
    rounding (~1e-5) move the cumulative sums, and with them an inverse-CDF draw, by a few
    ids. Rounds are therefore compared in order and must match exactly (accept count and
    emitted ids) up to the first round that differs; that round must differ in a way such
    rounding explains: an emitted id within DRAW_DRIFT ids of the oracle's (a draft,
    replacement or bonus draw moved along the CDF), or an accept decision whose oracle
    ratio u q(d) / p(d) lies within RATIO_MARGIN of 1. Later rounds, which continue from
    different tokens, are not compared. Returns (tokens compared, note)."""
    if got[0] != want[0]:
        if abs(int(got[0]) - int(want[0])) <= DRAW_DRIFT:
            return 0, f"first draw {got[0]} vs {want[0]}"
        raise AssertionError(f"first token {got[0]} vs oracle {want[0]}")
    pos = 1
    for r, rec in enumerate(recs):
        if pos >= budget:
            break
        ga = gpu_log[r] if r < len(gpu_log) else -1
        if gpu_drafts is not None and r < len(gpu_drafts):
            # The drafts both loops proposed this round: any difference is the draft's own
            # inverse-CDF draw moving, which must stay within DRAW_DRIFT ids.
            gd = [int(x) for x in gpu_drafts[r]]
            for j, (a, b) in enumerate(zip(gd, rec["drafts"])):
                if a != b:
                    if abs(a - b) <= DRAW_DRIFT and (ga >= j or rec["a"] >= j):
                        ok = all(x == y for x, y in zip(got[pos: pos + j], rec["emitted"][:j]))
                        if ok:
                            return pos + j, f"round {r}: draft draw {a} vs {b}"
                    if abs(a - b) > DRAW_DRIFT:
                        raise AssertionError(f"round {r}: drafts {gd} vs oracle {rec['drafts']}")
                    break
        go = [int(x) for x in got[pos: pos + ga + 1]] if ga >= 0 else []
        wo = rec["emitted"][: budget - pos]
        if ga == rec["a"] and go == wo:
            pos += rec["a"] + 1
            continue
        # Ids both sides emitted from the same kind of draw: the accepted drafts before the
        # first differing decision, or every id when the accept counts agree.
        same = len(go) if ga == rec["a"] else min(ga, rec["a"])
        for i in range(min(same, len(go), len(wo))):
            if go[i] != wo[i]:
                if abs(go[i] - wo[i]) <= DRAW_DRIFT:
                    return pos + i, f"round {r}: draw {go[i]} vs {wo[i]}"
                raise AssertionError(f"round {r}: emitted {go} vs oracle {wo} (accepts {ga} vs {rec['a']})")
        j = min(ga, rec["a"])
        if ga != rec["a"] and "ratios" in rec and 0 <= j < len(rec["ratios"]) and \
                abs(rec["ratios"][j] - 1.0) < RATIO_MARGIN:
            return pos + j, f"round {r}: accept {ga} vs {rec['a']} (oracle ratio {rec['ratios'][j]:.4f})"
        if ga > rec["a"] and j < len(go) and go[j] != rec["drafts"][j] and abs(go[j] - rec["drafts"][j]) <= DRAW_DRIFT:
            # The GPU accepted a draft the oracle never proposed: the draft's own draw moved.
            return pos + j, f"round {r}: draft draw {go[j]} vs {rec['drafts'][j]}"
        raise AssertionError(f"round {r}: accepts {ga} vs oracle {rec['a']}, emitted {go} vs {wo}, "
                             f"ratios {rec.get('ratios')}")
    assert np.array_equal(np.asarray(got), np.asarray(want)), (got, want)
    return len(want), "equal"
@pytest.fixture(scope="module")
def cfg3_oracles(smollm_dirs):
    return oracle.Model(smollm_dirs[0]), oracle.Model(smollm_dirs[1])


@pytest.fixture(scope="module")
def cfg3_greedy(cfg3_oracles):
    # The target's own greedy decode of the 16 prompts with the oracle's top-2 margins and
    # runner-ups: greedy speculation must reproduce it.
    prompts = [ve.prompt(1 + b, 49152, 32) for b in range(16)]
    return cfg3_oracles[0].generate_batch(prompts, 32, threads=os.cpu_count() or 1)


@pytest.mark.parametrize("k", [4, 8])
@pytest.mark.parametrize("mode", [ve.SPEC_GREEDY, ve.SPEC_REJECTION])
def test_config3_b16_matches_oracle(smollm_dirs, cfg3_oracles, cfg3_greedy, k, mode):
    # B = 16 sequences (prompt seeds 1..16, 32 tokens), 32 generated tokens each: the
    # verify pass is B (k + 1) = 80 / 144 vectors on the tcgen05 GEMV. Accept counts per
    # round and tokens bit-exact against the oracle's loop (sequences on host threads).
    # Greedy: a sequence whose target decode meets an oracle near-tie (top-2 logit gap
    # below common.TIE_MARGIN) is compared up to that decision only.
    B, budget, seed = 16, 32, 3
    prompts = [ve.prompt(1 + b, 49152, 32) for b in range(B)]
    t = ve.Engine(smollm_dirs[0], max_batch=B * (k + 1), max_len=32 + budget + k + 8)
    d = ve.Engine(smollm_dirs[1], max_batch=B, max_len=32 + budget + k + 8, share=t)
    try:
        got, st, log, drafts = t.spec_generate(d, prompts, budget, k=k, mode=mode, seed=seed, log_rounds=64,
                                               draft_log=True)
        acceptance = t.metrics().speculative_acceptance
    finally:
        close(t, d)
    want, want_log, recs = spec_oracle.spec_generate(*cfg3_oracles, prompts, budget, k,
                                                     rejection=(mode == ve.SPEC_REJECTION), seed=seed,
                                                     threads=os.cpu_count() or 1, records=True)
    ties = []
    for s in range(B):
        gpu_log = [int(a) for a in log[:, s] if a >= 0]
        if mode == ve.SPEC_REJECTION:
            gpu_drafts = [drafts[r, s] for r in range(drafts.shape[0]) if log[r, s] >= 0]
            n, note = rejection_rounds_agree(got[s], gpu_log, want[s], recs[s], budget, gpu_drafts)
            if note != "equal":
                ties.append((s, n, note))
            continue
        if mode == ve.SPEC_GREEDY:
            g_tokens, _, g_margins, g_second = cfg3_greedy
            assert np.array_equal(want[s], g_tokens[s])  # the oracle's loop equals plain greedy
            n, note = greedy_tokens_agree(got[s], want[s], g_margins[s], g_second[s])
            if note != "equal":
                ties.append((s, note))
                # Rounds that ended before the tie decided the same tokens.
                done, r = 0, 0
                while r < len(want_log[s]) and done + want_log[s][r] + 1 <= n:
                    assert gpu_log[r] == want_log[s][r], (s, r, gpu_log, want_log[s])
                    done += want_log[s][r] + 1
                    r += 1
                continue
        assert gpu_log == want_log[s], (s, gpu_log, want_log[s])
        assert np.array_equal(got[s], want[s]), (s, got[s], want[s])
    orc_rate = sum(sum(r["a"] for r in rr) for rr in recs) / max(1, sum(k * len(rr) for rr in recs))
    print(f"config 3 k={k} mode={mode}: acceptance gpu {st.accepted / st.drafted:.3f} oracle {orc_rate:.3f}; "
          f"divergences {ties}")
    if mode == ve.SPEC_GREEDY:
        assert len(ties) <= 2
    else:
        # Draws over these near-uniform distributions drift (see rejection_rounds_agree), so
        # the acceptance rate, not every sampled id, is what both loops must share.
        assert abs(st.accepted / st.drafted - orc_rate) < 0.05
    # The partial acceptance the noisy draft is meant to give, reported by the target's
    # SnapshotMetrics (the reference fixes it at -1).
    assert 0 < st.accepted < st.drafted
    assert acceptance == pytest.approx(st.accepted / st.drafted, rel=1e-6)
