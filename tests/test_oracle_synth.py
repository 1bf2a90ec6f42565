"""The oracle's own seeded inputs and generation loops, without a GPU.

The CPU side of every parity check and the benchmark's reference arm build their
synthetic models and prompts inside the oracle (test infrastructure), so they never load
the product's libraries. These tests pin those generators to the engine's (the bytes the
CUDA path reads), and the stop rules and the multi-threaded batch to the one-at-a-time
loop.
"""
import numpy as np
import pytest

import oracle
from voxelengine import engine as ve

TINY = dict(vocab=512, hidden=128, inter=256, layers=2, heads=2, kv_heads=1, max_pos=64)


def test_generators_match_the_engine():
    assert np.array_equal(oracle.normal_f16(2, 1.0, 4099), ve.normal_f16(2, 1.0, 4099))
    assert np.array_equal(oracle.normal_f16(4, 0.02, 1000), ve.normal_f16(4, 0.02, 1000))
    assert np.array_equal(oracle.prompt(1, 49152, 32), ve.prompt(1, 49152, 32))
    assert np.array_equal(oracle.permutation(3, 513), ve.permutation(3, 513))
    assert np.array_equal(oracle.uniforms(9, 300), ve.uniforms(9, 300))


@pytest.mark.parametrize("kw", [dict(), dict(int8=True), dict(noise_seed=6, noise_std=0.004),
                                dict(tied=False)])
def test_synth_model_matches_the_written_model(tmp_path, kw):
    # Same draw order and rounding: the in-memory oracle model and the oracle loaded from
    # the engine-written safetensors generate identical tokens with identical margins.
    d = ve.synth_model(str(tmp_path / "m"), seed=7, **kw, **TINY)
    from_file = oracle.Model(d)
    in_memory = oracle.Model.synth(seed=7, **kw, **TINY)
    p = oracle.prompt(5, TINY["vocab"], 6)
    a, ma = from_file.generate(p, 12)
    b, mb = in_memory.generate(p, 12)
    assert np.array_equal(a, b) and np.array_equal(ma, mb)
    st1, st2 = from_file.state(16), in_memory.state(16)
    l1, t1 = st1.forward(int(p[0]), trace=True)
    l2, t2 = st2.forward(int(p[0]), trace=True)
    assert np.array_equal(l1, l2) and np.array_equal(t1, t2)


def test_stop_rules():
    m = oracle.Model.synth(seed=3, **TINY)
    p = oracle.prompt(2, TINY["vocab"], 5)
    full, _ = m.generate(p, 20)
    # No stop id: the same tokens as the plain loop.
    toks, _, hit = m.generate_stop(p, 20, eos=-1)
    assert np.array_equal(toks, full) and not hit
    # Stop id = the 8th token: generation ends at its first occurrence, inclusive.
    eos = int(full[7])
    first = int(np.argmax(full == eos))
    toks, _, hit = m.generate_stop(p, 20, eos=eos)
    assert hit and toks.size == first + 1 and np.array_equal(toks, full[: first + 1])
    # maxPos: seqLen + 1 >= max_pos ends the loop after max_pos - len(prompt) tokens.
    toks, _, hit = m.generate_stop(p, 20, max_pos=12, eos=-1)
    assert not hit and toks.size == 12 - p.size and np.array_equal(toks, full[: toks.size])


def test_batch_equals_one_at_a_time():
    m = oracle.Model.synth(seed=4, **TINY)
    prompts = [oracle.prompt(10 + s, TINY["vocab"], 3 + s % 4) for s in range(7)]
    out, counts, margins, second = m.generate_batch(prompts, 9, threads=3)
    for s, p in enumerate(prompts):
        want, mg = m.generate(p, 9)
        assert counts[s] == 9
        assert np.array_equal(out[s], want) and np.array_equal(margins[s], mg)
    # The runner-up of each step: the best other token, its logit margin behind the winner.
    st = m.state(32)
    lg = None
    for i, t in enumerate(prompts[0]):
        lg, _ = st.forward(int(t))
    order = np.argsort(-lg.astype(np.float64), kind="stable")
    assert order[0] == out[0][0] and order[1] == second[0][0]
    assert np.float32(lg[order[0]] - lg[order[1]]) == margins[0][0]
