"""CPU checks of the oracle's sliding window (orc_state_set_window), the checker of the
engine's ring-of-pages KV cache: a window at least as long as the sequence changes
nothing; a short one changes the logits exactly from the first position whose window
no longer starts at 0."""
import numpy as np
import pytest

import oracle
from voxelengine import engine as ve

SMALL = dict(vocab=512, hidden=128, inter=256, layers=2, heads=4, kv_heads=2, max_pos=256)


@pytest.fixture(scope="module")
def small(tmp_path_factory):
    return oracle.Model(ve.synth_model(str(tmp_path_factory.mktemp("win") / "m"), seed=3, **SMALL))


def run(small, tokens, page=0, ring=0):
    st = small.state(len(tokens) + 1)
    if ring:
        st.set_window(page, ring)
    return [st.forward(int(t))[0] for t in tokens]


def test_long_window_is_no_window(small):
    toks = ve.prompt(1, SMALL["vocab"], 40)
    a, b = run(small, toks), run(small, toks, 16, 3)  # 48 tokens of window >= 40
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_short_window_starts_after_the_ring_fills(small):
    toks = ve.prompt(2, SMALL["vocab"], 60)
    page, ring = 8, 3
    a, b = run(small, toks), run(small, toks, page, ring)
    # Position t sees [max(0, t // page - ring + 1) * page, t]: identical logits while that
    # start is 0 (t < ring * page), different afterwards.
    for t in range(len(toks)):
        same = np.array_equal(a[t], b[t])
        assert same == (t < ring * page), t
