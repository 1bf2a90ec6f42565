"""The lane arithmetic of the persistent step's eight-row lm_head reduction, restated in
numpy float32 (no GPU).

`lm_dot8` in csrc/decode.cu reduces the eight per-lane row sums of a warp together: at the
xor-16 level each lane keeps four rows and sends the other four, at xor 8 two, at xor 4
one, then two plain levels; lane l ends with row (l >> 2) & 7. Its tokens are compared
with the oracle's by the GPU engine tests; this file checks the claim that lets it replace
eight `warp_sum`s without changing any logit: every level adds the same pair of partial
sums as `warp_sum` (v += shfl_xor(v, o) for o = 16, 8, 4, 2, 1), so each row's total is
bit-identical.
"""
import numpy as np

LANES = np.arange(32)


def warp_sum_rows(acc):
    s = acc.copy()
    for o in (16, 8, 4, 2, 1):
        s = (s + s[LANES ^ o]).astype(np.float32)
    return s


def lm_dot8_reduce(acc):
    b4, b3, b2 = (LANES & 16) != 0, (LANES & 8) != 0, (LANES & 4) != 0
    u = np.zeros((32, 4), np.float32)
    for i in range(4):
        send = np.where(b4, acc[:, i], acc[:, i + 4])
        u[:, i] = np.where(b4, acc[:, i + 4], acc[:, i]) + send[LANES ^ 16]
    t = np.zeros((32, 2), np.float32)
    for i in range(2):
        send = np.where(b3, u[:, i], u[:, i + 2])
        t[:, i] = np.where(b3, u[:, i + 2], u[:, i]) + send[LANES ^ 8]
    send = np.where(b2, t[:, 0], t[:, 1])
    x = (np.where(b2, t[:, 1], t[:, 0]) + send[LANES ^ 4]).astype(np.float32)
    x = (x + x[LANES ^ 2]).astype(np.float32)
    return (x + x[LANES ^ 1]).astype(np.float32)


def test_transposed_reduction_is_bit_identical_to_warp_sum():
    rng = np.random.default_rng(5)
    row = (LANES >> 2) & 7
    for _ in range(500):
        scale = rng.choice([1e-3, 1.0, 1e3])
        acc = (rng.standard_normal((32, 8)) * scale).astype(np.float32)
        want = warp_sum_rows(acc)[LANES, row]
        got = lm_dot8_reduce(acc)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
