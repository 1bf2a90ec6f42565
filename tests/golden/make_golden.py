"""Regenerates tests/golden/harness_kats.npz.

The reference ships no golden files: its known-answer tests are the seeded,
generated kernel tests of src/app/Opure_TestHarness.cpp, which draw inputs from a
xorshift64 `Rng` (:36-47) and compute the expected values inline, in fp32, next to
each GPU dispatch. This script restates both -- the Rng in pure Python (independent
of the C oracle's own Rng) and each inline expectation with float32 scalar arithmetic
in the harness's operation order -- and stores inputs and expectations:

  gemv      TestGEMV        :1176-1229  64x128, seed 0xC0FFEE01
  gemvq     TestGEMVQuant   :1244-1311  64x128 int8, scaleW 0.0137, seed 0x9A17BEEF
  rms       TestRMSNorm     :1314-1361  d 256, eps 1e-5, seed 0xBADF00D2
  swiglu    TestSwiGLU      :1364-1400  n 64, seed 0x5EED1234
  add       TestAdd         :1403-1433  n 64, seed 0x77777777
  addres    TestAddRes      :1554-1586  n 64, seed 0xADDE5EED
  argmax    TestArgMax      :1436-1471  49152, seed 0x13571357
  attn{hd}  TestAttentionAt :1479-1547  4 q heads, 2 kv heads, 7 keys, maxSeq 64,
                                         seed 0xABCDEF01 ^ (hd * 2654435761) (uint32)

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os

import numpy as np

F = np.float32
HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "harness_kats.npz")
MASK64 = (1 << 64) - 1


class Rng:
    """Opure_TestHarness.cpp:36-47."""

    def __init__(self, seed: int):
        self.s = seed if seed else 1

    def next_u32(self) -> int:
        s = self.s
        s ^= (s << 13) & MASK64
        s ^= s >> 7
        s ^= (s << 17) & MASK64
        self.s = s
        return s >> 32

    def next_f(self) -> np.float32:
        # static_cast<float>(u32) / 2147483648.0f - 1.0f, each step rounded to float.
        return F(F(self.next_u32()) / F(2147483648.0)) - F(1.0)

    def fill(self, n: int, mul: float = 1.0, add: float = 0.0) -> np.ndarray:
        out = np.empty(n, F)
        m, a = F(mul), F(add)
        for i in range(n):
            v = self.next_f()
            if mul != 1.0:
                v = F(v * m)
            if add != 0.0:
                v = F(v + a)
            out[i] = v
        return out


def gemv():
    rng = Rng(0xC0FFEE01)
    W = rng.fill(64 * 128).reshape(64, 128)
    X = rng.fill(128)
    ref = np.empty(64, F)
    for o in range(64):
        acc = F(0.0)
        for i in range(128):
            acc = F(acc + F(W[o, i] * X[i]))
        ref[o] = acc
    return dict(gemv_W=W, gemv_X=X, gemv_ref=ref)


def gemvq():
    rng = Rng(0x9A17BEEF)
    q = np.empty(64 * 128, np.int8)
    for n in range(q.size):
        v = int(F(rng.next_f() * F(127.0)))  # truncation toward zero, as static_cast<int>
        v -= 63
        q[n] = ((v + 128) & 0xFF) - 128       # static_cast<int8_t>: two's-complement wrap
    q = q.reshape(64, 128)
    X = np.empty(128, F)
    for i in range(128):
        X[i] = F(F(rng.next_f() * F(2.0)) - F(1.0))
    sw, sx = F(0.0137), F(1.0)
    ref = np.empty(64, F)
    for o in range(64):
        acc = F(0.0)
        for i in range(128):
            acc = F(acc + F(F(q[o, i]) * X[i]))
        ref[o] = F(F(acc * sw) * sx)
    return dict(gemvq_q=q, gemvq_X=X, gemvq_ref=ref, gemvq_scale_w=np.array(sw))


def rms():
    rng = Rng(0xBADF00D2)
    X = rng.fill(256)
    G = rng.fill(256, mul=0.5)
    ss = 0.0
    for i in range(256):
        ss += float(X[i]) * float(X[i])  # double accumulation
    eps = F(1e-5)
    inv = F(F(1.0) / F(np.sqrt(F(F(ss / 256) + eps))))
    ref = np.array([F(F(X[i] * inv) * G[i]) for i in range(256)], F)
    return dict(rms_X=X, rms_G=G, rms_ref=ref, rms_eps=np.array(eps))


def swiglu():
    rng = Rng(0x5EED1234)
    G = rng.fill(64, mul=3.0)
    U = rng.fill(64)
    ref = np.empty(64, F)
    for i in range(64):
        s = F(F(1.0) / F(F(1.0) + np.exp(-G[i])))
        ref[i] = F(F(G[i] * s) * U[i])
    return dict(swiglu_G=G, swiglu_U=U, swiglu_ref=ref)


def add():
    rng = Rng(0x77777777)
    A = rng.fill(64)
    B = rng.fill(64)
    return dict(add_A=A, add_B=B, add_ref=(A + B).astype(F))


def addres():
    rng = Rng(0xADDE5EED)
    X = rng.fill(64, mul=2.0, add=-1.0)
    R = rng.fill(64, mul=2.0, add=-1.0)
    return dict(addres_X=X, addres_R=R, addres_ref=(X + R).astype(F))


def argmax():
    rng = Rng(0x13571357)
    L = rng.fill(49152, mul=5.0)
    best, bi = F(-1e30), 0
    for i in range(L.size):
        if L[i] > best:
            best, bi = L[i], i
    return dict(argmax_L=L, argmax_val=np.array(best), argmax_idx=np.array(bi, np.uint32))


def attention(hd: int):
    nh, nkv, nseq, nmax = 4, 2, 7, 64
    seed = 0xABCDEF01 ^ ((hd * 2654435761) & 0xFFFFFFFF)
    rng = Rng(seed)
    Q = rng.fill(nh * hd).reshape(nh, hd)
    K = rng.fill(nkv * nmax * hd).reshape(nkv, nmax, hd)
    V = rng.fill(nkv * nmax * hd).reshape(nkv, nmax, hd)
    ref = np.zeros((nh, hd), F)
    group = nh // nkv
    for h in range(nh):
        kvh = h // group
        m, l = F(-1e30), F(0.0)
        acc = np.zeros(hd, F)
        for s in range(nseq):
            score = F(0.0)
            for d in range(hd):
                score = F(score + F(Q[h, d] * K[kvh, s, d]))
            nm = m if m > score else score
            corr = F(0.0) if m <= F(-1e29) else F(np.exp(F(m - nm)))
            pv = F(np.exp(F(score - nm)))
            l = F(F(l * corr) + pv)
            acc = (acc * corr).astype(F) + (pv * V[kvh, s]).astype(F)
            acc = acc.astype(F)
            m = nm
        ref[h] = (acc / l).astype(F)
    p = f"attn{hd}_"
    return {p + "Q": Q, p + "K": K, p + "V": V, p + "ref": ref}


def main():
    data = {}
    for fn in (gemv, gemvq, rms, swiglu, add, addres, argmax):
        data.update(fn())
    for hd in (32, 64, 96, 128, 160, 192, 224, 256):
        data.update(attention(hd))
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    main()
