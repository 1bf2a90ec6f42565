"""CPU restatement of the speculative decoding loop (test infrastructure: the checker of
the GPU loop in tests/ and the CPU baseline of the config-3 bench; never product code).

Follows the engine's SpecGenerate contract (opure-voxelengine_b200/host/spec_decode.h)
sequence by sequence on the oracle's scalar forward: the draft proposes k tokens from
position p (after recomputing position p-1), the target evaluates positions p..p+k, and
oracle.spec_accept_* decides; both states are rolled back by truncation. Uniforms come
from the harness Rng (Opure_TestHarness.cpp:36-47) seeded per sequence as
seed ^ (s * 0x9E3779B97F4A7C15), drawn per round as u_draft[k], u_accept[k], u_final.
"""
import numpy as np

import oracle

GOLDEN = 0x9E3779B97F4A7C15
MASK = (1 << 64) - 1


class Rng:
    def __init__(self, seed: int):
        self.s = (seed & MASK) or 1

    def u32(self) -> int:
        s = self.s
        s ^= (s << 13) & MASK
        s ^= s >> 7
        s ^= (s << 17) & MASK
        self.s = s
        return s >> 32

    def uniform(self) -> float:
        return float(np.float32(self.u32() / 4294967296.0))


def argmax(logits) -> int:
    return int(oracle.argmax(np.asarray(logits, np.float32)[None])[0][0])


def spec_generate(target: oracle.Model, draft: oracle.Model, prompts, budget: int, k: int,
                  rejection: bool, seed: int = 0, threads: int = 1, records: bool = False):
    """Returns (tokens [n][budget], accept counts per round [n][rounds]), and with
    records=True also per sequence a list of per-round records: the drafted tokens, the
    accepted count, the emitted tokens and (rejection) each draft's acceptance ratio
    u_accept * q(d) / p(d) (accepted when <= 1). With threads > 1 the sequences run
    concurrently on host threads, each computing serially (the models are only read;
    every sequence has its own states and uniform stream)."""
    if threads > 1 and len(prompts) > 1:
        from concurrent.futures import ThreadPoolExecutor

        def one(s):
            oracle.thread_serial(True)
            return _spec_one(target, draft, s, prompts[s], budget, k, rejection, seed)
        with ThreadPoolExecutor(max_workers=min(threads, len(prompts))) as ex:
            res = list(ex.map(one, range(len(prompts))))
    else:
        res = [_spec_one(target, draft, s, p, budget, k, rejection, seed) for s, p in enumerate(prompts)]
    out = (np.array([r[0] for r in res], np.int32), [r[1] for r in res])
    return out + ([r[2] for r in res],) if records else out


def _prob(logits, i: int) -> float:
    """softmax(logits)[i] in double."""
    z = np.asarray(logits, np.float64)
    e = np.exp(z - z.max())
    return float(e[i] / e.sum())


def _spec_one(target, draft, s, prompt, budget, k, rejection, seed):
    """One sequence of the loop (sequence index s picks its uniform stream)."""
    rng = Rng(seed ^ ((s * GOLDEN) & MASK))
    p0 = len(prompt)
    cap = p0 + budget + k + 2
    ts, ds = target.state(cap), draft.state(cap)
    lt = None
    for i, tok in enumerate(prompt):
        lt, _ = ts.forward(int(tok), logits=(i == p0 - 1))
        ds.forward(int(tok), logits=False)
    first = oracle.sample_softmax(lt, rng.uniform()) if rejection else argmax(lt)
    out, log, recs = [first], [], []
    p, t, prev = p0, first, int(prompt[-1])
    while len(out) < budget:
        ud = [rng.uniform() for _ in range(k)] if rejection else None
        ua = [rng.uniform() for _ in range(k)] if rejection else None
        uf = rng.uniform() if rejection else None
        ds.truncate(p - 1)
        ds.forward(prev, logits=False)
        drafts, dlog, cur = [], [], t
        for j in range(k):
            lq, _ = ds.forward(cur)
            d = oracle.sample_softmax(lq, ud[j]) if rejection else argmax(lq)
            drafts.append(d)
            dlog.append(lq)
            cur = d
        ts.truncate(p)
        tl = np.stack([ts.forward(tok)[0] for tok in [t] + drafts])
        if rejection:
            a, toks = oracle.spec_accept_rejection(tl, np.stack(dlog), np.array(drafts), np.array(ua, np.float32), uf)
        else:
            a, toks = oracle.spec_accept_greedy(tl, np.array(drafts))
        log.append(int(a))
        rec = {"drafts": [int(d) for d in drafts], "a": int(a), "emitted": [int(x) for x in toks[: a + 1]]}
        if rejection:
            rec["ratios"] = [float(ua[j]) * _prob(dlog[j], drafts[j]) / max(_prob(tl[j], drafts[j]), 1e-300)
                             for j in range(k)]
        recs.append(rec)
        for i in range(a + 1):
            if len(out) < budget:
                out.append(int(toks[i]))
        prev = int(toks[a - 1]) if a > 0 else t
        t = int(toks[a])
        p += a + 1
    return out, log, recs
