"""opure_attention_static: attention for callers that may not allocate device memory.

Some hosts cannot call cudaMalloc from library code: a plugin whose host application owns
the GPU memory budget, or a real-time decode loop that cannot stall on an allocation (which
synchronises the device). opure_attention_static takes the same inputs and outputs as
opure_attention but keeps its split partials in a fixed buffer inside the library. This file
runs last (pytest collects it after the others) and must pass on its own or after them: two
calls in a row, different shapes, each checked against opure_attention on the same inputs
and against the CPU oracle.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from common import rel_err
from voxelengine import cuda as cu

pytestmark = pytest.mark.gpu
STATIC_LIMIT = 8 << 20  # OPURE_ATTN_STATIC_SCRATCH_BYTES


@pytest.fixture(scope="module")
def ctx():
    c = cu.Ctx(0)
    yield c
    c.close()


def problem(ctx, B, ctxlen, page, seed, nh=9, nkv=3, hd=64):
    rng = np.random.default_rng(seed)
    maxp = -(-ctxlen // page)
    npages = B * maxp + 3
    perm = rng.permutation(npages)[: B * maxp].reshape(B, maxp).astype(np.int32)
    pool = oracle.f32_to_f16(rng.standard_normal((npages, 2, nkv, page, hd)).astype(np.float32))
    q = rng.standard_normal((B, 1, nh, hd)).astype(np.float32)
    lens = np.array([ctxlen - 13 * b for b in range(B)], np.int32)
    bufs = dict(q=ctx.to_device(q), pool=ctx.to_device(pool), pt=ctx.to_device(perm),
                seq=ctx.to_device(np.arange(B, dtype=np.int32)), len=ctx.to_device(lens))
    a = cu.AttnArgs()
    a.q, a.seq, a.seq_len = bufs["q"].ptr, bufs["seq"].ptr, bufs["len"].ptr
    a.n, a.n_q, a.n_heads, a.scale, a.max_ctx = B, 1, nh, 1.0, int(lens.max())
    a.kv = cu.KvLayout(bufs["pool"].ptr, bufs["pt"].ptr, npages, maxp, page, nkv, hd)
    want = oracle.attention_paged(q, pool, perm, lens, page, nh, nkv, hd)
    return a, q.shape, bufs, want


def run(ctx, a, shape, static):
    out = ctx.buffer(int(np.prod(shape)) * 4).fill(0xFF)
    a.out = out.ptr
    if static:
        a.scratch, a.scratch_bytes = None, 0
        cu.check(cu.lib().opure_attention_static(ctx.h, C.byref(a)), "opure_attention_static")
    else:
        sb = cu.attention_scratch_bytes(a.n, a.n_q, a.n_heads, a.kv.n_kv, a.kv.head_dim, a.max_ctx)
        scratch = ctx.buffer(sb).fill(0)
        a.scratch, a.scratch_bytes = scratch.ptr, sb
        ctx.attention(a)
    got = out.download(np.float32, shape)
    assert ctx.last_error() == 0
    return got


def test_static_scratch_matches_allocating_entry_point_twice(ctx):
    # Two calls in a row with different shapes: the second must not see the first's
    # leftover counters or partials.
    for B, L, page, seed in ((3, 1000, 16, 1), (8, 2048, 64, 2)):
        a, shape, _, want_cpu = problem(ctx, B, L, page, seed)
        want = run(ctx, a, shape, static=False)
        got = run(ctx, a, shape, static=True)
        assert not np.isnan(got).any()
        assert rel_err(got, want) < 1e-3
        assert rel_err(got, want_cpu) < 1e-3


def test_static_scratch_refuses_oversized_calls(ctx):
    # 4096 entries: far more (entry, kv head, split) partials than the fixed buffer holds.
    # Every input and output is sized for all 4096 entries (each reads sequence 0's one
    # page), so even a call that were wrongly accepted would stay inside its buffers.
    n, nh, hd = 4096, 9, 64
    a, _, bufs, _ = problem(ctx, 1, 64, 64, 3)
    q = ctx.to_device(np.zeros((n, 1, nh, hd), np.float32))
    seq = ctx.to_device(np.zeros(n, np.int32))
    lens = ctx.to_device(np.full(n, 64, np.int32))
    out = ctx.buffer(n * nh * hd * 4)
    a.q, a.seq, a.seq_len, a.out, a.n = q.ptr, seq.ptr, lens.ptr, out.ptr, n
    need = cu.attention_scratch_bytes(a.n, 1, a.n_heads, 3, 64, a.max_ctx)
    assert need > STATIC_LIMIT
    st = cu.lib().opure_attention_static(ctx.h, C.byref(a))
    assert st == cu.ERR_UNSUPPORTED
    assert ctx.last_error() == 0
