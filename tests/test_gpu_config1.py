"""BASELINE config 1 at its own sizes: paged flash-decode attention, 9 query heads / 3 KV
heads, head_dim 64, fp16 Q/K/V drawn N(0, 1) from seed 2, page size 64, the page table a
seeded permutation (seed 3) of the physical pages, against the CPU oracle.

Seed-2 stream order: the queries [B][9][64], then the page pool in memory order
[page][K|V][kv head][slot][dim]. Contexts of 8192 and 32768 tokens run the split-K
path with 3072-token splits (the split policy's long-context rule); each sequence's
length is the configuration's context minus a small per-sequence offset, so splits end
mid-page. Gate: max error <= 1e-3 x max|oracle| (the per-kernel relative gate).
"""
import os

import numpy as np
import pytest

import oracle
from common import rel_err
from voxelengine import cuda as cu

pytestmark = pytest.mark.gpu
oracle.set_threads(os.cpu_count() or 1)
NH, NKV, HD, P = 9, 3, 64, 64
REL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    c = cu.Ctx(0)
    yield c
    c.close()


def config1_inputs(B, ctxlen):
    pages = B * (ctxlen // P)
    n_q = B * NH * HD
    draws = oracle.normal_f16(2, 1.0, n_q + pages * 2 * NKV * P * HD)
    q = oracle.f16_to_f32(draws[:n_q]).reshape(B, 1, NH, HD)
    pool = draws[n_q:].reshape(pages, 2, NKV, P, HD)
    table = oracle.permutation(3, pages).reshape(B, ctxlen // P)
    lens = np.array([ctxlen - (b * 13) % 97 for b in range(B)], np.uint32)
    return q, pool, table, lens


def run_attention(ctx, q, pool, table, lens, split_tokens=0):
    B = q.shape[0]
    max_ctx = int(lens.max())
    dq, dp, dpt = ctx.to_device(q), ctx.to_device(pool), ctx.to_device(table.astype(np.int32))
    dseq = ctx.to_device(np.arange(B, dtype=np.int32))
    dlen = ctx.to_device(lens.astype(np.int32))
    dout = ctx.buffer(q.size * 4).fill(0xFF)
    a = cu.AttnArgs()
    a.q, a.out, a.seq, a.seq_len = dq.ptr, dout.ptr, dseq.ptr, dlen.ptr
    a.n, a.n_q, a.n_heads, a.scale, a.max_ctx = B, 1, NH, 1.0, max_ctx
    a.kv = cu.KvLayout(dp.ptr, dpt.ptr, pool.shape[0], table.shape[1], P, NKV, HD)
    a.split_tokens = split_tokens
    sb = cu.attention_scratch_bytes(B, 1, NH, NKV, HD, max_ctx, split_tokens)
    scratch = ctx.buffer(sb).fill(0)
    a.scratch, a.scratch_bytes = scratch.ptr, sb
    ctx.attention(a)
    out = dout.download(np.float32, q.shape)
    assert ctx.last_error() == 0
    for b in (dq, dp, dpt, dseq, dlen, dout, scratch):
        b.free()
    return out


@pytest.mark.parametrize("B,ctxlen", [(8, 8192), (8, 32768), (64, 8192), (64, 32768)])
def test_config1_attention_matches_oracle(ctx, B, ctxlen):
    q, pool, table, lens = config1_inputs(B, ctxlen)
    got = run_attention(ctx, q, pool, table, lens)
    want = oracle.attention_paged(q, pool, table, lens, P, NH, NKV, HD)
    assert not np.isnan(got).any()
    err = rel_err(got, want)
    assert err < REL, err


def test_config1_forced_short_splits(ctx):
    # The same data through 128-token splits: many more partial states to merge.
    q, pool, table, lens = config1_inputs(8, 8192)
    got = run_attention(ctx, q, pool, table, lens, split_tokens=128)
    want = oracle.attention_paged(q, pool, table, lens, P, NH, NKV, HD)
    assert rel_err(got, want) < REL
