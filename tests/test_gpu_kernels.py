"""CUDA kernels vs the CPU oracle, through the C ABI (libopure_cuda.so).

Each test mirrors one of the reference harness's kernel tests
(src/app/Opure_TestHarness.cpp) or one BASELINE config, runs the sm_100a kernel through
its extern "C" entry point, and compares with the oracle on the same inputs:
  - the harness's own criterion (Compare, :70-101) where the kernel's inputs are exact;
  - the per-kernel gate, max error <= 1e-3 x max|reference|, everywhere;
  - bit-exact for indices (ArgMax, accept/reject decisions, sampled tokens).
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from common import compare, kats, rel_err
from voxelengine import cuda as cu

pytestmark = pytest.mark.gpu
REL = 1e-3          # per-kernel relative gate
K = kats()


@pytest.fixture(scope="module")
def ctx():
    c = cu.Ctx(0)
    yield c
    c.close()


def f16(a):
    return oracle.f32_to_f16(np.asarray(a, np.float32))


def gemv_gpu(ctx, w, x, dtype=cu.W_F16, scale=1.0, pro=cu.PRO_NONE, gain=None, eps=1e-5,
             epi=cu.EPI_STORE, residual=None, rows=None):
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    nvec, cols = x.shape
    rows = rows if rows is not None else w.shape[0]
    dw, dx = ctx.to_device(w), ctx.to_device(x)
    dy = ctx.buffer(nvec * rows * 4).fill(0xFF)
    a = cu.GemvArgs()
    a.w, a.w_dtype, a.scale_w, a.scale_x = dw.ptr, dtype, scale, 1.0
    a.rows, a.cols, a.nvec = rows, cols, nvec
    a.x, a.x_stride, a.y, a.y_stride = dx.ptr, cols, dy.ptr, rows
    a.prologue, a.epilogue, a.eps = pro, epi, eps
    if gain is not None:
        a.norm_gain = ctx.to_device(gain).ptr
    if residual is not None:
        a.residual = ctx.to_device(np.ascontiguousarray(residual, np.float32)).ptr
    keys = None
    if epi == cu.EPI_ARGMAX:
        keys = ctx.buffer(8 * nvec).fill(0)
        a.argmax_keys = keys.ptr
    ctx.gemv(a)
    y = dy.download(np.float32, (nvec, rows))
    assert ctx.last_error() == 0
    if keys is not None:
        idx = ctx.buffer(4 * nvec)
        ctx.call("opure_argmax_decode", C.c_void_p(keys.ptr), nvec, C.c_void_p(idx.ptr), None)
        return y, idx.download(np.uint32, nvec)
    return y


# ---- reference harness KATs ------------------------------------------------------
def test_gemv_kat(ctx):
    # TestGEMV 64x128 (:1176-1229). The kernel streams fp16 weights, so W is rounded
    # to fp16 and the oracle runs on the same values.
    w = f16(K["gemv_W"])
    y = gemv_gpu(ctx, w, K["gemv_X"])[0]
    want = oracle.gemv_f16(w, K["gemv_X"])
    ok, *_ = compare(y, want)
    assert ok and rel_err(y, want) < REL


def test_gemv_quant_kat(ctx):
    # TestGEMVQuant (:1244-1311): exact int8 inputs, so the harness's own expectation
    # applies directly.
    q = K["gemvq_q"]
    sw = float(K["gemvq_scale_w"])
    y = gemv_gpu(ctx, q, K["gemvq_X"], dtype=cu.W_Q8, scale=sw)[0]
    ok, max_abs, rms = compare(y, K["gemvq_ref"])
    assert ok, (max_abs, rms)
    assert rel_err(y, oracle.gemv_q8(q, sw, K["gemvq_X"])) < REL


def test_rmsnorm_kat(ctx):
    x, g = K["rms_X"], f16(K["rms_G"])
    dx, dg, dy = ctx.to_device(x), ctx.to_device(g), ctx.buffer(x.nbytes).fill(0xFF)
    ctx.call("opure_rmsnorm", C.c_void_p(dx.ptr), C.c_void_p(dg.ptr), C.c_void_p(dy.ptr),
             x.size, 1, float(K["rms_eps"]))
    y = dy.download(np.float32, x.shape)
    want = oracle.rmsnorm(x, oracle.f16_to_f32(g), float(K["rms_eps"]))
    ok, *_ = compare(y, want)
    assert ok and rel_err(y, want) < REL


def test_swiglu_kat(ctx):
    g, u = K["swiglu_G"], K["swiglu_U"]
    dg, du, dh = ctx.to_device(g), ctx.to_device(u), ctx.buffer(g.nbytes).fill(0xFF)
    ctx.call("opure_swiglu", C.c_void_p(dg.ptr), C.c_void_p(du.ptr), C.c_void_p(dh.ptr), g.size)
    h = dh.download(np.float32, g.shape)
    ok, max_abs, rms = compare(h, K["swiglu_ref"])
    assert ok, (max_abs, rms)


@pytest.mark.parametrize("name", ["add", "addres"])
def test_add_kat(ctx, name):
    a, b = (K["add_A"], K["add_B"]) if name == "add" else (K["addres_X"], K["addres_R"])
    da, db, dd = ctx.to_device(a), ctx.to_device(b), ctx.buffer(a.nbytes).fill(0xFF)
    ctx.call("opure_add", C.c_void_p(da.ptr), C.c_void_p(db.ptr), C.c_void_p(dd.ptr), a.size)
    assert np.array_equal(dd.download(np.float32, a.shape), K[f"{name}_ref"])


def test_argmax_kat(ctx):
    L = K["argmax_L"]
    dl, di, dv = ctx.to_device(L), ctx.buffer(4), ctx.buffer(4)
    ctx.call("opure_argmax", C.c_void_p(dl.ptr), L.size, 1, C.c_void_p(di.ptr), C.c_void_p(dv.ptr))
    assert di.download(np.uint32, 1)[0] == K["argmax_idx"]
    assert dv.download(np.float32, 1)[0] == K["argmax_val"]


def test_argmax_ties_nan_rows(ctx):
    x = np.zeros((3, 4096), np.float32)
    x[0, [7, 4000, 9]] = 5.0            # tie: lowest index wins
    x[1, :] = np.nan
    x[1, 123] = -1.0                     # NaN never wins
    x[2, 4095] = 1e-30
    dl, di, dv = ctx.to_device(x), ctx.buffer(12), ctx.buffer(12)
    ctx.call("opure_argmax", C.c_void_p(dl.ptr), 4096, 3, C.c_void_p(di.ptr), C.c_void_p(dv.ptr))
    idx = di.download(np.uint32, 3)
    want, _ = oracle.argmax(x)
    assert list(idx) == list(want) == [7, 123, 4095]


def paged_from_planes(k_plane, v_plane, page_size, perm):
    """Scatter [n_kv][S][hd] planes into the page pool through page table `perm`."""
    n_kv, S, hd = k_plane.shape
    npages = -(-S // page_size)
    pool = np.zeros((int(perm.max()) + 1, 2, n_kv, page_size, hd), np.uint16)
    for lp in range(npages):
        n = min(page_size, S - lp * page_size)
        pool[perm[lp], 0, :, :n] = f16(k_plane[:, lp * page_size: lp * page_size + n])
        pool[perm[lp], 1, :, :n] = f16(v_plane[:, lp * page_size: lp * page_size + n])
    return pool


def attention_gpu(ctx, q, pool, page_table, seq_lens, page_size, n_heads, n_kv, hd,
                  n_q=1, scale=1.0, split_tokens=0):
    """q [n, n_q, n_heads, hd]; pool uint16 page pool; page_table [n, max_pages]."""
    n = q.shape[0]
    max_ctx = int(np.max(seq_lens)) + n_q - 1
    dq, dp = ctx.to_device(q.astype(np.float32)), ctx.to_device(pool)
    dpt = ctx.to_device(page_table.astype(np.int32))
    dseq = ctx.to_device(np.arange(n, dtype=np.int32))
    dlen = ctx.to_device(np.asarray(seq_lens, np.int32))
    dout = ctx.buffer(q.size * 4).fill(0xFF)
    sb = cu.attention_scratch_bytes(n, n_q, n_heads, n_kv, hd, max_ctx, split_tokens)
    scratch = ctx.buffer(sb).fill(0)
    a = cu.AttnArgs()
    a.q, a.out, a.seq, a.seq_len = dq.ptr, dout.ptr, dseq.ptr, dlen.ptr
    a.n, a.n_q, a.n_heads, a.scale, a.max_ctx = n, n_q, n_heads, scale, max_ctx
    a.split_tokens, a.scratch, a.scratch_bytes = split_tokens, scratch.ptr, sb
    a.kv = cu.KvLayout(dp.ptr, dpt.ptr, pool.shape[0], page_table.shape[1], page_size, n_kv, hd)
    ctx.attention(a)
    out = dout.download(np.float32, q.shape)
    assert ctx.last_error() == 0
    return out


@pytest.mark.parametrize("hd", [32, 64, 96, 128, 160, 192, 224, 256])
def test_attention_kat(ctx, hd):
    # TestAttentionAt (:1479-1547): 4 q heads, 2 kv heads, 7 keys, maxSeq 64. The
    # cache is fp16 here, so K/V are rounded and the oracle sees the same values.
    p = f"attn{hd}_"
    Q, Kp, Vp = K[p + "Q"], K[p + "K"], K[p + "V"]
    perm = np.array([0], np.int32)
    pool = paged_from_planes(Kp[:, :7], Vp[:, :7], 64, perm)
    got = attention_gpu(ctx, Q[None, None], pool, perm[None], [7], 64, 4, 2, hd)[0, 0]
    want = oracle.attention_paged(Q[None, None], pool, perm[None], [7], 64, 4, 2, hd)[0, 0]
    ok, *_ = compare(got, want)
    assert ok and rel_err(got, want) < REL
    # Against the harness's own fp32 expectation the only extra error is the fp16 cache.
    assert rel_err(got, K[p + "ref"]) < 2e-2


# ---- paged attention (small points; full sweep in bench) --------
@pytest.mark.parametrize("B,ctxlen,page", [(1, 512, 64), (8, 2048, 64), (3, 1000, 16),
                                           (2, 300, 128), (1, 5, 32)])
def test_paged_attention_permuted(ctx, B, ctxlen, page):
    rng = np.random.default_rng(B * 7919 + ctxlen)
    nh, nkv, hd = 9, 3, 64
    maxp = -(-ctxlen // page)
    npages = B * maxp + 5
    perm = rng.permutation(npages)[: B * maxp].reshape(B, maxp).astype(np.int32)
    pool = f16(rng.standard_normal((npages, 2, nkv, page, hd)).astype(np.float32))
    q = rng.standard_normal((B, 1, nh, hd)).astype(np.float32)
    lens = np.array([ctxlen - (b * 37) % max(ctxlen // 2, 1) for b in range(B)], np.int32)
    got = attention_gpu(ctx, q, pool, perm, lens, page, nh, nkv, hd)
    want = oracle.attention_paged(q, pool, perm, lens, page, nh, nkv, hd)
    assert rel_err(got, want) < REL


@pytest.mark.parametrize("page", [16, 64, 128])
def test_attention_masks_poisoned_tail(ctx, page):
    # Every pool byte outside the sequences' tokens is NaN (fp16 0xFFFF): whole pages are
    # staged into shared memory, so masked rows must contribute nothing, not NaN * 0.
    rng = np.random.default_rng(page)
    B, nh, nkv, hd = 3, 9, 3, 64
    lens = np.array([1, page + 3, 5 * page - 1], np.int32)
    maxp = -(-int(lens.max()) // page)
    npages = B * maxp + 2
    perm = rng.permutation(npages)[: B * maxp].reshape(B, maxp).astype(np.int32)
    pool = np.full((npages, 2, nkv, page, hd), 0xFFFF, np.uint16)
    for b in range(B):
        for t in range(int(lens[b])):
            pg, r = perm[b, t // page], t % page
            pool[pg, :, :, r] = f16(rng.standard_normal((2, nkv, hd)).astype(np.float32))
    q = rng.standard_normal((B, 1, nh, hd)).astype(np.float32)
    got = attention_gpu(ctx, q, pool, perm, lens, page, nh, nkv, hd)
    want = oracle.attention_paged(q, pool, perm, lens, page, nh, nkv, hd)
    assert not np.isnan(got).any()
    assert rel_err(got, want) < REL


def test_attention_large_batch_long_context(ctx):
    # Config-1 shape at a size the oracle finishes quickly: 64 sequences, several splits.
    rng = np.random.default_rng(77)
    B, nh, nkv, hd, page, L = 64, 9, 3, 64, 64, 1024
    maxp = L // page
    perm = rng.permutation(B * maxp).reshape(B, maxp).astype(np.int32)
    pool = f16(rng.standard_normal((B * maxp, 2, nkv, page, hd)).astype(np.float32))
    q = rng.standard_normal((B, 1, nh, hd)).astype(np.float32)
    lens = np.array([L - (b * 29) % 700 for b in range(B)], np.int32)
    got = attention_gpu(ctx, q, pool, perm, lens, page, nh, nkv, hd)
    want = oracle.attention_paged(q, pool, perm, lens, page, nh, nkv, hd)
    assert rel_err(got, want) < REL


def test_attention_multi_query_causal(ctx):
    # Speculative verify: 5 queries, query j sees seq_len + j keys.
    rng = np.random.default_rng(11)
    B, nq, nh, nkv, hd, page, L = 2, 5, 9, 3, 64, 16, 70
    maxp = -(-(L + nq) // page)
    perm = rng.permutation(B * maxp).reshape(B, maxp).astype(np.int32)
    pool = f16(rng.standard_normal((B * maxp, 2, nkv, page, hd)).astype(np.float32) * 0.5)
    q = rng.standard_normal((B, nq, nh, hd)).astype(np.float32)
    lens = np.array([L, L - 9], np.int32)
    got = attention_gpu(ctx, q, pool, perm, lens, page, nh, nkv, hd, n_q=nq)
    want = oracle.attention_paged(q, pool, perm, lens, page, nh, nkv, hd)
    assert rel_err(got, want) < REL


def test_attention_forced_splits_and_scale(ctx):
    rng = np.random.default_rng(5)
    B, nh, nkv, hd, page, L = 2, 8, 8, 128, 64, 1500
    maxp = -(-L // page)
    perm = rng.permutation(B * maxp).reshape(B, maxp).astype(np.int32)
    pool = f16(rng.standard_normal((B * maxp, 2, nkv, page, hd)).astype(np.float32))
    q = rng.standard_normal((B, 1, nh, hd)).astype(np.float32)
    lens = np.array([L, 777], np.int32)
    scale = 1.0 / np.sqrt(hd)
    got = attention_gpu(ctx, q, pool, perm, lens, page, nh, nkv, hd, scale=scale, split_tokens=128)
    want = oracle.attention_paged(q, pool, perm, lens, page, nh, nkv, hd, scale=scale)
    assert rel_err(got, want) < REL


# ---- GEMV at the projection shapes ------------------------------
SHAPES = [(576, 576), (192, 576), (1536, 576), (576, 1536), (49152, 576)]


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("nvec", [1, 5, 9])
def test_gemv_shapes_f16(ctx, rows, cols, nvec):
    rng = np.random.default_rng(rows * 31 + cols + nvec)
    w = f16(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = oracle.f16_to_f32(f16(rng.standard_normal((nvec, cols)).astype(np.float32)))
    y = gemv_gpu(ctx, w, x)
    assert rel_err(y, oracle.gemv_f16(w, x)) < REL


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("nvec", [1, 5, 9])
def test_gemv_shapes_q8(ctx, rows, cols, nvec):
    rng = np.random.default_rng(rows * 17 + cols + nvec)
    w = f16(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    q, s = oracle.quantize_q8(w)
    x = oracle.f16_to_f32(f16(rng.standard_normal((nvec, cols)).astype(np.float32)))
    y = gemv_gpu(ctx, q, x, dtype=cu.W_Q8, scale=s)
    assert rel_err(y, oracle.gemv_q8(q, s, x)) < REL


def test_gemv_fused_rmsnorm_add(ctx):
    rng = np.random.default_rng(3)
    rows, cols, nvec = 576, 576, 3
    w = f16(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((nvec, cols)).astype(np.float32)
    g = f16(1.0 + 0.1 * rng.standard_normal(cols).astype(np.float32))
    res = rng.standard_normal((nvec, rows)).astype(np.float32)
    y = gemv_gpu(ctx, w, x, pro=cu.PRO_RMSNORM, gain=g, epi=cu.EPI_ADD, residual=res)
    xn = np.stack([oracle.rmsnorm(x[v], oracle.f16_to_f32(g), 1e-5) for v in range(nvec)])
    want = res + oracle.gemv_f16(w, xn)
    assert rel_err(y, want) < REL


def test_gemv_fused_swiglu(ctx):
    rng = np.random.default_rng(4)
    ff, cols = 1536, 576
    w = f16(rng.standard_normal((2 * ff, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((2, cols)).astype(np.float32)
    y = gemv_gpu(ctx, w, x, epi=cu.EPI_SWIGLU, rows=ff)
    gu = oracle.gemv_f16(w, x)
    want = np.stack([oracle.swiglu(gu[v, :ff], gu[v, ff:]) for v in range(2)])
    assert rel_err(y, want) < REL


def test_gemv_fused_argmax_lm_head(ctx):
    rng = np.random.default_rng(9)
    rows, cols, nvec = 49152, 576, 2
    w = f16(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((nvec, cols)).astype(np.float32)
    g = f16(np.ones(cols, np.float32))
    y, idx = gemv_gpu(ctx, w, x, pro=cu.PRO_RMSNORM, gain=g, epi=cu.EPI_ARGMAX)
    xn = np.stack([oracle.rmsnorm(x[v], np.ones(cols, np.float32), 1e-5) for v in range(nvec)])
    logits = oracle.gemv_f16(w, xn)
    assert rel_err(y, logits) < REL
    want, _ = oracle.argmax(logits)
    assert list(idx) == list(want)


def test_gemv_writes_every_output(ctx):
    # Poison-and-walk (Opure_VoxelEngine.cpp:625-636): outputs start as NaN bytes and
    # every element must be overwritten, including ragged row counts.
    rng = np.random.default_rng(2)
    for rows in (1, 3, 5, 17, 1027):
        w = f16(rng.standard_normal((rows, 64)).astype(np.float32))
        y = gemv_gpu(ctx, w, rng.standard_normal(64).astype(np.float32))
        assert not np.isnan(y).any()


# ---- tensor-core path (16..256 vectors per pass: batched decode, verify pass) ----------
# The vectors are split into fp16 hi + lo halves, so the result keeps fp32-GEMV accuracy:
# besides the 1e-3 gate, the error must stay within TC_REL of the double-precision oracle.
TC_REL = 2e-5


@pytest.mark.parametrize("rows,cols,nvec", [(576, 576, 16), (960, 576, 64), (576, 1536, 64),
                                            (192, 576, 144), (1000, 576, 300), (2048, 8192, 64)])
def test_gemv_tc_store(ctx, rows, cols, nvec):
    rng = np.random.default_rng(rows + cols + nvec)
    w = f16(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((nvec, cols)).astype(np.float32) * np.float32(3.0)
    y = gemv_gpu(ctx, w, x)
    want = oracle.gemv_f16(w, x)
    err = rel_err(y, want)
    assert err < TC_REL, err


def test_gemv_tc_rmsnorm_add(ctx):
    rng = np.random.default_rng(31)
    rows, cols, nvec = 576, 576, 64
    w = f16(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((nvec, cols)).astype(np.float32)
    x[3] *= 1e-4                                 # per-vector scales differ widely
    x[5] *= 1e3
    g = f16(1.0 + 0.1 * rng.standard_normal(cols).astype(np.float32))
    res = rng.standard_normal((nvec, rows)).astype(np.float32)
    y = gemv_gpu(ctx, w, x, pro=cu.PRO_RMSNORM, gain=g, epi=cu.EPI_ADD, residual=res)
    xn = np.stack([oracle.rmsnorm(x[v], oracle.f16_to_f32(g), 1e-5) for v in range(nvec)])
    want = res + oracle.gemv_f16(w, xn)
    assert rel_err(y, want) < TC_REL


def test_gemv_tc_unnormalised_scales(ctx):
    # Without a norm the per-vector power-of-two scale carries vectors far outside
    # fp16's range (and far below it) through the fp16 halves.
    rng = np.random.default_rng(32)
    rows, cols, nvec = 576, 1536, 32
    w = f16(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((nvec, cols)).astype(np.float32)
    x *= (10.0 ** rng.uniform(-6, 6, size=(nvec, 1))).astype(np.float32)
    y = gemv_gpu(ctx, w, x)
    want = oracle.gemv_f16(w, x)
    for v in range(nvec):
        assert rel_err(y[v], want[v]) < TC_REL, v


@pytest.mark.parametrize("nvec", [16, 64, 80])
def test_gemv_tc_swiglu(ctx, nvec):
    rng = np.random.default_rng(40 + nvec)
    ff, cols = 1536, 576
    w = f16(rng.standard_normal((2 * ff, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((nvec, cols)).astype(np.float32)
    g = f16(np.ones(cols, np.float32))
    y = gemv_gpu(ctx, w, x, pro=cu.PRO_RMSNORM, gain=g, epi=cu.EPI_SWIGLU, rows=ff)
    xn = np.stack([oracle.rmsnorm(x[v], np.ones(cols, np.float32), 1e-5) for v in range(nvec)])
    gu = oracle.gemv_f16(w, xn)
    want = np.stack([oracle.swiglu(gu[v, :ff], gu[v, ff:]) for v in range(nvec)])
    assert rel_err(y, want) < TC_REL


def test_gemv_tc_argmax_lm_head(ctx):
    rng = np.random.default_rng(41)
    rows, cols, nvec = 49152, 576, 64
    w = f16(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = rng.standard_normal((nvec, cols)).astype(np.float32)
    g = f16(np.ones(cols, np.float32))
    y, idx = gemv_gpu(ctx, w, x, pro=cu.PRO_RMSNORM, gain=g, epi=cu.EPI_ARGMAX)
    xn = np.stack([oracle.rmsnorm(x[v], np.ones(cols, np.float32), 1e-5) for v in range(nvec)])
    logits = oracle.gemv_f16(w, xn)
    assert rel_err(y, logits) < TC_REL
    want, _ = oracle.argmax(logits)
    assert list(idx) == list(want)


def test_gemv_tc_matches_cuda_core_path(ctx):
    # 15 vectors run on the CUDA-core GEMV, 16 on the tensor cores: same results to
    # within fp32 rounding.
    rng = np.random.default_rng(42)
    w = f16(rng.standard_normal((960, 576)).astype(np.float32) * 0.02)
    x = rng.standard_normal((16, 576)).astype(np.float32)
    y16 = gemv_gpu(ctx, w, x)
    y15 = gemv_gpu(ctx, w, x[:15])
    assert rel_err(y16[:15], y15) < TC_REL


def test_gemv_tc_chained_operands(ctx):
    """A decode layer's GEMV chain on packed operands: o_proj-style ADD producing the gained
    residual's packed form and per-tile sums of squares, gate;up with the RMSNorm applied from
    those sums and a packed SwiGLU output, down_proj ADD producing the next packed residual,
    and a normed STORE consumer. Each stage against the oracle on the previous stage's fp32
    output (what its packed operand encodes)."""
    rng = np.random.default_rng(43)
    n, h, ff = 64, 576, 1536
    w1 = f16(rng.standard_normal((h, h)).astype(np.float32) * 0.02)
    w2 = f16(rng.standard_normal((2 * ff, h)).astype(np.float32) * 0.02)
    w3 = f16(rng.standard_normal((h, ff)).astype(np.float32) * 0.02)
    w4 = f16(rng.standard_normal((960, h)).astype(np.float32) * 0.02)
    g2 = f16((0.5 + rng.random(h)).astype(np.float32))
    g4 = f16((0.5 + rng.random(h)).astype(np.float32))
    a = rng.standard_normal((n, h)).astype(np.float32)
    r = rng.standard_normal((n, h)).astype(np.float32) * 3.0
    tiles = (h + 127) // 128
    pk_res = ctx.buffer(cu.packed_bytes(n, h)).fill(0)
    pk_act = ctx.buffer(cu.packed_bytes(n, ff)).fill(0)
    ss = ctx.buffer(4 * tiles * n).fill(0xFF)
    dg2, dg4 = ctx.to_device(g2), ctx.to_device(g4)

    def call(w, rows, cols, x=None, x_packed=None, sums=None, pro=cu.PRO_NONE, epi=cu.EPI_STORE,
             residual=None, y_packed=None, y_gain=None, y_sumsq=None):
        dw = ctx.to_device(w)
        dy = ctx.buffer(n * rows * 4).fill(0xFF)
        args = cu.GemvArgs()
        args.w, args.w_dtype, args.rows, args.cols, args.nvec = dw.ptr, cu.W_F16, rows, cols, n
        if x is not None:
            dx = ctx.to_device(np.ascontiguousarray(x, np.float32))
            args.x, args.x_stride = dx.ptr, cols
        args.y, args.y_stride = dy.ptr, rows
        args.prologue, args.epilogue, args.eps = pro, epi, 1e-5
        if residual is not None:
            args.residual = ctx.to_device(np.ascontiguousarray(residual, np.float32)).ptr
        args.x_packed = x_packed.ptr if x_packed is not None else None
        args.x_sumsq = sums.ptr if sums is not None else None
        args.y_packed = y_packed.ptr if y_packed is not None else None
        args.y_pack_gain = y_gain.ptr if y_gain is not None else None
        args.y_sumsq = y_sumsq.ptr if y_sumsq is not None else None
        ctx.gemv(args)
        out = dy.download(np.float32, (n, rows))
        assert ctx.last_error() == 0
        return out

    # o_proj + residual from fp32 inputs, emitting g2 * x packed and the sums of squares.
    y1 = call(w1, h, h, x=a, epi=cu.EPI_ADD, residual=r, y_packed=pk_res, y_gain=dg2, y_sumsq=ss)
    assert rel_err(y1, r + oracle.gemv_f16(w1, a)) < TC_REL
    sums = ss.download(np.float32, (tiles, n)).sum(axis=0)
    assert np.allclose(sums, (y1.astype(np.float64) ** 2).sum(axis=1), rtol=1e-5)
    # gate;up + SwiGLU with the RMSNorm from the packed operand, emitting the activation.
    y2 = call(w2, ff, h, x_packed=pk_res, sums=ss, pro=cu.PRO_RMSNORM, epi=cu.EPI_SWIGLU, y_packed=pk_act)
    xn = np.stack([oracle.rmsnorm(y1[v], oracle.f16_to_f32(g2), 1e-5) for v in range(n)])
    gu = oracle.gemv_f16(w2, xn)
    want2 = np.stack([oracle.swiglu(gu[v, :ff], gu[v, ff:]) for v in range(n)])
    assert rel_err(y2, want2) < TC_REL
    # down_proj + residual from the packed activation, emitting g4 * x packed.
    y3 = call(w3, h, ff, x_packed=pk_act, epi=cu.EPI_ADD, residual=y1, y_packed=pk_res, y_gain=dg4, y_sumsq=ss)
    assert rel_err(y3, y1 + oracle.gemv_f16(w3, y2)) < TC_REL
    # A normed consumer of that (the next q;k;v).
    y4 = call(w4, 960, h, x_packed=pk_res, sums=ss, pro=cu.PRO_RMSNORM)
    xn4 = np.stack([oracle.rmsnorm(y3[v], oracle.f16_to_f32(g4), 1e-5) for v in range(n)])
    assert rel_err(y4, oracle.gemv_f16(w4, xn4)) < TC_REL


def test_gemv_tc_chained_out_of_range_is_reported(ctx):
    # A packed value beyond fp16's range cannot be represented: the kernel reports it in the
    # status word instead of writing an infinity.
    rng = np.random.default_rng(44)
    n, h = 16, 576
    w = f16(rng.standard_normal((h, h)).astype(np.float32) * 0.02)
    x = rng.standard_normal((n, h)).astype(np.float32)
    r = np.zeros((n, h), np.float32)
    r[3, 100] = 1.0e5
    pk = ctx.buffer(cu.packed_bytes(n, h)).fill(0)
    dw, dx, dr = ctx.to_device(w), ctx.to_device(x), ctx.to_device(r)
    dy = ctx.buffer(n * h * 4)
    args = cu.GemvArgs()
    args.w, args.w_dtype, args.rows, args.cols, args.nvec = dw.ptr, cu.W_F16, h, h, n
    args.x, args.x_stride, args.y, args.y_stride = dx.ptr, h, dy.ptr, h
    args.epilogue, args.residual, args.y_packed = cu.EPI_ADD, dr.ptr, pk.ptr
    ctx.gemv(args)
    ctx.sync()
    assert ctx.last_error() == cu.ERR_DEVICE_BOUNDS


def test_gemv_chained_needs_tensor_core_shape(ctx):
    # Fewer than 16 vectors run on the CUDA cores, which have no packed operands.
    n, h = 8, 576
    w = np.zeros((h, h), np.float16)
    pk = ctx.buffer(cu.packed_bytes(16, h)).fill(0)
    dw, dy = ctx.to_device(w), ctx.buffer(n * h * 4)
    args = cu.GemvArgs()
    args.w, args.w_dtype, args.rows, args.cols, args.nvec = dw.ptr, cu.W_F16, h, h, n
    args.x_packed, args.y, args.y_stride = pk.ptr, dy.ptr, h
    with pytest.raises(cu.OpureError) as e:
        ctx.gemv(args)
    assert e.value.status == cu.ERR_UNSUPPORTED


# ---- RoPE + KV append, embedding ------------------------------------------------------
@pytest.mark.parametrize("pos", [0, 1, 157, 4095])
def test_rope_kv_append(ctx, pos):
    rng = np.random.default_rng(pos + 1)
    nh, nkv, hd, page = 9, 3, 64, 64
    q = rng.standard_normal((1, nh * hd)).astype(np.float32)
    k = rng.standard_normal((1, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((1, nkv * hd)).astype(np.float32)
    maxp = pos // page + 1
    perm = rng.permutation(maxp + 2)[:maxp].astype(np.int32)
    pool = np.zeros((maxp + 2, 2, nkv, page, hd), np.uint16)
    stride = (nh + 2 * nkv) * hd + 8          # padded row: the kernel honours the stride
    qkv = np.zeros((1, stride), np.float32)
    qkv[0, : nh * hd], qkv[0, nh * hd:(nh + nkv) * hd] = q[0], k[0]
    qkv[0, (nh + nkv) * hd:(nh + 2 * nkv) * hd] = v[0]
    dqkv, dq = ctx.to_device(qkv), ctx.buffer(nh * hd * 4).fill(0xFF)
    dpool, dpt = ctx.to_device(pool), ctx.to_device(perm[None])
    dseq, dpos = ctx.to_device(np.array([0], np.int32)), ctx.to_device(np.array([pos], np.int32))
    kv = cu.KvLayout(dpool.ptr, dpt.ptr, maxp + 2, maxp, page, nkv, hd)
    ctx.call("opure_rope_kv_append", C.c_void_p(dqkv.ptr), stride, C.c_void_p(dq.ptr),
             C.c_void_p(dseq.ptr), C.c_void_p(dpos.ptr), 1, nh, 10000.0, C.byref(kv))
    gq = dq.download(np.float32, (nh * hd,))
    gpool = dpool.download(np.uint16, pool.shape)
    wq = oracle.rope(q[0], nh, hd, pos, 10000.0)
    wk = oracle.rope(k[0], nkv, hd, pos, 10000.0)
    assert rel_err(gq, wq) < 1e-6
    slot = gpool[perm[pos // page], :, :, pos % page]
    # fp16 of the rotated key may differ by one ulp where fp32 rounding of the rotation
    # straddles an fp16 tie; compare as fp16 values.
    assert np.abs(oracle.f16_to_f32(slot[0]).ravel() - wk).max() <= 1e-3 * np.abs(wk).max()
    assert np.array_equal(slot[1], f16(v[0]).reshape(nkv, hd))
    assert ctx.last_error() == 0


def test_rope_kv_out_of_range_page_is_refused(ctx):
    # A position past the page table is refused by the kernel's own bounds check and
    # reported through the status word; nothing is written.
    nh, nkv, hd, page = 9, 3, 64, 16
    pool = np.zeros((2, 2, nkv, page, hd), np.uint16)
    stride = (nh + 2 * nkv) * hd
    dqkv, dq = ctx.buffer(stride * 4).fill(0), ctx.buffer(nh * hd * 4).fill(0)
    dpool, dpt = ctx.to_device(pool), ctx.to_device(np.array([[0, 1]], np.int32))
    dseq, dpos = ctx.to_device(np.array([0], np.int32)), ctx.to_device(np.array([40], np.int32))
    kv = cu.KvLayout(dpool.ptr, dpt.ptr, 2, 2, page, nkv, hd)
    ctx.call("opure_rope_kv_append", C.c_void_p(dqkv.ptr), stride, C.c_void_p(dq.ptr),
             C.c_void_p(dseq.ptr), C.c_void_p(dpos.ptr), 1, nh, 10000.0, C.byref(kv))
    assert ctx.last_error() == cu.ERR_DEVICE_BOUNDS
    assert ctx.last_error() == 0  # cleared by the read
    assert not dpool.download(np.uint16, pool.shape).any()


def test_embedding(ctx):
    rng = np.random.default_rng(8)
    V, d = 1000, 576
    E = f16(rng.standard_normal((V, d)).astype(np.float32) * 0.02)
    toks = np.array([0, 999, 17, 17], np.int32)
    dE, dt, dout = ctx.to_device(E), ctx.to_device(toks), ctx.buffer(4 * d * 4)
    ctx.call("opure_embedding", C.c_void_p(dE.ptr), V, C.c_void_p(dt.ptr), 4, d, C.c_void_p(dout.ptr))
    assert np.array_equal(dout.download(np.float32, (4, d)), oracle.f16_to_f32(E[toks]))


# ---- speculative accept / sampling ----------------------------------------------------
def test_spec_accept_greedy_and_rejection(ctx):
    rng = np.random.default_rng(21)
    S, k, V = 4, 4, 4096
    tl = rng.standard_normal((S, k + 1, V)).astype(np.float32) * 3
    dl = (tl[:, :k] + rng.standard_normal((S, k, V)).astype(np.float32) * 0.8).astype(np.float32)
    draft = np.zeros((S, k), np.int32)
    for s in range(S):
        for i in range(k):
            draft[s, i] = int(np.argmax(tl[s, i])) if (s + i) % 3 else int(np.argmax(dl[s, i]))
    ua = rng.random((S, k)).astype(np.float32)
    uf = rng.random(S).astype(np.float32)
    for mode in (cu.SPEC_GREEDY, cu.SPEC_REJECTION):
        d_tl, d_dl, d_dr = ctx.to_device(tl), ctx.to_device(dl), ctx.to_device(draft)
        d_ua, d_uf = ctx.to_device(ua), ctx.to_device(uf)
        d_out, d_acc = ctx.buffer(S * (k + 1) * 4).fill(0xFF), ctx.buffer(S * 4)
        a = cu.SpecArgs(mode, S, k, V, d_tl.ptr, d_dl.ptr, d_dr.ptr, d_ua.ptr, d_uf.ptr,
                        d_out.ptr, d_acc.ptr)
        ctx.spec_accept(a)
        out = d_out.download(np.int32, (S, k + 1))
        acc = d_acc.download(np.int32, S)
        for s in range(S):
            if mode == cu.SPEC_GREEDY:
                wa, wt = oracle.spec_accept_greedy(tl[s], draft[s])
            else:
                wa, wt = oracle.spec_accept_rejection(tl[s], dl[s], draft[s], ua[s], uf[s])
            assert acc[s] == wa, (mode, s)
            assert list(out[s, : wa + 1]) == list(wt), (mode, s)


def test_sample_softmax(ctx):
    rng = np.random.default_rng(6)
    R, V = 16, 49152
    lg = rng.standard_normal((R, V)).astype(np.float32) * 2
    u = rng.random(R).astype(np.float32)
    d_l, d_u, d_o = ctx.to_device(lg), ctx.to_device(u), ctx.buffer(R * 4)
    ctx.call("opure_sample_softmax", C.c_void_p(d_l.ptr), V, R, C.c_void_p(d_u.ptr), C.c_void_p(d_o.ptr))
    got = d_o.download(np.int32, R)
    want = [oracle.sample_softmax(lg[r], float(u[r])) for r in range(R)]
    assert list(got) == want


# ---- ABI error paths -------------------------------------------------------------------
def test_invalid_arguments_are_refused(ctx):
    a = cu.GemvArgs()
    with pytest.raises(cu.OpureError) as e:
        ctx.gemv(a)
    assert e.value.status == cu.ERR_INVALID_ARG
    assert ctx.last_error() == 0


def test_injected_failure(ctx):
    cu.lib().opure_debug_inject_failure(ctx.h, 1, 1)
    ctx.sync()                                   # consumes the one allowed call
    with pytest.raises(cu.OpureError) as e:
        ctx.sync()
    assert e.value.status == cu.ERR_INJECTED
    ctx.sync()                                   # disarmed again
