"""The whole decode path on the GPU (libopure_engine -> libopure_cuda) vs the CPU oracle.

Mirrors the reference's model-level checks (Opure_TestHarness.cpp:588-1059): logits vs
the CPU reference, the per-layer residual trace, argmax agreement and generation --
here on seeded synthetic models, with multi-token prompts, positions > 0 (RoPE), paged
KV with shuffled page tables, batches and int8 weights, which the reference never tests.
Gates: token ids bit-exact; logits max_abs <= 2e-2 and <= 1e-3 relative; the
reference's own rms criterion is reported alongside.
"""
import os

import numpy as np
import pytest

import oracle
from common import compare, greedy_tokens_agree, rel_err
from voxelengine import engine as ve

pytestmark = pytest.mark.gpu
oracle.set_threads(os.cpu_count() or 1)

SMALL = dict(vocab=4096, hidden=576, inter=1536, layers=3, heads=9, kv_heads=3, max_pos=512)
HD128 = dict(vocab=2048, hidden=512, inter=1024, layers=2, heads=4, kv_heads=2, max_pos=512)


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    root = tmp_path_factory.mktemp("models")
    return {
        "small": ve.synth_model(str(root / "small"), seed=21, **SMALL),
        "q8": ve.synth_model(str(root / "q8"), seed=21, int8=True, **SMALL),
        "hd128": ve.synth_model(str(root / "hd128"), seed=22, **HD128),
    }


@pytest.fixture(scope="module")
def small(models):
    return oracle.Model(models["small"])


def assert_tokens(got, want, margins):
    got, want = np.asarray(got), np.asarray(want)
    if not np.array_equal(got, want):
        i = int(np.argmax(got != want))
        raise AssertionError(f"first token mismatch at step {i}: gpu {got[i]} oracle {want[i]} "
                             f"(oracle top-2 margin there {margins[i]:.3e})")


def test_generate_matches_oracle(models, small):
    p = ve.prompt(1, SMALL["vocab"], 12)
    with ve.Engine(models["small"], max_len=64) as eng:
        out, t = eng.generate([p], 24)
    want, margins = small.generate(p, 24)
    assert_tokens(out[0], want, margins)
    assert t.decode_steps == 24 and t.decode_ms > 0


def test_forward_logits_and_argmax(models, small):
    p = ve.prompt(7, SMALL["vocab"], 9)
    with ve.Engine(models["small"], max_len=64) as eng:
        logits = eng.forward_logits(p)
        am = eng.forward_argmax(p)
    st = small.state(64)
    for i, t in enumerate(p):
        lg, _ = st.forward(int(t), logits=(i == len(p) - 1))
    assert np.abs(logits - lg).max() <= 2e-2
    assert rel_err(logits, lg) < 1e-3
    ok, max_abs, rms = compare(logits, lg)
    print(f"logits vs oracle: max_abs {max_abs:.3e} rms {rms:.3e} reference-criterion {ok}")
    assert am == int(np.argmax(lg))


def test_layer_trace(models, small):
    # RunLayersTraced vs ForwardTraced (Opure_TestHarness.cpp:956-987): the residual after
    # every layer for one token at position 0.
    with ve.Engine(models["small"], max_len=16) as eng:
        tr = eng.trace(123, SMALL["layers"])
    _, want = small.state(16).forward(123, logits=False, trace=True)
    for layer in range(SMALL["layers"]):
        assert np.abs(tr[layer] - want[layer]).max() <= 1e-3, layer


def test_batch_of_independent_sequences(models, small):
    prompts = [ve.prompt(s, SMALL["vocab"], n) for s, n in ((2, 5), (3, 11), (4, 8))]
    with ve.Engine(models["small"], max_batch=3, max_len=64) as eng:
        out, _ = eng.generate(prompts, 16)
    for b, p in enumerate(prompts):
        want, margins = small.generate(p, 16)
        assert_tokens(out[b], want, margins)


def test_batch_beyond_one_gemv_pass(models, small):
    # 12 vectors: the GEMV stages at most 9 input vectors per pass.
    prompts = [ve.prompt(100 + s, SMALL["vocab"], 4) for s in range(12)]
    with ve.Engine(models["small"], max_batch=12, max_len=32) as eng:
        out, _ = eng.generate(prompts, 6)
    for b in (0, 5, 11):
        want, margins = small.generate(prompts[b], 6)
        assert_tokens(out[b], want, margins)


@pytest.mark.parametrize("n", [16, 40])
def test_tensor_core_batch_matches_oracle(models, small, n):
    # n >= 16 vectors take the per-layer kernels with the tensor-core GEMV path
    # (pack + tcgen05 GEMM per projection), ragged prompts.
    prompts = [ve.prompt(300 + s, SMALL["vocab"], 3 + s % 7) for s in range(n)]
    with ve.Engine(models["small"], max_batch=n, max_len=40) as eng:
        out, _ = eng.generate(prompts, 12)
    for b in range(0, n, 3):
        want, margins = small.generate(prompts[b], 12)
        assert_tokens(out[b], want, margins)


def test_host_driven_decode_steps(models):
    # Prefill + DecodeStep with the token/position copied in and the argmax read back
    # each step (Opure_VoxelEngine.cpp:765-800) equals the device-driven loop.
    p = ve.prompt(5, SMALL["vocab"], 6)
    with ve.Engine(models["small"], max_len=64) as eng:
        ref, _ = eng.generate([p], 10)
        nxt = eng.prefill(p)  # the prompt's argmax = first generated token
        toks = [nxt]
        for i in range(9):
            nxt = int(eng.decode_step([toks[-1]], [len(p) + i])[0])
            toks.append(nxt)
    assert toks == list(ref[0])


@pytest.mark.parametrize("page_size,seed,graphs", [(16, 3, True), (128, 0, True), (64, 9, False)])
def test_paging_and_graph_modes(models, small, page_size, seed, graphs):
    p = ve.prompt(9, SMALL["vocab"], 20)
    with ve.Engine(models["small"], max_len=96, page_size=page_size, page_seed=seed,
                   use_graphs=graphs) as eng:
        out, _ = eng.generate([p], 40)
    want, margins = small.generate(p, 40)
    assert_tokens(out[0], want, margins)


def test_int8_model(models):
    m = oracle.Model(models["q8"])
    p = ve.prompt(1, SMALL["vocab"], 10)
    with ve.Engine(models["q8"], max_len=64) as eng:
        out, _ = eng.generate([p], 16)
        logits = eng.forward_logits(p)
    want, margins = m.generate(p, 16)
    assert_tokens(out[0], want, margins)
    st = m.state(64)
    for i, t in enumerate(p):
        lg, _ = st.forward(int(t), logits=(i == len(p) - 1))
    assert rel_err(logits, lg) < 1e-3


def test_head_dim_128(models):
    m = oracle.Model(models["hd128"])
    p = ve.prompt(2, HD128["vocab"], 7)
    with ve.Engine(models["hd128"], max_len=64) as eng:
        out, _ = eng.generate([p], 20)
    want, margins = m.generate(p, 20)
    assert_tokens(out[0], want, margins)


def test_poisoned_buffers_do_not_leak(models, small):
    # Poison-and-walk (Opure_TestHarness.cpp:794-870): every activation the step reads
    # must have been written by the step itself.
    p = ve.prompt(4, SMALL["vocab"], 5)
    with ve.Engine(models["small"], max_len=32) as eng:
        eng.poison(float("nan"))
        out, _ = eng.generate([p], 8)
    want, margins = small.generate(p, 8)
    assert_tokens(out[0], want, margins)


def test_config0_smollm_full_size(smollm_dirs):
    # SmolLM-135M shape, weights N(0, 0.02) seed 0, 32-token prompt
    # seed 1, prefill then 128 greedy decode steps, batch 1, paged fp16 KV.
    d = smollm_dirs[0]
    p = ve.prompt(1, 49152, 32)
    with ve.Engine(d, max_len=256) as eng:
        out, t = eng.generate([p], 128)
    with ve.Engine(d, max_len=256, prefill_chunk=32) as eng:
        out_c, tc = eng.generate([p], 128)   # the 32-token prompt as one tensor-core step
    want, margins = oracle.Model(d).generate(p, 128)
    print(f"cfg0: decode {t.decode_ms / 128 * 1e3:.1f} us/token, prefill {t.prefill_ms:.2f} ms per-token "
          f"vs {tc.prefill_ms:.2f} ms chunked, min oracle margin {margins.min():.3e}")
    assert_tokens(out[0], want, margins)
    assert_tokens(out_c[0], want, margins)


# ---- the fused latency path (opure_decode_fused) ------------------------------------
@pytest.mark.parametrize("batch", [1, 2, 4, 8])
def test_fused_path_matches_oracle(models, small, batch):
    prompts = [ve.prompt(40 + b, SMALL["vocab"], 6 + 2 * b) for b in range(batch)]
    with ve.Engine(models["small"], max_batch=batch, max_len=96, path=ve.PATH_FUSED) as eng:
        out, _ = eng.generate(prompts, 30)
    for b in range(batch):
        want, margins = small.generate(prompts[b], 30)
        assert_tokens(out[b], want, margins)


def test_fused_and_per_op_paths_agree(models, small):
    p = ve.prompt(77, SMALL["vocab"], 17)
    res = {}
    for path in (ve.PATH_FUSED, ve.PATH_UNFUSED):
        with ve.Engine(models["small"], max_len=64, path=path) as eng:
            res[path] = (eng.generate([p], 20)[0][0], eng.forward_logits(p))
    assert np.array_equal(res[ve.PATH_FUSED][0], res[ve.PATH_UNFUSED][0])
    assert rel_err(res[ve.PATH_FUSED][1], res[ve.PATH_UNFUSED][1]) < 1e-4
    st = small.state(64)
    for i, t in enumerate(p):
        lg, _ = st.forward(int(t), logits=(i == len(p) - 1))
    assert rel_err(res[ve.PATH_FUSED][1], lg) < 1e-3


@pytest.mark.parametrize("batch", [1, 4])
def test_persistent_and_layer_kernels_agree(models, small, batch):
    # The single persistent kernel per step (PATH_FUSED on this shape) against the same
    # phases as three kernels per layer: identical tokens (the residual sums are
    # fixed-point, so both are order-independent) and logits equal to fp32 rounding.
    prompts = [ve.prompt(90 + b, SMALL["vocab"], 13) for b in range(batch)]
    res = {}
    for path in (ve.PATH_FUSED, ve.PATH_FUSED_LAYERS):
        with ve.Engine(models["small"], max_batch=batch, max_len=64, path=path) as eng:
            res[path] = eng.generate(prompts, 24)[0]
            lg = eng.forward_logits(prompts[0]) if batch == 1 else None
            res[(path, "lg")] = lg
    assert np.array_equal(res[ve.PATH_FUSED], res[ve.PATH_FUSED_LAYERS])
    if batch == 1:
        assert rel_err(res[(ve.PATH_FUSED, "lg")], res[(ve.PATH_FUSED_LAYERS, "lg")]) < 1e-5
    want, margins = small.generate(prompts[0], 24)
    assert_tokens(res[ve.PATH_FUSED][0], want, margins)


def test_fused_head_dim_128(models):
    m = oracle.Model(models["hd128"])
    p = ve.prompt(3, HD128["vocab"], 9)
    with ve.Engine(models["hd128"], max_len=64, path=ve.PATH_FUSED) as eng:
        out, _ = eng.generate([p], 20)
    want, margins = m.generate(p, 20)
    assert_tokens(out[0], want, margins)


def test_fused_host_driven_steps(models):
    p = ve.prompt(6, SMALL["vocab"], 5)
    with ve.Engine(models["small"], max_len=64, path=ve.PATH_FUSED) as eng:
        ref, _ = eng.generate([p], 8)
        toks = [eng.prefill(p)]
        for i in range(7):
            toks.append(int(eng.decode_step([toks[-1]], [len(p) + i])[0]))
    assert toks == list(ref[0])


@pytest.mark.parametrize("batch", [1, 2, 4])
def test_int8_persistent_path_matches_oracle(models, batch):
    # GEMV_Quant weights on the persistent step kernel (int8 slices streamed through the same
    # shared-memory slots, each dot product scaled by its tensor's scale) against the oracle,
    # and against the per-op int8 kernels.
    m = oracle.Model(models["q8"])
    prompts = [ve.prompt(500 + b, SMALL["vocab"], 9 + 3 * b) for b in range(batch)]
    with ve.Engine(models["q8"], max_batch=batch, max_len=80, path=ve.PATH_FUSED) as eng:
        out, _ = eng.generate(prompts, 24)
    with ve.Engine(models["q8"], max_batch=batch, max_len=80, path=ve.PATH_UNFUSED) as eng:
        per_op, _ = eng.generate(prompts, 24)
    for b in range(batch):
        want, margins = m.generate(prompts[b], 24)
        assert_tokens(out[b], want, margins)
    assert np.array_equal(out, per_op)


def test_int8_layer_kernels_are_refused(models):
    # int8 runs on the persistent kernel only; the three-kernels-per-layer path refuses it.
    with pytest.raises(Exception):
        ve.Engine(models["q8"], max_len=32, path=ve.PATH_FUSED_LAYERS)


def test_config0_int8_full_size(tmp_path_factory):
    # The config-0 model quantised per tensor (absmax / 127) decodes its 128 tokens on the
    # persistent kernel as the oracle does on the same int8 weights.
    d = ve.synth_model(str(tmp_path_factory.mktemp("cfg0q8")), seed=0, int8=True)
    p = ve.prompt(1, 49152, 32)
    with ve.Engine(d, max_len=256) as eng:
        out, _ = eng.generate([p], 128)
    want, _, margins, second = oracle.Model(d).generate_batch([p], 128, threads=os.cpu_count() or 1)
    n, note = greedy_tokens_agree(out[0], want[0], margins[0], second[0])
    print(f"cfg0 int8: {note}")
    assert n >= 64


@pytest.mark.parametrize("n,length", [(2, 200), (16, 130)])
def test_synthetic_long_context_matches_oracle(models, small, n, length):
    # Seeded KV contexts written on the device (opure_kv_synth) decode like the oracle
    # given the same values through load_kv; n = 16 runs the tensor-core GEMV path.
    c = SMALL
    first = ve.prompt(77, c["vocab"], n)
    with ve.Engine(models["small"], max_batch=n, max_len=length + 16) as eng:
        eng.synth_context(n, length, length + 12, 9, first)
        # A step's output enters the history as the next step's input: 9 steps leave 8.
        eng.run_steps(n, 9)
        eng.sync()
        got = [eng.read_tokens(v, length + 1, 8) for v in range(n)]
    for v in (0, n - 1):
        st = small.state(length + 16)
        st.load_kv(ve.synth_kv(9, v, c["layers"], c["kv_heads"], length, c["hidden"] // c["heads"]), length)
        tok, want, margins = int(first[v]), [], []
        for _ in range(8):
            lg, _ = st.forward(tok)
            tok = int(oracle.argmax(lg[None])[0][0])
            want.append(tok)
            top = np.sort(lg)[-2:]
            margins.append(float(top[1] - top[0]))
        assert_tokens(got[v], want, margins)


@pytest.mark.parametrize("chunk", [16, 64])
def test_chunked_prefill_matches_oracle(models, small, chunk):
    # Prompts of different lengths prefilled as steps of up to `chunk` token vectors
    # (several sequences per step, causal attention inside the step, tensor-core GEMMs
    # from 16 vectors), then self-driving decode: the oracle's tokens for every sequence.
    lens = (40, 17, 33)
    prompts = [ve.prompt(60 + i, SMALL["vocab"], n) for i, n in enumerate(lens)]
    with ve.Engine(models["small"], max_batch=3, max_len=96, prefill_chunk=chunk) as eng:
        got, t = eng.generate(prompts, 12)
    assert t.prefill_steps == -(-sum(lens) // chunk)
    for i, p in enumerate(prompts):
        want, margins = small.generate(p, 12)
        assert_tokens(got[i], want, margins)


def test_chunked_prefill_then_host_steps(models, small):
    # Prefill (chunked) followed by the reference's host-driven DecodeStep loop.
    p = ve.prompt(71, SMALL["vocab"], 21)
    want, margins = small.generate(p, 6)
    with ve.Engine(models["small"], max_len=64, prefill_chunk=16) as eng:
        tok = eng.prefill(p)
        got = [tok]
        for i in range(5):
            tok = int(eng.decode_step([tok], [len(p) + i])[0])
            got.append(tok)
    assert_tokens(got, want, margins)


# ---- sliding-window KV cache (pages recycled as a ring) ------------------------------
def windowed_oracle(small, prompt, budget, page, ring):
    """Greedy generation on the oracle with the same window (orc_state_set_window)."""
    st = small.state(len(prompt) + budget + 2)
    st.set_window(page, ring)
    lg = None
    for i, t in enumerate(prompt):
        lg, _ = st.forward(int(t), logits=(i == len(prompt) - 1))
    out, margins = [], []
    for j in range(budget):
        top = np.partition(lg, -2)[-2:]
        tok = int(oracle.argmax(lg[None])[0][0])
        out.append(tok)
        margins.append(float(abs(top[1] - top[0])))
        if j + 1 < budget:
            lg, _ = st.forward(tok)
    return np.array(out), np.array(margins)


@pytest.mark.parametrize("path,n", [(ve.PATH_AUTO, 1), (ve.PATH_AUTO, 3), (ve.PATH_FUSED_LAYERS, 2),
                                    (ve.PATH_UNFUSED, 2), (ve.PATH_AUTO, 17)])
def test_sliding_window_matches_oracle(models, small, path, n):
    # 16-token pages, a 3-page window: after 48 tokens every new page overwrites the
    # sequence's oldest one and attention covers the last 2 whole pages + the current one.
    # n = 1 / 3 run the persistent kernel, n = 17 the per-layer tensor-core path.
    page, ring, budget = 16, 3, 70
    prompts = [ve.prompt(500 + s, SMALL["vocab"], 9 + s % 4) for s in range(n)]
    with ve.Engine(models["small"], max_batch=n, max_len=96, page_size=page, kv_window=page * ring,
                   path=path) as eng:
        out, _ = eng.generate(prompts, budget)
    for b in sorted({0, n - 1}):
        want, margins = windowed_oracle(small, prompts[b], budget, page, ring)
        assert_tokens(out[b], want, margins)
    # The window matters: without it the oracle's tokens differ after the first wrap.
    full, _ = small.generate(prompts[0], budget)
    want0, _ = windowed_oracle(small, prompts[0], budget, page, ring)
    assert not np.array_equal(full, want0)


def test_sliding_window_chunked_prefill_and_limits(models, small):
    page, ring = 16, 3
    p = ve.prompt(600, SMALL["vocab"], 40)
    with ve.Engine(models["small"], max_len=128, page_size=page, kv_window=page * ring, prefill_chunk=16) as eng:
        out, _ = eng.generate([p], 60)
    want, margins = windowed_oracle(small, p, 60, page, ring)
    assert_tokens(out[0], want, margins)
    with pytest.raises(Exception):  # a prompt longer than the window cannot be chunk-prefilled
        with ve.Engine(models["small"], max_len=128, page_size=page, kv_window=page * ring,
                       prefill_chunk=16) as eng:
            eng.generate([ve.prompt(601, SMALL["vocab"], 60)], 4)
    with pytest.raises(Exception):  # not a multiple of the page size
        ve.Engine(models["small"], max_len=128, page_size=page, kv_window=40)


@pytest.mark.parametrize("window", [0, 48])
def test_chunked_prefill_with_poisoned_buffers(models, small, window):
    # A chunked prefill step has more token vectors than there are sequences: every vector's
    # step state (flags, known length) must be set by the host for that step, not left from
    # earlier use of the slot. Poison-and-walk with every slot marked self-driving, NaN
    # activations and NaN chained operands; one prompt in a two-sequence engine.
    page = 16
    p = ve.prompt(600, SMALL["vocab"], 40)
    kw = dict(kv_window=window) if window else {}
    with ve.Engine(models["small"], max_batch=2, max_len=128, page_size=page, prefill_chunk=16, **kw) as eng:
        eng.poison(float("nan"))
        out, _ = eng.generate([p], 12)
    want, margins = windowed_oracle(small, p, 12, page, window // page) if window else small.generate(p, 12)
    assert_tokens(out[0], want, margins)


# ---- Generate's stop rules (Opure_VoxelEngine.cpp:904,918-933) ------------------------
def _with_config(src, dst, **edits):
    """A model directory sharing src's weights with config.json edited."""
    import json
    os.makedirs(dst, exist_ok=True)
    cfg = json.load(open(os.path.join(src, "config.json")))
    cfg.update(edits)
    with open(os.path.join(dst, "config.json"), "w") as f:
        json.dump(cfg, f)
    link = os.path.join(dst, "model.safetensors")
    if not os.path.exists(link):
        os.symlink(os.path.join(src, "model.safetensors"), link)
    return dst


@pytest.mark.parametrize("batch,chunk", [(1, 0), (3, 0), (3, 16)])
def test_generate_stops_on_eos(models, small, tmp_path, batch, chunk):
    # The stop id (config.json's eos_token_id) is the 10th token of sequence 0's free run:
    # that sequence stops at its first occurrence, inclusive; the others stop wherever it
    # first appears in theirs, or run the whole budget.
    prompts = [ve.prompt(300 + s, SMALL["vocab"], 7 + 3 * s) for s in range(batch)]
    eos = int(small.generate(prompts[0], 40)[0][9])
    d = _with_config(models["small"], str(tmp_path / "eos"), eos_token_id=eos)
    m = oracle.Model(d)
    with ve.Engine(d, max_batch=batch, max_len=96, prefill_chunk=chunk) as eng:
        out, counts, hit, _ = eng.generate_stop(prompts, 40)
    for s, p in enumerate(prompts):
        want, margins, want_hit = m.generate_stop(p, 40)
        assert counts[s] == want.size and bool(hit[s]) == want_hit, (s, counts[s], want.size)
        assert_tokens(out[s, : counts[s]], want, margins)
        assert (out[s, counts[s]:] == -1).all()
    assert hit[0] and counts[0] <= 10


def test_generate_stops_at_max_positions(models, small, tmp_path):
    # max_position_embeddings 48: a prompt of length n gets 48 - n tokens (seqLen + 1 >=
    # maxPos ends the loop), whatever the budget.
    d = _with_config(models["small"], str(tmp_path / "maxpos"), max_position_embeddings=48)
    m = oracle.Model(d)
    prompts = [ve.prompt(400 + s, SMALL["vocab"], 20 + 8 * s) for s in range(2)]
    with ve.Engine(d, max_batch=2) as eng:
        out, counts, hit, _ = eng.generate_stop(prompts, 64)
    for s, p in enumerate(prompts):
        want, margins, _ = m.generate_stop(p, 64)
        assert want.size == 48 - p.size and counts[s] == want.size and not hit[s]
        assert_tokens(out[s, : counts[s]], want, margins)


# ---- BASELINE config 0 at batch 64 (the tensor-core path) ------------------------------
def test_config0_bs64_full_size(smollm_dirs):
    # All 64 config-0 sequences (prompt seeds 1..64, 32 tokens) decode 128 tokens in one
    # batch on the tcgen05 GEMV path; every fourth sequence is checked against the oracle
    # (16 sequences, run one per host thread).
    d = smollm_dirs[0]
    prompts = [ve.prompt(1 + b, 49152, 32) for b in range(64)]
    with ve.Engine(d, max_batch=64, max_len=168) as eng:
        out, _ = eng.generate(prompts, 128)
    checked = list(range(0, 64, 4))
    want, counts, margins, second = oracle.Model(d).generate_batch([prompts[b] for b in checked], 128,
                                                                   threads=os.cpu_count() or 1)
    notes = []
    for i, b in enumerate(checked):
        assert counts[i] == 128
        n, note = greedy_tokens_agree(out[b], want[i], margins[i], second[i])
        notes.append(note)
    ties = [x for x in notes if x != "equal"]
    print(f"bs64: {len(checked) - len(ties)} of {len(checked)} sequences equal for 128 tokens; {ties}")
    assert len(ties) <= 2
