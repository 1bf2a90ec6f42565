"""Tensor-parallel decode (BASELINE config 4's second variant) on 2 GPUs vs the oracle.

Each rank is a spawned process with its own GPU, ctx and NCCL communicator (the 128-byte
id comes from the parent); every rank holds its shard of a small Llama-shaped model and
the ranks all-reduce the o_proj / down_proj partial sums and the argmax keys each step.
Gates: every rank generates the oracle's tokens exactly (the unsharded model on the CPU).
Skipped with fewer than 2 GPUs.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

import oracle
from voxelengine import cuda as cu
from voxelengine import engine as ve

pytestmark = pytest.mark.gpu
oracle.set_threads(os.cpu_count() or 1)

MHA = dict(vocab=4096, hidden=512, inter=1024, layers=2, heads=8, kv_heads=8, max_pos=256)
GQA = dict(vocab=4096, hidden=512, inter=1024, layers=2, heads=8, kv_heads=4, max_pos=256)


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


needs2 = pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")


def _rank_main(rank, n, uid, model, prompt, budget, q):
    try:
        import sys
        repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [repo, os.path.join(repo, "opure-voxelengine_b200")]
        from voxelengine import cuda as cu2
        from voxelengine import engine as ve2
        ctx = cu2.Ctx(rank)
        comm = cu2.Comm(ctx, n, rank, uid, timeout_ms=60000)
        out = {}
        if model is None:
            # All-reduce check: rank r contributes r + i; the sum is known.
            buf = ctx.to_device(np.arange(1000, dtype=np.float32) + rank)
            comm.allreduce_sum(buf, 1000)
            keys = ctx.to_device(np.array([rank + 1, 5 - rank], np.uint64))
            comm.allreduce_max_u64(keys, 2)
            ctx.sync()
            out["sum"] = buf.download(np.float32, 1000)
            out["max"] = keys.download(np.uint64, 2)
        else:
            eng = ve2.Engine(model, max_len=64, comm=comm)
            toks, _ = eng.generate([prompt], budget)
            out["tokens"] = toks[0]
            out["stream_bytes"] = eng.info.stream_bytes
            eng.close()
        comm.close()
        ctx.close()
        q.put((rank, out))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, {"error": repr(e)}))


def _run(n, model=None, prompt=None, budget=0):
    uid = cu.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, n, uid, model, prompt, budget, q)) for r in range(n)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(n):
        r, out = q.get(timeout=300)
        res[r] = out
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r, out in res.items():
        assert "error" not in out, (r, out)
    return res


@needs2
def test_allreduce_two_ranks():
    res = _run(2)
    for r in range(2):
        assert np.array_equal(res[r]["sum"], 2 * np.arange(1000, dtype=np.float32) + 1)
        assert list(res[r]["max"]) == [2, 5]


@needs2
@pytest.mark.parametrize("shape", ["mha", "gqa"])
def test_tensor_parallel_generate_matches_oracle(tmp_path, shape):
    spec = MHA if shape == "mha" else GQA
    model = ve.synth_model(str(tmp_path / shape), seed=31, **spec)
    prompt = ve.prompt(5, spec["vocab"], 10)
    res = _run(2, model, prompt, 16)
    want, margins = oracle.Model(model).generate(prompt, 16)
    for r in range(2):
        got = np.asarray(res[r]["tokens"])
        if not np.array_equal(got, want):
            i = int(np.argmax(got != want))
            raise AssertionError(f"rank {r}: first mismatch at {i}: {got[i]} vs {want[i]} "
                                 f"(oracle top-2 margin {margins[i]:.3e})")
    # Each shard streams its share of the matrices (+ the whole norms).
    full = ve.inspect(model).stream_bytes
    assert res[0]["stream_bytes"] < full
