"""The multi-rank paths of bench.py with two gloo ranks on the CPU (no GPU).

bench.py runs one process per GPU under torchrun. Independent sequences are split across
ranks with no collective on the data path; the ranks only meet at barriers and at the
max-over-ranks timing and sum-over-ranks token reductions. These tests run those pieces as
two spawned processes over gloo (127.0.0.1): every sequence is assigned to exactly one
rank, the reductions agree on every rank, and `--impl reference` does no work on rank 1.
"""
import io
import multiprocessing as mp
import os
import socket
import sys
from contextlib import redirect_stdout

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                          RANK=str(rank), LOCAL_RANK=str(rank))
        sys.path.insert(0, REPO)
        import bench
        import torch.distributed as dist
        w, r, local = bench.dist_init()
        out = {"world": w, "rank": r, "local": local}
        out["shards"] = {t: bench.shard(t, w, r) for t in (1, 2, 7, 512, 513)}
        out["max"] = bench.allreduce_max(w, 1.5 * (r + 1))
        out["sum"] = bench.allreduce_sum(w, float(10 + r))
        bench.barrier(w)
        gathered = [None] * w
        dist.all_gather_object(gathered, out["shards"])
        out["all_shards"] = gathered
        if r == 1:
            # The reference arm runs on rank 0 only; other ranks exit without work.
            class Args:
                steps, warmup, batch, gpus = 2, 3, 1, w
            buf = io.StringIO()
            with redirect_stdout(buf):
                ret = bench.run_reference(Args(), w, r)
            out["ref_rank1"] = (ret, buf.getvalue())
        bench.barrier(w)
        dist.destroy_process_group()
        q.put((rank, out))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, {"error": repr(e)}))


def test_two_gloo_ranks_shard_and_reduce():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert "error" not in res[r], res[r]
        assert (res[r]["world"], res[r]["rank"]) == (world, r)
        assert res[r]["max"] == 3.0
        assert res[r]["sum"] == 21.0
    # Every sequence of every total belongs to exactly one rank, in contiguous ranges.
    gathered = res[0]["all_shards"]
    assert gathered == res[1]["all_shards"]
    for total in (1, 2, 7, 512, 513):
        covered = []
        for r in range(world):
            first, count = gathered[r][total]
            covered += list(range(first, first + count))
        assert covered == list(range(total)), total
    assert res[1]["ref_rank1"] == (None, "")


@pytest.mark.parametrize("total,world", [(512, 8), (513, 8), (5, 8), (64, 3)])
def test_shard_covers_every_sequence_once(total, world):
    sys.path.insert(0, REPO)
    import bench
    spans = [bench.shard(total, world, r) for r in range(world)]
    flat = [i for first, count in spans for i in range(first, first + count)]
    assert flat == list(range(total))
    counts = [c for _, c in spans]
    assert max(counts) - min(counts) <= 1
